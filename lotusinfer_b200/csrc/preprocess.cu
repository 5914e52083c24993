// Input preprocessing of the reference's classification demo
// (demo/image_classification.cpp:9-44, done there on the CPU with OpenCV) as
// one memory-bound kernel: 8-bit BGR HWC images -> bilinear resize (the
// cv::resize INTER_LINEAR geometry: half-pixel centres, source index clamped
// to the edge) -> RGB -> /255 -> centre crop -> (x - mean) / std, written as
// the NCHW fp32 batch the graph input takes.  One thread per output element
// of a row run; the resize is evaluated only at the cropped pixels.  Every
// float operation is rounded on its own (no contraction), in the order of the
// CPU oracle, so the two agree to the last bits.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace lotus_impl {

namespace {

struct Axis {
  int i0, i1;
  float a;
};

__device__ __forceinline__ Axis axis_of(int d, int n_src, float scale) {
  const float f = __fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(d), 0.5f), scale), 0.5f);
  const float s = floorf(f);
  Axis r;
  r.a = __fsub_rn(f, s);
  r.i0 = static_cast<int>(s);
  if (r.i0 < 0) {
    r.i0 = 0;
    r.a = 0.f;
  }
  if (r.i0 >= n_src - 1) {
    r.i0 = n_src - 1;
    r.a = 0.f;
  }
  r.i1 = min(r.i0 + 1, n_src - 1);
  return r;
}

struct PrepParams {
  const uint8_t* src;
  float* dst;
  int n, h, w, rh, rw, ch, cw, y0, x0;
  float mean[3], stdv[3];
};

__global__ void preprocess_kernel(const PrepParams p) {
  const int64_t total = static_cast<int64_t>(p.n) * 3 * p.ch * p.cw;
  const float sy = __fdiv_rn(static_cast<float>(p.h), static_cast<float>(p.rh));
  const float sx = __fdiv_rn(static_cast<float>(p.w), static_cast<float>(p.rw));
  const float inv255 = 1.0f / 255.0f;  // the float nearest 1/255, as the oracle
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int x = static_cast<int>(i % p.cw);
    int64_t t = i / p.cw;
    const int y = static_cast<int>(t % p.ch);
    t /= p.ch;
    const int c = static_cast<int>(t % 3);
    const int img = static_cast<int>(t / 3);
    const Axis ay = axis_of(p.y0 + y, p.h, sy);
    const Axis ax = axis_of(p.x0 + x, p.w, sx);
    const uint8_t* base = p.src + static_cast<int64_t>(img) * p.h * p.w * 3 + (2 - c);  // BGR -> RGB
    const float p00 = base[(static_cast<int64_t>(ay.i0) * p.w + ax.i0) * 3];
    const float p01 = base[(static_cast<int64_t>(ay.i0) * p.w + ax.i1) * 3];
    const float p10 = base[(static_cast<int64_t>(ay.i1) * p.w + ax.i0) * 3];
    const float p11 = base[(static_cast<int64_t>(ay.i1) * p.w + ax.i1) * 3];
    const float bx = __fsub_rn(1.0f, ax.a), by = __fsub_rn(1.0f, ay.a);
    const float top = __fadd_rn(__fmul_rn(bx, p00), __fmul_rn(ax.a, p01));
    const float bot = __fadd_rn(__fmul_rn(bx, p10), __fmul_rn(ax.a, p11));
    const float v = __fmul_rn(__fadd_rn(__fmul_rn(by, top), __fmul_rn(ay.a, bot)), inv255);
    p.dst[i] = __fdiv_rn(__fsub_rn(v, p.mean[c]), p.stdv[c]);
  }
}

}  // namespace

cudaError_t launch_preprocess(const uint8_t* src, int n, int h, int w, int rh, int rw, int ch, int cw,
                              const float* mean, const float* stdv, float* dst, cudaStream_t s) {
  PrepParams p;
  p.src = src;
  p.dst = dst;
  p.n = n;
  p.h = h;
  p.w = w;
  p.rh = rh;
  p.rw = rw;
  p.ch = ch;
  p.cw = cw;
  p.y0 = rh / 2 - ch / 2 > 0 ? rh / 2 - ch / 2 : 0;
  p.x0 = rw / 2 - cw / 2 > 0 ? rw / 2 - cw / 2 : 0;
  for (int c = 0; c < 3; ++c) {
    p.mean[c] = mean[c];
    p.stdv[c] = stdv[c];
  }
  const int64_t total = static_cast<int64_t>(n) * 3 * ch * cw;
  const int64_t want = (total + 255) / 256;
  const int grid = static_cast<int>(want < num_sms() * 16 ? want : num_sms() * 16);
  preprocess_kernel<<<grid, 256, 0, s>>>(p);
  note_launch();
  return cudaGetLastError();
}

}  // namespace lotus_impl
