// Bandwidth-bound pooling kernels on NHWC fp16 activations.
//
// Each thread owns one output pixel x 8 channels (one 16-byte vector), so a
// warp reads and writes contiguous channel runs of neighbouring pixels.
//
// Reference counterparts: source/operator/maxpool2d.cu:16-66 (whose padding
// taps leave the running max uninitialised when tap (0,0) is padding; here
// padding is -inf as in PyTorch) and source/operator/adaptive_avgpool2d.cu:15-52
// with the window start/size set in source/layer/layer_adaptive_avgpool2d.cu:42-46
// (integer stride; here PyTorch's [floor(i*H/OH), ceil((i+1)*H/OH)) windows,
// which agree with the reference for ResNet's 7x7 -> 1x1).

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace lotus_impl {

using namespace lotus_dev;

// IT is the index type: 32-bit when every element offset fits (the common
// case; 64-bit division in the grid-stride loop dominated the kernel), else 64-bit.
// KS = 3: the window is 3x3 at compile time, so the nine tap loads are
// unrolled and in flight together (with runtime kh/kw each load waits for the
// loop control of the one before); KS = 0: any window.
template <typename IT, int KS>
__global__ void maxpool_nhwc_kernel(const __half* __restrict__ x, int xs, __half* __restrict__ y, int n, int c, int cs,
                                    int h, int w, int oh, int ow, int kh, int kw, int sh, int sw, int ph, int pw,
                                    int act) {
  if (KS > 0) {
    kh = KS;
    kw = KS;
  }
  const int groups = cs / 8;
  const IT total = static_cast<IT>(n) * oh * ow * groups;
  for (IT i = blockIdx.x * static_cast<IT>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<IT>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(i % groups);
    const IT pix = i / groups;
    const int ox = static_cast<int>(pix % ow);
    const IT t = pix / ow;
    const int oy = static_cast<int>(t % oh);
    const int img = static_cast<int>(t / oh);
    float m[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) m[j] = -INFINITY;
    const int y0 = oy * sh - ph, x0 = ox * sw - pw;
    const __half* xb = x + static_cast<IT>(img) * h * w * xs + g * 8;
#pragma unroll
    for (int r = 0; r < (KS > 0 ? KS : kh); ++r) {
      const int iy = y0 + r;
      if (iy < 0 || iy >= h) continue;
#pragma unroll
      for (int s = 0; s < (KS > 0 ? KS : kw); ++s) {
        const int ix = x0 + s;
        if (ix < 0 || ix >= w) continue;
        float f[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(xb + (static_cast<IT>(iy) * w + ix) * xs)), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) m[j] = fmaxf(m[j], f[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) m[j] = (g * 8 + j < c) ? act_fn(m[j], act) : 0.f;
    reinterpret_cast<uint4*>(y + pix * cs)[g] = pack8(m);
  }
}

__global__ void adaptive_avgpool_nhwc_kernel(const __half* __restrict__ x, void* __restrict__ y, int n, int c, int cs,
                                             int h, int w, int oh, int ow, int act, int out_f32) {
  const int groups = cs / 8;
  const size_t total = static_cast<size_t>(n) * oh * ow * groups;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(i % groups);
    const size_t pix = i / groups;
    const int ox = static_cast<int>(pix % ow);
    const size_t t = pix / ow;
    const int oy = static_cast<int>(t % oh);
    const int img = static_cast<int>(t / oh);
    const int hs = (oy * h) / oh, he = ((oy + 1) * h + oh - 1) / oh;
    const int ws = (ox * w) / ow, we = ((ox + 1) * w + ow - 1) / ow;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const __half* xb = x + static_cast<size_t>(img) * h * w * cs + g * 8;
    for (int iy = hs; iy < he; ++iy) {
      for (int ix = ws; ix < we; ++ix) {
        float f[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(xb + (static_cast<size_t>(iy) * w + ix) * cs)), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += f[j];
      }
    }
    const float inv = 1.0f / static_cast<float>((he - hs) * (we - ws));
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = (g * 8 + j < c) ? act_fn(acc[j] * inv, act) : 0.f;
    if (out_f32) {
      float* yr = static_cast<float*>(y) + pix * c;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (g * 8 + j < c) yr[g * 8 + j] = acc[j];
    } else {
      reinterpret_cast<uint4*>(static_cast<__half*>(y) + pix * cs)[g] = pack8(acc);
    }
  }
}

// Large windows (a global pool such as ResNet's 7x7 -> 1x1): one block per
// output pixel, its threads laid out as (pixel slice, channel group) so that a
// warp reads consecutive 16-byte channel groups and each thread sums every
// S-th pixel of the window.  The S partial sums are added in slice order in
// shared memory.  Requires cs/8 <= blockDim.x.
__global__ void __launch_bounds__(256) adaptive_avgpool_window_kernel(const __half* __restrict__ x,
                                                                      void* __restrict__ y, int c, int cs, int h,
                                                                      int w, int oh, int ow, int act, int out_f32) {
  __shared__ float red[256 * 8];
  if (threadIdx.x == 0) griddep_launch();
  griddep_wait();  // the activations of the kernel before
  const int groups = cs / 8;
  const int slices = static_cast<int>(blockDim.x) / groups;
  const int g = static_cast<int>(threadIdx.x) % groups;
  const int sl = static_cast<int>(threadIdx.x) / groups;
  const int pix = blockIdx.x;
  const int ox = pix % ow;
  const int t = pix / ow;
  const int oy = t % oh;
  const int img = t / oh;
  const int hs = (oy * h) / oh, he = ((oy + 1) * h + oh - 1) / oh;
  const int ws = (ox * w) / ow, we = ((ox + 1) * w + ow - 1) / ow;
  const int wn = we - ws;
  const int cnt = (he - hs) * wn;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (sl < slices) {
    const __half* xb = x + static_cast<size_t>(img) * h * w * cs + g * 8;
#pragma unroll 4
    for (int k = sl; k < cnt; k += slices) {
      const int iy = hs + k / wn;
      const int ix = ws + k % wn;
      float f[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(xb + (static_cast<size_t>(iy) * w + ix) * cs)), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) red[threadIdx.x * 8 + j] = acc[j];
  }
  __syncthreads();
  if (sl != 0) return;
  for (int s2 = 1; s2 < slices; ++s2) {
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] += red[(s2 * groups + g) * 8 + j];
  }
  const float inv = 1.0f / static_cast<float>(cnt);
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = (g * 8 + j < c) ? act_fn(acc[j] * inv, act) : 0.f;
  if (out_f32) {
    float* yr = static_cast<float*>(y) + static_cast<size_t>(pix) * c;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (g * 8 + j < c) yr[g * 8 + j] = acc[j];
  } else {
    reinterpret_cast<uint4*>(static_cast<__half*>(y) + static_cast<size_t>(pix) * cs)[g] = pack8(acc);
  }
}

cudaError_t launch_maxpool(const void* x, int x_stride, void* y, int n, int c, int cs, int h, int w, int oh, int ow,
                           int kh, int kw, int sh, int sw, int ph, int pw, int act, cudaStream_t s) {
  const size_t total = static_cast<size_t>(n) * oh * ow * (cs / 8);
  const bool small = static_cast<size_t>(n) * h * w * x_stride < (1u << 31) && total < (1u << 31);
  if (small && kh == 3 && kw == 3)
    maxpool_nhwc_kernel<int, 3><<<grid_for(total, 256, 32), 256, 0, s>>>(
        static_cast<const __half*>(x), x_stride, static_cast<__half*>(y), n, c, cs, h, w, oh, ow, kh, kw, sh, sw, ph,
        pw, act);
  else if (small)
    maxpool_nhwc_kernel<int, 0><<<grid_for(total, 256, 32), 256, 0, s>>>(
        static_cast<const __half*>(x), x_stride, static_cast<__half*>(y), n, c, cs, h, w, oh, ow, kh, kw, sh, sw, ph,
        pw, act);
  else
    maxpool_nhwc_kernel<size_t, 0><<<grid_for(total, 256), 256, 0, s>>>(
        static_cast<const __half*>(x), x_stride, static_cast<__half*>(y), n, c, cs, h, w, oh, ow, kh, kw, sh, sw, ph,
        pw, act);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_adaptive_avgpool(const void* x, void* y, int n, int c, int cs, int h, int w, int oh, int ow,
                                    int act, int out_f32, cudaStream_t s) {
  const size_t total = static_cast<size_t>(n) * oh * ow * (cs / 8);
  const size_t pixels = static_cast<size_t>(n) * oh * ow;
  if (cs / 8 <= 256 && (h / oh) * (w / ow) >= 16 && pixels < (1u << 31) && static_cast<size_t>(h) * w * cs < (1u << 31)) {
    const cudaError_t e = launch_pdl(adaptive_avgpool_window_kernel, dim3(static_cast<unsigned>(pixels)), dim3(256), 0,
                                     s, static_cast<const __half*>(x), y, c, cs, h, w, oh, ow, act, out_f32);
    note_launch();
    return e != cudaSuccess ? e : cudaGetLastError();
  }
  adaptive_avgpool_nhwc_kernel<<<grid_for(total, 256), 256, 0, s>>>(static_cast<const __half*>(x), y, n, c, cs, h, w,
                                                                    oh, ow, act, out_f32);
  note_launch();
  return cudaGetLastError();
}

}  // namespace lotus_impl
