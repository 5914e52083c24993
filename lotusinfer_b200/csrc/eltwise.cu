// Elementwise / data-movement kernels on NHWC fp16 activations:
// residual add + activation, channel concatenation, and the two helpers of the
// transposed convolution (bias fill for output pixels no input reaches, and a
// direct output-stationary kernel for stride < kernel, where taps overlap).
//
// Reference counterparts: source/operator/add.cu:14-26 (Add + act),
// source/layer/concatenate.cpp:20-35 (per-sample cudaMemcpy concat along C),
// source/operator/transposed_conv2d.cu:17-140.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace lotus_impl {

using namespace lotus_dev;

__global__ void add_act_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b, uint4* __restrict__ y,
                               size_t vecs, int c, int cs, int act) {
  const int groups = cs / 8;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < vecs;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(i % groups);
    float fa[8], fb[8];
    unpack8(__ldg(a + i), fa);
    unpack8(__ldg(b + i), fb);
#pragma unroll
    for (int j = 0; j < 8; ++j) fa[j] = (g * 8 + j < c) ? act_fn(fa[j] + fb[j], act) : 0.f;
    y[i] = pack8(fa);
  }
}

// y[p, 0:ca] = a[p, 0:ca], y[p, ca:ca+cb] = b[p, 0:cb]; 16-byte moves when the
// channel offsets allow it, element moves otherwise.
__global__ void concat_kernel(const __half* __restrict__ a, int csa, const __half* __restrict__ b, int csb,
                              __half* __restrict__ y, int ca, int cb, int csy, size_t pixels) {
  const size_t total = pixels * csy;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t p = i / csy;
    const int ch = static_cast<int>(i - p * csy);
    __half v = __float2half_rn(0.f);
    if (ch < ca)
      v = a[p * csa + ch];
    else if (ch < ca + cb)
      v = b[p * csb + (ch - ca)];
    y[i] = v;
  }
}

__global__ void concat_vec_kernel(const uint4* __restrict__ a, int ga, const uint4* __restrict__ b, int gb,
                                  uint4* __restrict__ y, size_t pixels) {
  const int gy = ga + gb;
  const size_t total = pixels * gy;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t p = i / gy;
    const int g = static_cast<int>(i - p * gy);
    y[i] = g < ga ? __ldg(a + p * ga + g) : __ldg(b + p * gb + (g - ga));
  }
}

__global__ void tconv_fill_bias_kernel(__half* __restrict__ y, int ys, const float* __restrict__ bias, int cout,
                                       int cs, size_t pixels, int act) {
  const int groups = cs / 8;
  const size_t total = pixels * groups;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(i % groups);
    float f[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = g * 8 + j;
      f[j] = c < cout ? act_fn(bias ? bias[c] : 0.f, act) : 0.f;
    }
    reinterpret_cast<uint4*>(y + (i / groups) * ys)[g] = pack8(f);
  }
}

// Output-stationary transposed convolution for any stride/kernel/padding.
// Weights are the GEMM-prepacked rows ((ky*kw + kx)*cout + co) x k_pad.
__global__ void tconv_direct_kernel(const __half* __restrict__ x, const __half* __restrict__ wp, int k_pad,
                                    const float* __restrict__ bias, __half* __restrict__ y, int ys, int n, int cin,
                                    int csi,
                                    int h, int w, int cout, int cso, int oh, int ow, int kh, int kw, int sh, int sw,
                                    int ph, int pw, int act) {
  const size_t total = static_cast<size_t>(n) * oh * ow * cso;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int co = static_cast<int>(i % cso);
    const size_t pix = i / cso;
    const int ox = static_cast<int>(pix % ow);
    const size_t t = pix / ow;
    const int oy = static_cast<int>(t % oh);
    const int img = static_cast<int>(t / oh);
    if (co >= cout) {
      y[pix * ys + co] = __float2half_rn(0.f);
      continue;
    }
    float acc = bias ? bias[co] : 0.f;
    for (int ky = 0; ky < kh; ++ky) {
      const int ty = oy + ph - ky;
      if (ty < 0 || ty % sh) continue;
      const int iy = ty / sh;
      if (iy >= h) continue;
      for (int kx = 0; kx < kw; ++kx) {
        const int tx = ox + pw - kx;
        if (tx < 0 || tx % sw) continue;
        const int ix = tx / sw;
        if (ix >= w) continue;
        const __half* xp = x + ((static_cast<size_t>(img) * h + iy) * w + ix) * csi;
        const __half* wr = wp + (static_cast<size_t>(ky * kw + kx) * cout + co) * k_pad;
        for (int ci = 0; ci < cin; ++ci) acc += __half2float(xp[ci]) * __half2float(wr[ci]);
      }
    }
    y[pix * ys + co] = __float2half_rn(act_fn(acc, act));
  }
}

cudaError_t launch_add_act(const void* a, const void* b, void* y, size_t pixels, int c, int cs, int act,
                           cudaStream_t s) {
  const size_t vecs = pixels * (cs / 8);
  add_act_kernel<<<grid_for(vecs, 256), 256, 0, s>>>(static_cast<const uint4*>(a), static_cast<const uint4*>(b),
                                                     static_cast<uint4*>(y), vecs, c, cs, act);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_concat(const void* a, int csa, const void* b, int csb, void* y, int ca, int cb, int csy,
                          size_t pixels, cudaStream_t s) {
  if (ca == csa && cb == csb && (ca % 8) == 0 && (cb % 8) == 0 && csy == ca + cb) {
    concat_vec_kernel<<<grid_for(pixels * (csy / 8), 256), 256, 0, s>>>(
        static_cast<const uint4*>(a), ca / 8, static_cast<const uint4*>(b), cb / 8, static_cast<uint4*>(y), pixels);
  } else {
    concat_kernel<<<grid_for(pixels * csy, 256), 256, 0, s>>>(static_cast<const __half*>(a), csa,
                                                              static_cast<const __half*>(b), csb,
                                                              static_cast<__half*>(y), ca, cb, csy, pixels);
  }
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_tconv_fill_bias(void* y, int y_stride, const float* bias, int cout, int cs, size_t pixels, int act,
                                   cudaStream_t s) {
  tconv_fill_bias_kernel<<<grid_for(pixels * (cs / 8), 256), 256, 0, s>>>(static_cast<__half*>(y), y_stride, bias,
                                                                          cout, cs, pixels, act);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_tconv_direct(const void* x, const void* wp, int k_pad, const float* bias, void* y, int y_stride,
                                int n, int cin, int csi, int h, int w_, int cout, int cso, int oh, int ow, int kh,
                                int kw, int sh, int sw, int ph, int pw, int act, cudaStream_t s) {
  const size_t total = static_cast<size_t>(n) * oh * ow * cso;
  tconv_direct_kernel<<<grid_for(total, 256), 256, 0, s>>>(static_cast<const __half*>(x),
                                                           static_cast<const __half*>(wp), k_pad, bias,
                                                           static_cast<__half*>(y), y_stride, n, cin, csi, h, w_,
                                                           cout, cso, oh,
                                                           ow, kh, kw, sh, sw, ph, pw, act);
  note_launch();
  return cudaGetLastError();
}

}  // namespace lotus_impl
