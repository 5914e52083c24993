// Load-time weight prepacking and NCHW fp32 <-> NHWC fp16 layout conversion.
//
// The reference keeps every tensor NCHW fp32 (include/tensor.hpp:13-40,
// weights uploaded as-is in source/layer/layer_conv2d.cu:21); the tensor-core
// path wants K-major fp16 operands, so weights are converted once here with
// round-to-nearest-even and activations cross the layout boundary only at the
// graph input and output.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace lotus_impl {

using namespace lotus_dev;

// Conv: OIHW fp32 -> [cout, k_pad] fp16 with k = (r*kw + s)*cs_in + c.
__global__ void conv_prepack_kernel(const float* __restrict__ w, __half* __restrict__ wp, int cout, int cin, int kh,
                                    int kw, int cs_in, int k_pad) {
  const size_t total = static_cast<size_t>(cout) * k_pad;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int co = static_cast<int>(i / k_pad);
    const int k = static_cast<int>(i - static_cast<size_t>(co) * k_pad);
    const int tap = k / cs_in;
    const int c = k - tap * cs_in;
    float v = 0.f;
    if (tap < kh * kw && c < cin) {
      const int r = tap / kw, s = tap - (tap / kw) * kw;
      v = w[((static_cast<size_t>(co) * cin + c) * kh + r) * kw + s];
    }
    wp[i] = __float2half_rn(v);
  }
}

// Transposed conv: [cin, cout, kh, kw] fp32 -> rows j = (ky*kw + kx)*cout + co,
// columns ci (k_pad = roundup(cs_in, 64)).
__global__ void tconv_prepack_kernel(const float* __restrict__ w, __half* __restrict__ wp, int cin, int cout, int kh,
                                     int kw, int k_pad) {
  const size_t rows = static_cast<size_t>(kh) * kw * cout;
  const size_t total = rows * k_pad;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(i / k_pad);
    const int ci = static_cast<int>(i - static_cast<size_t>(j) * k_pad);
    const int tap = j / cout;
    const int co = j - tap * cout;
    const int ky = tap / kw, kx = tap - (tap / kw) * kw;
    float v = 0.f;
    if (ci < cin) v = w[((static_cast<size_t>(ci) * cout + co) * kh + ky) * kw + kx];
    wp[i] = __float2half_rn(v);
  }
}

// Linear: [out, in] fp32 -> [out, k_pad] fp16; optional (c,h,w)->(h,w,c)
// column permutation for a flattened NHWC input.
__global__ void linear_prepack_kernel(const float* __restrict__ w, __half* __restrict__ wp, int in_f, int out_f,
                                      int k_pad, int fc_c, int fc_h, int fc_w) {
  const size_t total = static_cast<size_t>(out_f) * k_pad;
  const bool perm = fc_c > 0 && fc_h > 0 && fc_w > 0;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int o = static_cast<int>(i / k_pad);
    const int k = static_cast<int>(i - static_cast<size_t>(o) * k_pad);
    float v = 0.f;
    if (k < in_f) {
      int src = k;
      if (perm) {
        const int c = k % fc_c;
        const int hw = k / fc_c;  // h*fc_w + w
        src = c * fc_h * fc_w + hw;
      }
      v = w[static_cast<size_t>(o) * in_f + src];
    }
    wp[i] = __float2half_rn(v);
  }
}

// One thread per pixel: coalesced fp32 plane reads, 16-byte fp16 writes.
__global__ void nchw_to_nhwc_kernel(const float* __restrict__ x, __half* __restrict__ y, int n, int c, int hw,
                                    int cs) {
  const size_t pixels = static_cast<size_t>(n) * hw;
  for (size_t p = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; p < pixels;
       p += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t img = p / hw;
    const size_t off = p - img * hw;
    const float* xs = x + img * c * static_cast<size_t>(hw) + off;
    uint4* yd = reinterpret_cast<uint4*>(y + p * cs);
    for (int c0 = 0; c0 < cs; c0 += 8) {
      float f[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = (c0 + j < c) ? __ldg(xs + static_cast<size_t>(c0 + j) * hw) : 0.f;
      yd[c0 / 8] = pack8(f);
    }
  }
}

__global__ void nhwc_to_nchw_kernel(const __half* __restrict__ x, float* __restrict__ y, int n, int c, int hw,
                                    int cs) {
  const size_t pixels = static_cast<size_t>(n) * hw;
  for (size_t p = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; p < pixels;
       p += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t img = p / hw;
    const size_t off = p - img * hw;
    float* yd = y + img * c * static_cast<size_t>(hw) + off;
    const uint4* xs = reinterpret_cast<const uint4*>(x + p * cs);
    for (int c0 = 0; c0 < c; c0 += 8) {
      float f[8];
      unpack8(xs[c0 / 8], f);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + j < c) yd[static_cast<size_t>(c0 + j) * hw] = f[j];
    }
  }
}

// Space-to-depth of a zero-padded NCHW fp32 image batch into NHWC fp16:
// y[n, i, j, (a*f + b)*c + ch] = xpad[n, ch, f*i + a, f*j + b] with
// xpad[.., u, v] = x[.., u - pad_h, v - pad_w] inside the image, 0 outside;
// channels c*f*f .. cs-1 are zero.  One thread per output pixel.
// FF/CC > 0 fix the factor and the channel count at compile time (the
// 3-channel factor-2 ResNet stem): the loops unroll and all loads of a pixel
// are in flight together; 0 = runtime values.
template <typename IT, int FF, int CC>
__global__ void space_to_depth_kernel(const float* __restrict__ x, __half* __restrict__ y, int n, int c, int h, int w,
                                      int f, int pad_h, int pad_w, int oh, int ow, int cs) {
  if (FF > 0) f = FF;
  if (CC > 0) c = CC;
  const IT pixels = static_cast<IT>(n) * oh * ow;
  const IT plane = static_cast<IT>(h) * w;
  for (IT p = blockIdx.x * static_cast<IT>(blockDim.x) + threadIdx.x; p < pixels;
       p += static_cast<IT>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(p % ow);
    const IT t = p / ow;
    const int i = static_cast<int>(t % oh);
    const int img = static_cast<int>(t / oh);
    const float* xb = x + static_cast<IT>(img) * c * plane;
    uint4* yd = reinterpret_cast<uint4*>(y + p * cs);
    // channel order (a, b, ch): consecutive threads (consecutive j) read
    // consecutive f-wide runs of one input row, so each warp load coalesces
    float v[8];
    int q = 0, vec = 0;
#pragma unroll
    for (int a = 0; a < (FF > 0 ? FF : f); ++a) {
      const int u = f * i + a - pad_h;
      const bool row_ok = u >= 0 && u < h;
#pragma unroll
      for (int b = 0; b < (FF > 0 ? FF : f); ++b) {
        const int col = f * j + b - pad_w;
        const bool ok = row_ok && col >= 0 && col < w;
        const float* src = xb + static_cast<IT>(u) * w + col;
#pragma unroll
        for (int ch = 0; ch < (CC > 0 ? CC : c); ++ch) {
          v[q++] = ok ? __ldg(src + ch * plane) : 0.f;
          if (q == 8) {
            yd[vec++] = pack8(v);
            q = 0;
          }
        }
      }
    }
    // pad channels c*f*f .. cs-1
    while (vec * 8 < cs) {
      for (; q < 8; ++q) v[q] = 0.f;
      yd[vec++] = pack8(v);
      q = 0;
    }
  }
}

cudaError_t launch_space_to_depth(const float* x, void* y, int n, int c, int h, int w, int f, int pad_h, int pad_w,
                                  int oh, int ow, int cs, cudaStream_t s) {
  const size_t pixels = static_cast<size_t>(n) * oh * ow;
  const bool small = static_cast<size_t>(n) * c * h * w < (1u << 31) && pixels * cs < (1u << 31);
  if (small && f == 2 && c == 3)
    space_to_depth_kernel<int, 2, 3><<<grid_for(pixels, 256, 32), 256, 0, s>>>(x, static_cast<__half*>(y), n, c, h, w,
                                                                               f, pad_h, pad_w, oh, ow, cs);
  else if (small)
    space_to_depth_kernel<int, 0, 0><<<grid_for(pixels, 256, 32), 256, 0, s>>>(x, static_cast<__half*>(y), n, c, h, w,
                                                                               f, pad_h, pad_w, oh, ow, cs);
  else
    space_to_depth_kernel<size_t, 0, 0><<<grid_for(pixels, 256), 256, 0, s>>>(x, static_cast<__half*>(y), n, c, h, w,
                                                                              f, pad_h, pad_w, oh, ow, cs);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_conv_prepack(const float* w, void* wp, int cout, int cin, int kh, int kw, int cs_in, int k_pad,
                                cudaStream_t s) {
  const size_t total = static_cast<size_t>(cout) * k_pad;
  conv_prepack_kernel<<<grid_for(total, 256), 256, 0, s>>>(w, static_cast<__half*>(wp), cout, cin, kh, kw, cs_in,
                                                           k_pad);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_tconv_prepack(const float* w, void* wp, int cin, int cout, int kh, int kw, int cs_in, int k_pad,
                                 cudaStream_t s) {
  (void)cs_in;
  const size_t total = static_cast<size_t>(kh) * kw * cout * k_pad;
  tconv_prepack_kernel<<<grid_for(total, 256), 256, 0, s>>>(w, static_cast<__half*>(wp), cin, cout, kh, kw, k_pad);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_linear_prepack(const float* w, void* wp, int in_f, int out_f, int k_pad, int fc_c, int fc_h,
                                  int fc_w, cudaStream_t s) {
  const size_t total = static_cast<size_t>(out_f) * k_pad;
  linear_prepack_kernel<<<grid_for(total, 256), 256, 0, s>>>(w, static_cast<__half*>(wp), in_f, out_f, k_pad, fc_c,
                                                             fc_h, fc_w);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_nchw_to_nhwc(const float* x, void* y, int n, int c, int h, int w, int cs, cudaStream_t s) {
  const size_t pixels = static_cast<size_t>(n) * h * w;
  nchw_to_nhwc_kernel<<<grid_for(pixels, 256), 256, 0, s>>>(x, static_cast<__half*>(y), n, c, h * w, cs);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_nhwc_to_nchw(const void* x, float* y, int n, int c, int h, int w, int cs, cudaStream_t s) {
  const size_t pixels = static_cast<size_t>(n) * h * w;
  nhwc_to_nchw_kernel<<<grid_for(pixels, 256), 256, 0, s>>>(static_cast<const __half*>(x), y, n, c, h * w, cs);
  note_launch();
  return cudaGetLastError();
}

}  // namespace lotus_impl
