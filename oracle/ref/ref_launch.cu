// Launch wrappers around the reference's own operator kernels (test
// infrastructure only).  Each wrapper repeats the per-sample launch loop of
// the reference layer that calls the kernel, with the reference's grid/block
// helpers, then synchronises.  Compiled with the reference sources (left where
// they lie) into oracle/_ref/libref_ops.so by oracle/ref/Makefile; used only
// to generate golden fixtures on a GPU.
#include "operator/adaptive_avgpool2d.cuh"
#include "operator/add.cuh"
#include "operator/conv2d.cuh"
#include "operator/fused_gemv_add_bias.cuh"
#include "operator/gemm_tensorcore.cuh"
#include "operator/maxpool2d.cuh"
#include "operator/transposed_conv2d.cuh"

using lotus::ActivationFunction;

extern "C" {

// Conv2dLayer::Forward, source/layer/layer_conv2d.cu:37-73 (padded sizes passed).
int ref_conv2d(const float* x, const float* w, const float* b, float* y, int n, int c, int h, int wd, int cout,
               int kh, int kw, int sh, int sw, int ph, int pw, int act) {
  const uint32_t oh = (h + 2 * ph - kh) / sh + 1, ow = (wd + 2 * pw - kw) / sw + 1;
  for (int i = 0; i < n; ++i) {
    lotus::Conv2d<<<lotus::MakeConv2dGrid(cout, oh, ow), lotus::MakeConv2dBlock()>>>(
        x + (size_t)i * c * h * wd, w, b != nullptr, b, y + (size_t)i * cout * oh * ow, cout, c, kh, kw, c, h + 2 * ph,
        wd + 2 * pw, cout, oh, ow, sh, sw, ph, pw, static_cast<ActivationFunction>(act));
  }
  return static_cast<int>(cudaDeviceSynchronize());
}

// TransposedConv2dLayer::Forward, source/layer/layer_transposed_conv2d.cu:37-72.
int ref_tconv2d(const float* x, const float* w, const float* b, float* y, int n, int cin, int h, int wd, int cout,
                int kh, int kw, int sh, int sw, int act) {
  const uint32_t oh = (h - 1) * sh + kh, ow = (wd - 1) * sw + kw;
  for (int i = 0; i < n; ++i) {
    lotus::TransConv2d<<<lotus::MakeTransposedConv2dGrid(cout, oh, ow, 0, 0), lotus::MakeTransposedConv2dBlock()>>>(
        x + (size_t)i * cin * h * wd, w, b != nullptr, b, y + (size_t)i * cout * oh * ow, cout, cin, kh, kw, cin, h,
        wd, cout, oh, ow, sh, sw, 0, 0, static_cast<ActivationFunction>(act));
  }
  return static_cast<int>(cudaDeviceSynchronize());
}

// Maxpool2dLayer::Forward, source/layer/layer_maxpool2d.cu:29-60 (padding 0).
int ref_maxpool2d(const float* x, float* y, int n, int c, int h, int wd, int k, int s, int act) {
  const uint32_t oh = (h - k) / s + 1, ow = (wd - k) / s + 1;
  for (int i = 0; i < n; ++i) {
    lotus::Maxpool2d<<<lotus::MakeMP2dGrid(c, oh, ow), lotus::MakeMP2dBlock()>>>(
        x + (size_t)i * c * h * wd, y + (size_t)i * c * oh * ow, k, k, c, h, wd, 0, 0, s, s, oh, ow,
        static_cast<ActivationFunction>(act));
  }
  return static_cast<int>(cudaDeviceSynchronize());
}

// AdaptiveAvgpool2dLayer::Forward with its window parameters,
// source/layer/layer_adaptive_avgpool2d.cu:23-57.
int ref_adaptive_avgpool2d(const float* x, float* y, int n, int c, int h, int wd, int oh, int ow, int act) {
  const uint32_t kh = (h + oh - 1) / oh, kw = (wd + ow - 1) / ow;
  const float sh = (h - kh) / oh, sw = (wd - kw) / ow;
  for (int i = 0; i < n; ++i) {
    lotus::AdaptiveAvgpool2d<<<lotus::MakeAAP2dGrid(c, oh, ow), lotus::MakeAAP2dBlock()>>>(
        x + (size_t)i * c * h * wd, y + (size_t)i * c * oh * ow, kh, kw, c, h, wd, sh, sw, oh, ow,
        static_cast<ActivationFunction>(act));
  }
  return static_cast<int>(cudaDeviceSynchronize());
}

// ExpressionLayer add, source/layer/expression.cu:29-50.
int ref_add(const float* a, const float* b, float* y, int count, int act) {
  lotus::Add<<<lotus::MakeAddGrid(count), lotus::MakeAddBlock()>>>(a, b, y, count,
                                                                     static_cast<ActivationFunction>(act));
  return static_cast<int>(cudaDeviceSynchronize());
}

// Gemm called once with m rows (requires m <= n: the grid helper sizes both
// dimensions by n, source/operator/gemm_tensorcore.cu:6-9).
int ref_gemm(const float* a, const float* w, const float* bias, float* c, int m, int n, int k, int act) {
  if (m > n) return -1;
  lotus::Gemm<<<lotus::MakeGemmGrid(m, n), lotus::MakeGemmBlock()>>>(a, w, bias != nullptr, bias, c, m, n, k,
                                                                    static_cast<ActivationFunction>(act));
  return static_cast<int>(cudaDeviceSynchronize());
}

// Fgemva on its element-wise load path only (weight_w % 4 != 0) and with
// weight_h a multiple of 8 (no row guard on its store).
int ref_gemv(const float* x, const float* w, const float* bias, float* y, int h, int wd, int act) {
  if (wd % 4 == 0 || h % 8 != 0) return -1;
  lotus::Fgemva<<<lotus::MakeSFgemvaGrid(h), lotus::MakeSFgemvaBlock()>>>(x, w, bias, y, h, wd, bias != nullptr,
                                                                          static_cast<ActivationFunction>(act));
  return static_cast<int>(cudaDeviceSynchronize());
}

}  // extern "C"
