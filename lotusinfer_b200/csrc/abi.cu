// C ABI entry points (include/lotus_ops.h): argument validation, shape
// arithmetic, dispatch to the kernels, status codes and error strings.
//
// The reference checks nothing at its launch sites (e.g.
// source/layer/layer_conv2d.cu:60-69 launches without cudaGetLastError) and
// aborts through glog CHECK on host-side shape errors
// (include/lotus_utils.hpp:28-32).  Here every entry point validates its
// arguments, returns a negative status instead of launching on bad input, and
// reports launch failures.

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>

#include <cuda_runtime.h>

#include "../../include/lotus_ops.h"
#include "kernels.h"

namespace lotus_impl {

static std::atomic<uint64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

static thread_local std::string t_last_error;

int set_error(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

static int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}
static int ok() {
  t_last_error.clear();
  return LOTUS_OK;
}
static int cuda_status(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(LOTUS_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return ok();
}
static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
static int cs_of(int c) { return (c + 7) / 8 * 8; }
static int round64(long v) { return static_cast<int>((v + 63) / 64 * 64); }

static constexpr long kMaxIndex = 0x7FFFFFFFL;

static int check_conv_desc(const lotus_conv2d_desc* d, int* oh, int* ow) {
  if (!d) return fail(LOTUS_ERR_INVALID, "conv2d: null descriptor");
  if (d->n <= 0 || d->c_in <= 0 || d->h <= 0 || d->w <= 0 || d->c_out <= 0 || d->kh <= 0 || d->kw <= 0)
    return fail(LOTUS_ERR_INVALID, "conv2d: sizes must be positive");
  if (d->stride_h <= 0 || d->stride_w <= 0 || d->pad_h < 0 || d->pad_w < 0)
    return fail(LOTUS_ERR_INVALID, "conv2d: stride must be positive and padding non-negative");
  if (d->act < 0 || d->act > 2) return fail(LOTUS_ERR_INVALID, "conv2d: unknown activation");
  if (d->out_kind != LOTUS_OUT_NHWC_F16 && d->out_kind != LOTUS_OUT_ROWS_F32)
    return fail(LOTUS_ERR_INVALID, "conv2d: unknown out_kind");
  const long eh = static_cast<long>(d->h) + 2L * d->pad_h - d->kh;
  const long ew = static_cast<long>(d->w) + 2L * d->pad_w - d->kw;
  if (eh < 0 || ew < 0) return fail(LOTUS_ERR_INVALID, "conv2d: kernel larger than padded input");
  *oh = static_cast<int>(eh / d->stride_h + 1);
  *ow = static_cast<int>(ew / d->stride_w + 1);
  if (d->kh > 255 || d->kw > 255) return fail(LOTUS_ERR_UNSUPPORTED, "conv2d: kernel side > 255");
  if (cs_of(d->c_in) > 65535) return fail(LOTUS_ERR_UNSUPPORTED, "conv2d: more than 65535 input channels");
  if (static_cast<long>(d->n) * *oh * *ow > kMaxIndex) return fail(LOTUS_ERR_UNSUPPORTED, "conv2d: too many pixels");
  return ok();
}

}  // namespace lotus_impl

using namespace lotus_impl;

extern "C" {

const char* lotus_last_error_string(void) { return t_last_error.c_str(); }

uint64_t lotus_launch_count(void) { return g_launches.load(); }

int lotus_device_error(void) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "device_error: synchronize");
  return read_device_error();
}

int lotus_channel_stride(int c) { return c <= 0 ? 0 : cs_of(c); }

int lotus_conv2d_out_hw(const lotus_conv2d_desc* d, int* oh, int* ow) {
  int a, b;
  const int st = check_conv_desc(d, &a, &b);
  if (st != LOTUS_OK) return st;
  if (oh) *oh = a;
  if (ow) *ow = b;
  return ok();
}

size_t lotus_conv2d_packed_weight_bytes(const lotus_conv2d_desc* d) {
  if (!d || d->c_out <= 0 || d->kh <= 0 || d->kw <= 0 || d->c_in <= 0) return 0;
  const long k_pad = round64(static_cast<long>(d->kh) * d->kw * cs_of(d->c_in));
  return static_cast<size_t>(d->c_out) * k_pad * 2;
}

int lotus_conv2d_prepack(const float* w_oihw, void* w_packed, const lotus_conv2d_desc* d, cudaStream_t stream) {
  int oh, ow;
  const int st = check_conv_desc(d, &oh, &ow);
  if (st != LOTUS_OK) return st;
  if (!w_oihw || !w_packed) return fail(LOTUS_ERR_INVALID, "conv2d_prepack: null pointer");
  const int cs = cs_of(d->c_in);
  const int k_pad = round64(static_cast<long>(d->kh) * d->kw * cs);
  return cuda_status(launch_conv_prepack(w_oihw, w_packed, d->c_out, d->c_in, d->kh, d->kw, cs, k_pad, stream),
                     "conv2d_prepack");
}

// Kernel arguments of a conv described by `d` (shape already checked).
static ConvTcArgs conv_args(const void* x, const void* w_packed, const float* bias, const void* residual, void* y,
                            const lotus_conv2d_desc* d, int oh, int ow) {
  ConvTcArgs a{};
  a.x = x;
  a.w_packed = w_packed;
  a.bias = bias;
  a.residual = residual;
  a.y = y;
  a.H = d->h;
  a.W = d->w;
  a.Cs_in = cs_of(d->c_in);
  a.OH = oh;
  a.OW = ow;
  a.kh = d->kh;
  a.kw = d->kw;
  a.sh = d->stride_h;
  a.sw = d->stride_w;
  a.ph = d->pad_h;
  a.pw = d->pad_w;
  a.n_cols = d->c_out;
  a.k_pad = round64(static_cast<long>(d->kh) * d->kw * a.Cs_in);
  a.Cs_out = cs_of(d->c_out);
  a.M = d->n * oh * ow;
  a.act = d->act;
  a.out_kind = d->out_kind;
  return a;
}

// The row-stacked kernel takes 64-channel stride-1 layers (ResNet stage 1)
// when the batch gives every SM at least two output rows of work; smaller
// launches go to the general kernel, which can split K.  LOTUS_CONV_ROWS=0
// or 1 forces the choice (tests); a forced general-kernel staging mode
// (LOTUS_CONV_AMODE) implies 0.
static bool use_rows_conv(const ConvTcArgs& a, int n) {
  const char* err = "";
  if (conv_rows_check(a, n, &err) != 0) return false;
  const char* env = std::getenv("LOTUS_CONV_ROWS");
  if (env != nullptr && env[0] == '0') return false;
  if (env == nullptr && std::getenv("LOTUS_CONV_AMODE") != nullptr) return false;  // a forced general-kernel path
  if (env != nullptr && env[0] == '1') return true;
  const int ipt = a.OW + a.kw - 1 <= 64 ? 2 : 1;
  return static_cast<long>((n + ipt - 1) / ipt) * a.OH >= 2L * num_sms();
}

// The CTA-pair kernel takes NHWC fp16 convs over 64-channel multiples with
// at least 128 output channels when its pair tiles fill every SM pair at
// least once: 256 x 256 pair tiles above 128 output channels, 512 x 128 pair
// tiles (two M tiles a CTA) at 128 (one M tile a CTA with 128 columns was
// measured slower than the general kernel: too little MMA per loaded stage).  Smaller launches go to the general kernel, which can split K.
// LOTUS_CONV_PAIR=0 or 1 forces the choice (1: 256 columns when Cout > 128,
// else 128); a forced general-kernel staging mode (LOTUS_CONV_AMODE)
// implies 0.
static int pair_conv_bn(const ConvTcArgs& a) {
  const char* env = std::getenv("LOTUS_CONV_PAIR");
  if (env != nullptr && env[0] == '0') return 0;
  if (env == nullptr && std::getenv("LOTUS_CONV_AMODE") != nullptr) return 0;
  const char* err = "";
  if (conv_pair_check(a, 128, &err) != 0 || a.n_cols < 128) return 0;
  const int bn = a.n_cols > 128 ? 256 : 128;
  if (env != nullptr && env[0] == '1') return bn;
  const long pairs = num_sms() / 2;
  const long m_tiles = (a.M + 127) / 128;
  const long m_groups = bn == 256 ? (m_tiles + 1) / 2 : (m_tiles + 3) / 4;  // M tiles a pair tile covers: 2 or 4
  // 512 x 128 pair tiles beat the general kernel on ResNet stage 2: 1x1/2
  // 0.031 vs 0.039 ms, and since the pair epilogue hands TMEM back early and
  // compiles the residual add in or out, the K = 1152 3x3 layers too (54.2 vs
  // 59.6 us, 64.7 vs 67.7 us with the residual)
  return m_groups * ((a.n_cols + bn - 1) / bn) >= pairs ? bn : 0;
}

static int conv_fwd_impl(const void* x, const void* w_packed, const float* bias, const void* residual, void* y,
                         const lotus_conv2d_desc* d, void* workspace, size_t workspace_bytes, cudaStream_t stream,
                         int y_stride = 0, bool pair_split = true) {
  int oh, ow;
  const int st = check_conv_desc(d, &oh, &ow);
  if (st != LOTUS_OK) return st;
  if (y_stride != 0 && (d->out_kind != LOTUS_OUT_NHWC_F16 || y_stride < cs_of(d->c_out) || y_stride % 8 != 0))
    return fail(LOTUS_ERR_INVALID,
                "conv2d: an output pixel stride needs the NHWC fp16 output, a multiple of 8 and >= roundup(c_out, 8)");
  if (!x || !w_packed || !y) return fail(LOTUS_ERR_INVALID, "conv2d: null x, w or y");
  if (!aligned16(x) || !aligned16(w_packed) || !aligned16(y) || (residual && !aligned16(residual)))
    return fail(LOTUS_ERR_INVALID, "conv2d: x, w, y and residual must be 16-byte aligned");
  if (residual && d->out_kind != LOTUS_OUT_NHWC_F16)
    return fail(LOTUS_ERR_INVALID, "conv2d: residual needs the NHWC fp16 output");
  if (d->out_kind == LOTUS_OUT_ROWS_F32 && (reinterpret_cast<uintptr_t>(y) & 3u))
    return fail(LOTUS_ERR_INVALID, "conv2d: fp32 output must be 4-byte aligned");
  if (workspace && !aligned16(workspace)) return fail(LOTUS_ERR_INVALID, "conv2d: workspace must be 16-byte aligned");
  ConvTcArgs a = conv_args(x, w_packed, bias, residual, y, d, oh, ow);
  a.ws = static_cast<float*>(workspace);
  a.ws_bytes = workspace ? workspace_bytes : 0;
  a.y_stride = y_stride;
  const char* err = "";
  if (use_rows_conv(a, d->n)) {
    const int rr = conv_rows_launch(a, d->n, stream, &err);
    if (rr != 0) return fail(rr == -2 ? LOTUS_ERR_UNSUPPORTED : LOTUS_ERR_CUDA, std::string("conv2d: ") + err);
    return ok();
  }
  if (const int bn = pair_conv_bn(a)) {
    // the pair kernel splits its last wave over K when the workspace holds
    // conv_pair_workspace_bytes; pair_split = false keeps it whole
    ConvTcArgs pa = a;
    if (!pair_split) {
      pa.ws = nullptr;
      pa.ws_bytes = 0;
    }
    const int rr = conv_pair_launch(pa, bn, stream, &err);
    if (rr != 0) return fail(rr == -2 ? LOTUS_ERR_UNSUPPORTED : LOTUS_ERR_CUDA, std::string("conv2d: ") + err);
    return ok();
  }
  const int r = conv_tc_launch(a, stream, &err);
  if (r != 0) return fail(r == -2 ? LOTUS_ERR_UNSUPPORTED : LOTUS_ERR_CUDA, std::string("conv2d: ") + err);
  return ok();
}

int lotus_conv2d_fwd(const void* x, const void* w_packed, const float* bias, const void* residual, void* y,
                     const lotus_conv2d_desc* d, cudaStream_t stream) {
  return conv_fwd_impl(x, w_packed, bias, residual, y, d, nullptr, 0, stream);
}

int lotus_conv2d_fwd_ws(const void* x, const void* w_packed, const float* bias, const void* residual, void* y,
                        const lotus_conv2d_desc* d, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return conv_fwd_impl(x, w_packed, bias, residual, y, d, workspace, workspace_bytes, stream);
}

int lotus_conv2d_fwd_slice(const void* x, const void* w_packed, const float* bias, const void* residual, void* y,
                           int y_pixel_stride, const lotus_conv2d_desc* d, void* workspace, size_t workspace_bytes,
                           cudaStream_t stream) {
  if (y_pixel_stride <= 0) return fail(LOTUS_ERR_INVALID, "conv2d_slice: pixel stride must be positive");
  return conv_fwd_impl(x, w_packed, bias, residual, y, d, workspace, workspace_bytes, stream, y_pixel_stride);
}

int lotus_conv2d_fwd_noalloc(const void* x, const void* w_packed, const float* bias, const void* residual, void* y,
                             const lotus_conv2d_desc* d, cudaStream_t stream) {
  static_assert(kNoAllocScratchBytes == LOTUS_NOALLOC_SCRATCH_BYTES, "scratch size in the header");
  int oh, ow;
  const int st = check_conv_desc(d, &oh, &ow);
  if (st != LOTUS_OK) return st;
  const size_t need = lotus_conv2d_workspace_bytes(d);
  if (need > kNoAllocScratchBytes)
    return fail(LOTUS_ERR_UNSUPPORTED, "conv2d_noalloc: this shape's split-K needs " + std::to_string(need) +
                                           " bytes of scratch, above the " + std::to_string(kNoAllocScratchBytes) +
                                           " built into the library; use lotus_conv2d_fwd_ws with a caller workspace");
  float* scratch = nullptr;
  if (need > 0) {
    const char* err = "";
    if (conv_tc_noalloc_scratch(&scratch, &err) != 0)
      return fail(LOTUS_ERR_CUDA, std::string("conv2d_noalloc: scratch set-up: ") + err);
  }
  return conv_fwd_impl(x, w_packed, bias, residual, y, d, scratch, scratch ? kNoAllocScratchBytes : 0, stream, 0,
                       /*pair_split=*/false);
}

size_t lotus_conv2d_workspace_bytes(const lotus_conv2d_desc* d) {
  int oh, ow;
  if (check_conv_desc(d, &oh, &ow) != LOTUS_OK) return 0;
  // placeholder non-null, 16-aligned pointers: planning reads no memory
  void* fake = reinterpret_cast<void*>(static_cast<uintptr_t>(256));
  ConvTcArgs a = conv_args(fake, fake, nullptr, nullptr, fake, d, oh, ow);
  size_t need = 0;
  const char* err = "";
  if (conv_tc_launch(a, nullptr, &err, &need) != 0) return 0;
  ok();
  return need;
}

// The general kernel's split-K need, or, for launches the CTA-pair kernel
// takes, the workspace it uses to split the K loop of its last wave of tiles
// (optional: with less the pair kernel runs unsplit, which is why
// lotus_conv2d_workspace_bytes leaves it out).
size_t lotus_conv2d_workspace_bytes_max(const lotus_conv2d_desc* d) {
  int oh, ow;
  if (check_conv_desc(d, &oh, &ow) != LOTUS_OK) return 0;
  void* fake = reinterpret_cast<void*>(static_cast<uintptr_t>(256));
  ConvTcArgs a = conv_args(fake, fake, nullptr, nullptr, fake, d, oh, ow);
  if (!use_rows_conv(a, d->n))
    if (const int bn = pair_conv_bn(a)) {
      ok();
      return conv_pair_workspace_bytes(a, bn);
    }
  return lotus_conv2d_workspace_bytes(d);
}

// ------------------------------------------------------------------ tconv
static int check_tconv(const lotus_tconv2d_desc* d, int* oh, int* ow) {
  if (!d) return fail(LOTUS_ERR_INVALID, "tconv2d: null descriptor");
  if (d->n <= 0 || d->c_in <= 0 || d->h <= 0 || d->w <= 0 || d->c_out <= 0 || d->kh <= 0 || d->kw <= 0)
    return fail(LOTUS_ERR_INVALID, "tconv2d: sizes must be positive");
  if (d->stride_h <= 0 || d->stride_w <= 0 || d->pad_h < 0 || d->pad_w < 0 || d->out_pad_h < 0 || d->out_pad_w < 0)
    return fail(LOTUS_ERR_INVALID, "tconv2d: bad stride/padding");
  if (d->out_pad_h >= d->stride_h || d->out_pad_w >= d->stride_w)
    return fail(LOTUS_ERR_INVALID, "tconv2d: output_padding must be smaller than stride");
  if (d->act < 0 || d->act > 2) return fail(LOTUS_ERR_INVALID, "tconv2d: unknown activation");
  const long a = static_cast<long>(d->h - 1) * d->stride_h - 2L * d->pad_h + d->kh + d->out_pad_h;
  const long b = static_cast<long>(d->w - 1) * d->stride_w - 2L * d->pad_w + d->kw + d->out_pad_w;
  if (a <= 0 || b <= 0) return fail(LOTUS_ERR_INVALID, "tconv2d: empty output");
  if (static_cast<long>(d->n) * a * b > kMaxIndex || static_cast<long>(d->n) * d->h * d->w > kMaxIndex)
    return fail(LOTUS_ERR_UNSUPPORTED, "tconv2d: too many pixels");
  if (static_cast<long>(d->kh) * d->kw * d->c_out > 65535)
    return fail(LOTUS_ERR_UNSUPPORTED, "tconv2d: kh*kw*c_out > 65535");
  *oh = static_cast<int>(a);
  *ow = static_cast<int>(b);
  return ok();
}

int lotus_tconv2d_out_hw(const lotus_tconv2d_desc* d, int* oh, int* ow) {
  int a, b;
  const int st = check_tconv(d, &a, &b);
  if (st != LOTUS_OK) return st;
  if (oh) *oh = a;
  if (ow) *ow = b;
  return ok();
}

size_t lotus_tconv2d_packed_weight_bytes(const lotus_tconv2d_desc* d) {
  if (!d || d->c_out <= 0 || d->kh <= 0 || d->kw <= 0 || d->c_in <= 0) return 0;
  return static_cast<size_t>(d->kh) * d->kw * d->c_out * round64(cs_of(d->c_in)) * 2;
}

int lotus_tconv2d_prepack(const float* w, void* w_packed, const lotus_tconv2d_desc* d, cudaStream_t stream) {
  int oh, ow;
  const int st = check_tconv(d, &oh, &ow);
  if (st != LOTUS_OK) return st;
  if (!w || !w_packed) return fail(LOTUS_ERR_INVALID, "tconv2d_prepack: null pointer");
  const int cs = cs_of(d->c_in);
  return cuda_status(
      launch_tconv_prepack(w, w_packed, d->c_in, d->c_out, d->kh, d->kw, cs, round64(cs), stream), "tconv2d_prepack");
}

static int tconv_fwd_impl(const void* x, const void* w_packed, const float* bias, void* y, int y_stride,
                          const lotus_tconv2d_desc* d, cudaStream_t stream) {
  int oh, ow;
  const int st = check_tconv(d, &oh, &ow);
  if (st != LOTUS_OK) return st;
  if (!x || !w_packed || !y) return fail(LOTUS_ERR_INVALID, "tconv2d: null x, w or y");
  if (!aligned16(x) || !aligned16(w_packed) || !aligned16(y))
    return fail(LOTUS_ERR_INVALID, "tconv2d: x, w and y must be 16-byte aligned");
  const int cs_in = cs_of(d->c_in), cs_out = cs_of(d->c_out);
  if (y_stride == 0) y_stride = cs_out;
  if (y_stride < cs_out || y_stride % 8 != 0)
    return fail(LOTUS_ERR_INVALID, "tconv2d: output pixel stride must be a multiple of 8 and >= roundup(c_out, 8)");
  const int k_pad = round64(cs_in);
  const size_t out_pixels = static_cast<size_t>(d->n) * oh * ow;
  const bool no_overlap = d->stride_h >= d->kh && d->stride_w >= d->kw;
  if (!no_overlap) {
    return cuda_status(launch_tconv_direct(x, w_packed, k_pad, bias, y, y_stride, d->n, d->c_in, cs_in, d->h, d->w,
                                           d->c_out, cs_out, oh, ow, d->kh, d->kw, d->stride_h, d->stride_w, d->pad_h,
                                           d->pad_w, d->act, stream),
                       "tconv2d(direct)");
  }
  const bool full_cover = d->stride_h == d->kh && d->stride_w == d->kw && d->out_pad_h == 0 && d->out_pad_w == 0;
  if (!full_cover || cs_out != d->c_out) {
    const cudaError_t e = launch_tconv_fill_bias(y, y_stride, bias, d->c_out, cs_out, out_pixels, d->act, stream);
    if (e != cudaSuccess) return cuda_status(e, "tconv2d(fill)");
  }
  ConvTcArgs a{};
  a.x = x;
  a.w_packed = w_packed;
  a.bias = bias;
  a.residual = nullptr;
  a.y = y;
  a.H = d->h;
  a.W = d->w;
  a.Cs_in = cs_in;
  a.OH = d->h;
  a.OW = d->w;
  a.kh = 1;
  a.kw = 1;
  a.sh = 1;
  a.sw = 1;
  a.ph = 0;
  a.pw = 0;
  a.n_cols = d->kh * d->kw * d->c_out;
  a.k_pad = k_pad;
  a.Cs_out = cs_out;
  a.M = d->n * d->h * d->w;
  a.act = d->act;
  a.out_kind = 2;
  a.t_oh = oh;
  a.t_ow = ow;
  a.t_sh = d->stride_h;
  a.t_sw = d->stride_w;
  a.t_ph = d->pad_h;
  a.t_pw = d->pad_w;
  a.t_kw = d->kw;
  a.t_cout = d->c_out;
  a.y_stride = y_stride;
  const char* err = "";
  const int r = conv_tc_launch(a, stream, &err);
  if (r != 0) return fail(r == -2 ? LOTUS_ERR_UNSUPPORTED : LOTUS_ERR_CUDA, std::string("tconv2d: ") + err);
  return ok();
}

int lotus_tconv2d_fwd(const void* x, const void* w_packed, const float* bias, void* y, const lotus_tconv2d_desc* d,
                      cudaStream_t stream) {
  return tconv_fwd_impl(x, w_packed, bias, y, 0, d, stream);
}

int lotus_tconv2d_fwd_slice(const void* x, const void* w_packed, const float* bias, void* y, int y_pixel_stride,
                            const lotus_tconv2d_desc* d, cudaStream_t stream) {
  if (y_pixel_stride <= 0) return fail(LOTUS_ERR_INVALID, "tconv2d_slice: pixel stride must be positive");
  return tconv_fwd_impl(x, w_packed, bias, y, y_pixel_stride, d, stream);
}

// ------------------------------------------------------------------ linear
size_t lotus_linear_packed_weight_bytes(int in_features, int out_features) {
  if (in_features <= 0 || out_features <= 0) return 0;
  return static_cast<size_t>(out_features) * round64(in_features) * 2;
}

int lotus_linear_prepack(const float* w, void* w_packed, int in_features, int out_features, int fc_c, int fc_h,
                         int fc_w, cudaStream_t stream) {
  if (!w || !w_packed) return fail(LOTUS_ERR_INVALID, "linear_prepack: null pointer");
  if (in_features <= 0 || out_features <= 0) return fail(LOTUS_ERR_INVALID, "linear_prepack: sizes must be positive");
  if ((fc_c > 0 || fc_h > 0 || fc_w > 0) && static_cast<long>(fc_c) * fc_h * fc_w != in_features)
    return fail(LOTUS_ERR_INVALID, "linear_prepack: fc_c*fc_h*fc_w != in_features");
  return cuda_status(
      launch_linear_prepack(w, w_packed, in_features, out_features, round64(in_features), fc_c, fc_h, fc_w, stream),
      "linear_prepack");
}

static int check_linear(const void* x, const void* w, void* y, int m, int in_f, int out_f, int act, int out_kind) {
  if (!x || !w || !y) return fail(LOTUS_ERR_INVALID, "linear: null x, w or y");
  if (m <= 0 || in_f <= 0 || out_f <= 0) return fail(LOTUS_ERR_INVALID, "linear: sizes must be positive");
  if (act < 0 || act > 2) return fail(LOTUS_ERR_INVALID, "linear: unknown activation");
  if (out_kind != LOTUS_OUT_NHWC_F16 && out_kind != LOTUS_OUT_ROWS_F32)
    return fail(LOTUS_ERR_INVALID, "linear: unknown out_kind");
  if (!aligned16(x) || !aligned16(w) || !aligned16(y))
    return fail(LOTUS_ERR_INVALID, "linear: x, w and y must be 16-byte aligned");
  return ok();
}

// GEMM kernel arguments of a Linear layer (M = batch rows).
static ConvTcArgs gemm_args(const void* x, const void* w_packed, const float* bias, void* y, int m, int in_features,
                            int out_features, int act, int out_kind) {
  ConvTcArgs a{};
  a.x = x;
  a.w_packed = w_packed;
  a.bias = bias;
  a.y = y;
  a.H = 1;
  a.W = 1;
  a.Cs_in = cs_of(in_features);
  a.OH = 1;
  a.OW = 1;
  a.kh = a.kw = a.sh = a.sw = 1;
  a.ph = a.pw = 0;
  a.n_cols = out_features;
  a.k_pad = round64(in_features);
  a.Cs_out = cs_of(out_features);
  a.M = m;
  a.act = act;
  a.out_kind = out_kind;
  return a;
}

static int gemm_fwd_impl(const void* x, const void* w_packed, const float* bias, void* y, int m, int in_features,
                         int out_features, int act, int out_kind, void* workspace, size_t workspace_bytes,
                         cudaStream_t stream) {
  const int st = check_linear(x, w_packed, y, m, in_features, out_features, act, out_kind);
  if (st != LOTUS_OK) return st;
  if (workspace && !aligned16(workspace)) return fail(LOTUS_ERR_INVALID, "gemm: workspace must be 16-byte aligned");
  ConvTcArgs a = gemm_args(x, w_packed, bias, y, m, in_features, out_features, act, out_kind);
  a.ws = static_cast<float*>(workspace);
  a.ws_bytes = workspace ? workspace_bytes : 0;
  const char* err = "";
  const int r = conv_tc_launch(a, stream, &err);
  if (r != 0) return fail(r == -2 ? LOTUS_ERR_UNSUPPORTED : LOTUS_ERR_CUDA, std::string("gemm: ") + err);
  return ok();
}

int lotus_gemm_bias_fwd(const void* x, const void* w_packed, const float* bias, void* y, int m, int in_features,
                        int out_features, int act, int out_kind, cudaStream_t stream) {
  return gemm_fwd_impl(x, w_packed, bias, y, m, in_features, out_features, act, out_kind, nullptr, 0, stream);
}

int lotus_linear_fwd(const void* x, const void* w_packed, const float* bias, void* y, int m, int in_features,
                     int out_features, int act, int out_kind, cudaStream_t stream) {
  return lotus_linear_fwd_ws(x, w_packed, bias, y, m, in_features, out_features, act, out_kind, nullptr, 0, stream);
}

size_t lotus_linear_workspace_bytes(int m, int in_features, int out_features) {
  if (m <= 8 || in_features <= 0 || out_features <= 0) return 0;  // the GEMV path needs none
  void* fake = reinterpret_cast<void*>(static_cast<uintptr_t>(256));
  ConvTcArgs a = gemm_args(fake, fake, nullptr, fake, m, in_features, out_features, 0, LOTUS_OUT_ROWS_F32);
  size_t need = 0;
  const char* err = "";
  if (conv_tc_launch(a, nullptr, &err, &need) != 0) return 0;
  ok();
  return need;
}

int lotus_linear_fwd_ws(const void* x, const void* w_packed, const float* bias, void* y, int m, int in_features,
                        int out_features, int act, int out_kind, void* workspace, size_t workspace_bytes,
                        cudaStream_t stream) {
  const int st = check_linear(x, w_packed, y, m, in_features, out_features, act, out_kind);
  if (st != LOTUS_OK) return st;
  if (m > 8)
    return gemm_fwd_impl(x, w_packed, bias, y, m, in_features, out_features, act, out_kind, workspace, workspace_bytes,
                         stream);
  const bool f16 = out_kind == LOTUS_OUT_NHWC_F16;
  const int ldy = f16 ? cs_of(out_features) : out_features;
  cudaError_t e = launch_gemv(w_packed, 1, round64(in_features), x, 1, cs_of(in_features), bias, y, f16 ? 1 : 0, ldy,
                              m, out_features, in_features, act, stream);
  if (e == cudaSuccess && f16 && ldy != out_features)
    e = cudaMemset2DAsync(static_cast<char*>(y) + static_cast<size_t>(out_features) * 2, static_cast<size_t>(ldy) * 2, 0,
                          static_cast<size_t>(ldy - out_features) * 2, m, stream);
  return cuda_status(e, "linear(gemv)");
}

int lotus_gemv_bias_fwd(const void* w, int w_dtype, const void* x, int x_dtype, const float* bias, void* y,
                        int y_dtype, int batch, int h_out, int w_in, int act, cudaStream_t stream) {
  if (!w || !x || !y) return fail(LOTUS_ERR_INVALID, "gemv: null w, x or y");
  if (batch <= 0 || batch > 8 || h_out <= 0 || w_in <= 0)
    return fail(LOTUS_ERR_INVALID, "gemv: need 1 <= batch <= 8 and positive sizes");
  if ((w_dtype != 0 && w_dtype != 1) || (x_dtype != 0 && x_dtype != 1) || (y_dtype != 0 && y_dtype != 1))
    return fail(LOTUS_ERR_INVALID, "gemv: dtype must be 0 (fp32) or 1 (fp16)");
  if (act < 0 || act > 2) return fail(LOTUS_ERR_INVALID, "gemv: unknown activation");
  const int ldw = w_dtype ? round64(w_in) : w_in;
  const int ldx = x_dtype ? cs_of(w_in) : w_in;
  const int ldy = y_dtype ? cs_of(h_out) : h_out;
  cudaError_t e = launch_gemv(w, w_dtype, ldw, x, x_dtype, ldx, bias, y, y_dtype, ldy, batch, h_out, w_in, act, stream);
  if (e == cudaSuccess && y_dtype && ldy != h_out)
    e = cudaMemset2DAsync(static_cast<char*>(y) + static_cast<size_t>(h_out) * 2, static_cast<size_t>(ldy) * 2, 0,
                          static_cast<size_t>(ldy - h_out) * 2, batch, stream);
  return cuda_status(e, "gemv");
}

// ------------------------------------------------------------------ pooling
int lotus_maxpool2d_out_hw(const lotus_pool2d_desc* d, int* oh, int* ow) {
  if (!d) return fail(LOTUS_ERR_INVALID, "maxpool2d: null descriptor");
  if (d->n <= 0 || d->c <= 0 || d->h <= 0 || d->w <= 0 || d->kh <= 0 || d->kw <= 0 || d->stride_h <= 0 ||
      d->stride_w <= 0 || d->pad_h < 0 || d->pad_w < 0)
    return fail(LOTUS_ERR_INVALID, "maxpool2d: bad sizes");
  if (2 * d->pad_h > d->kh || 2 * d->pad_w > d->kw)
    return fail(LOTUS_ERR_INVALID, "maxpool2d: padding must be at most half the kernel");
  const int eh = d->h + 2 * d->pad_h - d->kh, ew = d->w + 2 * d->pad_w - d->kw;
  if (eh < 0 || ew < 0) return fail(LOTUS_ERR_INVALID, "maxpool2d: kernel larger than padded input");
  if (oh) *oh = eh / d->stride_h + 1;
  if (ow) *ow = ew / d->stride_w + 1;
  return ok();
}

static int maxpool_impl(const void* x, int x_stride, void* y, const lotus_pool2d_desc* d, cudaStream_t stream) {
  int oh, ow;
  const int st = lotus_maxpool2d_out_hw(d, &oh, &ow);
  if (st != LOTUS_OK) return st;
  if (d->act < 0 || d->act > 2) return fail(LOTUS_ERR_INVALID, "maxpool2d: unknown activation");
  if (!x || !y || !aligned16(x) || !aligned16(y)) return fail(LOTUS_ERR_INVALID, "maxpool2d: bad x or y pointer");
  if (x_stride == 0) x_stride = cs_of(d->c);
  if (x_stride < cs_of(d->c) || x_stride % 8 != 0)
    return fail(LOTUS_ERR_INVALID, "maxpool2d: input pixel stride must be a multiple of 8 and >= roundup(c, 8)");
  return cuda_status(launch_maxpool(x, x_stride, y, d->n, d->c, cs_of(d->c), d->h, d->w, oh, ow, d->kh, d->kw,
                                    d->stride_h, d->stride_w, d->pad_h, d->pad_w, d->act, stream),
                     "maxpool2d");
}

int lotus_maxpool2d_fwd(const void* x, void* y, const lotus_pool2d_desc* d, cudaStream_t stream) {
  return maxpool_impl(x, 0, y, d, stream);
}

int lotus_maxpool2d_fwd_strided(const void* x, int x_pixel_stride, void* y, const lotus_pool2d_desc* d,
                                cudaStream_t stream) {
  if (x_pixel_stride <= 0) return fail(LOTUS_ERR_INVALID, "maxpool2d_strided: pixel stride must be positive");
  return maxpool_impl(x, x_pixel_stride, y, d, stream);
}

// Row-conv arguments of a conv (+ pool) request, or an error status.
static int row_conv_args(const lotus_conv2d_desc* d, const lotus_pool2d_desc* pool, ConvRowArgs* a) {
  int oh, ow;
  const int st = check_conv_desc(d, &oh, &ow);
  if (st != LOTUS_OK) return st;
  if (d->out_kind != LOTUS_OUT_NHWC_F16)
    return fail(LOTUS_ERR_UNSUPPORTED, "conv2d_maxpool: NHWC fp16 output only");
  if (d->stride_h != 1 || d->stride_w != 1 || d->pad_h != 0 || d->pad_w != 0)
    return fail(LOTUS_ERR_UNSUPPORTED, "conv2d_maxpool: stride 1, no padding only");
  if (pool) {
    int ph, pw;
    const int ps = lotus_maxpool2d_out_hw(pool, &ph, &pw);
    if (ps != LOTUS_OK) return ps;
    if (pool->n != d->n || pool->c != d->c_out || pool->h != oh || pool->w != ow)
      return fail(LOTUS_ERR_INVALID, "conv2d_maxpool: pool input must be the conv output");
    if (pool->kh != 3 || pool->kw != 3 || pool->stride_h != 2 || pool->stride_w != 2 || pool->pad_h != 1 ||
        pool->pad_w != 1)
      return fail(LOTUS_ERR_UNSUPPORTED, "conv2d_maxpool: 3x3 / stride 2 / pad 1 pooling only");
    // max commutes with the monotone activations, but a second activation after
    // the pool is only the identity for ReLU after ReLU
    if (!(pool->act == LOTUS_ACT_NONE || (pool->act == LOTUS_ACT_RELU && d->act == LOTUS_ACT_RELU)))
      return fail(LOTUS_ERR_UNSUPPORTED, "conv2d_maxpool: activation after the pool");
  }
  a->N = d->n;
  a->H = d->h;
  a->W = d->w;
  a->Cs_in = cs_of(d->c_in);
  a->kh = d->kh;
  a->kw = d->kw;
  a->Cout = d->c_out;
  a->Cs_out = cs_of(d->c_out);
  a->act = d->act;
  a->pool = pool ? 1 : 0;
  const char* err = "";
  if (conv_row_check(*a, &err) != 0) return fail(LOTUS_ERR_UNSUPPORTED, std::string("conv2d_maxpool: ") + err);
  return ok();
}

int lotus_conv2d_maxpool_supported(const lotus_conv2d_desc* d, const lotus_pool2d_desc* pool) {
  ConvRowArgs a{};
  return row_conv_args(d, pool, &a);
}

int lotus_conv2d_maxpool_fwd(const void* x, const void* w_packed, const float* bias, void* y,
                             const lotus_conv2d_desc* d, const lotus_pool2d_desc* pool, cudaStream_t stream) {
  ConvRowArgs a{};
  const int st = row_conv_args(d, pool, &a);
  if (st != LOTUS_OK) return st;
  if (!x || !w_packed || !y) return fail(LOTUS_ERR_INVALID, "conv2d_maxpool: null x, w or y");
  if (!aligned16(x) || !aligned16(w_packed) || !aligned16(y))
    return fail(LOTUS_ERR_INVALID, "conv2d_maxpool: x, w and y must be 16-byte aligned");
  a.x = x;
  a.w_packed = w_packed;
  a.bias = bias;
  a.y = y;
  const char* err = "";
  const int r = conv_row_launch(a, stream, &err);
  if (r != 0) return fail(r == -2 ? LOTUS_ERR_UNSUPPORTED : LOTUS_ERR_CUDA, std::string("conv2d_maxpool: ") + err);
  return ok();
}

int lotus_preprocess_bgr_u8(const uint8_t* src, int n, int src_h, int src_w, int resize_h, int resize_w, int crop_h,
                            int crop_w, const float* mean, const float* stdv, float* dst, cudaStream_t stream) {
  if (!src || !dst) return fail(LOTUS_ERR_INVALID, "preprocess: null src or dst");
  if (n <= 0 || src_h <= 0 || src_w <= 0 || resize_h <= 0 || resize_w <= 0 || crop_h <= 0 || crop_w <= 0)
    return fail(LOTUS_ERR_INVALID, "preprocess: sizes must be positive");
  if (crop_h > resize_h || crop_w > resize_w) return fail(LOTUS_ERR_INVALID, "preprocess: crop larger than the resize");
  if (static_cast<int64_t>(n) * src_h * src_w * 3 > (int64_t(1) << 40))
    return fail(LOTUS_ERR_UNSUPPORTED, "preprocess: input too large");
  static const float kMean[3] = {0.485f, 0.456f, 0.406f};
  static const float kStd[3] = {0.229f, 0.224f, 0.225f};
  const float* m = mean ? mean : kMean;
  const float* sd = stdv ? stdv : kStd;
  for (int c = 0; c < 3; ++c)
    if (!(sd[c] != 0.f)) return fail(LOTUS_ERR_INVALID, "preprocess: std must be non-zero");
  return cuda_status(launch_preprocess(src, n, src_h, src_w, resize_h, resize_w, crop_h, crop_w, m, sd, dst, stream),
                     "preprocess");
}

int lotus_adaptive_avgpool2d_fwd(const void* x, void* y, int n, int c, int h, int w, int oh, int ow, int act,
                                 int out_f32, cudaStream_t stream) {
  if (!x || !y || !aligned16(x) || !aligned16(y)) return fail(LOTUS_ERR_INVALID, "adaptive_avgpool2d: bad pointer");
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0 || oh <= 0 || ow <= 0)
    return fail(LOTUS_ERR_INVALID, "adaptive_avgpool2d: sizes must be positive");
  if (act < 0 || act > 2) return fail(LOTUS_ERR_INVALID, "adaptive_avgpool2d: unknown activation");
  return cuda_status(launch_adaptive_avgpool(x, y, n, c, cs_of(c), h, w, oh, ow, act, out_f32 ? 1 : 0, stream),
                     "adaptive_avgpool2d");
}

// ------------------------------------------------------------------ eltwise
int lotus_add_act_fwd(const void* x1, const void* x2, void* y, size_t pixels, int c, int act, cudaStream_t stream) {
  if (!x1 || !x2 || !y || !aligned16(x1) || !aligned16(x2) || !aligned16(y))
    return fail(LOTUS_ERR_INVALID, "add: bad pointer");
  if (c <= 0) return fail(LOTUS_ERR_INVALID, "add: channels must be positive");
  if (act < 0 || act > 2) return fail(LOTUS_ERR_INVALID, "add: unknown activation");
  if (pixels == 0) return ok();
  return cuda_status(launch_add_act(x1, x2, y, pixels, c, cs_of(c), act, stream), "add");
}

int lotus_concat_channels_fwd(const void* a, int ca, const void* b, int cb, void* y, int n, int h, int w,
                              cudaStream_t stream) {
  if (!a || !b || !y) return fail(LOTUS_ERR_INVALID, "concat: null pointer");
  if (ca <= 0 || cb <= 0 || n <= 0 || h <= 0 || w <= 0) return fail(LOTUS_ERR_INVALID, "concat: bad sizes");
  const size_t pixels = static_cast<size_t>(n) * h * w;
  return cuda_status(launch_concat(a, cs_of(ca), b, cs_of(cb), y, ca, cb, cs_of(ca + cb), pixels, stream), "concat");
}

int lotus_nchw_f32_to_nhwc_f16(const float* x, void* y, int n, int c, int h, int w, cudaStream_t stream) {
  if (!x || !y || !aligned16(y)) return fail(LOTUS_ERR_INVALID, "nchw_to_nhwc: bad pointer");
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0) return fail(LOTUS_ERR_INVALID, "nchw_to_nhwc: bad sizes");
  return cuda_status(launch_nchw_to_nhwc(x, y, n, c, h, w, cs_of(c), stream), "nchw_to_nhwc");
}

int lotus_space_to_depth_f16(const float* x, void* y, int n, int c, int h, int w, int factor, int pad_h, int pad_w,
                             int out_h, int out_w, cudaStream_t stream) {
  if (!x || !y || !aligned16(y)) return fail(LOTUS_ERR_INVALID, "space_to_depth: bad pointer");
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0 || factor <= 0 || pad_h < 0 || pad_w < 0 || out_h <= 0 || out_w <= 0)
    return fail(LOTUS_ERR_INVALID, "space_to_depth: bad sizes");
  return cuda_status(launch_space_to_depth(x, y, n, c, h, w, factor, pad_h, pad_w, out_h, out_w,
                                           cs_of(c * factor * factor), stream),
                     "space_to_depth");
}

int lotus_nhwc_f16_to_nchw_f32(const void* x, float* y, int n, int c, int h, int w, cudaStream_t stream) {
  if (!x || !y || !aligned16(x)) return fail(LOTUS_ERR_INVALID, "nhwc_to_nchw: bad pointer");
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0) return fail(LOTUS_ERR_INVALID, "nhwc_to_nchw: bad sizes");
  return cuda_status(launch_nhwc_to_nchw(x, y, n, c, h, w, cs_of(c), stream), "nhwc_to_nchw");
}

}  // extern "C"
