// Host-side declarations of the kernel launchers behind the C ABI.
// Everything here is internal; the public surface is include/lotus_ops.h.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace lotus_impl {

// Counts every kernel launch issued by the library (exported through
// lotus_launch_count()).
void note_launch();

struct ConvTcArgs {
  const void* x;          // NHWC fp16 [.., H, W, Cs_in]
  const void* w_packed;   // [n_cols, k_pad] fp16
  const float* bias;      // [bias length] or null
  const void* residual;   // NHWC fp16 like y, or null
  void* y;
  int H, W, Cs_in;
  int OH, OW;             // GEMM pixel grid (conv output, or tconv input grid)
  int kh, kw, sh, sw, ph, pw;
  int n_cols;             // GEMM N (Cout, or kh*kw*Cout for the tconv scatter)
  int k_pad;              // multiple of 64
  int Cs_out;             // pixel stride of an NHWC fp16 output
  int M;                  // GEMM M
  int act;
  int out_kind;           // 0 NHWC fp16, 1 fp32 rows, 2 tconv scatter
  int block_n;            // 0 = choose
  int t_oh, t_ow, t_sh, t_sw, t_ph, t_pw, t_kw, t_cout;
  float* ws = nullptr;    // split-K workspace (fp32) or null
  size_t ws_bytes = 0;
  int y_stride = 0;       // pixel stride of an NHWC fp16 output (0 = Cs_out)
};

// Launches the conv / GEMM kernel (and the split-K reduction when it splits).
// With ws_need != null it only plans: *ws_need = the workspace bytes the
// split-K plan for `a` wants (0 = no split), nothing is launched.
int conv_tc_launch(const ConvTcArgs& a, cudaStream_t stream, const char** err, size_t* ws_need = nullptr);

// Built-in split-K scratch of lotus_conv2d_fwd_noalloc (LOTUS_NOALLOC_SCRATCH_BYTES).
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
// Device address of that scratch on the current device; the first call on a
// device looks it up (cudaGetSymbolAddress).  0 = ok, < 0 = error in *err.
int conv_tc_noalloc_scratch(float** ptr, const char** err);
// Returns and clears the device error word of every kernel file (first
// non-zero code, 0 = none, -1 = unreadable).
int read_device_error();

// Shared host helpers (conv_tc.cu): a driver entry point by name, the tiled
// tensor-map encoder, the current device's SM count, the bounded-wait limit
// of a launch (LOTUS_WAIT_LIMIT or the default) and the process-unique id of
// the current CUDA context (0 = none).
void* driver_fn(const char* name);
// LOTUS_PDL=0 turns programmatic dependent launch off (default on).
bool pdl_enabled();
// Launch that allows programmatic dependent launch (the kernel must call
// griddep_wait() before touching data earlier kernels wrote).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}
PFN_cuTensorMapEncodeTiled_v12000 encode_tiled();
PFN_cuTensorMapEncodeIm2col_v12000 encode_im2col();
int num_sms();
uint32_t wait_limit_from_env();
uint64_t current_context_id();

// conv_row.cu: the row-tile conv (stride 1, no padding, Cs_in*kw == 64,
// OW <= 128, Cout <= 64) with an optional fused 3x3 / stride-2 / pad-1 max
// pool of its activated output.
struct ConvRowArgs {
  const void* x;          // NHWC fp16 [N, H, W, Cs_in]
  const void* w_packed;   // [Cout, kh*64] fp16 (the conv prepack)
  const float* bias;      // [Cout] or null
  void* y;                // NHWC fp16 [N, OH, OW, Cs_out] or pooled [N, PH, PW, Cs_out]
  int N, H, W, Cs_in, kh, kw, Cout, Cs_out, act;
  int pool;               // 0 none, 1 max pool 3x3 / stride 2 / pad 1
};
// 0 when the row kernel takes this shape, else -2 with the reason in *err.
int conv_row_check(const ConvRowArgs& a, const char** err);
int conv_row_launch(const ConvRowArgs& a, cudaStream_t stream, const char** err);
int conv_row_read_device_error();

// conv_rows.cu: the row-stacked conv for stride-1 convs over 64-channel
// pixels (kernels up to 3x3, padding below the kernel size, <= 64 output
// channels, output rows <= 128 pixels, dense NHWC fp16 output, optional
// residual): ResNet stage 1.  `n` is the batch.  check: 0 when it takes the
// shape, else -2 with the reason in *err.
int conv_rows_check(const ConvTcArgs& a, int n, const char** err);
int conv_rows_launch(const ConvTcArgs& a, int n, cudaStream_t stream, const char** err);
int conv_rows_read_device_error();

// conv_pair.cu: the conv on CTA pairs (tcgen05 cta_group::2) for inputs
// with a multiple of 64 channels, NHWC fp16 output (optional residual, any
// kernel / stride / padding the im2col TMA takes), output channels <= 1024.
// `bn` = 256 (256 x 256 pair tiles) or 128 (512 x 128 pair tiles: two M
// tiles a CTA).  check: 0 when it takes the
// shape, else -2 with the reason in *err.
int conv_pair_check(const ConvTcArgs& a, int bn, const char** err);
int conv_pair_launch(const ConvTcArgs& a, int bn, cudaStream_t stream, const char** err);
// Workspace bytes the pair kernel uses to split its last wave over K (0: it
// does not split this shape); without that much workspace it runs unsplit.
size_t conv_pair_workspace_bytes(const ConvTcArgs& a, int bn);
// conv_tc.cu: the split-K reduction into an NHWC fp16 output.
cudaError_t launch_splitk_reduce(const float* ws, int splits, int rows, int ws_ld, const float* bias,
                                 const __half* residual, __half* y, int M, int cout, int cs_out, int y_stride,
                                 int act, cudaStream_t stream);
int conv_pair_read_device_error();

// pack.cu
cudaError_t launch_conv_prepack(const float* w, void* wp, int cout, int cin, int kh, int kw, int cs_in, int k_pad,
                                cudaStream_t s);
cudaError_t launch_tconv_prepack(const float* w, void* wp, int cin, int cout, int kh, int kw, int cs_in, int k_pad,
                                 cudaStream_t s);
cudaError_t launch_linear_prepack(const float* w, void* wp, int in_f, int out_f, int k_pad, int fc_c, int fc_h,
                                  int fc_w, cudaStream_t s);
cudaError_t launch_nchw_to_nhwc(const float* x, void* y, int n, int c, int h, int w, int cs, cudaStream_t s);
cudaError_t launch_space_to_depth(const float* x, void* y, int n, int c, int h, int w, int f, int pad_h, int pad_w,
                                  int oh, int ow, int cs, cudaStream_t s);
cudaError_t launch_nhwc_to_nchw(const void* x, float* y, int n, int c, int h, int w, int cs, cudaStream_t s);

// pool.cu
// x_stride: input pixel stride (elements; a channel slice of a wider tensor), cs: output pixel stride
cudaError_t launch_maxpool(const void* x, int x_stride, void* y, int n, int c, int cs, int h, int w, int oh, int ow,
                           int kh, int kw, int sh, int sw, int ph, int pw, int act, cudaStream_t s);
cudaError_t launch_adaptive_avgpool(const void* x, void* y, int n, int c, int cs, int h, int w, int oh, int ow,
                                    int act, int out_f32, cudaStream_t s);

// eltwise.cu
cudaError_t launch_add_act(const void* a, const void* b, void* y, size_t pixels, int c, int cs, int act,
                           cudaStream_t s);
cudaError_t launch_concat(const void* a, int csa, const void* b, int csb, void* y, int ca, int cb, int csy,
                          size_t pixels, cudaStream_t s);
cudaError_t launch_tconv_fill_bias(void* y, int y_stride, const float* bias, int cout, int cs, size_t pixels, int act,
                                   cudaStream_t s);
cudaError_t launch_tconv_direct(const void* x, const void* wp, int k_pad, const float* bias, void* y, int y_stride,
                                int n, int cin, int csi, int h, int w_, int cout, int cso, int oh, int ow, int kh,
                                int kw, int sh, int sw, int ph, int pw, int act, cudaStream_t s);

// preprocess.cu
cudaError_t launch_preprocess(const uint8_t* src, int n, int h, int w, int rh, int rw, int ch, int cw,
                              const float* mean, const float* stdv, float* dst, cudaStream_t s);

// gemv.cu
cudaError_t launch_gemv(const void* w, int w_f16, int ldw, const void* x, int x_f16, int ldx, const float* bias,
                        void* y, int y_f16, int ldy, int batch, int h_out, int w_in, int act, cudaStream_t s);

}  // namespace lotus_impl
