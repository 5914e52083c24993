/*
 * lotus_ops.h - C ABI of the B200 (sm_100a) dense-contraction operators.
 *
 * Each entry point replaces one `__global__` operator of lotusInfer together
 * with its `Make*Grid/Make*Block` launch helpers (include/operator/*.cuh in
 * the reference).  Differences from the reference interface, all deliberate:
 *   - one call per layer for the whole batch (the reference launches once per
 *     sample, e.g. source/layer/layer_conv2d.cu:43-70);
 *   - an explicit cudaStream_t and an int status (0 = OK, < 0 = error; the
 *     text is in lotus_last_error_string()) instead of unchecked launches;
 *   - activations inside the network are NHWC fp16 with the channel stride
 *     padded to a multiple of 8 ("Cs"); layout conversion entry points move
 *     NCHW fp32 tensors (the reference's Tensor format) in and out;
 *   - weights are prepacked once at load time into K-major fp16.
 * All pointers are device pointers owned by the caller.  No entry point
 * allocates device memory.
 */
#ifndef LOTUS_OPS_H_
#define LOTUS_OPS_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define LOTUS_OK 0
#define LOTUS_ERR_INVALID (-1)     /* bad shape, pointer or alignment */
#define LOTUS_ERR_UNSUPPORTED (-2) /* valid request outside this build's kernels */
#define LOTUS_ERR_CUDA (-3)        /* a CUDA runtime/driver call failed */

/* Activation, same values as lotus::ActivationFunction
 * (reference include/lotus_utils.hpp:44-48). */
#define LOTUS_ACT_NONE 0
#define LOTUS_ACT_RELU 1
#define LOTUS_ACT_SIGMOID 2

/* Output element type / layout of a contraction. */
#define LOTUS_OUT_NHWC_F16 0   /* [N, OH, OW, Cs_out] fp16, pad channels zeroed */
#define LOTUS_OUT_ROWS_F32 1   /* [N*OH*OW, Cout] fp32 rows (logits, GEMM C) */

/* Convolution descriptor.  Fields mirror the scalar arguments of the
 * reference Conv2d kernel (include/operator/conv2d.cuh:11-21), but H/W are
 * the real input sizes, not padded ones, and the batch is explicit. */
typedef struct lotus_conv2d_desc {
  int n;          /* batch */
  int c_in;       /* input channels */
  int h, w;       /* input height / width */
  int c_out;      /* output channels */
  int kh, kw;     /* kernel size */
  int stride_h, stride_w;
  int pad_h, pad_w;
  int act;        /* LOTUS_ACT_* */
  int out_kind;   /* LOTUS_OUT_* */
} lotus_conv2d_desc;

/* Output spatial size of a convolution described by `d`. */
int lotus_conv2d_out_hw(const lotus_conv2d_desc* d, int* oh, int* ow);

/* Channel stride of an NHWC fp16 activation with `c` channels. */
int lotus_channel_stride(int c);

/* Bytes of a prepacked conv weight: c_out rows of K_pad fp16, where
 * K_pad = roundup(kh*kw*Cs_in, 64). */
size_t lotus_conv2d_packed_weight_bytes(const lotus_conv2d_desc* d);

/* Prepack OIHW fp32 weights (reference layout, source/layer/layer_conv2d.cu:21)
 * into K-major fp16 rows, k = (r*kw + s)*Cs_in + c, zero padded. */
int lotus_conv2d_prepack(const float* w_oihw, void* w_packed, const lotus_conv2d_desc* d,
                         cudaStream_t stream);

/* y = act(conv(x, w) + bias [+ residual]).
 * Replaces lotus::Conv2d (reference source/operator/conv2d.cu:17-187 and the
 * unlinked source/operator/conv2d_tensorcore.cu:18-152) plus the separate
 * residual Add (source/operator/add.cu:14-26) that follows it in ResNet.
 * x: NHWC fp16 [n, h, w, Cs_in]; w_packed from lotus_conv2d_prepack; bias fp32
 * [c_out] or NULL; residual NHWC fp16 with y's shape or NULL (only with
 * LOTUS_OUT_NHWC_F16); y per d->out_kind.  Implicit GEMM on tcgen05 tensor
 * cores: fp16 operands, fp32 accumulation in TMEM. */
int lotus_conv2d_fwd(const void* x, const void* w_packed, const float* bias, const void* residual, void* y,
                     const lotus_conv2d_desc* d, cudaStream_t stream);

/* Split-K form of lotus_conv2d_fwd for launches with too few output tiles to
 * fill the GPU (small batches, late layers): the K loop is split over CTAs
 * that write fp32 partial tiles into `workspace`, and a second kernel sums
 * them (in split order, deterministically) and applies bias, residual and
 * activation.  lotus_conv2d_workspace_bytes(d) is the workspace size the
 * split for this shape wants (0 = it does not split); with a smaller or null
 * workspace the call runs unsplit, exactly like lotus_conv2d_fwd.  The
 * workspace is caller-owned device memory, 16-byte aligned; it is scratch
 * between the two kernels of one call, so calls sharing it must not overlap
 * on the GPU.  The same reference kernels as lotus_conv2d_fwd. */
size_t lotus_conv2d_workspace_bytes(const lotus_conv2d_desc* d);
/* The workspace lotus_conv2d_fwd_ws can use for this shape: the split-K need
 * above, or, for the large launches that run as 2-SM pair tiles, the fp32
 * partial sums of the last wave of tiles split over K (so that the wave keeps
 * every SM pair busy) and finished by the same reduction.  Optional: with
 * less workspace those launches run unsplit.  Split and unsplit results
 * differ only by the fp32 summation order. */
size_t lotus_conv2d_workspace_bytes_max(const lotus_conv2d_desc* d);
int lotus_conv2d_fwd_ws(const void* x, const void* w_packed, const float* bias, const void* residual, void* y,
                        const lotus_conv2d_desc* d, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* lotus_conv2d_fwd_ws writing a channel slice of a wider NHWC fp16 tensor
 * (LOTUS_OUT_NHWC_F16 only): y points at the slice's first channel (16-byte
 * aligned) and consecutive output pixels are y_pixel_stride elements apart (a
 * multiple of 8, >= roundup(c_out, 8)); only the slice's channels are written
 * (a residual, if any, keeps its own dense stride).  The graph uses it to
 * write a conv's output straight into its half of a torch.cat buffer
 * (reference source/layer/concatenate.cpp:20-35 copies it there instead). */
int lotus_conv2d_fwd_slice(const void* x, const void* w_packed, const float* bias, const void* residual, void* y,
                           int y_pixel_stride, const lotus_conv2d_desc* d, void* workspace, size_t workspace_bytes,
                           cudaStream_t stream);

/* lotus_conv2d_fwd_ws without a caller workspace, for callers that cannot
 * allocate device memory: cudaMalloc / cudaFree can synchronise the device and
 * can fail, so code that runs inside a latency-critical serving loop, inside a
 * host framework that owns the device memory pool, or anywhere a
 * mid-inference out-of-memory must not happen cannot call it.  The split-K
 * partial sums go to a scratch area compiled into this library,
 * LOTUS_NOALLOC_SCRATCH_BYTES (8 MiB) per GPU, which every GPU that loads the
 * library holds until the process exits; nothing is allocated per call.
 * A shape whose split needs more than that is rejected with
 * LOTUS_ERR_UNSUPPORTED (lotus_conv2d_workspace_bytes tells beforehand); a
 * shape that does not split runs like lotus_conv2d_fwd.  The first call on a
 * device (with that device current) looks up the scratch's device address;
 * make it before any stream capture.  All calls share the one scratch, so
 * calls whose kernels can overlap on the GPU (other streams, other host
 * threads) race: the caller serialises them.  Each call writes every partial
 * sum before reading it, so nothing needs clearing between calls.  No
 * counterpart in the reference (it has no split-K). */
#define LOTUS_NOALLOC_SCRATCH_BYTES (8u << 20)
int lotus_conv2d_fwd_noalloc(const void* x, const void* w_packed, const float* bias, const void* residual, void* y,
                             const lotus_conv2d_desc* d, cudaStream_t stream);

/* Transposed convolution (PyTorch ConvTranspose2d semantics, dilation 1).
 * Replaces lotus::TransConv2d (reference source/operator/transposed_conv2d.cu:17-140,
 * launched from source/layer/layer_transposed_conv2d.cu:37-72). */
typedef struct lotus_tconv2d_desc {
  int n, c_in, h, w, c_out, kh, kw;
  int stride_h, stride_w;
  int pad_h, pad_w;                 /* crop on each side */
  int out_pad_h, out_pad_w;         /* PyTorch output_padding */
  int act;
} lotus_tconv2d_desc;

int lotus_tconv2d_out_hw(const lotus_tconv2d_desc* d, int* oh, int* ow);
size_t lotus_tconv2d_packed_weight_bytes(const lotus_tconv2d_desc* d);
/* Prepack [Cin, Cout, kh, kw] fp32 (PyTorch ConvTranspose2d layout) weights. */
int lotus_tconv2d_prepack(const float* w_iokk, void* w_packed, const lotus_tconv2d_desc* d, cudaStream_t stream);
/* x NHWC fp16 [n,h,w,Cs_in] -> y NHWC fp16 [n,oh,ow,Cs_out]. */
int lotus_tconv2d_fwd(const void* x, const void* w_packed, const float* bias, void* y, const lotus_tconv2d_desc* d,
                      cudaStream_t stream);
/* lotus_tconv2d_fwd writing a channel slice of a wider NHWC fp16 tensor: y
 * points at the slice's first channel (16-byte aligned) and consecutive output
 * pixels are y_pixel_stride elements apart (a multiple of 8, >=
 * roundup(c_out, 8)); only the slice's channels are written.  The graph uses
 * it to write a transposed conv's output straight into its half of a
 * torch.cat buffer (reference source/layer/concatenate.cpp:20-35 copies it
 * there instead). */
int lotus_tconv2d_fwd_slice(const void* x, const void* w_packed, const float* bias, void* y, int y_pixel_stride,
                            const lotus_tconv2d_desc* d, cudaStream_t stream);

/* Linear y[m, n] = act(sum_k x[m, k] * W[n, k] + b[n]), the reference Gemm
 * (source/operator/gemm_tensorcore.cu:18-169, called from
 * source/layer/linear.cu:33-51) with M = batch.  x is fp16 rows [m, Kx]
 * (Kx = in_features; a flattened NHWC activation is passed as is).
 * out_kind selects fp16 rows (LOTUS_OUT_NHWC_F16 with 1x1 spatial, row stride
 * Cs(n)) or fp32 rows.  Small M runs the HBM-bound GEMV, larger M the
 * tcgen05 GEMM. */
size_t lotus_linear_packed_weight_bytes(int in_features, int out_features);
/* Prepack W [out, in] fp32.  If (fc_c, fc_h, fc_w) are all > 0 the input is
 * a flattened NCHW [fc_c, fc_h, fc_w] tensor in the model but NHWC in this
 * runtime, and the weight columns are permuted from (c,h,w) to (h,w,c). */
int lotus_linear_prepack(const float* w, void* w_packed, int in_features, int out_features, int fc_c, int fc_h,
                         int fc_w, cudaStream_t stream);
int lotus_linear_fwd(const void* x, const void* w_packed, const float* bias, void* y, int m, int in_features,
                     int out_features, int act, int out_kind, cudaStream_t stream);
/* Split-K form of lotus_linear_fwd (GEMM path, m > 8), same contract as
 * lotus_conv2d_fwd_ws. */
size_t lotus_linear_workspace_bytes(int m, int in_features, int out_features);
int lotus_linear_fwd_ws(const void* x, const void* w_packed, const float* bias, void* y, int m, int in_features,
                        int out_features, int act, int out_kind, void* workspace, size_t workspace_bytes,
                        cudaStream_t stream);
/* Forced variants for per-operator tests and benches. */
int lotus_gemm_bias_fwd(const void* x, const void* w_packed, const float* bias, void* y, int m, int in_features,
                        int out_features, int act, int out_kind, cudaStream_t stream);

/* Fused GEMV + bias + act, the reference Fgemva
 * (source/operator/fused_gemv_add_bias.cu:16-108): y[b, h] = act(W[h,:] . x[b,:] + bias[h]).
 * W fp32 [h_out, w_in] row-major (w_dtype 0) or a fp16 linear-prepacked
 * weight (w_dtype 1).  x fp32 (x_dtype 0) or fp16 (1) rows [batch, w_in],
 * y fp32 (y_dtype 0) or fp16 (1) rows [batch, ldy].  batch <= 8. */
int lotus_gemv_bias_fwd(const void* w, int w_dtype, const void* x, int x_dtype, const float* bias, void* y,
                        int y_dtype, int batch, int h_out, int w_in, int act, cudaStream_t stream);

/* Max pooling, NHWC fp16, padding acts as -inf (PyTorch semantics; the
 * reference kernel is source/operator/maxpool2d.cu:16-66). */
typedef struct lotus_pool2d_desc {
  int n, c, h, w;
  int kh, kw, stride_h, stride_w, pad_h, pad_w;
  int act;
} lotus_pool2d_desc;
int lotus_maxpool2d_out_hw(const lotus_pool2d_desc* d, int* oh, int* ow);
int lotus_maxpool2d_fwd(const void* x, void* y, const lotus_pool2d_desc* d, cudaStream_t stream);
/* Max pooling of a channel slice of a wider NHWC fp16 tensor: x points at the
 * slice's first channel and consecutive pixels are x_pixel_stride elements
 * apart (a multiple of 8, >= roundup(c, 8)); y as lotus_maxpool2d_fwd.  Lets
 * a pool read the encoder half of a U-Net concatenation buffer in place. */
int lotus_maxpool2d_fwd_strided(const void* x, int x_pixel_stride, void* y, const lotus_pool2d_desc* d,
                                cudaStream_t stream);

/* Convolution with the max pool that follows it fused into its epilogue:
 * y = maxpool3x3/2/pad1(act(conv(x, w) + bias)), NHWC fp16 in and out
 * ([n, ph, pw, Cs(c_out)] with the pool's output size).  Replaces the
 * reference's Conv2d launch followed by its Maxpool2d launch on the conv's
 * output (source/operator/conv2d.cu:17-187, source/operator/maxpool2d.cu:16-66,
 * one after the other in source/graph.cpp:84-109); the full-size conv output
 * is never written.  Pooling pads with -inf (PyTorch semantics).  `pool` NULL
 * runs the same row kernel without the pool (y is then the conv output).
 * Supported: stride-1 convs without padding whose kernel row is one 64-wide
 * K block (Cs(c_in) * kw == 64, e.g. the space-to-depth ResNet stem: 12
 * channels padded to 16, 4x4 kernel), output rows of at most 128 pixels, at
 * most 64 output channels, kh <= 6, the pool 3x3 / stride 2 / pad 1 with no
 * activation of its own (or ReLU after a ReLU conv).
 * lotus_conv2d_maxpool_supported returns LOTUS_OK for a request the fused
 * kernel takes, else LOTUS_ERR_UNSUPPORTED / LOTUS_ERR_INVALID with the reason
 * in lotus_last_error_string(); it launches nothing. */
int lotus_conv2d_maxpool_supported(const lotus_conv2d_desc* d, const lotus_pool2d_desc* pool);
int lotus_conv2d_maxpool_fwd(const void* x, const void* w_packed, const float* bias, void* y,
                             const lotus_conv2d_desc* d, const lotus_pool2d_desc* pool, cudaStream_t stream);

/* Adaptive average pooling, NHWC fp16 in; PyTorch windows
 * [floor(i*H/OH), ceil((i+1)*H/OH)).  Output NHWC fp16 (out_f32 = 0) or
 * fp32 rows [n, oh*ow*c] in NHWC order (out_f32 = 1).  Replaces
 * source/operator/adaptive_avgpool2d.cu:15-52. */
int lotus_adaptive_avgpool2d_fwd(const void* x, void* y, int n, int c, int h, int w, int oh, int ow, int act,
                                 int out_f32, cudaStream_t stream);

/* y = act(x1 + x2) over `pixels` NHWC fp16 pixels of `c` channels (channel
 * stride Cs(c); pad channels are written as zero).  Replaces
 * source/operator/add.cu:14-26. */
int lotus_add_act_fwd(const void* x1, const void* x2, void* y, size_t pixels, int c, int act, cudaStream_t stream);

/* Channel concatenation of two NHWC fp16 tensors (torch.cat dim=1 in NCHW
 * terms; reference source/layer/concatenate.cpp:20-35). */
int lotus_concat_channels_fwd(const void* a, int ca, const void* b, int cb, void* y, int n, int h, int w,
                              cudaStream_t stream);

/* Layout conversion between the reference's NCHW fp32 tensors and the
 * runtime's NHWC fp16 activations. */
int lotus_nchw_f32_to_nhwc_f16(const float* x, void* y, int n, int c, int h, int w, cudaStream_t stream);
int lotus_nhwc_f16_to_nchw_f32(const void* x, float* y, int n, int c, int h, int w, cudaStream_t stream);

/* Space-to-depth of a zero-padded NCHW fp32 batch into NHWC fp16:
 * y[n, i, j, (a*factor + b)*c + ch] = x[n, ch, factor*i + a - pad_h, factor*j + b - pad_w]
 * (zero outside the image), for i < out_h, j < out_w; channel stride
 * Cs(c*factor^2).  A stride-`factor` conv with kernel k on x equals a
 * stride-1 conv with kernel ceil(k/factor) on y; the graph uses this for
 * 3-channel strided stem convs.  No reference counterpart (the reference runs
 * the stem as a direct conv, source/operator/conv2d.cu:17-187). */
int lotus_space_to_depth_f16(const float* x, void* y, int n, int c, int h, int w, int factor, int pad_h, int pad_w,
                             int out_h, int out_w, cudaStream_t stream);

/* Input preprocessing of the reference's classification demo
 * (demo/image_classification.cpp:9-44, done there on the CPU with OpenCV):
 * n decoded 8-bit BGR images (HWC, all src_h x src_w, rows of src_w*3 bytes,
 * device memory) -> bilinear resize to resize_h x resize_w with the
 * cv::resize INTER_LINEAR geometry (half-pixel centres, source index clamped
 * to the edge) -> BGR to RGB -> /255 -> centre crop crop_h x crop_w at
 * (max(0, resize/2 - crop/2)) -> (x - mean[c]) / std[c] -> NCHW fp32
 * [n, 3, crop_h, crop_w] in dst, the graph input format.  mean / std: 3 floats
 * each in RGB order, or NULL for the reference's ImageNet constants
 * (0.485, 0.456, 0.406) / (0.229, 0.224, 0.225).  The resize is evaluated in
 * fp32 without rounding to 8 bits in between (OpenCV's 8-bit path does), so
 * results differ from the demo by at most one 8-bit step before the
 * normalisation.  The demo's 256 -> 224 pipeline is resize 256 x 256, crop
 * 224 x 224. */
int lotus_preprocess_bgr_u8(const uint8_t* src, int n, int src_h, int src_w, int resize_h, int resize_w, int crop_h,
                            int crop_w, const float* mean, const float* stdv, float* dst, cudaStream_t stream);

/* Last error of the calling thread, "" if none. */
const char* lotus_last_error_string(void);

/* Returns and clears the device-side error word (a bounded wait inside a
 * kernel expired); 0 means none.  Synchronises the current device. */
int lotus_device_error(void);

/* Number of kernels launched by this library in this process (all devices). */
uint64_t lotus_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* LOTUS_OPS_H_ */
