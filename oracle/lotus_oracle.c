/*
 * CPU oracle for the lotusInfer dense-contraction hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this file; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline legs do, and only as the checker.
 *
 * Pinned against the reference itself: the reference's own operator kernels,
 * compiled from its sources by oracle/ref/Makefile and run on a GPU by
 * tests/golden/make_golden.py, produced tests/golden/ref_ops.npz;
 * tests/test_golden_cpu.py requires these functions to reproduce those
 * outputs (bit for bit on integer-valued and fp16-exact inputs).  Also
 * checked against hand-computed answers, the reference GEMM test's
 * deterministic inputs and torch CPU.
 *
 * Plain C restatements (fp32 NCHW, OpenMP over the outermost independent
 * loop) of the host-side reference loops the reference's per-operator tests
 * compare against, with PyTorch semantics where the reference kernels are
 * known to be wrong (noted per function).  Every function cites the file and
 * lines of the reference it follows.
 */
#include <float.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* Activation: reference include/lotus_utils.hpp:44-48 (enum NONE/RELU/SIGMOID)
 * applied after the bias as in source/operator/conv2d.cu:174-182. */
static inline float oracle_act(float v, int act) {
  if (act == 1) return v > 0.f ? v : 0.f;
  if (act == 2) return 1.f / (1.f + expf(-v));
  return v;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/*
 * conv2d: y[n,co,oh,ow] = act(b[co] + sum_{ci,r,s} w[co,ci,r,s] * xpad[n,ci,oh*sh+r,ow*sw+s]
 *                              [+ residual[n,co,oh,ow]])
 * Follows test/test_conv2d.cu:8-48 (zero-padded input, window x kernel sum
 * plus bias) with the activation epilogue of source/operator/conv2d.cu:168-185.
 * The optional residual is the ResNet `pnnx.Expression add` + ReLU pair
 * (source/operator/add.cu:14-26 on the conv output) folded into one call:
 * y = act(conv + b + residual).
 */
void oracle_conv2d(const float* x, const float* w, const float* b, const float* residual, float* y, int n, int c,
                   int h, int wd, int cout, int kh, int kw, int sh, int sw, int ph, int pw, int act) {
  const int oh = (h + 2 * ph - kh) / sh + 1;
  const int ow = (wd + 2 * pw - kw) / sw + 1;
  const long plane = (long)oh * ow;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int in = 0; in < n; ++in) {
    for (int co = 0; co < cout; ++co) {
      float* out = y + ((long)in * cout + co) * plane;
      const float bias = b ? b[co] : 0.f;
      for (long i = 0; i < plane; ++i) out[i] = bias;
      for (int ci = 0; ci < c; ++ci) {
        const float* xp = x + ((long)in * c + ci) * h * wd;
        for (int r = 0; r < kh; ++r) {
          for (int s = 0; s < kw; ++s) {
            const float wv = w[(((long)co * c + ci) * kh + r) * kw + s];
            /* output columns whose input column lies inside the image */
            int ow_lo = 0;
            while (ow_lo < ow && ow_lo * sw - pw + s < 0) ++ow_lo;
            int ow_hi = ow;
            while (ow_hi > ow_lo && (ow_hi - 1) * sw - pw + s >= wd) --ow_hi;
            for (int yy = 0; yy < oh; ++yy) {
              const int ih = yy * sh - ph + r;
              if (ih < 0 || ih >= h) continue;
              const float* xr = xp + (long)ih * wd + (s - pw);
              float* orow = out + (long)yy * ow;
              if (sw == 1) {
                for (int xx = ow_lo; xx < ow_hi; ++xx) orow[xx] += wv * xr[xx];
              } else {
                for (int xx = ow_lo; xx < ow_hi; ++xx) orow[xx] += wv * xr[(long)xx * sw];
              }
            }
          }
        }
      }
      const float* res = residual ? residual + ((long)in * cout + co) * plane : NULL;
      for (long i = 0; i < plane; ++i) out[i] = oracle_act(out[i] + (res ? res[i] : 0.f), act);
    }
  }
}

/*
 * Transposed conv2d, PyTorch ConvTranspose2d semantics (dilation 1):
 * full[n,co,iy*sh+ky,ix*sw+kx] += x[n,ci,iy,ix] * w[ci,co,ky,kx], accumulated
 * in double, then cropped by `ph/pw` on each side, output size
 * (H-1)*sh - 2*ph + kh + oph, then + bias and act.
 * Follows the scatter-add check of test/test_transposed_conv2d.cu:20-50
 * (double accumulator, crop by padding); output_padding follows PyTorch
 * (the reference layer passes output_padding as the crop,
 * source/layer/layer_transposed_conv2d.cu:123-124).
 */
void oracle_tconv2d(const float* x, const float* w, const float* b, float* y, int n, int cin, int h, int wd, int cout,
                    int kh, int kw, int sh, int sw, int ph, int pw, int oph, int opw, int act) {
  const int oh = (h - 1) * sh - 2 * ph + kh + oph;
  const int ow = (wd - 1) * sw - 2 * pw + kw + opw;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int in = 0; in < n; ++in) {
    for (int co = 0; co < cout; ++co) {
      double* acc = (double*)calloc((size_t)oh * ow, sizeof(double));
      for (int ci = 0; ci < cin; ++ci) {
        const float* xp = x + ((long)in * cin + ci) * h * wd;
        for (int ky = 0; ky < kh; ++ky) {
          for (int kx = 0; kx < kw; ++kx) {
            const double wv = w[(((long)ci * cout + co) * kh + ky) * kw + kx];
            for (int iy = 0; iy < h; ++iy) {
              const int oy = iy * sh + ky - ph;
              if (oy < 0 || oy >= oh) continue;
              for (int ix = 0; ix < wd; ++ix) {
                const int ox = ix * sw + kx - pw;
                if (ox < 0 || ox >= ow) continue;
                acc[(long)oy * ow + ox] += wv * xp[(long)iy * wd + ix];
              }
            }
          }
        }
      }
      float* out = y + ((long)in * cout + co) * oh * ow;
      const double bias = b ? b[co] : 0.0;
      for (long i = 0; i < (long)oh * ow; ++i) out[i] = oracle_act((float)(acc[i] + bias), act);
      free(acc);
    }
  }
}

/*
 * GEMV: y[b,hh] = act(sum_k W[hh,k] * x[b,k] + bias[hh]) for `batch` rows of x.
 * Follows test/test_fused_gemv_add_bias.cu:12-31 (row dot product + bias).
 */
void oracle_gemv(const float* wmat, const float* x, const float* bias, float* y, int batch, int hout, int win,
                 int act) {
#pragma omp parallel for schedule(static)
  for (int hh = 0; hh < hout; ++hh) {
    const float* wr = wmat + (long)hh * win;
    for (int bb = 0; bb < batch; ++bb) {
      const float* xr = x + (long)bb * win;
      float acc = 0.f;
      for (int k = 0; k < win; ++k) acc += wr[k] * xr[k];
      y[(long)bb * hout + hh] = oracle_act(acc + (bias ? bias[hh] : 0.f), act);
    }
  }
}

/*
 * GEMM: C[m,nn] = act(sum_k A[m,k] * B[nn,k] + bias[nn]), B the Linear weight
 * [out, in].  Follows test/test_gemm.cu:50 (input * weight^T + bias) with
 * M = batch rows (one call per layer, not per sample).
 */
void oracle_gemm(const float* a, const float* bmat, const float* bias, float* c, int m, int nn, int k, int act) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < m; ++i) {
    const float* ar = a + (long)i * k;
    for (int j = 0; j < nn; ++j) {
      const float* br = bmat + (long)j * k;
      float acc = 0.f;
      for (int t = 0; t < k; ++t) acc += ar[t] * br[t];
      c[(long)i * nn + j] = oracle_act(acc + (bias ? bias[j] : 0.f), act);
    }
  }
}

/*
 * Max pooling with -inf padding (PyTorch).  The reference test pads with
 * zeros and takes the window amax (test/test_maxpool2d.cu:8-34), which equals
 * this only for non-negative inputs; its kernel leaves the max uninitialised
 * when tap (0,0) is padding (source/operator/maxpool2d.cu:38,48-52).
 * `zero_pad` = 1 reproduces the test's zero-padded amax.
 */
void oracle_maxpool2d(const float* x, float* y, int n, int c, int h, int wd, int kh, int kw, int sh, int sw, int ph,
                      int pw, int act, int zero_pad) {
  const int oh = (h + 2 * ph - kh) / sh + 1;
  const int ow = (wd + 2 * pw - kw) / sw + 1;
#pragma omp parallel for collapse(2) schedule(static)
  for (int in = 0; in < n; ++in) {
    for (int ch = 0; ch < c; ++ch) {
      const float* xp = x + ((long)in * c + ch) * h * wd;
      float* out = y + ((long)in * c + ch) * oh * ow;
      for (int yy = 0; yy < oh; ++yy) {
        for (int xx = 0; xx < ow; ++xx) {
          float m = -INFINITY;
          for (int r = 0; r < kh; ++r) {
            const int iy = yy * sh - ph + r;
            for (int s = 0; s < kw; ++s) {
              const int ix = xx * sw - pw + s;
              float v;
              if (iy < 0 || iy >= h || ix < 0 || ix >= wd) {
                if (!zero_pad) continue;
                v = 0.f;
              } else {
                v = xp[(long)iy * wd + ix];
              }
              if (v > m) m = v;
            }
          }
          out[(long)yy * ow + xx] = oracle_act(m, act);
        }
      }
    }
  }
}

/*
 * Adaptive average pooling with PyTorch windows
 * [floor(i*H/OH), ceil((i+1)*H/OH)).  For ResNet's 7x7 -> 1x1 this equals the
 * reference layer (kernel = ceil(H/OH), source/layer/layer_adaptive_avgpool2d.cu:42-46).
 */
void oracle_adaptive_avgpool2d(const float* x, float* y, int n, int c, int h, int wd, int oh, int ow, int act) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int in = 0; in < n; ++in) {
    for (int ch = 0; ch < c; ++ch) {
      const float* xp = x + ((long)in * c + ch) * h * wd;
      float* out = y + ((long)in * c + ch) * oh * ow;
      for (int i = 0; i < oh; ++i) {
        const int hs = (i * h) / oh, he = ((i + 1) * h + oh - 1) / oh;
        for (int j = 0; j < ow; ++j) {
          const int ws = (j * wd) / ow, we = ((j + 1) * wd + ow - 1) / ow;
          float acc = 0.f;
          for (int iy = hs; iy < he; ++iy)
            for (int ix = ws; ix < we; ++ix) acc += xp[(long)iy * wd + ix];
          out[(long)i * ow + j] = oracle_act(acc / (float)((he - hs) * (we - ws)), act);
        }
      }
    }
  }
}

/*
 * The reference's own fixed-window average pooling as its test checks it
 * (test/test_adaptive_avgpool2d.cu:8-29 with the parameters of :36-50):
 * window k = ceil(H/OH), start = round(i * stride), stride = (float)(int)((H-k)/OH).
 * Used only to document where the reference departs from PyTorch.
 */
void oracle_avgpool_reference_windows(const float* x, float* y, int c, int h, int wd, int oh, int ow) {
  const int kh = (h + oh - 1) / oh, kw = (wd + ow - 1) / ow;
  const float sh = (float)((h - kh) / oh), sw = (float)((wd - kw) / ow);
  for (int ch = 0; ch < c; ++ch) {
    for (int i = 0; i < oh; ++i) {
      for (int j = 0; j < ow; ++j) {
        const int y0 = (int)roundf(i * sh), x0 = (int)roundf(j * sw);
        float acc = 0.f;
        for (int r = 0; r < kh; ++r)
          for (int s = 0; s < kw; ++s) acc += x[((long)ch * h + y0 + r) * wd + x0 + s];
        y[((long)ch * oh + i) * ow + j] = acc / (float)(kh * kw);
      }
    }
  }
}

/* y = act(x1 + x2); test/test_add.cu:7-21 with the act of source/operator/add.cu:14-26. */
void oracle_add(const float* x1, const float* x2, float* y, long count, int act) {
#pragma omp parallel for schedule(static)
  for (long i = 0; i < count; ++i) y[i] = oracle_act(x1[i] + x2[i], act);
}

/* torch.cat(dim=1) of two NCHW tensors (source/layer/concatenate.cpp:20-35). */
void oracle_concat(const float* a, int ca, const float* b, int cb, float* y, int n, long hw) {
  for (int in = 0; in < n; ++in) {
    memcpy(y + (long)in * (ca + cb) * hw, a + (long)in * ca * hw, sizeof(float) * ca * hw);
    memcpy(y + ((long)in * (ca + cb) + ca) * hw, b + (long)in * cb * hw, sizeof(float) * cb * hw);
  }
}
