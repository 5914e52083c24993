// Implicit-GEMM convolution on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// GEMM view (NHWC activations):
//   M = N*OH*OW output pixels, N_gemm = Cout, K = kh*kw*Cs_in ordered (r, s, c).
//   A[m, k] = x[n, oh*sh - ph + r, ow*sw - pw + s, c]   (zero outside the image)
//   B[co, k] = prepacked weight row co (K-major fp16, K padded to 64).
//   D[m, co] accumulates in TMEM (fp32), M tile = 128 lanes, N tile = BLOCK_N columns.
//
// One CTA computes one 128 x BLOCK_N output tile with 6 warps:
//   warps 0-3  A producers: gather the im2col rows with 16-byte cp.async
//              (zero-fill for padding) into the 128B-swizzled K-major layout,
//              then become the epilogue (TMEM -> registers -> bias, residual,
//              activation -> fp16/fp32 global stores);
//   warp 4     B producer: one elected thread issues TMA tiled loads of the
//              weight tile;
//   warp 5     allocates TMEM; one elected thread issues tcgen05.mma
//              (M=128, N=BLOCK_N, K=16) and commits stage releases.
// Stages are guarded by full/empty mbarriers; all waits are bounded.
//
// The same kernel runs the Linear GEMM (a 1x1 "image") and the stride==kernel
// transposed convolution (a 1x1 conv over Cin with N_gemm = kh*kw*Cout, whose
// epilogue scatters each column to its (ky, kx) output pixel).
//
// Reference counterparts: source/operator/conv2d.cu:17-187 (fp32 SIMT conv,
// the kernel the reference actually links), source/operator/conv2d_tensorcore.cu:18-152
// (WMMA conv), source/operator/gemm_tensorcore.cu:18-169 (Linear GEMM),
// source/operator/transposed_conv2d.cu:17-140; epilogue order bias -> act as
// in conv2d.cu:168-185, residual added before the activation as the
// Expression add + ReLU pair of models/resnet/resnet18.pnnx.param does.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "ptx.cuh"
#include "kernels.h"

namespace lotus_impl {

using namespace lotus_dev;

constexpr int kBlockM = 128;
constexpr int kBlockK = 64;                     // fp16 elements = one 128-byte swizzle row
constexpr int kABytes = kBlockM * kBlockK * 2;  // 16 KB per stage
constexpr int kThreads = 192;
constexpr int kLag = 2;                         // cp.async groups a producer keeps in flight

struct ConvTcParams {
  const __half* x;
  const float* bias;
  const __half* residual;
  void* y;
  int H, W, Cs_in;
  int OH, OW;
  int kh, kw, sh, sw, ph, pw;
  int Cout;      // columns with real outputs (N_gemm)
  int Cs_out;    // pixel stride of the NHWC fp16 output
  int M;
  int KB;        // number of 64-wide K blocks
  int act;
  int out_kind;  // 0 NHWC fp16, 1 fp32 rows, 2 transposed-conv scatter (NHWC fp16)
  // transposed-conv scatter geometry
  int t_oh, t_ow, t_sh, t_sw, t_ph, t_pw, t_kw, t_cout;
};

template <int BN, int STAGES>
struct SmemLayout {
  static constexpr int kBBytes = BN * kBlockK * 2;
  static constexpr int kAOff = 0;
  static constexpr int kBOff = STAGES * kABytes;
  static constexpr int kBarOff = kBOff + STAGES * kBBytes;
  static constexpr int kMiscOff = kBarOff + (2 * STAGES + 1) * 8;
  static constexpr int kTableOff = (kMiscOff + 16 + 15) & ~15;
  // +1024 for manual alignment of the dynamic smem base
  static constexpr int bytes(int table_entries) { return kTableOff + table_entries * 4 + 1024; }
};

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int BN, int STAGES, bool FAST>
__global__ void __launch_bounds__(kThreads, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const ConvTcParams p) {
  using L = SmemLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + L::kAOff;
  uint8_t* sB = smem + L::kBOff;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);
  uint32_t* ktable = reinterpret_cast<uint32_t*>(smem + L::kTableOff);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int m0 = blockIdx.x * kBlockM;
  const int n0 = blockIdx.y * BN;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 128 + 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) tma_prefetch_desc(&tmap_w);
  if (!FAST) {
    // K-chunk table: one entry per 8-channel chunk, (r, s, c) or invalid.
    const int nchunks = p.KB * 8;
    const int taps = p.kh * p.kw;
    for (int kc = tid; kc < nchunks; kc += kThreads) {
      const int k = kc * 8;
      const int tap = k / p.Cs_in;
      uint32_t e = 0xFFFFFFFFu;
      if (tap < taps) {
        const int c = k - tap * p.Cs_in;
        const int r = tap / p.kw;
        const int s = tap - r * p.kw;
        e = (uint32_t(r) << 24) | (uint32_t(s) << 16) | uint32_t(c);
      }
      ktable[kc] = e;
    }
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 4) {
    // ------------------------------------------------------------ A producer
    const int row = tid;  // 0..127
    const int m = m0 + row;
    const bool mvalid = m < p.M;
    const int ohw = p.OH * p.OW;
    int n_img = 0, oh = 0, ow = 0;
    if (mvalid) {
      n_img = m / ohw;
      const int rem = m - n_img * ohw;
      oh = rem / p.OW;
      ow = rem - oh * p.OW;
    }
    const int ih0 = oh * p.sh - p.ph;
    const int iw0 = ow * p.sw - p.pw;
    const __half* xb = p.x + static_cast<int64_t>(n_img) * p.H * p.W * p.Cs_in;
    const uint32_t swz = row & 7;
    const uint32_t a_row = smem_u32(sA) + row * 128;
    int r = 0, s = 0, c0 = 0;
    bool ok_run = true;
    for (int kb = 0; kb < p.KB; ++kb) {
      const int st = kb % STAGES;
      const uint32_t it = kb / STAGES;
      if (kb >= STAGES) {
        if (*abort_flag || !mbar_wait(&empty[st], (it - 1) & 1, kErrWaitEmpty)) {
          *abort_flag = 1;
          ok_run = false;
          break;
        }
      }
      const uint32_t dst = a_row + st * kABytes;
      if (FAST) {
        const int ih = ih0 + r, iw = iw0 + s;
        const bool ok = mvalid && (unsigned)ih < (unsigned)p.H && (unsigned)iw < (unsigned)p.W;
        const __half* src = ok ? xb + (static_cast<int64_t>(ih) * p.W + iw) * p.Cs_in + c0 : p.x;
        const uint32_t nb = ok ? 16u : 0u;
#pragma unroll
        for (int j = 0; j < 8; ++j) cp_async_16(dst + ((j ^ swz) << 4), ok ? src + j * 8 : src, nb);
        c0 += kBlockK;
        if (c0 == p.Cs_in) {
          c0 = 0;
          if (++s == p.kw) {
            s = 0;
            ++r;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t e = ktable[kb * 8 + j];
          const int rr = int(e >> 24), ss = int((e >> 16) & 0xFF), cc = int(e & 0xFFFF);
          const int ih = ih0 + rr, iw = iw0 + ss;
          const bool ok = (e != 0xFFFFFFFFu) && mvalid && (unsigned)ih < (unsigned)p.H &&
                          (unsigned)iw < (unsigned)p.W;
          const __half* src = ok ? xb + (static_cast<int64_t>(ih) * p.W + iw) * p.Cs_in + cc : p.x;
          cp_async_16(dst + ((j ^ swz) << 4), src, ok ? 16u : 0u);
        }
      }
      cp_async_commit();
      if (kb >= kLag) {
        cp_async_wait<kLag>();
        fence_proxy_async_smem();
        mbar_arrive(&full[(kb - kLag) % STAGES]);
      }
    }
    cp_async_wait_all();
    fence_proxy_async_smem();
    if (ok_run) {
      const int first = p.KB > kLag ? p.KB - kLag : 0;
      for (int kb = first; kb < p.KB; ++kb) mbar_arrive(&full[kb % STAGES]);
    }

    // ------------------------------------------------------------ epilogue
    __syncwarp();
    bool acc_ok = false;
    if (!*abort_flag) acc_ok = mbar_wait(accf, 0, kErrWaitAccum);
    if (!acc_ok) *abort_flag = 1;
    tc_fence_after();
    const int erow = warp * 32 + lane;
    const int em = m0 + erow;
    const bool evalid = acc_ok && em < p.M;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);

    // scatter geometry for out_kind 2
    int sc_n = 0, sc_iy = 0, sc_ix = 0;
    if (p.out_kind == 2 && evalid) {
      const int hw = p.OH * p.OW;  // the GEMM "output" grid is the tconv input grid
      sc_n = em / hw;
      const int rem = em - sc_n * hw;
      sc_iy = rem / p.OW;
      sc_ix = rem - sc_iy * p.OW;
    }

#pragma unroll 1
    for (int cc = 0; cc < BN / 32; ++cc) {
      uint32_t v[32];
      __syncwarp();
      tmem_ld_32x32b_x32(t_lane + cc * 32, v);  // warp-collective: every lane executes it
      tmem_ld_wait();
      if (!evalid) continue;
      const int colbase = n0 + cc * 32;
      if (p.out_kind == 0) {
        __half* yrow = reinterpret_cast<__half*>(p.y) + static_cast<int64_t>(em) * p.Cs_out;
        const __half* rrow = p.residual ? p.residual + static_cast<int64_t>(em) * p.Cs_out : nullptr;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int cg = colbase + g * 8;
          if (cg >= p.Cs_out) break;
          float f[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(v[g * 8 + j]);
          if (rrow) {
            const uint4 rv = *reinterpret_cast<const uint4*>(rrow + cg);
            const __half2* rh = reinterpret_cast<const __half2*>(&rv);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 rf = __half22float2(rh[j]);
              f[2 * j] += rf.x;
              f[2 * j + 1] += rf.y;
            }
          }
          uint32_t packed[4];
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            const int c_a = cg + j, c_b = cg + j + 1;
            float a = 0.f, b = 0.f;
            if (c_a < p.Cout) a = apply_act(f[j] + (p.bias ? __ldg(p.bias + c_a) : 0.f), p.act);
            if (c_b < p.Cout) b = apply_act(f[j + 1] + (p.bias ? __ldg(p.bias + c_b) : 0.f), p.act);
            packed[j / 2] = pack_half2(a, b);
          }
          *reinterpret_cast<uint4*>(yrow + cg) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        }
      } else if (p.out_kind == 1) {
        float* yrow = reinterpret_cast<float*>(p.y) + static_cast<int64_t>(em) * p.Cout;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int col = colbase + j;
          if (col < p.Cout)
            yrow[col] = apply_act(__uint_as_float(v[j]) + (p.bias ? __ldg(p.bias + col) : 0.f), p.act);
        }
      } else {
        // transposed conv: column -> (tap, co) -> output pixel
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int cg = colbase + g * 8;
          if (cg >= p.Cout) break;
          const int tap = cg / p.t_cout;
          const int co = cg - tap * p.t_cout;
          const int ky = tap / p.t_kw, kx = tap - ky * p.t_kw;
          const int oy = sc_iy * p.t_sh + ky - p.t_ph;
          const int ox = sc_ix * p.t_sw + kx - p.t_pw;
          if ((unsigned)oy >= (unsigned)p.t_oh || (unsigned)ox >= (unsigned)p.t_ow) continue;
          __half* ypix = reinterpret_cast<__half*>(p.y) +
                         ((static_cast<int64_t>(sc_n) * p.t_oh + oy) * p.t_ow + ox) * p.Cs_out;
          if ((p.t_cout & 7) == 0) {
            uint32_t packed[4];
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              const float a = apply_act(__uint_as_float(v[g * 8 + j]) + (p.bias ? __ldg(p.bias + co + j) : 0.f), p.act);
              const float b =
                  apply_act(__uint_as_float(v[g * 8 + j + 1]) + (p.bias ? __ldg(p.bias + co + j + 1) : 0.f), p.act);
              packed[j / 2] = pack_half2(a, b);
            }
            *reinterpret_cast<uint4*>(ypix + co) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          } else {
            for (int j = 0; j < 8; ++j) {
              const int col = cg + j;
              if (col >= p.Cout) break;
              const int tp = col / p.t_cout;
              const int c2 = col - tp * p.t_cout;
              const int ky2 = tp / p.t_kw, kx2 = tp - ky2 * p.t_kw;
              const int oy2 = sc_iy * p.t_sh + ky2 - p.t_ph;
              const int ox2 = sc_ix * p.t_sw + kx2 - p.t_pw;
              if ((unsigned)oy2 >= (unsigned)p.t_oh || (unsigned)ox2 >= (unsigned)p.t_ow) continue;
              __half* yp = reinterpret_cast<__half*>(p.y) +
                           ((static_cast<int64_t>(sc_n) * p.t_oh + oy2) * p.t_ow + ox2) * p.Cs_out;
              yp[c2] = __float2half_rn(
                  apply_act(__uint_as_float(v[g * 8 + j]) + (p.bias ? __ldg(p.bias + c2) : 0.f), p.act));
            }
          }
        }
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ B producer (TMA)
    if (lane == 0) {
      for (int kb = 0; kb < p.KB; ++kb) {
        const int st = kb % STAGES;
        const uint32_t it = kb / STAGES;
        if (kb >= STAGES) {
          if (*abort_flag || !mbar_wait(&empty[st], (it - 1) & 1, kErrWaitEmpty)) {
            *abort_flag = 1;
            break;
          }
        }
        mbar_arrive_expect_tx(&full[st], L::kBBytes);
        tma_load_2d(sB + st * L::kBBytes, &tmap_w, &full[st], kb * kBlockK, n0);
      }
    }
  } else {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16_m128(BN);
      bool ok_run = true;
      for (int kb = 0; kb < p.KB; ++kb) {
        const int st = kb % STAGES;
        const uint32_t it = kb / STAGES;
        if (*abort_flag || !mbar_wait(&full[st], it & 1, kErrWaitFull)) {
          *abort_flag = 1;
          ok_run = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_base = smem_u32(sA + st * kABytes);
        const uint32_t b_base = smem_u32(sB + st * L::kBBytes);
#pragma unroll
        for (int k = 0; k < kBlockK / 16; ++k) {
          umma_f16(tmem_base, make_sdesc_sw128(a_base + k * 32), make_sdesc_sw128(b_base + k * 32), idesc,
                   (kb | k) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[st]);
      }
      // Signal the epilogue even on abort so that it does not wait out its
      // own limit; it checks the abort flag before reading TMEM.
      umma_commit(accf);
      (void)ok_run;
    }
  }

  // All MMAs have completed once the epilogue has passed accf (or the CTA
  // aborted); TMEM can be released after everyone is done with it.
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, BN);
  }
}

// ---------------------------------------------------------------- host side

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2-D map over the packed weight [rows, k_pad] fp16, box {64, bn}, 128B swizzle.
static int make_weight_tmap(CUtensorMap* map, const void* w, int rows, int k_pad, int bn) {
  auto enc = get_encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k_pad), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(k_pad) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBlockK), static_cast<cuuint32_t>(bn)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(w), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

template <int BN, int STAGES, bool FAST>
static cudaError_t launch_impl(const CUtensorMap& map, const ConvTcParams& p, int n_rows, cudaStream_t stream) {
  using L = SmemLayout<BN, STAGES>;
  const int table = FAST ? 0 : p.KB * 8;
  const int smem = L::bytes(table);
  auto kern = conv_tc_kernel<BN, STAGES, FAST>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  dim3 grid((p.M + kBlockM - 1) / kBlockM, (n_rows + BN - 1) / BN);
  kern<<<grid, kThreads, smem, stream>>>(map, p);
  note_launch();
  return cudaGetLastError();
}

int conv_tc_launch(const ConvTcArgs& a, cudaStream_t stream, const char** err) {
  ConvTcParams p{};
  p.x = static_cast<const __half*>(a.x);
  p.bias = a.bias;
  p.residual = static_cast<const __half*>(a.residual);
  p.y = a.y;
  p.H = a.H;
  p.W = a.W;
  p.Cs_in = a.Cs_in;
  p.OH = a.OH;
  p.OW = a.OW;
  p.kh = a.kh;
  p.kw = a.kw;
  p.sh = a.sh;
  p.sw = a.sw;
  p.ph = a.ph;
  p.pw = a.pw;
  p.Cout = a.n_cols;
  p.Cs_out = a.Cs_out;
  p.M = a.M;
  p.KB = a.k_pad / kBlockK;
  p.act = a.act;
  p.out_kind = a.out_kind;
  p.t_oh = a.t_oh;
  p.t_ow = a.t_ow;
  p.t_sh = a.t_sh;
  p.t_sw = a.t_sw;
  p.t_ph = a.t_ph;
  p.t_pw = a.t_pw;
  p.t_kw = a.t_kw;
  p.t_cout = a.t_cout;

  const bool fast = (a.Cs_in % kBlockK) == 0;
  if (!fast && p.KB * 8 > 8192) {
    *err = "conv: K too large for the general gather path";
    return -2;
  }
  int bn = a.block_n;
  if (bn == 0) bn = a.n_cols <= 64 ? 64 : (a.n_cols <= 128 ? 128 : 128);
  CUtensorMap map;
  if (make_weight_tmap(&map, a.w_packed, a.n_cols, a.k_pad, bn) != 0) {
    *err = "conv: cuTensorMapEncodeTiled failed (driver entry point or arguments)";
    return -3;
  }
  cudaError_t e;
  if (bn == 64) {
    e = fast ? launch_impl<64, 4, true>(map, p, a.n_cols, stream) : launch_impl<64, 4, false>(map, p, a.n_cols, stream);
  } else if (bn == 128) {
    e = fast ? launch_impl<128, 3, true>(map, p, a.n_cols, stream)
             : launch_impl<128, 3, false>(map, p, a.n_cols, stream);
  } else if (bn == 256) {
    e = fast ? launch_impl<256, 4, true>(map, p, a.n_cols, stream)
             : launch_impl<256, 4, false>(map, p, a.n_cols, stream);
  } else {
    *err = "conv: unsupported block_n";
    return -2;
  }
  if (e != cudaSuccess) {
    *err = cudaGetErrorString(e);
    return -3;
  }
  return 0;
}

int read_device_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, lotus_dev::g_lotus_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) {
    int zero = 0;
    cudaMemcpyToSymbol(lotus_dev::g_lotus_device_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace lotus_impl
