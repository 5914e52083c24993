// Implicit-GEMM convolution on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// GEMM view (NHWC activations):
//   M = N*OH*OW output pixels, N_gemm = Cout, K = kh*kw*Cs_in ordered (r, s, c).
//   A[m, k] = x[n, oh*sh - ph + r, ow*sw - pw + s, c]   (zero outside the image)
//   B[co, k] = prepacked weight row co (K-major fp16, K padded to 64).
//   D[m, co] accumulates in TMEM (fp32): 128 lanes x BLOCK_N columns per tile.
//
// Persistent, warp-specialised kernel, one CTA per SM walking the output
// tiles (tile = m_tile * n_tiles + n_tile, so the N tiles of one pixel block
// run on neighbouring SMs and share the A rows through L2):
//   warps 0-7  epilogue (two warps per TMEM lane quarter, one per column
//              half): TMEM -> registers -> bias (staged in shared memory per
//              tile), residual, activation -> fp16 NHWC / fp32 rows /
//              transposed-conv scatter stores;
//   warp 8     allocates all 512 TMEM columns as a ring of 512/BLOCK_N
//              (at most 8) accumulators; one thread issues tcgen05.mma (M=128, N=BLOCK_N,
//              K=16) and commits stage / accumulator releases;
//   warps 10/11 (AMODE 1/2) a second MMA issuer and TMA producer pair with its
//              own half of the stages takes every other tile: one thread
//              issues at most one tcgen05.mma per ~80 cycles, so a single
//              issuer leaves the tensor pipe idle between MMAs;
//   warp 9     one thread issues the TMA loads: the weight tile always, and
//              the activation tile in im2col mode (AMODE 1: 3x3 / strided
//              convs with Cs_in % 64 == 0) or tiled mode (AMODE 2: 1x1 stride-1
//              convs and Linear, a plain [M, Cs_in] matrix);
//   warps 10-13 (AMODE 0 only) gather the im2col rows with 16-byte cp.async
//              for channel counts that are not a multiple of 64 (stem, U-Net
//              level 1), using a per-CTA table of (r, s, c) per 8-channel chunk.
//
// Resident-weight halo mode (AMODE 3): stride-1 convs with Cs_in of 16, 32 or
// 64 channels whose whole weight matrix fits in shared memory next to two or
// more activation buffers (the space-to-depth stem, ResNet stage 1, U-Net
// level 1-2).  The weights are loaded once per CTA.  The M axis of one image
// runs over positions q = oy * Wp + ox of the zero-padded input width
// Wp = W + 2*pw (columns ox >= OW are computed and dropped).  Output q under
// tap (r, s) reads padded input pixel q + r*Wp + s, so one tiled TMA box of R
// whole padded rows (Cs_in channels a row, swizzled at the row's width) holds
// the A operand of every tap of a 128-position tile: tap (r, s) is the same
// buffer with the descriptor start moved by (q0 % Wp + r*Wp + s) rows.  The
// swizzle is a function of the shared-memory address, so a start moved by
// whole rows reads what the TMA wrote.  The MMA thread waits once per tile
// instead of once per 64-wide K block.
//
// Streamed-weight halo mode (AMODE 4, selected with LOTUS_CONV_AMODE=4): the
// same padded-row halo for stride-1
// convs with Cs_in a multiple of 64 whose weights do not fit (ResNet stages
// 2-3): one 64-channel halo box per (tile, channel chunk) serves the kh*kw
// taps of that chunk, the weights stream per 64-wide K block in chunk-major
// order (all taps of chunk 0, then chunk 1, ...).  Two producer/MMA pipelines
// as in AMODE 1/2, each with its own weight stages and two halo buffers.
// Split-K (AMODE 0/1/2, when a launch has too few output tiles to fill the
// SMs and the caller passes a workspace): tile t = split * mn_tiles + mn,
// split s covers K blocks [s*kbs, (s+1)*kbs); the epilogue writes raw fp32
// partial tiles to the workspace and splitk_reduce_kernel sums them in split
// order and applies bias, residual and activation.
// The epilogue of tile i overlaps the main loop of the tiles after it.  Every wait is
// bounded; an expired wait records an error code and the CTA drains and exits.
//
// The same kernel runs the Linear GEMM (a 1x1 "image") and the stride==kernel
// transposed convolution (a 1x1 conv over Cin with N_gemm = kh*kw*Cout whose
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
#include <cstdlib>
#include <algorithm>
#include <atomic>
#include <mutex>

#include "kernels.h"
#include "ptx.cuh"

namespace lotus_impl {

using namespace lotus_dev;

constexpr int kBlockM = 128;
constexpr int kBlockK = 64;                     // fp16 elements = one 128-byte swizzle row
constexpr int kABytes = kBlockM * kBlockK * 2;  // 16 KB per stage
constexpr int kMaxTable = 2048;                 // gather-table entries (8-channel chunks): K <= 16384
constexpr int kBiasMax = 1024;                  // bias entries staged in shared memory
constexpr int kStageBytes = 32 * 64;            // per epilogue warp: 32 rows x 64 bytes of fp16 output

struct ConvTcParams {
  const __half* x;
  const float* bias;
  const __half* residual;
  void* y;
  int H, W, Cs_in;
  int OH, OW;
  int kh, kw, sh, sw, ph, pw;
  int Cout;      // GEMM N (columns with real outputs)
  int Cs_out;    // channels written per output pixel (roundup(Cout, 8)); the residual's pixel stride
  int y_stride;  // pixel stride of the NHWC fp16 output (>= Cs_out: a channel slice of a wider tensor)
  int M;
  int KB;        // number of 64-wide K blocks
  int act;
  int out_kind;  // 0 NHWC fp16, 1 fp32 rows, 2 transposed-conv scatter (NHWC fp16)
  int n_tiles;   // N tiles per M tile
  int tiles;     // total tiles
  int bias_smem; // 1: bias staged in shared memory (<= kBiasMax columns), 0: read from global
  // transposed-conv scatter geometry
  int t_oh, t_ow, t_sh, t_sw, t_ph, t_pw, t_kw, t_cout;
  // resident-weight halo mode geometry (AMODE 3)
  int Wp;           // padded input width W + 2*pw
  int tpi;          // 128-position tiles per image
  int halo_off;     // byte offset of the first halo buffer (after the weights)
  int halo_stride;  // bytes per halo buffer (multiple of 1024)
  int halo_slots;   // halo buffers in the ring (2..kHaloSlotsMax)
  int halo_bytes;   // bytes one halo box writes
  int a_rowbytes;   // Cs_in * 2: 32, 64 or 128
  int a_layout;     // tcgen05 descriptor swizzle code of that row width
  uint32_t wp_magic;  // ceil(2^32 / Wp) (Wp >= 2): q / Wp == __umulhi(q, wp_magic) for q * Wp < 2^32
  int cchunks;      // AMODE 4: 64-channel chunks per pixel (Cs_in / 64)
  // split-K
  int ksplit;       // K splits (1 = none)
  int kbs;          // K blocks per split
  int mn_tiles;     // output tiles (tiles = mn_tiles * ksplit)
  float* ws;        // [ksplit][ws_rows][ws_ld] fp32 partial sums
  int ws_rows;      // m_tiles * 128
  int ws_ld;        // n_tiles * BN
  // bounded waits: try_wait rounds before a wait gives up (kMaxWaitIters
  // unless LOTUS_WAIT_LIMIT says otherwise)
  uint32_t wait_limit;
  // test hook (LOTUS_TEST_WITHHOLD_ARRIVAL=1): CTA 0's producer skips its
  // first stage load, so the consumer's bounded wait must run out and the
  // kernel must report it and return; no fault and no unbounded wait
  int withhold_arrival;
};

// Output tile and K-block range of tile t (split-K: t = split * mn_tiles + mn).
struct TileK {
  int mn, split, kb0, nkb;
};
__device__ __forceinline__ TileK tile_k(const ConvTcParams& p, int t) {
  TileK r;
  r.split = t / p.mn_tiles;
  r.mn = t - r.split * p.mn_tiles;
  r.kb0 = r.split * p.kbs;
  r.nkb = p.KB - r.kb0 < p.kbs ? p.KB - r.kb0 : p.kbs;
  return r;
}

// Raw fp32 accumulator chunk (32 columns) into the split-K workspace.
__device__ __forceinline__ void store_partial(const ConvTcParams& p, const uint32_t (&v)[32], int split, int row,
                                              int col) {
  float4* dst = reinterpret_cast<float4*>(p.ws + (static_cast<size_t>(split) * p.ws_rows + row) * p.ws_ld + col);
#pragma unroll
  for (int j = 0; j < 8; ++j)
    dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]), __uint_as_float(v[4 * j + 2]),
                         __uint_as_float(v[4 * j + 3]));
}

constexpr int kHaloSlotsMax = 8;
// weights + halo ring (AMODE 3): what remains of the 227 KB of shared memory
// after the barriers, a 1 KB bias area and the 1 KB alignment slack
constexpr int kHaloRegion = 208 * 1024;
constexpr int kHaloBiasMax = 256;  // AMODE 3 has one N tile of at most 128 columns
// AMODE 4: weight stages + 2 x kHalo4Slots halo buffers, bias of up to 512 columns
constexpr int kHalo4Region = 204 * 1024;
constexpr int kHalo4BiasMax = 512;
constexpr int kHalo4Slots = 2;  // halo buffers per pipeline

template <int BN, int STAGES, int AMODE>
struct Cfg {
  // cp.async groups a gather thread keeps in flight before it signals a
  // stage (must stay below STAGES; two stages stay free for the tensor core)
  static constexpr int kLag = STAGES - 2;
  static constexpr int kEpiWarps = 8;                      // 2 per TMEM lane quarter
  // BN=64 outside the gather mode: the epilogue warps form two groups of
  // four that take alternate tiles (the gather mode's 448 threads leave 128
  // registers a thread, too few for a whole 64-column row set)
  static constexpr bool kEpiGroups = BN == 64 && AMODE != 0;
  // warps that drain each accumulator
  static constexpr int kEpiArrivals = kEpiGroups ? 4 : kEpiWarps;
  static constexpr int kMmaWarp = 8;
  static constexpr int kTmaWarp = 9;
  static constexpr int kGatherWarp0 = 10;                  // AMODE 0: warps 10-13
  // AMODE 3: three MMA-issuing warps (8, 10, 11) take tiles round robin;
  // one thread issues at most one tcgen05.mma per ~80 cycles whatever N is,
  // plus the integer work between two issues, so the short tap loops of
  // this mode need several issuers to keep the tensor pipe busy
  static constexpr int kMmaWarp2 = 10;
  // AMODE 1/2: two independent pipelines (producer warp 9 + MMA warp 8 and
  // producer warp 11 + MMA warp 10), each with half of the stages, take
  // alternate tiles and share the epilogue warps and the accumulator ring
  // (BN=256 tiles fill all of TMEM with two accumulators: one pipeline; an
  // N=256 MMA keeps the tensor pipe busier than one thread's issue cost)
  static constexpr int kRings = ((AMODE == 1 || AMODE == 2 || AMODE == 4) && BN <= 128) ? 2 : 1;
  static constexpr int kRingStages = STAGES / kRings;
  static constexpr int kTmaWarp2 = 11;
  static constexpr int kMmaIssuers = AMODE == 3 ? 3 : (kRings == 2 ? 2 : 1);
  static constexpr int kThreads = AMODE == 0 ? 448 : (AMODE == 3 ? 384 : (kRings == 2 ? 384 : 320));
  // issuer index of a warp (-1: not an issuer): warp 8 is issuer 0, warps
  // 10.. the others
  static __device__ __forceinline__ int issuer_of(int warp) {
    if (warp == kMmaWarp) return 0;
    if (kMmaIssuers > 1 && warp >= kMmaWarp2 && warp < kMmaWarp2 + kMmaIssuers - 1) return warp - kMmaWarp2 + 1;
    return -1;
  }
  static constexpr int kBBytes = BN * kBlockK * 2;
  static constexpr int kAOff = 0;
  // AMODE 3 keeps resident weights and the halo ring in one region at 0
  // AMODE 4 puts the weight stages at 0 and the halo buffers after them
  static constexpr int kBOff = AMODE == 3 ? kHaloRegion : (AMODE == 4 ? 0 : STAGES * kABytes);
  static constexpr int kBarOff =
      AMODE == 3 ? kHaloRegion : (AMODE == 4 ? kHalo4Region : kBOff + STAGES * kBBytes);
  // TMEM accumulator ring: all 512 columns (one CTA per SM), at most 8 tiles,
  // so the MMA runs several tiles ahead of the epilogue and the handoff
  // latency of one accumulator (commit -> TMEM load -> release) stays hidden
  static constexpr int kAccBufs = 512 / BN < 8 ? 512 / BN : 8;
  // full, empty, tfull[kAccBufs], tempty[kAccBufs], mma_done, hfull[kHaloSlotsMax], hempty[kHaloSlotsMax]
  static constexpr int kNumBars = 2 * STAGES + 2 * kAccBufs + 1 + 2 * kHaloSlotsMax;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kBiasOff = (kMiscOff + 16 + 15) & ~15;
  // per-warp output staging (NHWC fp16 stores), then the gather table
  static constexpr int kStageOff =
      kBiasOff + (AMODE == 3 ? kHaloBiasMax : (AMODE == 4 ? kHalo4BiasMax : kBiasMax)) * 4;
  static constexpr int kTableOff = kStageOff + kEpiWarps * kStageBytes;
  static constexpr int bytes(int table_entries) { return kTableOff + table_entries * 4 + 1024; }
  static constexpr uint32_t kTmemCols = kAccBufs * BN;
};

// K-major shared-memory descriptor for rows of `rowbytes` (32/64/128) bytes
// under the matching swizzle (`layout` 6/4/2); 8-row groups are 8*rowbytes
// apart.  LBO is unused: one MMA's K=16 slice lies inside one swizzle row.
__device__ __forceinline__ uint64_t make_sdesc_rows(uint32_t smem_addr, uint32_t rowbytes, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>((8u * rowbytes) >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(layout) << 61;
  return d;
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int ACT>
__device__ __forceinline__ float act_t(float v) {
  if (ACT == 1) return fmaxf(v, 0.0f);
  if (ACT == 2) return 1.0f / (1.0f + expf(-v));
  return v;
}

// Bias of column `c` of the tile (OUT 0/1) or of output channel `c` (OUT 2).
__device__ __forceinline__ float bias_of(const ConvTcParams& p, const float* sb, int n0, int c) {
  if (p.bias_smem) return sb[c];
  const int col = p.out_kind == 2 ? c : n0 + c;
  const int lim = p.out_kind == 2 ? p.t_cout : p.Cout;
  return (p.bias != nullptr && col < lim) ? __ldg(p.bias + col) : 0.f;
}

// NHWC fp16 epilogue of one 32-column chunk, warp-cooperative: every lane
// computes its row's 64 bytes (bias, residual, activation, pad channels zero),
// parks them in the warp's 32 x 64-byte staging buffer (16-byte chunks XOR-
// swizzled by row so that neither side has bank conflicts), and the warp then
// stores 8 rows x 64 contiguous bytes per instruction.  Storing 16 bytes per
// lane straight from the accumulator row would touch 32 partial sectors per
// instruction.  All 32 lanes must call it; `valid` = the lane's row is an
// output pixel (em is its row index).
template <int ACT>
__device__ __forceinline__ void epi_store_nhwc(const ConvTcParams& p, const uint32_t (&v)[32], int em, bool valid,
                                               int n0, int cl, const float* sb, bool full, const uint4* res,
                                               uint8_t* stg, int lane) {
  uint4* st = reinterpret_cast<uint4*>(stg);  // [32 rows][4 chunks]
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int c = cl + g * 8;  // column inside the tile
    float f[8];
    if (p.bias_smem) {
      const float4 b0 = *reinterpret_cast<const float4*>(sb + c);
      const float4 b1 = *reinterpret_cast<const float4*>(sb + c + 4);
      f[0] = b0.x; f[1] = b0.y; f[2] = b0.z; f[3] = b0.w;
      f[4] = b1.x; f[5] = b1.y; f[6] = b1.z; f[7] = b1.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = bias_of(p, sb, n0, c + j);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] += __uint_as_float(v[g * 8 + j]);
    if (res) {
      const __half2* rh = reinterpret_cast<const __half2*>(&res[g]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 rf = __half22float2(rh[j]);
        f[2 * j] += rf.x;
        f[2 * j + 1] += rf.y;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = act_t<ACT>(f[j]);
    if (!full) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (n0 + c + j >= p.Cout) f[j] = 0.f;  // pad channels stay zero
    }
    st[lane * 4 + ((g ^ (lane >> 1)) & 3)] = make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]),
                                                        pack_half2(f[4], f[5]), pack_half2(f[6], f[7]));
  }
  __syncwarp();
  const int row_em = valid ? em : -1;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 8 * i + (lane >> 2);  // staged row this lane stores
    const int c = lane & 3;             // and its 16-byte chunk
    const int em_r = __shfl_sync(0xffffffffu, row_em, r);
    const uint4 val = st[r * 4 + ((c ^ (r >> 1)) & 3)];
    const int col = n0 + cl + c * 8;
    if (em_r >= 0 && (full || col < p.Cs_out))
      *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(p.y) + static_cast<int64_t>(em_r) * p.y_stride + col) = val;
  }
  __syncwarp();  // the buffer is rewritten by the next chunk
}

template <int ACT_UNUSED = 0>
__device__ __forceinline__ void epi_store_nhwc_act(const ConvTcParams& p, const uint32_t (&v)[32], int em, bool valid,
                                                   int n0, int cl, const float* sb, bool full, const uint4* res,
                                                   uint8_t* stg, int lane) {
  if (p.act == 1)
    epi_store_nhwc<1>(p, v, em, valid, n0, cl, sb, full, res, stg, lane);
  else if (p.act == 0)
    epi_store_nhwc<0>(p, v, em, valid, n0, cl, sb, full, res, stg, lane);
  else
    epi_store_nhwc<2>(p, v, em, valid, n0, cl, sb, full, res, stg, lane);
}

// Epilogue of one 32-column chunk of one accumulator row.  `cl` is the
// chunk's first column inside the tile; `sb` points at the bias of the tile's
// first column (OUT 0/1, zero past Cout) or at bias[0] (OUT 2, indexed by the
// output channel); `full` says every column of the tile is < Cout.
template <int OUT, int ACT>
__device__ __forceinline__ void epi_chunk(const ConvTcParams& p, const uint32_t (&v)[32], int em, int n0, int cl,
                                          const float* sb, bool full, const uint4* res, int sc_n, int sc_iy,
                                          int sc_ix) {
  if (OUT == 0) {
    __half* yrow = reinterpret_cast<__half*>(p.y) + static_cast<int64_t>(em) * p.y_stride + n0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int c = cl + g * 8;  // column inside the tile
      if (!full && n0 + c >= p.Cs_out) break;
      float f[8];
      if (p.bias_smem) {
        const float4 b0 = *reinterpret_cast<const float4*>(sb + c);
        const float4 b1 = *reinterpret_cast<const float4*>(sb + c + 4);
        f[0] = b0.x; f[1] = b0.y; f[2] = b0.z; f[3] = b0.w;
        f[4] = b1.x; f[5] = b1.y; f[6] = b1.z; f[7] = b1.w;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = bias_of(p, sb, n0, c + j);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] += __uint_as_float(v[g * 8 + j]);
      if (res) {
        const __half2* rh = reinterpret_cast<const __half2*>(&res[g]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 rf = __half22float2(rh[j]);
          f[2 * j] += rf.x;
          f[2 * j + 1] += rf.y;
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = act_t<ACT>(f[j]);
      if (!full) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (n0 + c + j >= p.Cout) f[j] = 0.f;  // pad channels stay zero
      }
      *reinterpret_cast<uint4*>(yrow + c) = make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]),
                                                       pack_half2(f[4], f[5]), pack_half2(f[6], f[7]));
    }
  } else if (OUT == 1) {
    float* yrow = reinterpret_cast<float*>(p.y) + static_cast<int64_t>(em) * p.Cout + n0;
    if (full && (p.Cout & 3) == 0 && p.bias_smem) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 b = *reinterpret_cast<const float4*>(sb + cl + j);
        float4 o;
        o.x = act_t<ACT>(__uint_as_float(v[j]) + b.x);
        o.y = act_t<ACT>(__uint_as_float(v[j + 1]) + b.y);
        o.z = act_t<ACT>(__uint_as_float(v[j + 2]) + b.z);
        o.w = act_t<ACT>(__uint_as_float(v[j + 3]) + b.w);
        *reinterpret_cast<float4*>(yrow + cl + j) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + cl + j < p.Cout) yrow[cl + j] = act_t<ACT>(__uint_as_float(v[j]) + bias_of(p, sb, n0, cl + j));
    }
  } else {
    // transposed conv: GEMM column -> (tap, co) -> output pixel; sb holds bias[col % t_cout]
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int cg = n0 + cl + g * 8;
      if (cg >= p.Cout) break;
      if ((p.t_cout & 7) == 0) {
        const int tap = cg / p.t_cout;
        const int co = cg - tap * p.t_cout;
        const int ky = tap / p.t_kw, kx = tap - ky * p.t_kw;
        const int oy = sc_iy * p.t_sh + ky - p.t_ph;
        const int ox = sc_ix * p.t_sw + kx - p.t_pw;
        if ((unsigned)oy >= (unsigned)p.t_oh || (unsigned)ox >= (unsigned)p.t_ow) continue;
        __half* ypix = reinterpret_cast<__half*>(p.y) +
                       ((static_cast<int64_t>(sc_n) * p.t_oh + oy) * p.t_ow + ox) * p.y_stride;
        float f[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = act_t<ACT>(__uint_as_float(v[g * 8 + j]) + bias_of(p, sb, n0, co + j));
        *reinterpret_cast<uint4*>(ypix + co) = make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]),
                                                          pack_half2(f[4], f[5]), pack_half2(f[6], f[7]));
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
                       ((static_cast<int64_t>(sc_n) * p.t_oh + oy2) * p.t_ow + ox2) * p.y_stride;
          yp[c2] = __float2half_rn(act_t<ACT>(__uint_as_float(v[g * 8 + j]) + bias_of(p, sb, n0, c2)));
        }
      }
    }
  }
}

template <int OUT>
__device__ __forceinline__ void epi_chunk_act(const ConvTcParams& p, const uint32_t (&v)[32], int em, int n0, int cl,
                                              const float* sb, bool full, const uint4* res, int sc_n, int sc_iy,
                                              int sc_ix) {
  if (p.act == 1)
    epi_chunk<OUT, 1>(p, v, em, n0, cl, sb, full, res, sc_n, sc_iy, sc_ix);
  else if (p.act == 0)
    epi_chunk<OUT, 0>(p, v, em, n0, cl, sb, full, res, sc_n, sc_iy, sc_ix);
  else
    epi_chunk<OUT, 2>(p, v, em, n0, cl, sb, full, res, sc_n, sc_iy, sc_ix);
}

// q / Wp of a padded-grid position: with m = ceil(2^32 / d), floor(q * m /
// 2^32) == floor(q / d) whenever q * d < 2^32 (here q < 2^17, d <= 256).
__device__ __forceinline__ int div_wp(const ConvTcParams& p, int q) {
  return static_cast<int>(__umulhi(static_cast<uint32_t>(q), p.wp_magic));
}

template <int BN, int STAGES, int AMODE>
__global__ void __launch_bounds__(Cfg<BN, STAGES, AMODE>::kThreads, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
               const ConvTcParams p) {
  using C = Cfg<BN, STAGES, AMODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + C::kAOff;
  uint8_t* sB = smem + C::kBOff;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;        // [kAccBufs] accumulator ready for the epilogue
  uint64_t* tempty = tfull + C::kAccBufs;  // [kAccBufs] accumulator drained by the epilogue
  uint64_t* mma_done = tempty + C::kAccBufs;
  uint64_t* hfull = mma_done + 1;            // [kHaloSlotsMax] AMODE 3: halo buffer loaded
  uint64_t* hempty = hfull + kHaloSlotsMax;  // [kHaloSlotsMax] AMODE 3: halo buffer consumed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);
  float* s_bias = reinterpret_cast<float*>(smem + C::kBiasOff);
  uint8_t* s_stage = smem + C::kStageOff + (threadIdx.x >> 5) * kStageBytes;  // epilogue warps only
  uint32_t* ktable = reinterpret_cast<uint32_t*>(smem + C::kTableOff);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], AMODE == 0 ? 128 + 1 : 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < C::kAccBufs; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], C::kEpiArrivals);
    }
    mbar_init(mma_done, C::kMmaIssuers);
    for (int h = 0; h < kHaloSlotsMax; ++h) {
      mbar_init(&hfull[h], 1);
      mbar_init(&hempty[h], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == C::kTmaWarp && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    if (AMODE != 0) tma_prefetch_desc(&tmap_a);
  }
  if (AMODE == 0) {
    // K-chunk table: one entry per 8-channel chunk, (r, s, c) or invalid.
    const int nchunks = p.KB * 8;
    const int taps = p.kh * p.kw;
    for (int kc = tid; kc < nchunks; kc += C::kThreads) {
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
  // bias, once per CTA: columns [0, bias_len) (tconv: output channels), zero
  // past the real bias so float4 reads of a whole tile stay defined
  const int bias_len = p.out_kind == 2 ? p.t_cout : p.n_tiles * BN;
  for (int i = tid; p.bias_smem && i < bias_len; i += C::kThreads) {
    const int lim = p.out_kind == 2 ? p.t_cout : p.Cout;
    s_bias[i] = (p.bias != nullptr && i < lim) ? __ldg(p.bias + i) : 0.f;
  }
  if (warp == C::kMmaWarp) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int ohw = p.OH * p.OW;
  // set-up done: let the next kernel start being scheduled, then wait for
  // the kernels before this one (activations, residual, workspace)
  if (tid == 0) griddep_launch();
  griddep_wait();

  if (warp < C::kEpiWarps) {
    // ================================================================ epilogue
    // warp w reads TMEM lanes 32*(w%4).. (its hardware lane quarter) and the
    // columns of tile half w/4.
    constexpr int kHalf = BN / 2;
    constexpr int kResVecs = kHalf / 8;
    const int q = warp & 3;
    const int hcol = (warp >> 2) * kHalf;
    const int erow = q * 32 + lane;
    const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
    // split-K exists only in the staged modes: elsewhere its code compiles away
    constexpr bool kSplitable = AMODE <= 2;
    const bool has_res = p.residual != nullptr && p.out_kind == 0 && (!kSplitable || p.ksplit == 1);
    // output row of this thread in tile t (em) and whether it is a real pixel
    auto row_of = [&](int t, int& em, bool& rvalid) {
      if (AMODE != 3 && AMODE != 4) t = tile_k(p, t).mn;
      em = (t / p.n_tiles) * kBlockM + erow;
      rvalid = em < p.M;
      if (AMODE == 3 || AMODE == 4) {
        // position q of the padded-width grid -> output pixel
        const int mt = t / p.n_tiles;
        const int img = mt / p.tpi;
        const int q = (mt - img * p.tpi) * kBlockM + erow;
        const int oy = q / p.Wp;
        const int ox = q - oy * p.Wp;
        rvalid = oy < p.OH && ox < p.OW;
        em = (img * p.OH + oy) * p.OW + ox;
      }
    };
    // residual rows do not depend on the accumulator.  At BN=64 (epilogue-
    // bound layers) the rows of the next tile are loaded while this tile is
    // processed: a load issued only just before this tile's accumulator wait
    // exposes the full DRAM latency whenever the MMAs are ahead.  At BN=128
    // the second register set would spill, and the rows of the tile itself
    // are loaded ahead of its accumulator wait.
    constexpr bool kPipeRes = BN == 64;
    constexpr bool kChunked = BN > 128;
    auto load_res = [&](int t, uint4 (&r)[kResVecs]) {
      int em_t;
      bool ok_t;
      row_of(t, em_t, ok_t);
      const int n0_t = ((kSplitable ? tile_k(p, t).mn : t) % p.n_tiles) * BN;
      if (has_res && ok_t && t < p.tiles) {
        const uint4* rrow =
            reinterpret_cast<const uint4*>(p.residual + static_cast<int64_t>(em_t) * p.Cs_out + n0_t + hcol);
#pragma unroll
        for (int i = 0; i < kResVecs; ++i)
          r[i] = (n0_t + hcol + i * 8 < p.Cs_out) ? __ldg(rrow + i) : make_uint4(0, 0, 0, 0);
      }
    };
    if constexpr (C::kEpiGroups) {
    // BN=64: the two groups of four warps (0-3 and 4-7, one warp per TMEM
    // lane quarter in each) take alternate tiles, and a warp drains all 64
    // columns of its 32 rows.  A tile then costs one chain of accumulator
    // wait, loads, math and stores per warp instead of two half-width
    // chains, and the two groups' chains overlap.
    const int grp = warp >> 2;
    const int gx = static_cast<int>(gridDim.x);
    // halo mode (one N tile): image and tile-in-image of the group's tiles
    // t0, t0 + 2*gridDim.x, ... kept as counters, no division per tile
    int w_img = 0, w_ti = 0, g_img = 0, g_ti = 0;
    if (AMODE == 3) {
      const int t0 = static_cast<int>(blockIdx.x) + grp * gx;
      w_img = t0 / p.tpi;
      w_ti = t0 - w_img * p.tpi;
      g_img = (2 * gx) / p.tpi;
      g_ti = 2 * gx - g_img * p.tpi;
    }
    int lt = grp;
    for (int t = static_cast<int>(blockIdx.x) + grp * gx; t < p.tiles; t += 2 * gx, lt += 2) {
      const TileK tk = kSplitable ? tile_k(p, t) : TileK{t, 0, 0, p.KB};
      const int n0 = AMODE == 3 ? 0 : (tk.mn % p.n_tiles) * BN;
      const int ab = lt % C::kAccBufs;
      int em;
      bool rvalid;
      if (AMODE == 3) {
        const int q = w_ti * kBlockM + erow;
        const int oy = div_wp(p, q);
        const int ox = q - oy * p.Wp;
        rvalid = oy < p.OH && ox < p.OW;
        em = (w_img * p.OH + oy) * p.OW + ox;
        w_ti += g_ti;
        w_img += g_img;
        if (w_ti >= p.tpi) {
          w_ti -= p.tpi;
          ++w_img;
        }
      } else {
        row_of(t, em, rvalid);
      }
      const bool tile_full = n0 + BN <= p.Cout;
      // residual rows of both 32-column chunks, read ahead of the accumulator wait
      uint4 rc[2][4];
      if (has_res && rvalid) {
        const uint4* rrow = reinterpret_cast<const uint4*>(p.residual + static_cast<int64_t>(em) * p.Cs_out + n0);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          rc[i >> 2][i & 3] = (n0 + i * 8 < p.Cs_out) ? __ldg(rrow + i) : make_uint4(0, 0, 0, 0);
      }
      int sc_n = 0, sc_iy = 0, sc_ix = 0;
      if (p.out_kind == 2 && rvalid) {
        sc_n = em / ohw;
        const int rem = em - sc_n * ohw;
        sc_iy = rem / p.OW;
        sc_ix = rem - sc_iy * p.OW;
      }
      const bool ok = !*abort_flag && mbar_wait(&tfull[ab], (lt / C::kAccBufs) & 1, kErrWaitAccum, p.wait_limit);
      if (!ok) *abort_flag = 1;
      tc_fence_after();
      uint32_t v[2][32];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        __syncwarp();
        tmem_ld_32x32b_x32(tmem_base + t_lane + ab * BN + cc * 32, v[cc]);  // warp-collective
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[ab]);
      if (kSplitable && p.ksplit > 1) {
        if (ok) {
#pragma unroll
          for (int cc = 0; cc < 2; ++cc)
            store_partial(p, v[cc], tk.split, (tk.mn / p.n_tiles) * kBlockM + erow, n0 + cc * 32);
        }
        continue;
      }
      if (ok && rvalid) {
        const float* sb = p.out_kind == 2 ? s_bias : s_bias + n0;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const uint4* rp = has_res ? rc[cc] : nullptr;
          if (p.out_kind == 0)
            epi_chunk_act<0>(p, v[cc], em, n0, cc * 32, sb, tile_full, rp, sc_n, sc_iy, sc_ix);
          else if (p.out_kind == 1)
            epi_chunk_act<1>(p, v[cc], em, n0, cc * 32, sb, tile_full, rp, sc_n, sc_iy, sc_ix);
          else
            epi_chunk_act<2>(p, v[cc], em, n0, cc * 32, sb, tile_full, rp, sc_n, sc_iy, sc_ix);
        }
      }
    }
    } else {
    uint4 res[kResVecs], res_next[kPipeRes ? kResVecs : 1];
    if (kPipeRes) load_res(blockIdx.x, res);
    int lt = 0;
    for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++lt) {
      const TileK tk = kSplitable ? tile_k(p, t) : TileK{t, 0, 0, p.KB};
      const int n0 = (tk.mn % p.n_tiles) * BN;
      const int ab = lt % C::kAccBufs;
      int em;
      bool rvalid;
      row_of(t, em, rvalid);
      const bool tile_full = n0 + BN <= p.Cout;
      if (kPipeRes)
        load_res(t + static_cast<int>(gridDim.x), reinterpret_cast<uint4(&)[kResVecs]>(res_next));
      else if (!kChunked)
        load_res(t, res);
      int sc_n = 0, sc_iy = 0, sc_ix = 0;
      if (p.out_kind == 2 && rvalid) {
        sc_n = em / ohw;
        const int rem = em - sc_n * ohw;
        sc_iy = rem / p.OW;
        sc_ix = rem - sc_iy * p.OW;
      }
      const bool ok = !*abort_flag && mbar_wait(&tfull[ab], (lt / C::kAccBufs) & 1, kErrWaitAccum, p.wait_limit);
      if (!ok) *abort_flag = 1;
      tc_fence_after();
      if (kChunked) {
        // BN=256: 128 columns per warp, drained and stored 32 at a time (the
        // whole half would not fit in registers); the accumulator goes back
        // after the last chunk's load, its residual is read per chunk
        const float* sb = s_bias + n0;
#pragma unroll 1
        for (int cc = 0; cc < kHalf / 32; ++cc) {
          uint32_t vc[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tmem_base + t_lane + ab * BN + hcol + cc * 32, vc);  // warp-collective
          tmem_ld_wait();
          if (cc == kHalf / 32 - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[ab]);
          }
          const int cl = hcol + cc * 32;
          if (kSplitable && p.ksplit > 1) {
            if (ok) store_partial(p, vc, tk.split, (tk.mn / p.n_tiles) * kBlockM + erow, n0 + cl);
            continue;
          }
          uint4 rc[4];
          if (has_res && rvalid) {
            const uint4* rrow =
                reinterpret_cast<const uint4*>(p.residual + static_cast<int64_t>(em) * p.Cs_out + n0 + cl);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              rc[i] = (n0 + cl + i * 8 < p.Cs_out) ? __ldg(rrow + i) : make_uint4(0, 0, 0, 0);
          }
          if (p.out_kind == 0) {
            if (__all_sync(0xffffffffu, ok))
              epi_store_nhwc_act(p, vc, em, rvalid, n0, cl, sb, tile_full, has_res ? rc : nullptr, s_stage, lane);
          } else if (ok && rvalid) {
            epi_chunk_act<1>(p, vc, em, n0, cl, sb, tile_full, nullptr, 0, 0, 0);
          }
        }
        continue;
      }
      // drain this warp's share of the accumulator into registers, then hand
      // the TMEM buffer back to the MMA warp before the math and the stores
      uint32_t v[kHalf / 32][32];
#pragma unroll
      for (int cc = 0; cc < kHalf / 32; ++cc) {
        __syncwarp();
        tmem_ld_32x32b_x32(tmem_base + t_lane + ab * BN + hcol + cc * 32, v[cc]);  // warp-collective
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[ab]);
      if (kSplitable && p.ksplit > 1) {
        if (ok) {
#pragma unroll
          for (int cc = 0; cc < kHalf / 32; ++cc)
            store_partial(p, v[cc], tk.split, (tk.mn / p.n_tiles) * kBlockM + erow, n0 + hcol + cc * 32);
        }
        continue;
      }
      // staged stores at BN >= 128 (measured: faster for ResNet stages 2-4,
      // slower for the BN=64 halo layers, whose epilogue per tile is short)
      if (BN >= 128 && p.out_kind == 0 && __all_sync(0xffffffffu, ok)) {
        const float* sb = s_bias + n0;
#pragma unroll
        for (int cc = 0; cc < kHalf / 32; ++cc) {
          const uint4* rp = has_res ? &res[cc * 4] : nullptr;
          epi_store_nhwc_act(p, v[cc], em, rvalid, n0, hcol + cc * 32, sb, tile_full, rp, s_stage, lane);
        }
      } else if (ok && rvalid && (BN < 128 || p.out_kind != 0)) {
        const float* sb = p.out_kind == 2 ? s_bias : s_bias + n0;
#pragma unroll
        for (int cc = 0; cc < kHalf / 32; ++cc) {
          const int cl = hcol + cc * 32;
          const uint4* rp = has_res ? &res[cc * 4] : nullptr;
          if (p.out_kind == 0)
            epi_chunk_act<0>(p, v[cc], em, n0, cl, sb, tile_full, rp, sc_n, sc_iy, sc_ix);
          else if (p.out_kind == 1)
            epi_chunk_act<1>(p, v[cc], em, n0, cl, sb, tile_full, rp, sc_n, sc_iy, sc_ix);
          else
            epi_chunk_act<2>(p, v[cc], em, n0, cl, sb, tile_full, rp, sc_n, sc_iy, sc_ix);
        }
      }
      if (kPipeRes) {
#pragma unroll
        for (int i = 0; i < kResVecs; ++i) res[i] = res_next[kPipeRes ? i : 0];
      }
    }
    }
  } else if (C::issuer_of(warp) >= 0) {
    // ================================================================ MMA issuer(s)
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16_m128(BN);
      const int issuer = C::issuer_of(warp);  // several issuers: tiles with lt % n_iss == issuer
      // An issuer waiting on a halo buffer must never be two loads ahead of
      // the producer (a parity wait would then match the previous phase), so
      // AMODE 3 uses at most as many issuers as halo buffers; the others idle.
      const int n_iss = AMODE == 3 ? (p.halo_slots < C::kMmaIssuers ? p.halo_slots : C::kMmaIssuers) : C::kMmaIssuers;
      uint32_t it = 0, hc = 0;
      int lt = 0;
      bool ok = true;
      // AMODE 3: the resident weights land once, on full[0]
      if (AMODE == 3 && p.tiles > static_cast<int>(blockIdx.x)) ok = mbar_wait_relaxed(&full[0], 0, kErrWaitFull, p.wait_limit);
      // AMODE 3: tile-in-image, halo buffer and its phase of tile lt, and
      // lt % n_iss, kept as counters (no division per tile)
      int w_ti = 0, g_ti = 0, h_slot = 0, h_phase = 0, rr = 0;
      if (AMODE == 3) {
        w_ti = static_cast<int>(blockIdx.x) % p.tpi;
        g_ti = static_cast<int>(gridDim.x) % p.tpi;
      }
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, ++lt) {
        const int c_ti = w_ti, c_slot = h_slot, c_phase = h_phase;
        if (AMODE == 3) {
          w_ti += g_ti;
          if (w_ti >= p.tpi) w_ti -= p.tpi;
          if (++h_slot == p.halo_slots) {
            h_slot = 0;
            h_phase ^= 1;
          }
        }
        if (C::kMmaIssuers > 1) {
          const bool mine = rr == issuer;  // rr == lt % n_iss
          if (++rr == n_iss) rr = 0;
          if (!mine) continue;
        }
        const int ab = lt % C::kAccBufs;
        // no shared-memory loads (the abort flag included) in this loop: one
        // issued behind queued MMAs waits for them to drain; the waits are
        // relaxed for the same reason.  A stalled peer still ends the loop
        // through the bounded waits.
        if (!mbar_wait_relaxed(&tempty[ab], ((lt / C::kAccBufs) & 1) ^ 1, kErrWaitAccum, p.wait_limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ab * BN;
        if (AMODE == 3) {
          const int hs = c_slot;
          if (!mbar_wait_relaxed(&hfull[hs], static_cast<uint32_t>(c_phase), kErrWaitFull, p.wait_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // descriptors are built once per tile; a tap or K step only moves
          // the start-address field (16-byte units in the low bits; every
          // address stays below 232448 bytes, so the 14-bit field cannot carry)
          const int q0 = c_ti * kBlockM;
          const uint32_t rb = static_cast<uint32_t>(p.a_rowbytes);
          const uint32_t ox0 = static_cast<uint32_t>(q0 - div_wp(p, q0) * p.Wp);  // q0 % Wp
          const uint64_t a_desc =
              make_sdesc_rows(smem_u32(sA) + p.halo_off + hs * p.halo_stride + ox0 * rb, rb, p.a_layout);
          const uint64_t b_desc = make_sdesc_sw128(smem_u32(sA));
          const int csub = p.Cs_in >> 4;  // K=16 slices per tap
          const uint32_t row16 = rb >> 4, wp16 = static_cast<uint32_t>(p.Wp) * row16;
          int k0 = 0;
          for (int r = 0; r < p.kh; ++r) {
            for (int sx = 0; sx < p.kw; ++sx) {
              const uint64_t a_tap = a_desc + static_cast<uint32_t>(r) * wp16 + static_cast<uint32_t>(sx) * row16;
              for (int c = 0; c < csub; ++c, k0 += 16) {
                const uint32_t b_off16 = static_cast<uint32_t>((k0 >> 6) * (C::kBBytes >> 4) + ((k0 & 63) >> 3));
                umma_f16(d_tmem, a_tap + 2u * c, b_desc + b_off16, idesc, k0 != 0 ? 1u : 0u);
              }
            }
          }
          umma_commit(&hempty[hs]);
          umma_commit(&tfull[ab]);
          continue;
        }
        if (AMODE == 4) {
          const int q0 = ((t / p.n_tiles) % p.tpi) * kBlockM;
          const uint32_t row0 = static_cast<uint32_t>(q0 % p.Wp) * 8;  // 128-byte rows in 16-byte units
          const int taps = p.kh * p.kw;
          for (int cc = 0; cc < p.cchunks && ok; ++cc, ++hc) {
            const int hs = issuer * kHalo4Slots + static_cast<int>(hc % kHalo4Slots);
            if (!mbar_wait_relaxed(&hfull[hs], (hc / kHalo4Slots) & 1, kErrWaitFull, p.wait_limit)) {
              ok = false;
              break;
            }
            const uint64_t a_base = make_sdesc_sw128(smem_u32(sA) + p.halo_off + hs * p.halo_stride) + row0;
            int r = 0, sx = 0;
            for (int tap = 0; tap < taps; ++tap, ++it) {
              const int st = issuer * C::kRingStages + static_cast<int>(it % C::kRingStages);
              if (!mbar_wait_relaxed(&full[st], (it / C::kRingStages) & 1, kErrWaitFull, p.wait_limit)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t a_desc = a_base + static_cast<uint32_t>(r * p.Wp + sx) * 8u;
              const uint64_t b_desc = make_sdesc_sw128(smem_u32(sB + st * C::kBBytes));
#pragma unroll
              for (int k = 0; k < kBlockK / 16; ++k)
                umma_f16(d_tmem, a_desc + 2u * k, b_desc + 2u * k, idesc, (cc | tap | k) != 0 ? 1u : 0u);
              umma_commit(&empty[st]);
              if (++sx == p.kw) {
                sx = 0;
                ++r;
              }
            }
            if (ok) umma_commit(&hempty[hs]);
          }
          if (!ok) break;
          umma_commit(&tfull[ab]);
          continue;
        }
        const int nkb = tile_k(p, t).nkb;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int st = issuer * C::kRingStages + static_cast<int>(it % C::kRingStages);
          if (!mbar_wait_relaxed(&full[st], (it / C::kRingStages) & 1, kErrWaitFull, p.wait_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a_desc = make_sdesc_sw128(smem_u32(sA + st * kABytes));
          const uint64_t b_desc = make_sdesc_sw128(smem_u32(sB + st * C::kBBytes));
#pragma unroll
          for (int k = 0; k < kBlockK / 16; ++k) {  // K step = 32 bytes = 2 start-address units
            umma_f16(d_tmem, a_desc + 2u * k, b_desc + 2u * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[st]);
        }
        if (!ok) break;
        umma_commit(&tfull[ab]);
      }
      if (!ok) *abort_flag = 1;
      // every MMA this thread issued has completed once mma_done fires
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, kErrWaitFull, p.wait_limit);
    }
  } else if (warp == C::kTmaWarp || (C::kRings == 2 && warp == C::kTmaWarp2)) {
    // ================================================================ TMA producer(s)
    if (lane == 0) {
      const int ring = warp == C::kTmaWarp ? 0 : 1;  // kRings == 2: tiles with lt % 2 == ring
      uint32_t it = 0;
      constexpr uint32_t kTx = C::kBBytes + (AMODE != 0 ? kABytes : 0);
      bool ok = true;
      if (AMODE == 3 && p.tiles > static_cast<int>(blockIdx.x)) {
        // resident weights: every 64-wide K block of the (single) N tile
        mbar_arrive_expect_tx(&full[0], static_cast<uint32_t>(p.KB) * C::kBBytes);
        for (int kb = 0; kb < p.KB; ++kb) tma_load_2d(sA + kb * C::kBBytes, &tmap_w, &full[0], kb * kBlockK, 0);
        int lt = 0;
        // image, tile-in-image, halo buffer and phase of tile lt as counters
        int img = static_cast<int>(blockIdx.x) / p.tpi;
        int ti = static_cast<int>(blockIdx.x) - img * p.tpi;
        const int g_img = static_cast<int>(gridDim.x) / p.tpi;
        const int g_ti = static_cast<int>(gridDim.x) - g_img * p.tpi;
        int hs = 0, hph = 0;
        for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++lt) {
          if (*abort_flag || !mbar_wait(&hempty[hs], static_cast<uint32_t>(hph ^ 1), kErrWaitEmpty, p.wait_limit)) {
            ok = false;
            break;
          }
          const int q0 = ti * kBlockM;
          // test hook: CTA 0's first halo buffer never fills
          if (!(p.withhold_arrival && blockIdx.x == 0 && lt == 0)) {
            mbar_arrive_expect_tx(&hfull[hs], static_cast<uint32_t>(p.halo_bytes));
            tma_load_4d(sA + p.halo_off + hs * p.halo_stride, &tmap_a, &hfull[hs], 0, -p.pw, div_wp(p, q0) - p.ph,
                        img);
          }
          ti += g_ti;
          img += g_img;
          if (ti >= p.tpi) {
            ti -= p.tpi;
            ++img;
          }
          if (++hs == p.halo_slots) {
            hs = 0;
            hph ^= 1;
          }
        }
        // before the CTA may exit (an abort included), every TMA load this
        // thread issued has landed: the weights, and the last load of each
        // halo buffer (earlier ones were waited for through hempty)
        mbar_wait(&full[0], 0, kErrWaitFull, p.wait_limit);
        for (int j = lt - 1; j >= 0 && j >= lt - p.halo_slots; --j)
          mbar_wait(&hfull[j % p.halo_slots], (j / p.halo_slots) & 1, kErrWaitFull, p.wait_limit);
      }
      if (AMODE == 4) {
        // halo chunk h of this pipeline: tile lt = ring + 2 * (h / cchunks), chunk h % cchunks
        const int gx = static_cast<int>(gridDim.x), bx = static_cast<int>(blockIdx.x);
        const int my_tiles = p.tiles > bx ? (p.tiles - 1 - bx) / gx + 1 : 0;
        const int ring_tiles = my_tiles > ring ? (my_tiles - 1 - ring) / 2 + 1 : 0;
        const uint32_t n_h = static_cast<uint32_t>(ring_tiles) * p.cchunks;
        uint32_t h_issued = 0;
        auto issue_halo = [&](uint32_t h) -> bool {
          const int t = bx + (ring + 2 * static_cast<int>(h / p.cchunks)) * gx;
          const int cc = static_cast<int>(h % p.cchunks);
          const int mt = t / p.n_tiles;
          const int img = mt / p.tpi;
          const int q0 = (mt - img * p.tpi) * kBlockM;
          const int hs = ring * kHalo4Slots + static_cast<int>(h % kHalo4Slots);
          if (*abort_flag || !mbar_wait(&hempty[hs], ((h / kHalo4Slots) & 1) ^ 1, kErrWaitEmpty, p.wait_limit)) return false;
          mbar_arrive_expect_tx(&hfull[hs], static_cast<uint32_t>(p.halo_bytes));
          tma_load_4d(sA + p.halo_off + hs * p.halo_stride, &tmap_a, &hfull[hs], cc * kBlockK, -p.pw, q0 / p.Wp - p.ph,
                      img);
          ++h_issued;
          return true;
        };
        uint32_t h = 0;
        if (n_h > 0) ok = issue_halo(0);
        const int taps = p.kh * p.kw;
        for (int lt = ring; lt < my_tiles && ok; lt += 2) {
          const int t = bx + lt * gx;
          const int n0 = (t % p.n_tiles) * BN;
          for (int cc = 0; cc < p.cchunks && ok; ++cc, ++h) {
            for (int tap = 0; tap < taps; ++tap, ++it) {
              const int st = ring * C::kRingStages + static_cast<int>(it % C::kRingStages);
              if (*abort_flag || !mbar_wait(&empty[st], ((it / C::kRingStages) & 1) ^ 1, kErrWaitEmpty, p.wait_limit)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(C::kBBytes));
              tma_load_2d(sB + st * C::kBBytes, &tmap_w, &full[st], tap * p.Cs_in + cc * kBlockK, n0);
              // the next chunk's halo goes out after this chunk's first weight
              // block, a whole chunk ahead of its first MMA
              if (tap == 0 && h + 1 < n_h && !issue_halo(h + 1)) {
                ok = false;
                break;
              }
            }
          }
        }
        // the last halo loads of this pipeline have landed before the CTA may exit
        for (int j = static_cast<int>(h_issued) - 1; j >= 0 && j >= static_cast<int>(h_issued) - kHalo4Slots; --j)
          mbar_wait(&hfull[ring * kHalo4Slots + j % kHalo4Slots], (j / kHalo4Slots) & 1, kErrWaitFull, p.wait_limit);
      }
      int plt = 0;
      for (int t = blockIdx.x; t < p.tiles && ok && AMODE != 3 && AMODE != 4; t += gridDim.x, ++plt) {
        if (C::kRings == 2 && (plt & 1) != ring) continue;
        const TileK tk = tile_k(p, t);
        const int m0 = (tk.mn / p.n_tiles) * kBlockM;
        const int n0 = (tk.mn % p.n_tiles) * BN;
        int wst = 0, hst = 0, nimg = 0;
        if (AMODE == 1) {
          nimg = m0 / ohw;
          const int rem = m0 - nimg * ohw;
          const int oh = rem / p.OW;
          const int ow = rem - oh * p.OW;
          wst = ow * p.sw - p.pw;
          hst = oh * p.sh - p.ph;
        }
        // first K block of this split: its (tap, channel) position
        const int cpt = p.Cs_in / kBlockK;  // AMODE 1: 64-channel blocks per tap
        int c0 = 0, s = 0, r = 0;
        if (AMODE == 1) {
          const int tap0 = tk.kb0 / cpt;
          c0 = (tk.kb0 - tap0 * cpt) * kBlockK;
          r = tap0 / p.kw;
          s = tap0 - r * p.kw;
        }
        for (int kb = tk.kb0; kb < tk.kb0 + tk.nkb; ++kb, ++it) {
          const int st = ring * C::kRingStages + static_cast<int>(it % C::kRingStages);
          if (*abort_flag || !mbar_wait(&empty[st], ((it / C::kRingStages) & 1) ^ 1, kErrWaitEmpty, p.wait_limit)) {
            ok = false;
            break;
          }
          if (p.withhold_arrival && blockIdx.x == 0 && it == 0) continue;  // test hook: stage never fills
          mbar_arrive_expect_tx(&full[st], kTx);
          tma_load_2d(sB + st * C::kBBytes, &tmap_w, &full[st], kb * kBlockK, n0);
          if (AMODE == 1) {
            tma_load_im2col_4d(sA + st * kABytes, &tmap_a, &full[st], c0, wst, hst, nimg, static_cast<uint16_t>(s),
                               static_cast<uint16_t>(r));
            c0 += kBlockK;
            if (c0 == p.Cs_in) {
              c0 = 0;
              if (++s == p.kw) {
                s = 0;
                ++r;
              }
            }
          } else if (AMODE == 2) {
            tma_load_2d(sA + st * kABytes, &tmap_a, &full[st], kb * kBlockK, m0);
          }
        }
      }
      if (!ok) *abort_flag = 1;
      if (AMODE == 1 || AMODE == 2 || AMODE == 4) {
        // every TMA load this thread issued has landed before the CTA may exit
        // (the last kRingStages stages; earlier ones were waited for through
        // their empty barriers)
        for (int j = static_cast<int>(it) - 1; j >= 0 && j >= static_cast<int>(it) - C::kRingStages; --j)
          mbar_wait(&full[ring * C::kRingStages + j % C::kRingStages], (j / C::kRingStages) & 1, kErrWaitFull, p.wait_limit);
      }
    }
  } else if (AMODE == 0) {
    // ================================================================ A gather (cp.async)
    // Lane l of gather warp gw copies 16-byte chunk (l % 8) of rows
    // gw*32 + l/8 + 4*i (i = 0..7): one warp instruction moves four whole
    // 128-byte rows, which are contiguous in global memory whenever a K block
    // is one run of channels (or of space-to-depth taps).
    const int gt = tid - C::kGatherWarp0 * 32;  // 0..127
    const int gw = gt >> 5, gl = gt & 31;
    const int j = gl & 7;
    const int rbase = gw * 32 + (gl >> 3);
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
      const TileK tk = tile_k(p, t);
      const int m0 = (tk.mn / p.n_tiles) * kBlockM;
      int ih0[8], iw0[8];
      const __half* xb[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int m = m0 + rbase + 4 * i;
        ih0[i] = -(1 << 28);  // rows past M never pass the bounds check
        iw0[i] = 0;
        xb[i] = p.x;
        if (m < p.M) {
          const int n_img = m / ohw;
          const int rem = m - n_img * ohw;
          const int oh = rem / p.OW;
          const int ow = rem - oh * p.OW;
          ih0[i] = oh * p.sh - p.ph;
          iw0[i] = ow * p.sw - p.pw;
          xb[i] = p.x + static_cast<int64_t>(n_img) * p.H * p.W * p.Cs_in;
        }
      }
      for (int kb = tk.kb0; kb < tk.kb0 + tk.nkb; ++kb, ++it) {
        const int st = it % STAGES;
        if (*abort_flag || !mbar_wait(&empty[st], ((it / STAGES) & 1) ^ 1, kErrWaitEmpty, p.wait_limit)) {
          ok = false;
          break;
        }
        const uint32_t e = ktable[kb * 8 + j];
        const bool ek = e != 0xFFFFFFFFu;
        const int rr = int(e >> 24), ss = int((e >> 16) & 0xFF), cc = int(e & 0xFFFF);
        const uint32_t stage = smem_u32(sA) + st * kABytes;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int row = rbase + 4 * i;
          const int ih = ih0[i] + rr, iw = iw0[i] + ss;
          const bool okc = ek && (unsigned)ih < (unsigned)p.H && (unsigned)iw < (unsigned)p.W;
          const __half* src = okc ? xb[i] + (static_cast<int64_t>(ih) * p.W + iw) * p.Cs_in + cc : p.x;
          cp_async_16(stage + row * 128 + ((j ^ (row & 7)) << 4), src, okc ? 16u : 0u);
        }
        cp_async_commit();
        if (it >= C::kLag) {
          cp_async_wait<C::kLag>();
          fence_proxy_async_smem();
          mbar_arrive(&full[(it - C::kLag) % STAGES]);
        }
      }
    }
    cp_async_wait_all();
    fence_proxy_async_smem();
    if (ok) {
      for (uint32_t j = it > C::kLag ? it - C::kLag : 0; j < it; ++j) mbar_arrive(&full[j % STAGES]);
    } else {
      *abort_flag = 1;
    }
  }

  // TMEM is released after every warp is done with it (the MMA thread has
  // waited for all of its MMAs, the epilogue for all of its loads).
  tc_fence_before();
  __syncthreads();
  if (warp == C::kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------- host side

void* driver_fn(const char* name) {
  cudaDriverEntryPointQueryResult q;
  void* ptr = nullptr;
  if (cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
    return ptr;
  return nullptr;
}

constexpr int kMaxDevices = 64;

// Process-unique id of the calling thread's current CUDA context (cuCtxGetId),
// 0 if there is none or the driver does not say.  Per-device caches compare
// it to notice a context that was destroyed and recreated (cudaDeviceReset).
uint64_t current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    get_current = reinterpret_cast<GetCurrent>(driver_fn("cuCtxGetCurrent"));
    get_id = reinterpret_cast<GetId>(driver_fn("cuCtxGetId"));
  });
  if (!get_current || !get_id) return 0;
  // no runtime call that could initialise a context here: this runs inside
  // stream captures, where such calls are not allowed
  CUcontext c = nullptr;
  unsigned long long id = 0;
  if (get_current(&c) != CUDA_SUCCESS || c == nullptr || get_id(c, &id) != CUDA_SUCCESS) return 0;
  return static_cast<uint64_t>(id);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(driver_fn("cuTensorMapEncodeTiled"));
  });
  return fn;
}

PFN_cuTensorMapEncodeIm2col_v12000 encode_im2col() {
  static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(driver_fn("cuTensorMapEncodeIm2col"));
  });
  return fn;
}

// 2-D map over a row-major fp16 matrix [rows, cols] (row stride ld elements),
// box {64, box_rows}, 128B swizzle.  Columns past `cols` read as zero.
static int make_tmap_2d(CUtensorMap* map, const void* base, int rows, int cols, int ld, int box_rows) {
  auto enc = encode_tiled();
  if (!enc) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBlockK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// im2col map over the NHWC activation [N, H, W, Cs]: 128 pixels x 64 channels
// per load, bounding box [-pad, dim - 1 + pad - (k - 1)], traversal = stride.
static int make_tmap_im2col(CUtensorMap* map, const ConvTcArgs& a, int n_img) {
  auto enc = encode_im2col();
  if (!enc) return -1;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.Cs_in), static_cast<cuuint64_t>(a.W), static_cast<cuuint64_t>(a.H),
                        static_cast<cuuint64_t>(n_img)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(a.Cs_in) * 2, static_cast<cuuint64_t>(a.W) * a.Cs_in * 2,
                           static_cast<cuuint64_t>(a.H) * a.W * a.Cs_in * 2};
  int lower[2] = {-a.pw, -a.ph};
  int upper[2] = {a.pw - (a.kw - 1), a.ph - (a.kh - 1)};
  cuuint32_t estr[4] = {1, static_cast<cuuint32_t>(a.sw), static_cast<cuuint32_t>(a.sh), 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(a.x), dims, strides, lower, upper,
                   kBlockK, kBlockM, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// Halo map over the NHWC activation [N, H, W, Cs]: box of min(Cs, 64)
// channels x Wp pixels x R rows of one image, swizzled at the box row width;
// the kernel starts each box at pixel -pw so that its rows are whole
// zero-padded input rows (and at channel 64*chunk in AMODE 4).
static int make_tmap_halo(CUtensorMap* map, const ConvTcArgs& a, int n_img, int wp, int rows) {
  const int box_c = a.Cs_in < kBlockK ? a.Cs_in : kBlockK;
  auto enc = encode_tiled();
  if (!enc) return -1;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.Cs_in), static_cast<cuuint64_t>(a.W), static_cast<cuuint64_t>(a.H),
                        static_cast<cuuint64_t>(n_img)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(a.Cs_in) * 2, static_cast<cuuint64_t>(a.W) * a.Cs_in * 2,
                           static_cast<cuuint64_t>(a.H) * a.W * a.Cs_in * 2};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(box_c), static_cast<cuuint32_t>(wp), static_cast<cuuint32_t>(rows), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapSwizzle sw = box_c == 16 ? CU_TENSOR_MAP_SWIZZLE_32B
                                : box_c == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                              : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(a.x), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// Resident-weight halo plan of a conv at block width `bn`: fills the AMODE 3
// fields of `p` and returns the fraction of computed positions that are real
// outputs, or 0 when the layer does not fit the mode (stride 1, Cs_in of 16,
// 32 or 64, one N tile, weights plus two halo buffers within kHaloRegion).
static double halo_plan(const ConvTcArgs& a, int bn, ConvTcParams* p) {
  const int wp = a.W + 2 * a.pw;
  if (a.sh != 1 || a.sw != 1 || a.out_kind == 2 || a.n_cols > bn || wp < 2) return 0.0;
  if (a.Cs_in != 16 && a.Cs_in != 32 && a.Cs_in != 64) return 0.0;
  if (wp > 256 || a.OW != wp - a.kw + 1 || a.k_pad % kBlockK != 0) return 0.0;
  const long q = static_cast<long>(a.OH) * wp;
  const int tpi = static_cast<int>((q + kBlockM - 1) / kBlockM);
  if (static_cast<long long>(tpi) * kBlockM * wp >= (1ll << 32)) return 0.0;  // div_wp's exact range
  int max_off = 0;
  for (int j = 0; j < tpi; ++j) max_off = std::max(max_off, (j * kBlockM) % wp);
  const int rows = (max_off + (a.kh - 1) * wp + (a.kw - 1) + kBlockM - 1) / wp + 1;
  if (rows > 256) return 0.0;
  const int rb = a.Cs_in * 2;
  const int w_bytes = (a.k_pad / kBlockK) * bn * kBlockK * 2;
  const int halo_bytes = rb * wp * rows;
  const int stride = (halo_bytes + 1023) & ~1023;
  if (w_bytes >= kHaloRegion) return 0.0;
  const int slots = std::min(kHaloSlotsMax, (kHaloRegion - w_bytes) / stride);
  if (slots < 2) return 0.0;
  p->Wp = wp;
  p->tpi = tpi;
  p->halo_off = w_bytes;
  p->halo_stride = stride;
  p->halo_slots = slots;
  p->halo_bytes = halo_bytes;
  p->a_rowbytes = rb;
  p->a_layout = rb == 32 ? 6 : (rb == 64 ? 4 : 2);
  p->wp_magic = static_cast<uint32_t>(((1ull << 32) + wp - 1) / wp);
  return static_cast<double>(a.OH) * a.OW / (static_cast<double>(tpi) * kBlockM);
}

// Streamed-weight halo plan (AMODE 4) at block width `bn` with `stages`
// weight stages (split over the two pipelines): fills the halo fields of `p`
// and returns the fraction of computed positions that are real outputs, or 0
// when the layer does not fit (stride 1, Cs_in a multiple of 64, weight
// stages plus 2 x kHalo4Slots halo buffers within kHalo4Region).
static double halo4_plan(const ConvTcArgs& a, int bn, int stages, ConvTcParams* p) {
  const int wp = a.W + 2 * a.pw;
  if (a.sh != 1 || a.sw != 1 || a.out_kind == 2 || a.Cs_in % kBlockK != 0) return 0.0;
  if (wp > 256 || a.OW != wp - a.kw + 1 || a.k_pad != a.kh * a.kw * a.Cs_in) return 0.0;
  const long q = static_cast<long>(a.OH) * wp;
  const int tpi = static_cast<int>((q + kBlockM - 1) / kBlockM);
  int max_off = 0;
  for (int j = 0; j < tpi; ++j) max_off = std::max(max_off, (j * kBlockM) % wp);
  const int rows = (max_off + (a.kh - 1) * wp + (a.kw - 1) + kBlockM - 1) / wp + 1;
  if (rows > 256) return 0.0;
  const int halo_bytes = kBlockK * 2 * wp * rows;
  const int stride = (halo_bytes + 1023) & ~1023;
  const int w_bytes = stages * bn * kBlockK * 2;
  if (w_bytes + 2 * kHalo4Slots * stride > kHalo4Region) return 0.0;
  if ((a.out_kind == 2 ? a.t_cout : ((a.n_cols + bn - 1) / bn) * bn) > kHalo4BiasMax) return 0.0;
  p->Wp = wp;
  p->tpi = tpi;
  p->halo_off = w_bytes;
  p->halo_stride = stride;
  p->halo_slots = kHalo4Slots;
  p->halo_bytes = halo_bytes;
  p->a_rowbytes = kBlockK * 2;
  p->a_layout = 2;
  p->cchunks = a.Cs_in / kBlockK;
  return static_cast<double>(a.OH) * a.OW / (static_cast<double>(tpi) * kBlockM);
}

// Bounded-wait limit of a launch: LOTUS_WAIT_LIMIT try_wait rounds (1 .. 2^30)
// when set, kMaxWaitIters otherwise.
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("LOTUS_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

uint32_t wait_limit_from_env() {
  const char* e = std::getenv("LOTUS_WAIT_LIMIT");
  if (!e) return kMaxWaitIters;
  const long v = std::atol(e);
  return (v >= 1 && v <= (1L << 30)) ? static_cast<uint32_t>(v) : kMaxWaitIters;
}

// Split-K reduction: y[m, c] = act(bias[c] + sum_s ws[s][m][c] (+ residual)),
// eight channels per thread, summed in split order (deterministic).  NHWC
// fp16 output (pad channels written as zero) or fp32 rows.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int ws_rows, int ws_ld,
                                     const float* __restrict__ bias, const __half* __restrict__ residual,
                                     void* __restrict__ y, int M, int cout, int cs_out, int y_stride, int act,
                                     int out_kind) {
  if (threadIdx.x == 0) griddep_launch();
  griddep_wait();  // the partial sums of the kernel before
  const int groups = out_kind == 0 ? cs_out / 8 : (cout + 7) / 8;
  const int total = M * groups;  // < 2^31, checked by the launcher
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int m = i / groups;
    const int c0 = (i - m * groups) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int sp = 0; sp < splits; ++sp) {
      const float4* src = reinterpret_cast<const float4*>(ws + (static_cast<size_t>(sp) * ws_rows + m) * ws_ld + c0);
      const float4 a = __ldg(src), b = __ldg(src + 1);
      acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
      acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
    }
    float res[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (residual) {
      const uint4 r = __ldg(reinterpret_cast<const uint4*>(residual + static_cast<size_t>(m) * cs_out + c0));
      const __half2* rh = reinterpret_cast<const __half2*>(&r);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(rh[j]);
        res[2 * j] = f.x;
        res[2 * j + 1] = f.y;
      }
    }
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = c0 + j;
      const float v = acc[j] + ((bias != nullptr && c < cout) ? __ldg(bias + c) : 0.f) + res[j];
      o[j] = c < cout ? apply_act(v, act) : 0.f;
    }
    if (out_kind == 0) {
      *reinterpret_cast<uint4*>(static_cast<__half*>(y) + static_cast<size_t>(m) * y_stride + c0) =
          make_uint4(pack_half2(o[0], o[1]), pack_half2(o[2], o[3]), pack_half2(o[4], o[5]), pack_half2(o[6], o[7]));
    } else {
      float* yr = static_cast<float*>(y) + static_cast<size_t>(m) * cout;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + j < cout) yr[c0 + j] = o[j];
    }
  }
}

// Split-K reduction of `splits` fp32 partial tiles in ws[split][row][ws_ld]
// into an NHWC fp16 output of `rows` rows (bias, residual, activation; pad
// channels zero), on `stream`, allowing programmatic dependent launch.
cudaError_t launch_splitk_reduce(const float* ws, int splits, int rows, int ws_ld, const float* bias,
                                 const __half* residual, __half* y, int M, int cout, int cs_out, int y_stride,
                                 int act, cudaStream_t stream) {
  const size_t total = static_cast<size_t>(M) * (cs_out / 8);
  const unsigned grid =
      static_cast<unsigned>(std::min<size_t>((total + 255) / 256, static_cast<size_t>(num_sms()) * 8));
  cudaError_t e = launch_pdl(splitk_reduce_kernel, dim3(grid), dim3(256), 0, stream, ws, splits, rows, ws_ld, bias,
                             residual, static_cast<void*>(y), M, cout, cs_out, y_stride, act, 0);
  note_launch();
  return e != cudaSuccess ? e : cudaGetLastError();
}

// Split count for an output-tile grid of `mn` tiles over KB K blocks on `sms`
// SMs: none unless the grid fills at most half of the SMs; at least 4 K blocks
// per split; every split non-empty.
static int split_count(long mn, int kb_total, int sms, int* kbs) {
  *kbs = kb_total;
  if (mn * 2 > sms || kb_total < 8) return 1;
  const long s = std::min<long>(kb_total / 4, sms / mn);
  if (s < 2) return 1;
  *kbs = static_cast<int>((kb_total + s - 1) / s);
  return (kb_total + *kbs - 1) / *kbs;
}

// SM count of the current device, cached per device ordinal.
int num_sms() {
  static std::atomic<int> cache[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

template <int BN, int STAGES, int AMODE>
static cudaError_t launch_impl(const CUtensorMap& mw, const CUtensorMap& ma, const ConvTcParams& p,
                               cudaStream_t stream) {
  using C = Cfg<BN, STAGES, AMODE>;
  static_assert(C::bytes(AMODE == 0 ? kMaxTable : 0) <= 232448, "dynamic shared memory above 227 KB");
  const int smem = C::bytes(AMODE == 0 ? p.KB * 8 : 0);
  auto kern = conv_tc_kernel<BN, STAGES, AMODE>;
  // the shared-memory opt-in is a property of the function in one context:
  // set it once per device and again whenever that device's context changed
  // (a cudaDeviceReset creates a new one)
  static std::atomic<uint64_t> attr_ctx[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  const uint64_t ctx = current_context_id();
  if (ctx == 0 || attr_ctx[dev].load(std::memory_order_acquire) != ctx) {
    const cudaError_t ae = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                C::bytes(AMODE == 0 ? kMaxTable : 0));
    if (ae != cudaSuccess) return ae;
    attr_ctx[dev].store(ctx, std::memory_order_release);
  }
  const int grid = p.tiles < num_sms() ? p.tiles : num_sms();
  const cudaError_t le = launch_pdl(kern, dim3(grid), dim3(C::kThreads), smem, stream, mw, ma, p);
  note_launch();
  return le != cudaSuccess ? le : cudaGetLastError();
}

int conv_tc_launch(const ConvTcArgs& a, cudaStream_t stream, const char** err, size_t* ws_need) {
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
  p.y_stride = a.y_stride > 0 ? a.y_stride : a.Cs_out;
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
  p.wait_limit = wait_limit_from_env();
  const char* wh = std::getenv("LOTUS_TEST_WITHHOLD_ARRIVAL");
  p.withhold_arrival = (wh && std::atoi(wh) == 1) ? 1 : 0;

  int bn = a.block_n;
  if (bn == 0) {
    const char* env = std::getenv("LOTUS_CONV_BN");
    bn = env ? std::atoi(env) : 0;
  }
  const bool plain_gemm = a.kh == 1 && a.kw == 1 && a.sh == 1 && a.sw == 1 && a.ph == 0 && a.pw == 0;
  const int n_img = a.M / (a.OH * a.OW);
  const size_t x_bytes = static_cast<size_t>(n_img) * a.H * a.W * a.Cs_in * 2;
  // the im2col TMA path (below) takes 64-channel-aligned inputs of >= 128 KB
  const bool im2col_ok = !plain_gemm && a.Cs_in % kBlockK == 0 && x_bytes >= (128u << 10);
  const char* force = std::getenv("LOTUS_CONV_AMODE");
  const int forced = force ? std::atoi(force) : -1;
  if (bn != 64 && bn != 128 && bn != 256) bn = a.n_cols <= 64 ? 64 : (a.n_cols >= 256 && im2col_ok ? 256 : 128);
  // BN=256 exists for the im2col path only
  if (bn == 256 && (!im2col_ok || a.out_kind == 2 || (forced >= 0 && forced != 1))) bn = 128;
  p.n_tiles = (a.n_cols + bn - 1) / bn;
  const long m_tiles = (static_cast<long>(a.M) + kBlockM - 1) / kBlockM;
  if (m_tiles * p.n_tiles > 0x7FFFFFFFL) {
    *err = "conv: too many tiles";
    return -2;
  }
  p.tiles = static_cast<int>(m_tiles * p.n_tiles);
  p.bias_smem = (a.out_kind == 2 ? a.t_cout : p.n_tiles * bn) <= kBiasMax ? 1 : 0;

  // A operand: plain-GEMM tiles by 2-D TMA, im2col TMA for 64-channel-aligned
  // inputs, otherwise the cp.async gather.  Small inputs (< 128 KB) stay on
  // the gather path: the im2col map is only used on activation tensors at
  // least that large.
  int amode = 0;
  if (plain_gemm)
    amode = 2;
  else if (im2col_ok)
    amode = 1;
  // resident-weight halo mode where at least 70% of the computed positions are
  // real outputs (the padding columns and each image's last tile are waste)
  if (!plain_gemm && bn <= 128 && halo_plan(a, bn, &p) >= 0.70) amode = 3;
  // AMODE 4 only on request: with three weight stages per pipeline the
  // streamed weights, not the A bytes, bound these layers, and im2col is as
  // fast or faster on ResNet stages 2-3
  if (force && std::atoi(force) == 4 && amode == 1 && bn <= 128 && halo4_plan(a, bn, bn == 64 ? 8 : 6, &p) >= 0.70)
    amode = 4;
  if (force && std::atoi(force) == 0) amode = 0;
  if (force && std::atoi(force) == 1 && (amode == 3 || amode == 4))
    amode = a.Cs_in % kBlockK == 0 && x_bytes >= (128u << 10) ? 1 : 0;
  if (amode == 3) p.tiles = static_cast<int>(static_cast<long>(n_img) * p.tpi);
  if (amode == 4) p.tiles = static_cast<int>(static_cast<long>(n_img) * p.tpi * p.n_tiles);
  // split-K: launches whose output tiles fill at most half of the SMs split
  // their K loop when the caller passed a large enough workspace
  p.ksplit = 1;
  p.kbs = p.KB;
  p.mn_tiles = p.tiles;
  if ((amode == 0 || amode == 1 || amode == 2) && a.out_kind != 2) {
    int kbs = p.KB;
    const int sp = split_count(p.tiles, p.KB, num_sms(), &kbs);
    const size_t need = sp > 1 ? static_cast<size_t>(sp) * (m_tiles * kBlockM) * (p.n_tiles * bn) * 4 : 0;
    if (ws_need) {
      *ws_need = need;
      return 0;
    }
    if (sp > 1 && a.ws != nullptr && need <= a.ws_bytes && static_cast<long>(a.M) * (p.n_tiles * bn / 8) < (1L << 31)) {
      p.ksplit = sp;
      p.kbs = kbs;
      p.ws = a.ws;
      p.ws_rows = static_cast<int>(m_tiles * kBlockM);
      p.ws_ld = p.n_tiles * bn;
      p.tiles = p.mn_tiles * sp;
    }
  } else if (ws_need) {
    *ws_need = 0;
    return 0;
  }
  if (amode == 0 && p.KB * 8 > kMaxTable) {
    *err = "conv: K too large for the gather path";
    return -2;
  }

  CUtensorMap mw, ma;
  if (make_tmap_2d(&mw, a.w_packed, a.n_cols, a.k_pad, a.k_pad, bn) != 0) {
    *err = "conv: weight tensor map encoding failed";
    return -3;
  }
  ma = mw;  // unused by the gather path
  if (amode == 1 && make_tmap_im2col(&ma, a, n_img) != 0) {
    *err = "conv: im2col tensor map encoding failed";
    return -3;
  }
  if ((amode == 3 || amode == 4) && make_tmap_halo(&ma, a, n_img, p.Wp, p.halo_bytes / (p.a_rowbytes * p.Wp)) != 0) {
    *err = "conv: halo tensor map encoding failed";
    return -3;
  }
  if (amode == 2 && make_tmap_2d(&ma, a.x, a.M, a.Cs_in, a.Cs_in, kBlockM) != 0) {
    *err = "conv: activation tensor map encoding failed";
    return -3;
  }

  cudaError_t e = cudaErrorInvalidValue;
  if (bn == 256) {
    e = launch_impl<256, 4, 1>(mw, ma, p, stream);  // amode == 1 (see the BN choice above)
  } else if (bn == 64) {
    switch (amode) {
      case 0: e = launch_impl<64, 8, 0>(mw, ma, p, stream); break;
      case 1: e = launch_impl<64, 8, 1>(mw, ma, p, stream); break;
      case 2: e = launch_impl<64, 8, 2>(mw, ma, p, stream); break;
      case 4: e = launch_impl<64, 8, 4>(mw, ma, p, stream); break;
      default: e = launch_impl<64, 2, 3>(mw, ma, p, stream); break;
    }
  } else {
    switch (amode) {
      case 0: e = launch_impl<128, 6, 0>(mw, ma, p, stream); break;
      case 1: e = launch_impl<128, 6, 1>(mw, ma, p, stream); break;
      case 2: e = launch_impl<128, 6, 2>(mw, ma, p, stream); break;
      case 4: e = launch_impl<128, 6, 4>(mw, ma, p, stream); break;
      default: e = launch_impl<128, 2, 3>(mw, ma, p, stream); break;
    }
  }
  if (e == cudaSuccess && p.ksplit > 1) {
    const size_t total = static_cast<size_t>(a.M) * (a.out_kind == 0 ? a.Cs_out / 8 : (a.n_cols + 7) / 8);
    const unsigned grid = static_cast<unsigned>(std::min<size_t>((total + 255) / 256, static_cast<size_t>(num_sms()) * 8));
    e = launch_pdl(splitk_reduce_kernel, dim3(grid), dim3(256), 0, stream, static_cast<const float*>(p.ws), p.ksplit,
                   p.ws_rows, p.ws_ld, a.bias, static_cast<const __half*>(a.residual), a.y, a.M, a.n_cols, a.Cs_out,
                   p.y_stride, a.act, a.out_kind);
    note_launch();
    if (e == cudaSuccess) e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    *err = cudaGetErrorString(e);
    return -3;
  }
  return 0;
}

// Split-K scratch of lotus_conv2d_fwd_noalloc, for callers that cannot
// allocate device memory themselves.  Compiled into the library: every GPU
// that loads it holds these kNoAllocScratchBytes until the process exits.
// Host code must not pass the symbol itself to a kernel (on the host it is a
// stand-in, not a device address): conv_tc_noalloc_scratch() looks up the
// address per device.
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

int conv_tc_noalloc_scratch(float** ptr, const char** err) {
  static std::mutex mu;
  static float* addr[kMaxDevices] = {};
  static uint64_t addr_ctx[kMaxDevices] = {};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = "no usable current CUDA device";
    return -3;
  }
  const uint64_t ctx = current_context_id();
  std::lock_guard<std::mutex> lock(mu);
  // once per device, with that device current (the caller's current device),
  // and again when the device's context was recreated (after a
  // cudaDeviceReset the module and with it the scratch live elsewhere)
  if (addr[dev] == nullptr || ctx == 0 || addr_ctx[dev] != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *err = e != cudaSuccess ? cudaGetErrorString(e) : "cudaGetSymbolAddress returned null";
      return -3;
    }
    addr[dev] = static_cast<float*>(p);
    addr_ctx[dev] = ctx;
  }
  *ptr = addr[dev];
  return 0;
}

// Returns and clears this translation unit's device error word.
static int read_own_device_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, lotus_dev::g_lotus_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) {
    int zero = 0;
    cudaMemcpyToSymbol(lotus_dev::g_lotus_device_error, &zero, sizeof(int));
  }
  return v;
}

int read_device_error() {
  // every kernel file keeps its own error word; report the first non-zero
  // one and clear them all
  const int a = read_own_device_error();
  const int b = conv_row_read_device_error();
  const int c = conv_rows_read_device_error();
  const int d = conv_pair_read_device_error();
  return a != 0 ? a : b != 0 ? b : c != 0 ? c : d;
}

}  // namespace lotus_impl
