// Row-tile convolution on sm_100a tensor cores with an optional fused
// 3x3 / stride-2 / pad-1 max pool of its activated output.
//
// Scope: stride-1 convs without padding whose kernel row is exactly one
// 64-wide K block (Cs_in * kw == 64), output rows of at most 128 pixels and
// at most 64 output channels.  This is the ResNet-18 stem after the
// space-to-depth rewrite (4x4 kernel over 16-channel pixels, 112-pixel rows),
// whose output the reference feeds straight into a 3x3/2 max pool
// (source/operator/conv2d.cu:17-187 then source/operator/maxpool2d.cu:16-66,
// wired by source/graph.cpp:84-109).
//
// GEMM view: one tile = one output row (oy) of one image, M = 128 positions
// (ox = 0..127; ox >= OW are computed and dropped), N = Cout (<= 64),
// K = kh * 64.  In NHWC the kw taps of one kernel row read kw consecutive
// pixels, i.e. kw * Cs_in = 64 contiguous fp16 values starting at pixel
// (oy + r, ox).  A 4-D TMA map whose innermost dimension is those 64 values
// and whose next dimension steps ONE pixel (an overlapping stride) lands a
// whole input row as 128 rows of 128 bytes, 128B-swizzled: exactly the
// K-major A operand of kernel row r for every position of the tile, with a
// 1024-byte-aligned start.
//
// Stacked weights: input row y feeds output rows y, y-1, .., y-kh+1 through
// kernel rows 0..kh-1.  The kh weight blocks W_0..W_{kh-1} (64 rows each) lie
// one after the other in shared memory, i.e. they form one B operand of
// N = kh * 64 rows, so ONE set of 4 MMAs (K = 64 in steps of 16) per input
// row computes all kh partial products.  The accumulators sit in a TMEM ring
// of 8 blocks of 64 columns at DESCENDING positions: tile t (the t-th output
// row of the CTA) uses block P(t) = 7 - t % 8, so the blocks of tiles
// y, y-1, .., y-kh+1 are P(y), P(y)+1, .., P(y)+kh-1 (mod 8), contiguous
// except where the window wraps past block 7, where the MMA is split in two.
// Each input row is loaded once per CTA segment and read by one MMA group;
// every accumulator is zeroed by the epilogue (tcgen05.st) when it is
// drained, so every MMA accumulates.  For one output row the partial
// products are summed in kernel-row order, then K order, as a plain
// kernel-row loop would.
//
// Roles (608 threads):
//   warps 0-15  epilogue: warp w drains TMEM lane quarter w%4, columns
//               16*(w/4) .. +15, then zeroes them.  Without the pool: bias,
//               activation, fp16 store of the conv row.  With the pool:
//               fp16(acc + bias), its vertical max carried in registers from
//               row to row (a thread always holds the same ox and channels),
//               then once per pooled row the horizontal 3-wide max by warp
//               shuffles (lane 0's left neighbour comes from the previous
//               quarter through shared memory), then the activation of the
//               pooled pixel;
//   warp 16     TMEM allocation, MMA issuer (it waits on no mbarrier);
//   warp 17     TMA producer: the weights once, then input rows in order;
//   warp 18     the gate: the MMAs' mbarrier waits (tile block drained and
//               zeroed, input row landed), one named-barrier hand-off to the
//               issuer per input row (an mbarrier wait in the issuing warp is
//               held behind its queued MMAs).
// Each CTA owns a contiguous range of output units (pooled rows, or conv
// rows without the pool) over the whole batch, walked as per-image
// segments; with the pool a segment also computes the conv row just above
// its first pooled row (the shared row of two pooled windows).
//
// Barrier protocol (all waits bounded): rfull[slot] (TMA bytes), rempty[slot]
// (committed after the MMAs reading the row), tempty[block] (16 epilogue
// arrivals: drained and zeroed; the first phase completes after the initial
// zeroing), tfull[block] (committed after the last MMA of the tile's last
// input row), wfull for the weights.  The gate waits for a block only at
// the first input row of its tile; the tiles sharing an MMA window were all
// acquired before, and block P(t) is reused by tile t+8 only after tile t
// was drained and tile t+1 loaded (the release waits one tile), which needs
// the MMAs of input rows up to t+kh < t+8.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>

#include "kernels.h"
#include "ptx.cuh"

namespace lotus_impl {

using namespace lotus_dev;

namespace {

constexpr int kRowSlots = 8;                   // input-row ring
constexpr int kRowPos = 128;                   // positions (A rows) per tile
constexpr int kRowBox = 32;                    // positions per TMA box (one TMEM lane quarter)
constexpr int kRowMaxQPool = (kRowBox - 2) / 2;  // pooled columns per quarter (window centres on odd lanes)
constexpr int kSlotBytes = kRowPos * 128;      // one input row: 128 rows x 128 B
constexpr int kRowAcc = 8;                     // TMEM accumulator blocks of 64 columns
constexpr int kRowMaxKh = 6;                   // the MMA window (kh blocks) leaves two blocks for the epilogue
constexpr int kWBlockBytes = 64 * 128;         // one 64-wide K block of 64 weight rows
constexpr int kEpiWarps = 16;                  // 4 per TMEM lane quarter, 16 columns each
constexpr int kEpiCols = 64 / (kEpiWarps / 4);
constexpr int kIssuer = kEpiWarps, kProducer = kEpiWarps + 1, kGate = kEpiWarps + 2;
constexpr int kThreads = (kEpiWarps + 3) * 32;
constexpr uint32_t kRowBar = 1;  // named barrier of the gate / issuer hand-off (0 is __syncthreads)

// TMEM block of the CTA's t-th tile (descending, so one input row's MMA
// window over tiles y .. y-kh+1 is ascending and contiguous up to a wrap)
__device__ __forceinline__ int acc_block(int t) { return (kRowAcc - 1) - (t & (kRowAcc - 1)); }

struct RowParams {
  const float* bias;
  __half* y;
  int N, OH, OW, Cout, Cs_out, kh, act;
  int pool;          // 0: conv rows out, 1: fused 3x3/2 pad-1 max pool
  int PH, PW;        // pooled size (pool == 1)
  int units;         // N * (pool ? PH : OH)
  int w_bytes;       // kh * kWBlockBytes
  int qpool, qspan;  // pool: pooled columns per lane quarter, conv columns between quarters (2 * qpool)
  uint32_t wait_limit;
};

// Shared-memory layout (from the 1024-aligned base): weights, input-row ring,
// barriers, misc words, bias.
constexpr int kMaxWBytes = kRowMaxKh * kWBlockBytes;
constexpr int kRingOff = kMaxWBytes;  // weights first (only w_bytes of it used)
constexpr int kBarOff = kRingOff + kRowSlots * kSlotBytes;
constexpr int kNumBars = 1 + 2 * kRowSlots + 2 * kRowAcc + 1;
constexpr int kMiscOff = kBarOff + kNumBars * 8;
constexpr int kBiasOff = (kMiscOff + 16 + 15) & ~15;
constexpr int kSmemBytes = kBiasOff + 64 * 4 + 1024;
static_assert(kSmemBytes <= 232448, "row kernel shared memory above 227 KB");

// One segment of a CTA's units: image n, conv rows lo..hi.
struct Seg {
  int n, lo, hi;
};

// Next segment of the unit range [u, u1); advances u.
__device__ __forceinline__ bool next_seg(const RowParams& p, int& u, int u1, Seg& s) {
  if (u >= u1) return false;
  const int per = p.pool ? p.PH : p.OH;
  const int n = u / per;
  const int a = u - n * per;
  const int e = min(per, a + (u1 - u));
  s.n = n;
  if (p.pool) {
    // pooled row py covers conv rows 2py-1 .. 2py+1 (inside the image)
    s.lo = max(2 * a - 1, 0);
    s.hi = min(2 * e - 1, p.OH - 1);
  } else {
    s.lo = a;
    s.hi = e - 1;
  }
  u += e - a;
  return true;
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int ACT>
__device__ __forceinline__ float act_f(float v) {
  if (ACT == 1) return fmaxf(v, 0.0f);
  if (ACT == 2) return 1.0f / (1.0f + expf(-v));
  return v;
}

__device__ __forceinline__ uint32_t hmax2_u32(uint32_t a, uint32_t b) {
  __half2 x = *reinterpret_cast<__half2*>(&a), y = *reinterpret_cast<__half2*>(&b);
  __half2 m = __hmax2(x, y);
  return *reinterpret_cast<uint32_t*>(&m);
}
constexpr uint32_t kNegInf2 = 0xFC00FC00u;  // two fp16 -inf

// Epilogue warps.  Each thread keeps its 16 bias values in registers.
// Without the pool: act(acc + bias) -> fp16 store of the conv row.  With the
// pool: fp16(acc + bias) per conv row, the 3x3 window max on those fp16
// values (vertical in registers, horizontal by warp shuffles once per pooled
// row), then the activation of the pooled value.  Rounding to fp16 and the
// ReLU / identity activations are non-decreasing and ReLU commutes with the
// rounding, so this equals pooling the conv output the unfused kernels store,
// bit for bit (a sigmoid activation is applied to the rounded maximum).
//
// With the pool each TMEM lane quarter q holds its own overlapping range of
// conv columns, ox = qspan * q - 1 + lane (the producer lands A rows that
// way), so all three columns of every window it pools lie in the same warp:
// odd lanes 1, 3, .., qspan - 1 are the window centres (even ox) of pooled
// columns qpool * q .. qpool * q + qpool - 1.  Columns outside the conv map
// (ox = -1 on the left, ox >= OW) are the pool's -inf padding.  No warp
// waits for another.
//
// A drained accumulator block is zeroed with tcgen05.st right after it is
// read and released (wait::st, arrival on tempty) one tile later, after the
// next tile's TMEM load: the store completes under this tile's arithmetic.
// fp32 bias adds use the packed two-lane add (same rounding as two scalar
// adds).
template <int ACT>
__device__ __forceinline__ void epilogue(const RowParams& p, uint64_t* tfull, uint64_t* tempty, const float* s_bias,
                                         volatile int* abort_flag, uint32_t tmem_base, int u0, int u1) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3, cg = warp >> 2;
  const int ox = p.pool ? p.qspan * q - 1 + lane : kRowBox * q + lane;
  const bool xvalid = ox >= 0 && ox < p.OW;
  const int px = p.qpool * q + (lane >> 1);  // pooled column centred here (odd lanes)
  const bool centre = (lane & 1) != 0 && (lane >> 1) < p.qpool && px < p.PW;
  const int c0 = cg * kEpiCols;
  const bool pad = c0 + kEpiCols > p.Cout;  // this warp's columns reach past Cout (warp-uniform)
  float2 bias[kEpiCols / 2];
#pragma unroll
  for (int k = 0; k < kEpiCols / 2; ++k) bias[k] = make_float2(s_bias[c0 + 2 * k], s_bias[c0 + 2 * k + 1]);
  const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
  uint32_t carry[kEpiCols / 2], vmax[kEpiCols / 2];
#pragma unroll
  for (int k = 0; k < kEpiCols / 2; ++k) carry[k] = vmax[k] = kNegInf2;
  // every accumulator block starts at zero (the MMAs always accumulate)
#pragma unroll 1
  for (int b = 0; b < kRowAcc; ++b) tmem_st_zero_32x32b_x16(tmem_base + t_lane + b * 64 + c0);
  tmem_st_wait();
  tc_fence_before();
  __syncwarp();
  if (lane == 0)
    for (int b = 0; b < kRowAcc; ++b) mbar_arrive(&tempty[b]);
  int lt = 0;
  int pend = -1;  // block whose zeros are in flight, released after the next load
  int u = u0;
  Seg sg;
  while (next_seg(p, u, u1, sg)) {
    bool carry_ok = false;
    for (int oy = sg.lo; oy <= sg.hi; ++oy, ++lt) {
      const int ab = acc_block(lt);
      bool ok = true;
      if (lane == 0) ok = !*abort_flag && mbar_wait(&tfull[ab], (lt / kRowAcc) & 1, kErrWaitAccum, p.wait_limit);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      tc_fence_after();
      uint32_t r[kEpiCols];
      const uint32_t ta = tmem_base + t_lane + ab * 64 + c0;
      if (ok) {
        tmem_ld_32x32b_x16(ta, r);
        tmem_ld_wait();
      }
      if (pend >= 0) {  // the previous tile's block: its zeros are written
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[pend]);
      }
      if (ok) tmem_st_zero_32x32b_x16(ta);  // ready for tile lt + kRowAcc
      pend = ab;
      if (lane == 0 && !ok) *abort_flag = 1;
      if (!p.pool) {
        if (ok && xvalid) {
          uint32_t h[kEpiCols / 2];
#pragma unroll
          for (int k = 0; k < kEpiCols / 2; ++k) {
            const float2 v = __fadd2_rn(make_float2(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1])), bias[k]);
            float f0 = act_f<ACT>(v.x);
            float f1 = act_f<ACT>(v.y);
            if (pad && c0 + 2 * k >= p.Cout) f0 = 0.f;  // pad channels stay zero
            if (pad && c0 + 2 * k + 1 >= p.Cout) f1 = 0.f;
            h[k] = pack2(f0, f1);
          }
          __half* dst = p.y + ((static_cast<int64_t>(sg.n) * p.OH + oy) * p.OW + ox) * p.Cs_out + c0;
#pragma unroll
          for (int s = 0; s < kEpiCols / 8; ++s)
            if (c0 + 8 * s < p.Cs_out)
              *reinterpret_cast<uint4*>(dst + 8 * s) = make_uint4(h[4 * s], h[4 * s + 1], h[4 * s + 2], h[4 * s + 3]);
        }
      } else {
        // fp16(acc + bias) of this conv row; -inf outside the map (garbage
        // when !ok: never stored)
        uint32_t h[kEpiCols / 2];
#pragma unroll
        for (int k = 0; k < kEpiCols / 2; ++k) {
          const float2 v = __fadd2_rn(make_float2(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1])), bias[k]);
          h[k] = xvalid ? pack2(v.x, v.y) : kNegInf2;
        }
        // vertical max first, in registers (a thread always holds the same
        // ox and channels): carried row 2py-1, then 2py, then 2py+1
        bool close = false;  // this row completes a pooled row of the segment
        if (oy & 1) {
          if (oy != sg.lo) {  // (else it only carries into the segment's first pooled row)
#pragma unroll
            for (int k = 0; k < kEpiCols / 2; ++k) vmax[k] = hmax2_u32(vmax[k], h[k]);
            close = true;
          }
#pragma unroll
          for (int k = 0; k < kEpiCols / 2; ++k) carry[k] = h[k];
          carry_ok = true;
        } else {
#pragma unroll
          for (int k = 0; k < kEpiCols / 2; ++k) vmax[k] = carry_ok ? hmax2_u32(carry[k], h[k]) : h[k];
          close = oy == p.OH - 1;  // an odd-height map's last pooled row has no row below
        }
        if (close) {
          // horizontal 3-wide max at the centre lanes (ox - 1, ox, ox + 1 are
          // lanes l - 1, l, l + 1 of this warp)
          uint32_t o[kEpiCols / 2];
#pragma unroll
          for (int k = 0; k < kEpiCols / 2; ++k)
            o[k] = hmax2_u32(hmax2_u32(__shfl_up_sync(0xffffffffu, vmax[k], 1), vmax[k]),
                             __shfl_down_sync(0xffffffffu, vmax[k], 1));
          if (ok && centre) {
            if (ACT == 1) {
#pragma unroll
              for (int k = 0; k < kEpiCols / 2; ++k) o[k] = hmax2_u32(o[k], 0u);
            } else if (ACT == 2) {
#pragma unroll
              for (int k = 0; k < kEpiCols / 2; ++k) {
                const float2 f = __half22float2(*reinterpret_cast<__half2*>(&o[k]));
                o[k] = pack2(act_f<2>(f.x), act_f<2>(f.y));
              }
            }
            if (pad) {
#pragma unroll
              for (int k = 0; k < kEpiCols / 2; ++k) {
                if (c0 + 2 * k >= p.Cout) o[k] &= 0xFFFF0000u;  // pad channels stay zero
                if (c0 + 2 * k + 1 >= p.Cout) o[k] &= 0x0000FFFFu;
              }
            }
            __half* dst = p.y + ((static_cast<int64_t>(sg.n) * p.PH + (oy >> 1)) * p.PW + px) * p.Cs_out + c0;
#pragma unroll
            for (int s = 0; s < kEpiCols / 8; ++s)
              if (c0 + 8 * s < p.Cs_out)
                *reinterpret_cast<uint4*>(dst + 8 * s) =
                    make_uint4(o[4 * s], o[4 * s + 1], o[4 * s + 2], o[4 * s + 3]);
          }
        }
      }
    }
  }
  if (pend >= 0) {
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&tempty[pend]);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
conv_row_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                const RowParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* ring = smem + kRingOff;
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* rfull = wfull + 1;
  uint64_t* rempty = rfull + kRowSlots;
  uint64_t* tfull = rempty + kRowSlots;
  uint64_t* tempty = tfull + kRowAcc;
  uint64_t* mma_done = tempty + kRowAcc;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kMiscOff + 4);
  float* s_bias = reinterpret_cast<float*>(smem + kBiasOff);

  // warp index through a shuffle: the compiler then knows it is warp-uniform
  const int tid = threadIdx.x, warp = __shfl_sync(0xffffffffu, tid >> 5, 0), lane = tid & 31;
  // this CTA's units [u0, u1) (pooled rows or conv rows over the batch)
  const int u0 = static_cast<int>(static_cast<int64_t>(p.units) * blockIdx.x / gridDim.x);
  const int u1 = static_cast<int>(static_cast<int64_t>(p.units) * (blockIdx.x + 1) / gridDim.x);

  if (tid == 0) {
    mbar_init(wfull, 1);
    for (int s = 0; s < kRowSlots; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], 1);
    }
    for (int b = 0; b < kRowAcc; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (tid < 64) s_bias[tid] = (p.bias != nullptr && tid < p.Cout) ? __ldg(p.bias + tid) : 0.f;
  if (warp == kProducer && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == kIssuer) {
    tmem_alloc(tmem_slot, kRowAcc * 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (tid == 0) griddep_launch();  // set-up done: the next kernel may start being scheduled

  if (warp < kEpiWarps) {
    griddep_wait();  // its output buffer may still be in use by earlier kernels
    if (p.act == 1)
      epilogue<1>(p, tfull, tempty, s_bias, abort_flag, tmem_base, u0, u1);
    else if (p.act == 0)
      epilogue<0>(p, tfull, tempty, s_bias, abort_flag, tmem_base, u0, u1);
    else
      epilogue<2>(p, tfull, tempty, s_bias, abort_flag, tmem_base, u0, u1);
  } else if (warp == kProducer) {
    if (lane == 0) {
      bool ok = true;
      mbar_arrive_expect_tx(wfull, static_cast<uint32_t>(p.w_bytes));
      for (int r = 0; r < p.kh; ++r) tma_load_2d(sW + r * kWBlockBytes, &tmap_w, wfull, r * 64, 0);
      griddep_wait();  // the weights do not depend on earlier kernels; the input rows do
      uint32_t L = 0;
      int u = u0;
      Seg sg;
      const int x0 = p.pool ? -1 : 0, qstep = p.pool ? p.qspan : kRowBox;
      while (ok && next_seg(p, u, u1, sg)) {
        for (int yin = sg.lo; yin <= sg.hi + p.kh - 1; ++yin, ++L) {
          const uint32_t slot = L % kRowSlots;
          if (*abort_flag ||
              !mbar_wait(&rempty[slot], ((L / kRowSlots) & 1) ^ 1, kErrWaitEmpty, p.wait_limit)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&rfull[slot], kSlotBytes);
          // one 32-position box per TMEM lane quarter (pixel -1 and pixels
          // >= OW read as zeros)
          for (int qq = 0; qq < kRowPos / kRowBox; ++qq)
            tma_load_4d(ring + slot * kSlotBytes + qq * (kSlotBytes / 4), &tmap_x, &rfull[slot], 0, x0 + qq * qstep,
                        yin, sg.n);
        }
      }
      if (!ok) *abort_flag = 1;
      // every TMA load this thread issued has landed before the CTA may exit
      mbar_wait(wfull, 0, kErrWaitFull, p.wait_limit);
      for (int64_t j = static_cast<int64_t>(L) - 1; j >= 0 && j >= static_cast<int64_t>(L) - kRowSlots; --j)
        mbar_wait(&rfull[j % kRowSlots], static_cast<uint32_t>(j / kRowSlots) & 1, kErrWaitFull, p.wait_limit);
    }
  } else if (warp == kGate) {
    // Does every mbarrier wait the MMAs need and hands each input row to the
    // issuer through a named barrier (an mbarrier wait in the issuing warp
    // would be held behind its queued MMAs): the tile the row starts is
    // drained and zeroed, the row's slot is full.  One hand-off per input
    // row, also after an error (then with ok = false), so the two warps
    // always meet the same number of times.
    bool ok = true;
    if (lane == 0) ok = mbar_wait(wfull, 0, kErrWaitFull, p.wait_limit);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    uint32_t L = 0;
    int lt0 = 0;
    int u = u0;
    Seg sg;
    while (next_seg(p, u, u1, sg)) {
      const int ntiles = sg.hi - sg.lo + 1;
      for (int i = 0; i < ntiles + p.kh - 1; ++i, ++L) {
        const int ly = lt0 + i;
        if (lane == 0 && ok) {
          if (i < ntiles) ok = mbar_wait(&tempty[acc_block(ly)], (ly / kRowAcc) & 1, kErrWaitAccum, p.wait_limit);
          if (ok) ok = mbar_wait(&rfull[L % kRowSlots], (L / kRowSlots) & 1, kErrWaitFull, p.wait_limit);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok && lane == 0) *abort_flag = 1;
        bar_red_and(kRowBar, 64, ok);
      }
      lt0 += ntiles;
    }
  } else if (warp == kIssuer) {
    // The whole warp runs this loop (every value in it is warp-uniform); one
    // elected lane issues the MMAs and commits.  It waits on nothing but the
    // gate's per-row hand-off.
    bool ok = true;
    uint32_t L = 0;  // input rows consumed (ring position)
    int lt0 = 0;     // the segment's first tile
    int u = u0;
    Seg sg;
    const uint64_t b_base = make_sdesc_sw128(smem_u32(sW));
    while (next_seg(p, u, u1, sg)) {
      const int ntiles = sg.hi - sg.lo + 1;
      for (int i = 0; i < ntiles + p.kh - 1; ++i, ++L) {
        // input row sg.lo + i; it feeds tiles lt0 + i - j for kernel rows
        // j in [j_lo, j_hi] (the tiles of this segment)
        ok = bar_red_and(kRowBar, 64, true) && ok;
        if (!ok) continue;
        tc_fence_after();
        const int ly = lt0 + i;
        const uint32_t slot = L % kRowSlots;
        const uint64_t a_desc = make_sdesc_sw128(smem_u32(ring + slot * kSlotBytes));
        const int j_hi = min(p.kh - 1, i);
        const int blk0 = acc_block(ly);
        for (int j = max(0, i - (ntiles - 1)); j <= j_hi;) {
          // a run of blocks that neither wraps past block 7 nor exceeds N = 256
          const int blk = (blk0 + j) & (kRowAcc - 1);
          const int len = min(min(j_hi - j + 1, kRowAcc - blk), 4);
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(blk * 64);
          const uint64_t b_desc = b_base + static_cast<uint32_t>(j * (kWBlockBytes >> 4));
          const uint32_t idesc = make_idesc_f16_m128(static_cast<uint32_t>(len * 64));
          if (elect_one()) {
#pragma unroll
            for (int k = 0; k < 4; ++k)  // K step = 32 bytes = 2 start-address units
              umma_f16(d_tmem, a_desc + 2u * k, b_desc + 2u * k, idesc, 1u);
          }
          __syncwarp();
          j += len;
        }
        if (elect_one()) {
          umma_commit(&rempty[slot]);
          if (i >= p.kh - 1) umma_commit(&tfull[acc_block(ly - (p.kh - 1))]);  // its last input row
        }
        __syncwarp();
      }
      lt0 += ntiles;
    }
    // every MMA has completed once mma_done fires
    if (elect_one()) umma_commit(mma_done);
    __syncwarp();
    mbar_wait(mma_done, 0, kErrWaitFull, p.wait_limit);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kIssuer) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kRowAcc * 64);
  }
}

// Input rows of the NHWC activation as 64-value runs: element (e, x, y, n)
// is x[n, y, x + e / Cs_in, e % Cs_in], so dimension 0 (64 contiguous fp16 =
// kw pixels) overlaps the next pixel's run (stride Cs_in * 2 bytes).  Box
// {64, 32, 1, 1} = 4 KB (one TMEM lane quarter's A rows), 128B swizzle (inner
// box = swizzle span); x < OW keeps every run inside its image row, x >= OW
// and x = -1 read zeros.
int make_row_map(CUtensorMap* map, const ConvRowArgs& a, int ow) {
  auto enc = encode_tiled();
  if (!enc) return -1;
  const cuuint64_t px = static_cast<cuuint64_t>(a.Cs_in) * 2;
  cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(ow), static_cast<cuuint64_t>(a.H), static_cast<cuuint64_t>(a.N)};
  cuuint64_t strides[3] = {px, px * a.W, px * a.W * a.H};
  cuuint32_t box[4] = {64, kRowBox, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(a.x), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

int make_weight_map(CUtensorMap* map, const ConvRowArgs& a) {
  auto enc = encode_tiled();
  if (!enc) return -1;
  const int k_pad = a.kh * 64;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k_pad), static_cast<cuuint64_t>(a.Cout)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(k_pad) * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.w_packed), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

}  // namespace

int conv_row_check(const ConvRowArgs& a, const char** err) {
  if (a.Cs_in * a.kw != 64 || a.Cs_in % 8 != 0) {
    *err = "row conv: needs Cs_in * kw == 64";
    return -2;
  }
  if (a.kh < 1 || a.kh > kRowMaxKh || a.H < a.kh || a.W < a.kw) {
    *err = "row conv: kernel height outside 1..6 or larger than the input";
    return -2;
  }
  const int ow = a.W - a.kw + 1;
  if (ow > kRowPos) {
    *err = "row conv: output rows longer than 128 pixels";
    return -2;
  }
  if (a.Cout < 1 || a.Cout > 64 || a.Cs_out != (a.Cout + 7) / 8 * 8) {
    *err = "row conv: 1..64 output channels";
    return -2;
  }
  if (a.pool != 0 && a.pool != 1) {
    *err = "row conv: unknown pool";
    return -2;
  }
  if (a.pool == 1 && (ow - 1) / 2 + 1 > (kRowPos / kRowBox) * kRowMaxQPool) {
    *err = "row conv: pooled rows longer than 60 pixels";
    return -2;
  }
  if (static_cast<int64_t>(a.N) * (a.H - a.kh + 1) > 0x7FFFFFFF) {
    *err = "row conv: too many rows";
    return -2;
  }
  return 0;
}

int conv_row_launch(const ConvRowArgs& a, cudaStream_t stream, const char** err) {
  if (conv_row_check(a, err) != 0) return -2;
  RowParams p{};
  p.bias = a.bias;
  p.y = static_cast<__half*>(a.y);
  p.N = a.N;
  p.OH = a.H - a.kh + 1;
  p.OW = a.W - a.kw + 1;
  p.Cout = a.Cout;
  p.Cs_out = a.Cs_out;
  p.kh = a.kh;
  p.act = a.act;
  p.pool = a.pool;
  p.PH = (p.OH - 1) / 2 + 1;
  p.PW = (p.OW - 1) / 2 + 1;
  p.units = a.N * (a.pool ? p.PH : p.OH);
  p.w_bytes = a.kh * kWBlockBytes;
  p.qpool = (p.PW + (kRowPos / kRowBox) - 1) / (kRowPos / kRowBox);
  p.qspan = 2 * p.qpool;
  p.wait_limit = wait_limit_from_env();

  CUtensorMap mw, mx;
  if (make_weight_map(&mw, a) != 0) {
    *err = "row conv: weight tensor map encoding failed";
    return -3;
  }
  if (make_row_map(&mx, a, p.OW) != 0) {
    *err = "row conv: input-row tensor map encoding failed";
    return -2;
  }

  static std::atomic<uint64_t> attr_ctx[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *err = "row conv: no usable device";
    return -3;
  }
  const uint64_t ctx = current_context_id();
  if (ctx == 0 || attr_ctx[dev].load(std::memory_order_acquire) != ctx) {
    const cudaError_t ae = cudaFuncSetAttribute(conv_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                kSmemBytes);
    if (ae != cudaSuccess) {
      *err = cudaGetErrorString(ae);
      return -3;
    }
    attr_ctx[dev].store(ctx, std::memory_order_release);
  }
  const int grid = std::min(num_sms(), p.units);
  cudaError_t e = launch_pdl(conv_row_kernel, dim3(grid), dim3(kThreads), kSmemBytes, stream, mw, mx, p);
  note_launch();
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = cudaGetErrorString(e);
    return -3;
  }
  return 0;
}

int conv_row_read_device_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, lotus_dev::g_lotus_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) {
    int zero = 0;
    cudaMemcpyToSymbol(lotus_dev::g_lotus_device_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace lotus_impl
