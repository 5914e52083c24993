// Row-stacked convolution on sm_100a tensor cores for stride-1 convs over
// 64-channel NHWC inputs with at most 64 output channels and kernels up to
// 3x3 (ResNet-18 stage 1: 56x56, 64 -> 64 channels, 3x3, pad 1, with and
// without the folded residual add), output rows of at most 64 pixels (two
// images share a tile) or 128 pixels (one image a tile).
//
// The reference runs these layers as per-sample launches of its fp32 conv
// kernel (source/operator/conv2d.cu:17-187 from source/layer/layer_conv2d.cu:
// 43-70) followed by the Expression add + ReLU layer (source/layer/
// expression.cu:29-50) for the residual.
//
// GEMM view.  A tile is one output row oy of `ipt` images (ipt = 2 when
// OW + kw - 1 <= 64: A rows / TMEM lanes 0-63 hold image 2g, 64-127
// image 2g+1; ipt = 1: lanes 0-127 hold one image's row).  M = 128
// positions, N = Cout (<= 64), K = kh * kw * 64 channels.  Tap (j, s) of
// output row oy reads input row oy - ph + j at pixels ox + s - pw.
//
// A operands: per input row y the producer lands one 160-row slot (64
// channels a row, 128B-swizzled, 1024-aligned): with two images a tile, rows
// 0-63 hold pixels -pw .. 63-pw of image 2g and rows 64-159 pixels -pw ..
// 95-pw of image 2g+1; with one image, rows 0-159 hold pixels -pw .. 159-pw.
// Pixels outside the row (the left / right zero padding) and images past the
// batch read as zeros.  Tap column s is the same slot with the descriptor
// start moved by s rows (lane i reads slot row i + s = pixel ox + s - pw); a
// start inside a 1024-byte swizzle atom reads what the TMA wrote, since the
// swizzle is a function of the address, and costs no MMA throughput.  The
// two extra rows of image 2g's half are read only by lanes past OW.  Every
// input row is loaded once and read by one MMA group per tap column.
//
// Stacked weights, as in the stem's row kernel: input row y feeds output
// rows y + ph - j through kernel rows j = 0..kh-1.  The kh weight blocks of
// tap column s lie one after the other in shared memory (block s * kh + j),
// forming one B operand of N = kh * 64; the accumulators sit in a TMEM ring
// of 8 blocks of 64 columns at descending positions (tile t uses block
// 7 - t % 8), so the blocks of output rows y + ph, y + ph - 1, .. are
// ascending and contiguous up to a wrap past block 7, where the MMA splits.
// The input rows above and below the map (the vertical zero padding) are
// never loaded: their MMAs would add zeros.  Each accumulator is zeroed by
// the epilogue (tcgen05.st) when drained and the MMAs always accumulate, so
// one output pixel sums its taps in (j, s, k) order as a plain tap loop.
//
// Roles (608 threads): warps 0-15 epilogue (warp w drains TMEM lane quarter
// w % 4, columns 16 * (w / 4) .. +15: bias, residual, activation, fp16
// store), warp 16 TMEM allocation and MMA issue (warp-uniform loop, one
// elected lane issues; it waits on no mbarrier), warp 17 TMA producer
// (weights once, then input rows), warp 18 the gate: it does the MMAs'
// mbarrier waits and hands each input row to the issuer through a named
// barrier.
// Each CTA owns a contiguous range of units (image group, output row) walked
// as per-group segments.
//
// Barriers (all waits bounded): rfull / rempty per A-tile slot, tfull /
// tempty per TMEM block (the first tempty phase completes after the initial
// zeroing; a block is released one tile after it was drained), wfull for the
// weights.  The gate acquires a block when the first input row of its tile
// arrives; the issuer commits tfull after the tile's last input row; block P(t) is
// reused by tile t + 8 only after tile t + 1 was loaded by the epilogue,
// which needs input rows up to t + 1 - ph + kh - 1 < t + 8 - ph.
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

constexpr int kPos = 128;                  // A rows (positions) per tile
constexpr int kBox = 32;                   // positions per TMA box
constexpr int kSlotRows = kPos + kBox;     // A rows of a slot: 128 + room for the tap shifts
constexpr int kSlotBytes = kSlotRows * 128; // 20 KB
constexpr int kAcc = 8;                    // TMEM accumulator blocks of 64 columns
constexpr int kMaxK = 3;                   // kh, kw <= 3
constexpr int kWBlock = 64 * 128;          // 64 output channels x 64 K (one tap)
constexpr int kMaxSlots = 16;
constexpr int kEpiWarps = 16;
constexpr int kEpiCols = 64 / (kEpiWarps / 4);
constexpr int kIssuer = kEpiWarps, kProducer = kEpiWarps + 1, kGate = kEpiWarps + 2;
constexpr int kThreads = (kEpiWarps + 3) * 32;
constexpr uint32_t kRowBar = 1;  // named barrier of the gate / issuer hand-off (0 is __syncthreads)
constexpr int kHeadBytes = 1024;           // barriers, misc words, bias
constexpr int kSmemLimit = 232448;         // 227 KB opt-in

__device__ __forceinline__ int acc_block(int t) { return (kAcc - 1) - (t & (kAcc - 1)); }

struct RsParams {
  const float* bias;
  const __half* residual;  // NHWC [N, OH, OW, Cs_out] or null
  __half* y;               // NHWC [N, OH, OW, Cs_out]
  int N, H, OH, OW, Cout, Cs_out, kh, kw, ph, pw, act;
  int ipt;                 // images per tile (1 or 2)
  int units;               // ceil(N / ipt) * OH
  int slots;               // input-row ring slots
  int w_bytes;             // kh * kw * kWBlock
  uint32_t wait_limit;
};

// One segment of a CTA's units: image group g, output rows lo..hi.
struct Seg {
  int g, lo, hi;
};

__device__ __forceinline__ bool next_seg(const RsParams& p, int& u, int u1, Seg& s) {
  if (u >= u1) return false;
  const int g = u / p.OH;
  const int a = u - g * p.OH;
  const int e = min(p.OH, a + (u1 - u));
  s.g = g;
  s.lo = a;
  s.hi = e - 1;
  u += e - a;
  return true;
}

// Input rows a segment reads: [y_lo, y_hi] (the padding rows are skipped).
__device__ __forceinline__ int seg_ylo(const RsParams& p, const Seg& s) { return max(0, s.lo - p.ph); }
__device__ __forceinline__ int seg_yhi(const RsParams& p, const Seg& s) {
  return min(p.H - 1, s.hi - p.ph + p.kh - 1);
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

// Epilogue warps: out = act((acc + bias) + residual) in fp32 (the general
// conv kernel's order), fp16 store; pad channels zero.  The residual of a
// tile is read before its accumulator wait.  Drained blocks are zeroed and
// released one tile later (the store completes under the next tile's load).
template <int ACT, bool RES>
__device__ __forceinline__ void epilogue(const RsParams& p, uint64_t* tfull, uint64_t* tempty, const float* s_bias,
                                         volatile int* abort_flag, uint32_t tmem_base, int u0, int u1) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3, cg = warp >> 2;
  const int per = kPos / p.ipt;  // positions per image in a tile
  const int pos = q * 32 + lane;
  const int h = pos / per, ox = pos - h * per;
  const int c0 = cg * kEpiCols;
  const bool pad = c0 + kEpiCols > p.Cout;  // warp-uniform
  const bool cols = c0 < p.Cs_out;          // this warp's columns hold stored channels (warp-uniform)
  const bool two = c0 + 8 < p.Cs_out;       // ... and the second 8 of them
  float2 bias[kEpiCols / 2];
#pragma unroll
  for (int k = 0; k < kEpiCols / 2; ++k) bias[k] = make_float2(s_bias[c0 + 2 * k], s_bias[c0 + 2 * k + 1]);
  const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
#pragma unroll 1
  for (int b = 0; b < kAcc; ++b) tmem_st_zero_32x32b_x16(tmem_base + t_lane + b * 64 + c0);
  tmem_st_wait();
  tc_fence_before();
  __syncwarp();
  if (lane == 0)
    for (int b = 0; b < kAcc; ++b) mbar_arrive(&tempty[b]);
  int lt = 0, pend = -1;
  int u = u0;
  Seg sg;
  while (next_seg(p, u, u1, sg)) {
    const int n = sg.g * p.ipt + h;
    const bool valid = n < p.N && ox < p.OW && cols;
    const int64_t pix0 = static_cast<int64_t>(n) * p.OH * p.OW + ox;
    for (int oy = sg.lo; oy <= sg.hi; ++oy, ++lt) {
      const int ab = acc_block(lt);
      const int64_t off = (pix0 + static_cast<int64_t>(oy) * p.OW) * p.Cs_out + c0;
      uint4 rv[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
      if (RES && valid) {
        rv[0] = __ldg(reinterpret_cast<const uint4*>(p.residual + off));
        if (two) rv[1] = __ldg(reinterpret_cast<const uint4*>(p.residual + off + 8));
      }
      bool ok = true;
      if (lane == 0) ok = !*abort_flag && mbar_wait(&tfull[ab], (lt / kAcc) & 1, kErrWaitAccum, p.wait_limit);
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
      if (ok) tmem_st_zero_32x32b_x16(ta);  // ready for tile lt + kAcc
      pend = ab;
      if (lane == 0 && !ok) *abort_flag = 1;
      if (!(ok && valid)) continue;
      uint32_t o[kEpiCols / 2];
      const __half2* rh = reinterpret_cast<const __half2*>(rv);
#pragma unroll
      for (int k = 0; k < kEpiCols / 2; ++k) {
        float2 v = __fadd2_rn(make_float2(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1])), bias[k]);
        if (RES) v = __fadd2_rn(v, __half22float2(rh[k]));
        float f0 = act_f<ACT>(v.x), f1 = act_f<ACT>(v.y);
        if (pad && c0 + 2 * k >= p.Cout) f0 = 0.f;  // pad channels stay zero
        if (pad && c0 + 2 * k + 1 >= p.Cout) f1 = 0.f;
        o[k] = pack2(f0, f1);
      }
      __half* dst = p.y + off;
      *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
      if (two) *reinterpret_cast<uint4*>(dst + 8) = make_uint4(o[4], o[5], o[6], o[7]);
    }
  }
  if (pend >= 0) {
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&tempty[pend]);
  }
}

// The residual add compiled in or out (as in the pair kernel's epilogue).
template <int ACT>
__device__ __forceinline__ void epilogue_act(const RsParams& p, uint64_t* tfull, uint64_t* tempty,
                                             const float* s_bias, volatile int* abort_flag, uint32_t tmem_base,
                                             int u0, int u1) {
  if (p.residual != nullptr)
    epilogue<ACT, true>(p, tfull, tempty, s_bias, abort_flag, tmem_base, u0, u1);
  else
    epilogue<ACT, false>(p, tfull, tempty, s_bias, abort_flag, tmem_base, u0, u1);
}

__global__ void __launch_bounds__(kThreads, 1)
conv_rows_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                 const RsParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem);
  uint64_t* rfull = wfull + 1;
  uint64_t* rempty = rfull + kMaxSlots;
  uint64_t* tfull = rempty + kMaxSlots;
  uint64_t* tempty = tfull + kAcc;
  uint64_t* mma_done = tempty + kAcc;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 448);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 452);
  float* s_bias = reinterpret_cast<float*>(smem + 512);
  uint8_t* sW = smem + kHeadBytes;
  uint8_t* ring = sW + p.w_bytes;

  // warp index through a shuffle: the compiler then knows it is warp-uniform
  const int tid = threadIdx.x, warp = __shfl_sync(0xffffffffu, tid >> 5, 0), lane = tid & 31;
  const int u0 = static_cast<int>(static_cast<int64_t>(p.units) * blockIdx.x / gridDim.x);
  const int u1 = static_cast<int>(static_cast<int64_t>(p.units) * (blockIdx.x + 1) / gridDim.x);

  if (tid == 0) {
    mbar_init(wfull, 1);
    for (int s = 0; s < p.slots; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], 1);
    }
    for (int b = 0; b < kAcc; ++b) {
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
    tmem_alloc(tmem_slot, kAcc * 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (tid == 0) griddep_launch();  // set-up done: the next kernel may start being scheduled

  if (warp < kEpiWarps) {
    griddep_wait();  // residual and output buffers belong to earlier kernels
    if (p.act == 1)
      epilogue_act<1>(p, tfull, tempty, s_bias, abort_flag, tmem_base, u0, u1);
    else if (p.act == 0)
      epilogue_act<0>(p, tfull, tempty, s_bias, abort_flag, tmem_base, u0, u1);
    else
      epilogue_act<2>(p, tfull, tempty, s_bias, abort_flag, tmem_base, u0, u1);
  } else if (warp == kProducer) {
    if (lane == 0) {
      bool ok = true;
      // weight block of kernel row j, tap column s at block s * kh + j
      mbar_arrive_expect_tx(wfull, static_cast<uint32_t>(p.w_bytes));
      for (int s = 0; s < p.kw; ++s)
        for (int j = 0; j < p.kh; ++j)
          tma_load_2d(sW + (s * p.kh + j) * kWBlock, &tmap_w, wfull, (j * p.kw + s) * 64, 0);
      griddep_wait();  // the weights do not depend on earlier kernels; the input rows do
      uint32_t L = 0;
      int u = u0;
      Seg sg;
      while (ok && next_seg(p, u, u1, sg)) {
        const int yhi = seg_yhi(p, sg);
        for (int y = seg_ylo(p, sg); y <= yhi; ++y, ++L) {
          const uint32_t slot = L % p.slots;
          if (*abort_flag || !mbar_wait(&rempty[slot], ((L / p.slots) & 1) ^ 1, kErrWaitEmpty, p.wait_limit)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&rfull[slot], kSlotBytes);
          // five 32-row boxes: two for image 2g and three for image 2g+1,
          // or five of one image (the padding columns and images past the
          // batch read as zeros)
          for (int b = 0; b < kSlotRows / kBox; ++b) {
            const int hh = (p.ipt == 2 && b >= 2) ? 1 : 0;
            const int x = (b - 2 * hh) * kBox - p.pw;
            tma_load_4d(ring + slot * kSlotBytes + b * (kBox * 128), &tmap_x, &rfull[slot], 0, x, y,
                        sg.g * p.ipt + hh);
          }
        }
      }
      if (!ok) *abort_flag = 1;
      // every TMA load this thread issued has landed before the CTA may exit
      mbar_wait(wfull, 0, kErrWaitFull, p.wait_limit);
      for (int64_t j = static_cast<int64_t>(L) - 1; j >= 0 && j >= static_cast<int64_t>(L) - p.slots; --j)
        mbar_wait(&rfull[j % p.slots], static_cast<uint32_t>(j / p.slots) & 1, kErrWaitFull, p.wait_limit);
    }
  } else if (warp == kGate) {
    // Does every mbarrier wait the MMAs need and hands each input row to the
    // issuer through a named barrier (an mbarrier wait in the issuing warp
    // would be held behind its queued MMAs): the tiles the row starts are
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
      const int yhi = seg_yhi(p, sg);
      int next_acq = 0;
      for (int y = seg_ylo(p, sg); y <= yhi; ++y, ++L) {
        const int top = y + p.ph - sg.lo;
        const int j_lo = max(0, top - (ntiles - 1));
        if (lane == 0 && ok) {
          for (; ok && next_acq <= top - j_lo; ++next_acq) {
            const int t = lt0 + next_acq;
            ok = mbar_wait(&tempty[acc_block(t)], (t / kAcc) & 1, kErrWaitAccum, p.wait_limit);
          }
          if (ok) ok = mbar_wait(&rfull[L % p.slots], (L / p.slots) & 1, kErrWaitFull, p.wait_limit);
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
    uint32_t L = 0;  // input rows consumed (ring position)
    int lt0 = 0;     // the segment's first tile
    int u = u0;
    Seg sg;
    bool ok = true;
    const uint64_t b_base = make_sdesc_sw128(smem_u32(sW));
    while (next_seg(p, u, u1, sg)) {
      const int ntiles = sg.hi - sg.lo + 1;
      const int yhi = seg_yhi(p, sg);
      int next_done = 0;  // tiles (segment-relative) committed so far
      for (int y = seg_ylo(p, sg); y <= yhi; ++y, ++L) {
        // input row y feeds tiles top - j (top = the tile of kernel row 0),
        // kernel rows j in [j_lo, j_hi] that land inside the segment
        const int top = y + p.ph - sg.lo;
        const int j_lo = max(0, top - (ntiles - 1)), j_hi = min(p.kh - 1, top);
        ok = bar_red_and(kRowBar, 64, true) && ok;
        if (!ok) continue;
        tc_fence_after();
        const int blk0 = acc_block(lt0 + top);
        const uint32_t slot = L % p.slots;
        const uint64_t a_slot = make_sdesc_sw128(smem_u32(ring + slot * kSlotBytes));
        for (int s = 0; s < p.kw; ++s) {
          const uint64_t a_desc = a_slot + static_cast<uint32_t>(s * (128 >> 4));  // s rows in
          for (int j = j_lo; j <= j_hi;) {
            // a run of blocks that neither wraps past block 7 nor exceeds N = 256
            const int blk = (blk0 + j) & (kAcc - 1);
            const int len = min(min(j_hi - j + 1, kAcc - blk), 4);
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(blk * 64);
            const uint64_t b_desc = b_base + static_cast<uint32_t>((s * p.kh + j) * (kWBlock >> 4));
            const uint32_t idesc = make_idesc_f16_m128(static_cast<uint32_t>(len * 64));
            if (elect_one()) {
#pragma unroll
              for (int k = 0; k < 4; ++k)  // K step = 32 bytes = 2 start-address units
                umma_f16(d_tmem, a_desc + 2u * k, b_desc + 2u * k, idesc, 1u);
            }
            __syncwarp();
            j += len;
          }
        }
        if (elect_one()) umma_commit(&rempty[slot]);
        __syncwarp();
        // tiles whose last input row this was
        for (; next_done < ntiles && min(p.H - 1, sg.lo + next_done - p.ph + p.kh - 1) <= y; ++next_done) {
          if (elect_one()) umma_commit(&tfull[acc_block(lt0 + next_done)]);
          __syncwarp();
        }
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
    tmem_dealloc(tmem_base, kAcc * 64);
  }
}

// The 64-channel NHWC input as rows of pixels: box {64, 32, 1, 1} = 4 KB (32
// positions of one TMEM lane quarter), 128B swizzle; pixel coordinates
// below 0 or >= W and image coordinates >= N read as zeros.
int make_x_map(CUtensorMap* map, const ConvTcArgs& a, int n) {
  auto enc = encode_tiled();
  if (!enc) return -1;
  const cuuint64_t px = 128;
  cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(a.W), static_cast<cuuint64_t>(a.H), static_cast<cuuint64_t>(n)};
  cuuint64_t strides[3] = {px, px * a.W, px * a.W * a.H};
  cuuint32_t box[4] = {64, kBox, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(a.x), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// Prepacked weights [Cout, kh*kw*64] (K order: kernel row, tap column,
// channel): box {64, 64} = one tap of all (<= 64) output channels.
int make_w_map(CUtensorMap* map, const ConvTcArgs& a) {
  auto enc = encode_tiled();
  if (!enc) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.k_pad), static_cast<cuuint64_t>(a.n_cols)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.k_pad) * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.w_packed), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

int ring_slots(int w_bytes) {
  return std::min(kMaxSlots, (kSmemLimit - 1024 - kHeadBytes - w_bytes) / kSlotBytes);
}

}  // namespace

int conv_rows_check(const ConvTcArgs& a, int n, const char** err) {
  if (a.out_kind != 0 || (a.y_stride != 0 && a.y_stride != a.Cs_out)) {
    *err = "rows conv: dense NHWC fp16 output only";
    return -2;
  }
  if (a.Cs_in != 64 || a.sh != 1 || a.sw != 1) {
    *err = "rows conv: stride 1 over 64-channel pixels only";
    return -2;
  }
  if (a.kh < 1 || a.kh > kMaxK || a.kw < 1 || a.kw > kMaxK || a.ph < 0 || a.ph >= a.kh || a.pw < 0 ||
      a.pw >= a.kw || a.k_pad != a.kh * a.kw * 64) {
    *err = "rows conv: kernels up to 3x3 with padding below the kernel size";
    return -2;
  }
  if (a.n_cols < 1 || a.n_cols > 64 || a.Cs_out != (a.n_cols + 7) / 8 * 8) {
    *err = "rows conv: 1..64 output channels";
    return -2;
  }
  if (a.OW < 1 || a.OW > kPos || a.OH < 1 || n < 1) {
    *err = "rows conv: output rows of 1..128 pixels";
    return -2;
  }
  if (ring_slots(a.kh * a.kw * kWBlock) < 4) {
    *err = "rows conv: shared memory";
    return -2;
  }
  return 0;
}

int conv_rows_launch(const ConvTcArgs& a, int n, cudaStream_t stream, const char** err) {
  if (conv_rows_check(a, n, err) != 0) return -2;
  RsParams p{};
  p.bias = a.bias;
  p.residual = static_cast<const __half*>(a.residual);
  p.y = static_cast<__half*>(a.y);
  p.N = n;
  p.H = a.H;
  p.OH = a.OH;
  p.OW = a.OW;
  p.Cout = a.n_cols;
  p.Cs_out = a.Cs_out;
  p.kh = a.kh;
  p.kw = a.kw;
  p.ph = a.ph;
  p.pw = a.pw;
  p.act = a.act;
  // two images a tile when image 2g's lanes (ox < OW) never read past its
  // 64 slot rows (ox + kw - 1 <= 63)
  p.ipt = a.OW + a.kw - 1 <= kPos / 2 ? 2 : 1;
  p.units = (n + p.ipt - 1) / p.ipt * a.OH;
  p.w_bytes = a.kh * a.kw * kWBlock;
  p.slots = ring_slots(p.w_bytes);
  p.wait_limit = wait_limit_from_env();
  const int smem = 1024 + kHeadBytes + p.w_bytes + p.slots * kSlotBytes;

  CUtensorMap mw, mx;
  if (make_w_map(&mw, a) != 0) {
    *err = "rows conv: weight tensor map encoding failed";
    return -3;
  }
  if (make_x_map(&mx, a, n) != 0) {
    *err = "rows conv: input tensor map encoding failed";
    return -2;
  }
  static std::atomic<uint64_t> attr_ctx[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *err = "rows conv: no usable device";
    return -3;
  }
  const uint64_t ctx = current_context_id();
  if (ctx == 0 || attr_ctx[dev].load(std::memory_order_acquire) != ctx) {
    const cudaError_t ae =
        cudaFuncSetAttribute(conv_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (ae != cudaSuccess) {
      *err = cudaGetErrorString(ae);
      return -3;
    }
    attr_ctx[dev].store(ctx, std::memory_order_release);
  }
  const int grid = std::min(num_sms(), p.units);
  cudaError_t e = launch_pdl(conv_rows_kernel, dim3(grid), dim3(kThreads), smem, stream, mw, mx, p);
  note_launch();
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = cudaGetErrorString(e);
    return -3;
  }
  return 0;
}

}  // namespace lotus_impl

namespace lotus_impl {

int conv_rows_read_device_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, lotus_dev::g_lotus_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) {
    int zero = 0;
    cudaMemcpyToSymbol(lotus_dev::g_lotus_device_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace lotus_impl
