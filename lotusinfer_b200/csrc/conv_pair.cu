// Implicit-GEMM convolution on CTA pairs (tcgen05 cta_group::2) for convs
// over NHWC inputs whose channel count is a multiple of 64 (ResNet stages
// 2-4: 3x3 stride 1 and 2, 1x1 stride 2), with the fused bias, residual and
// activation epilogue and an NHWC fp16 output.
//
// Reference counterpart: source/operator/conv2d.cu:17-187 launched per
// sample from source/layer/layer_conv2d.cu:43-70, the residual from the
// Expression add + ReLU layer (source/layer/expression.cu:29-50).
//
// Why pairs.  A single-CTA tcgen05.mma (M = 128) reads its B operand (N rows
// of 32 bytes per K = 16 step) from shared memory at ~60 bytes a cycle,
// which keeps an N = 256 MMA at ~70% of the tensor rate and N = 128 at
// ~55%.  An M = 256 MMA issued for a CTA pair computes two 128-row halves,
// one per SM, and each SM supplies only half of B: per SM the A bytes stay
// the same and the B bytes halve, while the math per SM is unchanged.
//
// GEMM view: M = N*OH*OW output pixels, N_gemm = Cout, K = kh*kw*Cs_in in
// (tap, channel) order, A rows by im2col TMA, B = the prepacked K-major
// weights.  A pair tile is 256 M rows x BN columns: CTA rank r holds M rows
// 128r .. 128r+127 of it (its own A half, its own accumulator: 128 TMEM
// lanes x BN columns) and weight rows (output channels) BN/2*r .. +BN/2-1
// of the B operand.
//
// Roles (352 threads, both CTAs unless noted):
//   warps 0-7  epilogue: warp w drains TMEM lane quarter w % 4, column half
//              w / 4, in 32-column chunks: bias, residual, activation, fp16,
//              staged through shared memory into coalesced row stores; then
//              one arrival on the even CTA's tempty barrier;
//   warp 8     TMEM allocation (cta_group::2, both CTAs); in the even CTA
//              the MMA issuer: one M=256 MMA per K = 16 step, commits to the
//              barriers of both CTAs;
//   warp 9     TMA producer: this CTA's A half and B half of each stage, the
//              bytes counted on the even CTA's full barrier;
//   warp 10    (even CTA) the gate: waits on the even CTA's full and tempty
//              barriers and hands each 64-wide K block to the issuer through
//              named barriers (an mbarrier wait issued by the MMA-issuing
//              thread is held behind its queued MMAs; a named barrier is
//              not).  The hand-offs rotate over S + 1 barriers: the gate's
//              wait for K block h needs stage h mod S emptied by the MMAs of
//              block h - S, so the gate is never more than S blocks ahead and
//              never arrives twice on one barrier before the issuer took it.
//              After a failed wait the gate switches to bar.sync (lockstep)
//              and keeps handing off, so the issuer never waits forever.
// Every mbarrier wait is bounded.  Both CTAs meet at a cluster barrier after
// set-up and before teardown (a CTA must not exit while its peer's MMAs read
// its shared memory or its TMA signals the peer's barriers).
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

constexpr int kBlockM = 128;                    // M rows per CTA
constexpr int kBlockK = 64;                     // fp16 = one 128-byte swizzle row
constexpr int kABytes = kBlockM * kBlockK * 2;  // 16 KB
constexpr int kEpiWarps = 8;
constexpr int kMmaWarp = 8, kTmaWarp = 9, kGateWarp = 10;
constexpr int kThreads = 11 * 32;
constexpr int kStgBytes = 32 * 64;              // per epilogue warp: 32 rows x 32 fp16
constexpr int kBiasMax = 1024;
constexpr int kHeadBytes = 1024;                // barriers and misc words
constexpr int kSmemLimit = 232448;

// BN columns per pair tile; MT M tiles (of 128 rows) per CTA: a pair tile is
// 2 * MT * 128 rows x BN columns, one M = 256 MMA per M tile and K step, all
// MT of them reading the same B half.
template <int BN, int MT>
struct PairCfg {
  static constexpr int kBHalf = BN / 2;                    // weight rows per CTA
  static constexpr int kBBytes = kBHalf * kBlockK * 2;     // 8 or 16 KB
  static constexpr int kStage = MT * kABytes + kBBytes;
  static constexpr int kFixed = 1024 + kHeadBytes + kBiasMax * 4 + kEpiWarps * kStgBytes;
  static constexpr int kStages = std::min(8, (kSmemLimit - kFixed) / kStage);
  static constexpr int kQueue = kStages + 1;               // named barriers 1 .. kQueue
  static constexpr int kAccCols = BN * MT;                 // TMEM columns of one pair tile
  static constexpr int kAcc = 512 / kAccCols;              // TMEM accumulators
  static constexpr int kSmemBytes = kFixed + kStages * kStage;
  static_assert(kQueue <= 15, "named barriers");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory");
};

struct PairParams {
  const float* bias;
  const __half* residual;  // NHWC like y or null
  __half* y;
  int M, Cout, Cs_out, y_stride, act;
  int H, W, OH, OW, sh, sw, ph, pw, kh, kw, Cs_in;
  int KB;           // 64-wide K blocks
  int n_tiles;      // BN-column tiles
  int m_tiles;      // 128-row M tiles
  int pair_tiles;   // ceil(m_tiles / (2 * MT)) * n_tiles
  // Work units: pair tiles 0 .. full_units-1 whole, then each later tile as
  // ksplit units of kbs K blocks (the last wave's tiles, so that it keeps
  // every SM pair busy); a partial unit writes its raw fp32 sums to
  // ws[split][row - row0][ws_ld] and a split-K reduction finishes rows
  // row0 .. M-1.  ksplit == 1: every tile whole.
  int full_units, ksplit, kbs, units, row0, ws_ld;
  float* ws;
  uint32_t wait_limit;
};

// Work unit u: pair tile T, its K blocks kb0 .. kb0+nkb-1, and the split
// index of a partial unit (-1: the whole tile).
struct Unit {
  int T, kb0, nkb, split;
};
__device__ __forceinline__ Unit unit_of(const PairParams& p, int u) {
  Unit w;
  if (u < p.full_units) {
    w.T = u;
    w.kb0 = 0;
    w.nkb = p.KB;
    w.split = -1;
    return w;
  }
  const int v = u - p.full_units;
  const int t = v / p.ksplit;
  w.T = p.full_units + t;
  w.split = v - t * p.ksplit;
  w.kb0 = w.split * p.kbs;
  w.nkb = min(p.KB, w.kb0 + p.kbs) - w.kb0;
  return w;
}

// ------------------------------------------------------------ cluster PTX
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t map_to(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// Arrivals that order no memory accesses (no fence, so no wait for this
// thread's global stores to drain): for barriers that only hand back TMEM
// whose tcgen05.ld results are already in registers.
__device__ __forceinline__ void mbar_arrive_relaxed(uint64_t* bar) {
  asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(kWaitSuspendNs)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int err_code, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait_cluster(bar, parity)) return true;
  atomicExch(&g_lotus_device_error, err_code);
  return false;
}
__device__ __forceinline__ void named_arrive(uint32_t id, uint32_t count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ------------------------------------------------------------ pair tcgen05 / TMA
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[256 x N] (+)= A[256 x K] * B[N x K]^T over the pair: A rows 0-127 and B
// rows 0..N/2-1 from the even CTA's shared memory, the rest from the odd
// CTA's at the same offsets; D rows 0-127 in the even CTA's TMEM, 128-255 in
// the odd CTA's.
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// One arrival on the barrier at shared::cluster address `bar` once every
// pair MMA this thread issued so far is complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
// This CTA's half of a pair operand: the box lands in this CTA's shared
// memory, the bytes are counted on the even CTA's barrier `bar` (a
// shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* tmap, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_im2col_4d_pair(void* dst, const void* tmap, uint32_t bar, int c, int w,
                                                        int h, int n, uint16_t off_w, uint16_t off_h) {
  asm volatile(
      "cp.async.bulk.tensor.4d.im2col.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c), "r"(w), "r"(h), "r"(n), "h"(off_w), "h"(off_h)
      : "memory");
}

// Instruction descriptor, kind::f16, A = B = F16, D = F32, K-major, M = 256.
__host__ __device__ constexpr uint32_t idesc_pair(uint32_t n) {
  return (1u << 4) | ((n >> 3) << 17) | ((256u >> 4) << 24);
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <int ACT>
__device__ __forceinline__ float act_p(float v) {
  if (ACT == 1) return fmaxf(v, 0.0f);
  if (ACT == 2) return 1.0f / (1.0f + expf(-v));
  return v;
}

// One 32-column chunk of this lane's accumulator row: (acc + bias) +
// residual in fp32 (the general conv kernel's order), activation, fp16, pad
// channels zero.  The chunk is staged in the warp's 32 x 64-byte buffer
// (16-byte pieces XOR-swizzled by row) and stored as 8 rows x 64 contiguous
// bytes per instruction.  Warp-collective.
template <int ACT, bool RES>
__device__ __forceinline__ void store_chunk(const PairParams& p, const uint32_t (&v)[32], int em, bool valid,
                                            int col0, const float* s_bias, uint8_t* stg, int lane) {
  uint4* st = reinterpret_cast<uint4*>(stg);
  const bool full = col0 + 32 <= p.Cout;
  const int row_em = valid ? em : -1;
  uint4 res[4];
  if (RES) {
    // the chunk's residual rows, read as 8 rows x 64 contiguous bytes per
    // instruction into the staging buffer, then each lane takes its row
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 8 * i + (lane >> 2), c = lane & 3;
      const int em_r = __shfl_sync(0xffffffffu, row_em, r);
      uint4 val = make_uint4(0, 0, 0, 0);
      if (em_r >= 0 && col0 + c * 8 < p.Cs_out)
        val = __ldg(reinterpret_cast<const uint4*>(p.residual + static_cast<int64_t>(em_r) * p.Cs_out + col0 + c * 8));
      st[r * 4 + ((c ^ (r >> 1)) & 3)] = val;
    }
    __syncwarp();
#pragma unroll
    for (int g = 0; g < 4; ++g) res[g] = st[lane * 4 + ((g ^ (lane >> 1)) & 3)];
    __syncwarp();  // the buffer takes the output next
  }
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int c = col0 + 8 * g;
    float f[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = s_bias[c + j] + __uint_as_float(v[8 * g + j]);
    if (RES) {
      const __half2* rh = reinterpret_cast<const __half2*>(&res[g]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 rf = __half22float2(rh[j]);
        f[2 * j] += rf.x;
        f[2 * j + 1] += rf.y;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = act_p<ACT>(f[j]);
    if (!full) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c + j >= p.Cout) f[j] = 0.f;  // pad channels stay zero
    }
    st[lane * 4 + ((g ^ (lane >> 1)) & 3)] =
        make_uint4(pack_h2(f[0], f[1]), pack_h2(f[2], f[3]), pack_h2(f[4], f[5]), pack_h2(f[6], f[7]));
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 8 * i + (lane >> 2);  // staged row this lane stores
    const int c = lane & 3;             // and its 16-byte piece
    const int em_r = __shfl_sync(0xffffffffu, row_em, r);
    const uint4 val = st[r * 4 + ((c ^ (r >> 1)) & 3)];
    const int col = col0 + c * 8;
    if (em_r >= 0 && col < p.Cs_out)
      *reinterpret_cast<uint4*>(p.y + static_cast<int64_t>(em_r) * p.y_stride + col) = val;
  }
  __syncwarp();  // the buffer is rewritten by the next chunk
}

// One 32-column chunk of raw fp32 sums for the split-K reduction, at
// ws[split][em - row0][col0 ..]: two 16-column halves, each staged in the
// warp's 32 x 64-byte buffer like store_chunk and stored as 8 rows x 64
// contiguous bytes per instruction.  Warp-collective.
__device__ __forceinline__ void store_partial_chunk(const PairParams& p, const uint32_t (&v)[32], int em, bool valid,
                                                    int split, int col0, uint8_t* stg, int lane) {
  uint4* st = reinterpret_cast<uint4*>(stg);
  const int row_em = valid ? em : -1;
  float* base = p.ws + static_cast<int64_t>(split) * (p.M - p.row0) * p.ws_ld + col0;
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
    for (int g = 0; g < 4; ++g)
      st[lane * 4 + ((g ^ (lane >> 1)) & 3)] = make_uint4(v[16 * hf + 4 * g], v[16 * hf + 4 * g + 1],
                                                          v[16 * hf + 4 * g + 2], v[16 * hf + 4 * g + 3]);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 8 * i + (lane >> 2), c = lane & 3;
      const int em_r = __shfl_sync(0xffffffffu, row_em, r);
      const uint4 val = st[r * 4 + ((c ^ (r >> 1)) & 3)];
      if (em_r >= 0)
        *reinterpret_cast<uint4*>(base + static_cast<int64_t>(em_r - p.row0) * p.ws_ld + 16 * hf + 4 * c) = val;
    }
    __syncwarp();  // the buffer is rewritten next
  }
}

// Epilogue warps of both CTAs: this CTA's 128 rows of each pair tile.
template <int BN, int MT, int ACT, bool RES>
__device__ __forceinline__ void epilogue(const PairParams& p, uint64_t* tfull, uint64_t* tempty, const float* s_bias,
                                         uint8_t* stg, uint32_t tmem_base, uint32_t rank, volatile int* abort_flag) {
  using C = PairCfg<BN, MT>;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // warps 4h .. 4h+3 take half h of the tile's TMEM columns: with one M
  // tile a CTA, columns BN/2*h ..; with two, all BN columns of M tile h
  const int q = warp & 3, half = warp >> 2;
  const int mi = MT == 2 ? half : 0;                 // this warp's M tile
  const int col_base = MT == 2 ? 0 : half * (BN / 2);  // its first output column in the tile
  constexpr int kWarpCols = BN * MT / 2;
  const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
  const int pair0 = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  int lt = 0;
  for (int u = pair0; u < p.units; u += npairs, ++lt) {
    const Unit w = unit_of(p, u);
    const int mp = w.T / p.n_tiles, nt = w.T - mp * p.n_tiles;
    const int em = (((2 * mp + static_cast<int>(rank)) * MT + mi) * kBlockM) + q * 32 + lane;
    const bool valid = em < p.M;
    const int n0 = nt * BN;
    const int ab = lt % C::kAcc;
    if (RES && w.split < 0 && valid) {
      // pull this lane's residual row segment into L2 while the MMAs run
      const __half* rrow = p.residual + static_cast<int64_t>(em) * p.Cs_out;
      for (int c0 = n0 + col_base; c0 < min(n0 + col_base + kWarpCols, p.Cs_out); c0 += 64)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(rrow + c0));
    }
    bool ok = true;
    if (lane == 0) ok = !*abort_flag && mbar_wait(&tfull[ab], (lt / C::kAcc) & 1, kErrWaitAccum, p.wait_limit);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    tc_fence_after();
    // The accumulator goes back to the MMA warp (the ring lives on the even
    // CTA's barriers) right after this warp's last TMEM load, before its
    // last chunk is stored, with a relaxed arrival that waits for no stores.
    bool released = false;
    auto release = [&]() {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive_relaxed(&tempty[ab]);
        else
          mbar_arrive_remote_relaxed(map_to(&tempty[ab], 0));
      }
      released = true;
    };
#pragma unroll 1
    for (int c = 0; c < kWarpCols / 32; ++c) {
      const int col = col_base + c * 32;  // output column inside the tile
      if (!ok || n0 + col >= p.Cs_out) continue;  // warp-uniform
      uint32_t v[32];
      tmem_ld_32x32b_x32(tmem_base + t_lane + static_cast<uint32_t>(ab * C::kAccCols + half * kWarpCols + c * 32),
                         v);
      tmem_ld_wait();
      if (c + 1 == kWarpCols / 32 || n0 + col + 32 >= p.Cs_out) release();  // no TMEM load after this one
      if (w.split < 0)
        store_chunk<ACT, RES>(p, v, em, valid, n0 + col, s_bias, stg, lane);
      else  // a partial unit
        store_partial_chunk(p, v, em, valid, w.split, n0 + col, stg, lane);
    }
    if (!released) release();
    if (lane == 0 && !ok) *abort_flag = 1;
  }
}

// The residual add compiled in or out: a residual path that is only skipped
// at run time slowed the no-residual layers' epilogue (ResNet stage-2
// downsample 21.0 -> 24.2 us).
template <int BN, int MT, int ACT>
__device__ __forceinline__ void epilogue_act(const PairParams& p, uint64_t* tfull, uint64_t* tempty,
                                             const float* s_bias, uint8_t* stg, uint32_t tmem_base, uint32_t rank,
                                             volatile int* abort_flag) {
  if (p.residual != nullptr)
    epilogue<BN, MT, ACT, true>(p, tfull, tempty, s_bias, stg, tmem_base, rank, abort_flag);
  else
    epilogue<BN, MT, ACT, false>(p, tfull, tempty, s_bias, stg, tmem_base, rank, abort_flag);
}

template <int BN, int MT>
__global__ void __launch_bounds__(kThreads, 1)
conv_pair_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                 const PairParams p) {
  using C = PairCfg<BN, MT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // [kStages] even CTA: both halves of a stage landed
  uint64_t* empty = full + C::kStages;                 // [kStages] this CTA's stage consumed
  uint64_t* tfull = empty + C::kStages;                // [kAcc] this CTA's accumulator complete
  uint64_t* tempty = tfull + C::kAcc;                  // [kAcc] even CTA: drained by both epilogues
  uint64_t* mma_done = tempty + C::kAcc;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 960);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 964);
  float* s_bias = reinterpret_cast<float*>(smem + kHeadBytes);
  uint8_t* s_stg = smem + kHeadBytes + kBiasMax * 4;
  uint8_t* stages = s_stg + kEpiWarps * kStgBytes;  // 1024-aligned: 1024 + 4096 + 16384
  auto sA = [&](int st, int i) { return stages + st * C::kStage + i * kABytes; };
  auto sB = [&](int st) { return stages + st * C::kStage + MT * kABytes; };

  const int tid = threadIdx.x;
  const int warp = __shfl_sync(0xffffffffu, tid >> 5, 0), lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const int pair0 = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);

  if (tid == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);  // the even CTA's producer arrival + both CTAs' bytes
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < C::kAcc; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * kEpiWarps);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  for (int i = tid; i < kBiasMax; i += kThreads) s_bias[i] = (p.bias != nullptr && i < p.Cout) ? __ldg(p.bias + i) : 0.f;
  if (warp == kTmaWarp && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_a);
  }
  if (warp == kMmaWarp) {
    tmem_alloc_pair(tmem_slot, C::kAcc * C::kAccCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival or commit
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (tid == 0) griddep_launch();  // set-up done: the next kernel may start being scheduled

  if (warp < kEpiWarps) {
    griddep_wait();  // residual and output buffers belong to earlier kernels
    uint8_t* stg = s_stg + warp * kStgBytes;
    if (p.act == 1)
      epilogue_act<BN, MT, 1>(p, tfull, tempty, s_bias, stg, tmem_base, rank, abort_flag);
    else if (p.act == 0)
      epilogue_act<BN, MT, 0>(p, tfull, tempty, s_bias, stg, tmem_base, rank, abort_flag);
    else
      epilogue_act<BN, MT, 2>(p, tfull, tempty, s_bias, stg, tmem_base, rank, abort_flag);
  } else if (warp == kTmaWarp) {
    if (lane == 0) {
      griddep_wait();  // the activations of earlier kernels
      bool ok = true;
      uint32_t it = 0;
      const int ohw = p.OH * p.OW, cpt = p.Cs_in / kBlockK;
      for (int u = pair0; u < p.units && ok; u += npairs) {
        const Unit w = unit_of(p, u);
        const int mp = w.T / p.n_tiles, nt = w.T - mp * p.n_tiles;
        // this CTA's M tiles; past the last M tile (a pair tile that overhangs
        // the output) it loads the last real tile (those results are never
        // stored)
        int wst[MT], hst[MT], nimg[MT];
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          const int mt = min((2 * mp + static_cast<int>(rank)) * MT + i, p.m_tiles - 1);
          const int m0 = mt * kBlockM;
          nimg[i] = m0 / ohw;
          const int rem = m0 - nimg[i] * ohw;
          const int oh = rem / p.OW, ow = rem - oh * p.OW;
          wst[i] = ow * p.sw - p.pw;
          hst[i] = oh * p.sh - p.ph;
        }
        const int brow = nt * BN + static_cast<int>(rank) * C::kBHalf;
        // (tap, channel) position of the unit's first K block
        const int tap0 = w.kb0 / cpt;
        int c0 = (w.kb0 - tap0 * cpt) * kBlockK, r = tap0 / p.kw, s = tap0 - r * p.kw;
        for (int kb = w.kb0; kb < w.kb0 + w.nkb; ++kb, ++it) {
          const int st = static_cast<int>(it % C::kStages);
          if (*abort_flag || !mbar_wait(&empty[st], ((it / C::kStages) & 1) ^ 1, kErrWaitEmpty, p.wait_limit)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[st], 2u * C::kStage);
          const uint32_t fb = map_to(&full[st], 0);
          tma_load_2d_pair(sB(st), &tmap_w, fb, kb * kBlockK, brow);
#pragma unroll
          for (int i = 0; i < MT; ++i)
            tma_load_im2col_4d_pair(sA(st, i), &tmap_a, fb, c0, wst[i], hst[i], nimg[i], static_cast<uint16_t>(s),
                                    static_cast<uint16_t>(r));
          c0 += kBlockK;
          if (c0 == p.Cs_in) {
            c0 = 0;
            if (++s == p.kw) {
              s = 0;
              ++r;
            }
          }
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == kGateWarp) {
    if (rank == 0) {
      bool ok = true;
      uint32_t it = 0, h = 0;
      int lt = 0;
      for (int u = pair0; u < p.units; u += npairs, ++lt) {
        const Unit w = unit_of(p, u);
        const int ab = lt % C::kAcc;
        for (int kb = 0; kb < w.nkb; ++kb, ++it, ++h) {
          const int st = static_cast<int>(it % C::kStages);
          if (lane == 0 && ok) {
            if (kb == 0)
              ok = mbar_wait_cluster(&tempty[ab], ((lt / C::kAcc) & 1) ^ 1, kErrWaitAccum, p.wait_limit);
            if (ok) ok = mbar_wait(&full[st], (it / C::kStages) & 1, kErrWaitFull, p.wait_limit);
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          const uint32_t id = 1u + h % C::kQueue;
          if (ok) {
            named_arrive(id, 64);
          } else {
            if (lane == 0) *abort_flag = 1;
            named_sync(id, 64);  // lockstep from here on: never two arrivals ahead
          }
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (rank == 0) {
      // The whole warp runs this loop (warp-uniform values); one elected lane
      // issues and commits.  It waits only on the gate's named barriers.
      constexpr uint32_t idesc = idesc_pair(BN);
      uint32_t it = 0, h = 0;
      int lt = 0;
      for (int u = pair0; u < p.units; u += npairs, ++lt) {
        const Unit w = unit_of(p, u);
        const int ab = lt % C::kAcc;
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(ab * C::kAccCols);
        for (int kb = 0; kb < w.nkb; ++kb, ++it, ++h) {
          const int st = static_cast<int>(it % C::kStages);
          named_sync(1u + h % C::kQueue, 64);
          tc_fence_after();
          const uint64_t a_desc = make_sdesc_sw128(smem_u32(sA(st, 0)));
          const uint64_t b_desc = make_sdesc_sw128(smem_u32(sB(st)));
          if (elect_one()) {
#pragma unroll
            for (int k = 0; k < kBlockK / 16; ++k)  // K step = 32 bytes = 2 start-address units
#pragma unroll
              for (int i = 0; i < MT; ++i)  // M tile i: its A 16 KB further, its accumulator BN columns further
                umma_f16_pair(d_tmem + static_cast<uint32_t>(i * BN), a_desc + 2u * k + static_cast<uint32_t>(i * (kABytes >> 4)),
                              b_desc + 2u * k, idesc, (kb | k) != 0 ? 1u : 0u);
            umma_commit_pair(smem_u32(&empty[st]));  // this CTA's stage
            umma_commit_pair(map_to(&empty[st], 1));  // the odd CTA's stage
          }
          __syncwarp();
        }
        if (elect_one()) {
          umma_commit_pair(smem_u32(&tfull[ab]));
          umma_commit_pair(map_to(&tfull[ab], 1));
        }
        __syncwarp();
      }
      if (elect_one()) umma_commit_pair(smem_u32(mma_done));
      __syncwarp();
      mbar_wait(mma_done, 0, kErrWaitFull, p.wait_limit);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the pair's MMAs or loads may touch it
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::kAcc * C::kAccCols);
  }
}

// Weights [n_cols, k_pad] fp16: box {64, BN/2} (this CTA's half of a pair
// tile's output channels), rows past n_cols read as zero.
int make_w_map(CUtensorMap* map, const ConvTcArgs& a, int box_rows) {
  auto enc = encode_tiled();
  if (!enc) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.k_pad), static_cast<cuuint64_t>(a.n_cols)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.k_pad) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBlockK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.w_packed), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// im2col map over the NHWC activation [N, H, W, Cs]: 128 output pixels x 64
// channels per load, bounding box [-pad, dim - 1 + pad - (k - 1)],
// traversal stride = conv stride.
int make_im2col_map(CUtensorMap* map, const ConvTcArgs& a, int n_img) {
  auto enc = encode_im2col();
  if (!enc) return -1;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(a.Cs_in), static_cast<cuuint64_t>(a.W), static_cast<cuuint64_t>(a.H),
                        static_cast<cuuint64_t>(n_img)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(a.Cs_in) * 2, static_cast<cuuint64_t>(a.W) * a.Cs_in * 2,
                           static_cast<cuuint64_t>(a.H) * a.W * a.Cs_in * 2};
  int lower[2] = {-a.pw, -a.ph};
  int upper[2] = {a.pw - (a.kw - 1), a.ph - (a.kh - 1)};
  cuuint32_t estr[4] = {1, static_cast<cuuint32_t>(a.sw), static_cast<cuuint32_t>(a.sh), 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(a.x), dims, strides, lower,
                         upper, kBlockK, kBlockM, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// How the pair tiles are walked.  With `pairs` SM pairs, the tiles of the
// full waves are processed whole; when a workspace can be used, each tile of
// the last, partial wave is split over its K loop into k units (k = 2..4,
// each unit at least one K block), chosen when the round-robin makespan
// (full tile = 1, unit = its share of the K blocks) plus the split-K
// reduction it needs is estimated at least 8% below the unsplit makespan.
// The full part is a multiple of the N-tile count, so the split tiles cover
// whole output rows row0 .. M-1.  LOTUS_PAIR_SPLIT=0 never splits; =1 splits
// whenever that shortens the makespan, ignoring the reduction's cost.
struct PairPlan {
  int pair_tiles, full_units, ksplit, kbs, units, row0, ws_ld;
  size_t ws_bytes;  // 0 when nothing is split
};

PairPlan plan_pairs(const ConvTcArgs& a, int bn, int mt, int pairs, bool allow_split) {
  PairPlan pl{};
  const int KB = a.k_pad / kBlockK;
  const int n_tiles = (a.n_cols + bn - 1) / bn;
  const int m_tiles = (a.M + kBlockM - 1) / kBlockM;
  pl.pair_tiles = (m_tiles + 2 * mt - 1) / (2 * mt) * n_tiles;
  pl.full_units = pl.pair_tiles;
  pl.ksplit = 1;
  pl.kbs = KB;
  pl.units = pl.pair_tiles;
  pl.ws_ld = n_tiles * bn;
  const char* env = std::getenv("LOTUS_PAIR_SPLIT");
  if (!allow_split || pairs < 1 || (env != nullptr && env[0] == '0')) return pl;
  const bool force = env != nullptr && env[0] == '1';
  const int full = (pl.pair_tiles / pairs) * pairs / n_tiles * n_tiles;
  const int rem = pl.pair_tiles - full;
  if (rem <= 0) return pl;
  auto makespan = [&](int k, int kbs) {
    const int units = full + k * rem;
    double worst = 0;
    for (int q = 0; q < pairs && q < units; ++q) {
      double t = 0;
      for (int u = q; u < units; u += pairs) {
        if (u < full) {
          t += 1.0;
        } else {
          const int sp = (u - full) % k;
          t += static_cast<double>(std::min(KB, (sp + 1) * kbs) - sp * kbs) / KB;
        }
      }
      worst = std::max(worst, t);
    }
    return worst;
  };
  // Estimated time in microseconds: a pair tile at ~20 TFLOP/s (one SM
  // pair's share of the dense fp16 rate), the reduction as its HBM bytes at
  // ~6 TB/s (k fp32 partial rows read, fp16 rows written, the residual
  // read) plus ~2 us for its launch and tail.
  const double tile_us = 2.0 * (2 * mt * kBlockM) * bn * a.k_pad / 2.0e7;
  const int row0 = full / n_tiles * 2 * mt * kBlockM;
  auto reduce_us = [&](int k) {
    const double rows = static_cast<double>(a.M - row0);
    const double bytes = rows * (4.0 * k * pl.ws_ld + 2.0 * a.Cs_out * (a.residual != nullptr ? 2 : 1));
    return bytes / 6.0e6 + 2.0;
  };
  const double base = makespan(1, KB) * tile_us;
  int best_k = 1, best_kbs = KB;
  double best = base;
  for (int k = 2; k <= 4 && k <= KB; ++k) {
    const int kbs = (KB + k - 1) / k;
    const int keff = (KB + kbs - 1) / kbs;  // every unit gets at least one K block
    // LOTUS_PAIR_SPLIT=1: the split with the shortest makespan, whatever it costs
    const double t = makespan(keff, kbs) * tile_us + (force ? 0.0 : reduce_us(keff));
    if (t < best - 1e-9) {
      best = t;
      best_k = keff;
      best_kbs = kbs;
    }
  }
  if (best_k == 1 || (!force && best > 0.92 * base)) return pl;
  pl.full_units = full;
  pl.ksplit = best_k;
  pl.kbs = best_kbs;
  pl.units = full + best_k * rem;
  pl.row0 = row0;
  pl.ws_bytes = static_cast<size_t>(best_k) * (a.M - pl.row0) * pl.ws_ld * sizeof(float);
  return pl;
}

// Per device and context: the shared-memory opt-in of the kernel and the
// number of CTA pairs that can be resident at once (0 with *err set on
// failure).
template <int BN, int MT>
int resident_pairs(const char** err) {
  using C = PairCfg<BN, MT>;
  static std::atomic<uint64_t> attr_ctx[64];
  static std::atomic<int> max_pairs[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *err = "pair conv: no usable device";
    return 0;
  }
  const uint64_t ctx = current_context_id();
  if (ctx == 0 || attr_ctx[dev].load(std::memory_order_acquire) != ctx) {
    cudaError_t ae =
        cudaFuncSetAttribute(conv_pair_kernel<BN, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (ae != cudaSuccess) {
      *err = cudaGetErrorString(ae);
      return 0;
    }
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    int clusters = 0;
    ae = cudaOccupancyMaxActiveClusters(&clusters, conv_pair_kernel<BN, MT>, &cfg);
    if (ae != cudaSuccess || clusters < 1) {
      *err = ae != cudaSuccess ? cudaGetErrorString(ae) : "pair conv: no CTA pair fits an SM pair";
      return 0;
    }
    max_pairs[dev].store(clusters, std::memory_order_relaxed);
    attr_ctx[dev].store(ctx, std::memory_order_release);
  }
  return max_pairs[dev].load(std::memory_order_relaxed);
}

template <int BN, int MT>
int launch_bn(const ConvTcArgs& a, cudaStream_t stream, const char** err) {
  using C = PairCfg<BN, MT>;
  PairParams p{};
  p.bias = a.bias;
  p.residual = static_cast<const __half*>(a.residual);
  p.y = static_cast<__half*>(a.y);
  p.M = a.M;
  p.Cout = a.n_cols;
  p.Cs_out = a.Cs_out;
  p.y_stride = a.y_stride != 0 ? a.y_stride : a.Cs_out;
  p.act = a.act;
  p.H = a.H;
  p.W = a.W;
  p.OH = a.OH;
  p.OW = a.OW;
  p.sh = a.sh;
  p.sw = a.sw;
  p.ph = a.ph;
  p.pw = a.pw;
  p.kh = a.kh;
  p.kw = a.kw;
  p.Cs_in = a.Cs_in;
  p.KB = a.k_pad / kBlockK;
  p.n_tiles = (a.n_cols + BN - 1) / BN;
  p.m_tiles = (a.M + kBlockM - 1) / kBlockM;
  const int resident = resident_pairs<BN, MT>(err);
  if (resident < 1) return -3;
  // the split of the last wave needs the caller's workspace (and room in it)
  PairPlan pl = plan_pairs(a, BN, MT, resident, a.ws != nullptr);
  if (pl.ws_bytes > a.ws_bytes) pl = plan_pairs(a, BN, MT, resident, false);
  p.pair_tiles = pl.pair_tiles;
  p.full_units = pl.full_units;
  p.ksplit = pl.ksplit;
  p.kbs = pl.kbs;
  p.units = pl.units;
  p.row0 = pl.row0;
  p.ws_ld = pl.ws_ld;
  p.ws = pl.ksplit > 1 ? a.ws : nullptr;
  p.wait_limit = wait_limit_from_env();
  const int n_img = a.M / (a.OH * a.OW);

  CUtensorMap mw, ma;
  if (make_w_map(&mw, a, C::kBHalf) != 0) {
    *err = "pair conv: weight tensor map encoding failed";
    return -3;
  }
  if (make_im2col_map(&ma, a, n_img) != 0) {
    *err = "pair conv: im2col tensor map encoding failed";
    return -2;
  }
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  const int pairs = std::min(resident, p.units);
  cfg.gridDim = dim3(2 * pairs);
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, conv_pair_kernel<BN, MT>, mw, ma, p);
  note_launch();
  if (e == cudaSuccess && p.ksplit > 1)  // rows row0 .. M-1: sum the split units in order, bias, residual, act
    e = launch_splitk_reduce(p.ws, p.ksplit, a.M - p.row0, p.ws_ld, a.bias,
                             p.residual != nullptr ? p.residual + static_cast<int64_t>(p.row0) * p.Cs_out : nullptr,
                             p.y + static_cast<int64_t>(p.row0) * p.y_stride, a.M - p.row0, p.Cout, p.Cs_out,
                             p.y_stride, p.act, stream);
  if (e != cudaSuccess) {
    *err = cudaGetErrorString(e);
    return -3;
  }
  return 0;
}

template <int BN, int MT>
size_t workspace_bn(const ConvTcArgs& a) {
  const char* err = "";
  const int resident = resident_pairs<BN, MT>(&err);
  return resident < 1 ? 0 : plan_pairs(a, BN, MT, resident, true).ws_bytes;
}

}  // namespace

int conv_pair_check(const ConvTcArgs& a, int bn, const char** err) {
  if (bn != 128 && bn != 256) {
    *err = "pair conv: 128 or 256 columns per tile";
    return -2;
  }
  if (a.out_kind != 0) {
    *err = "pair conv: NHWC fp16 output only";
    return -2;
  }
  if (a.Cs_in % kBlockK != 0 || a.k_pad != a.kh * a.kw * a.Cs_in) {
    *err = "pair conv: input channels a multiple of 64";
    return -2;
  }
  if (a.n_cols < 1 || a.n_cols > kBiasMax || a.Cs_out != (a.n_cols + 7) / 8 * 8) {
    *err = "pair conv: 1..1024 output channels";
    return -2;
  }
  if (a.y_stride != 0 && (a.y_stride < a.Cs_out || a.y_stride % 8 != 0)) {
    *err = "pair conv: output pixel stride";
    return -2;
  }
  if (a.OH < 1 || a.OW < 1 || a.M < 1 || a.M % (a.OH * a.OW) != 0 || a.kh > 256 || a.kw > 256) {
    *err = "pair conv: shape";
    return -2;
  }
  return 0;
}

size_t conv_pair_workspace_bytes(const ConvTcArgs& a, int bn) {
  const char* err = "";
  if (conv_pair_check(a, bn, &err) != 0) return 0;
  return bn == 256 ? workspace_bn<256, 1>(a) : workspace_bn<128, 2>(a);
}

int conv_pair_launch(const ConvTcArgs& a, int bn, cudaStream_t stream, const char** err) {
  if (conv_pair_check(a, bn, err) != 0) return -2;
  // 128 columns: two M tiles a CTA (a 512 x 128 pair tile), so each weight
  // stage feeds two MMAs per K step
  return bn == 256 ? launch_bn<256, 1>(a, stream, err) : launch_bn<128, 2>(a, stream, err);
}

int conv_pair_read_device_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, lotus_dev::g_lotus_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (v != 0) {
    int zero = 0;
    cudaMemcpyToSymbol(lotus_dev::g_lotus_device_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace lotus_impl
