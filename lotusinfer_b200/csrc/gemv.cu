// HBM-bound fused GEMV + bias + activation for small batches (<= 8 rows).
//
// y[b, h] = act(sum_k W[h, k] * x[b, k] + bias[h])
//
// One warp owns one output row h: lanes stream the weight row with 16-byte
// loads (4 fp32 or 8 fp16 values), four loads in flight per lane, multiply
// each weight vector against every batch row of x (L1-resident), and reduce
// with warp shuffles.  The weight is read exactly once, so the kernel runs at
// the HBM roofline once enough rows are in flight.
//
// Reference counterpart: Fgemva + ReduceAdd, source/operator/fused_gemv_add_bias.cu:16-108
// (fp32, shared-memory tree reduction with block-wide barriers per 512 columns).

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"

namespace lotus_impl {

using namespace lotus_dev;

template <typename T>
struct Vec16;
template <>
struct Vec16<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float (&f)[8]) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p));
    f[0] = v.x;
    f[1] = v.y;
    f[2] = v.z;
    f[3] = v.w;
  }
  // streaming load for weights (read once)
  __device__ static void load_stream(const float* p, float (&f)[8]) {
    const float4 v = __ldcs(reinterpret_cast<const float4*>(p));
    f[0] = v.x;
    f[1] = v.y;
    f[2] = v.z;
    f[3] = v.w;
  }
};
template <>
struct Vec16<__half> {
  static constexpr int N = 8;
  __device__ static void load(const __half* p, float (&f)[8]) { unpack8(__ldg(reinterpret_cast<const uint4*>(p)), f); }
  __device__ static void load_stream(const __half* p, float (&f)[8]) {
    unpack8(__ldcs(reinterpret_cast<const uint4*>(p)), f);
  }
};

template <typename WT, typename XT, int B>
__global__ void __launch_bounds__(256) gemv_vec_kernel(const WT* __restrict__ w, int ldw, const XT* __restrict__ x,
                                                       int ldx, const float* __restrict__ bias, void* __restrict__ y,
                                                       int y_f16, int ldy, int batch, int h_out, int w_in, int act) {
  constexpr int V = Vec16<WT>::N;
  const int warps_per_block = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nvec = w_in / V;
  for (int h = blockIdx.x * warps_per_block + (threadIdx.x >> 5); h < h_out; h += gridDim.x * warps_per_block) {
    const WT* wr = w + static_cast<size_t>(h) * ldw;
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.f;
    int v = lane;
    for (; v + 3 * 32 < nvec; v += 4 * 32) {
      float wv[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) Vec16<WT>::load_stream(wr + (v + u * 32) * V, wv[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
#pragma unroll
        for (int b = 0; b < B; ++b) {
          if (b < batch) {
            float xv[8];
            if constexpr (sizeof(XT) == 4 && V == 8) {
              Vec16<float>::load(reinterpret_cast<const float*>(x) + static_cast<size_t>(b) * ldx + (v + u * 32) * V, xv);
              float xv2[8];
              Vec16<float>::load(reinterpret_cast<const float*>(x) + static_cast<size_t>(b) * ldx + (v + u * 32) * V + 4, xv2);
#pragma unroll
              for (int j = 0; j < 4; ++j) xv[4 + j] = xv2[j];
            } else if constexpr (sizeof(XT) == 2 && V == 4) {
              const __half2* hp = reinterpret_cast<const __half2*>(x + static_cast<size_t>(b) * ldx + (v + u * 32) * V);
              const float2 a0 = __half22float2(hp[0]), a1 = __half22float2(hp[1]);
              xv[0] = a0.x;
              xv[1] = a0.y;
              xv[2] = a1.x;
              xv[3] = a1.y;
            } else {
              Vec16<XT>::load(x + static_cast<size_t>(b) * ldx + (v + u * 32) * V, xv);
            }
#pragma unroll
            for (int j = 0; j < V; ++j) acc[b] = fmaf(wv[u][j], xv[j], acc[b]);
          }
        }
      }
    }
    for (; v < nvec; v += 32) {
      float wv[8];
      Vec16<WT>::load_stream(wr + v * V, wv);
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (b < batch) {
          const XT* xp = x + static_cast<size_t>(b) * ldx + v * V;
#pragma unroll
          for (int j = 0; j < V; ++j) {
            float xe;
            if constexpr (sizeof(XT) == 2)
              xe = __half2float(xp[j]);
            else
              xe = xp[j];
            acc[b] = fmaf(wv[j], xe, acc[b]);
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], o);
    }
    if (lane == 0) {
      const float bb = bias ? bias[h] : 0.f;
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (b < batch) {
          const float r = act_fn(acc[b] + bb, act);
          if (y_f16)
            static_cast<__half*>(y)[static_cast<size_t>(b) * ldy + h] = __float2half_rn(r);
          else
            static_cast<float*>(y)[static_cast<size_t>(b) * ldy + h] = r;
        }
      }
    }
  }
}

// Element-wise fallback for shapes or pointers that do not allow 16-byte loads.
template <typename WT, typename XT>
__global__ void gemv_scalar_kernel(const WT* __restrict__ w, int ldw, const XT* __restrict__ x, int ldx,
                                   const float* __restrict__ bias, void* __restrict__ y, int y_f16, int ldy, int batch,
                                   int h_out, int w_in, int act) {
  const int warps_per_block = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int h = blockIdx.x * warps_per_block + (threadIdx.x >> 5); h < h_out; h += gridDim.x * warps_per_block) {
    for (int b = 0; b < batch; ++b) {
      float acc = 0.f;
      for (int k = lane; k < w_in; k += 32) {
        float wf, xf;
        if constexpr (sizeof(WT) == 2) wf = __half2float(w[static_cast<size_t>(h) * ldw + k]);
        else wf = w[static_cast<size_t>(h) * ldw + k];
        if constexpr (sizeof(XT) == 2) xf = __half2float(x[static_cast<size_t>(b) * ldx + k]);
        else xf = x[static_cast<size_t>(b) * ldx + k];
        acc = fmaf(wf, xf, acc);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) {
        const float r = act_fn(acc + (bias ? bias[h] : 0.f), act);
        if (y_f16)
          static_cast<__half*>(y)[static_cast<size_t>(b) * ldy + h] = __float2half_rn(r);
        else
          static_cast<float*>(y)[static_cast<size_t>(b) * ldy + h] = r;
      }
    }
  }
}

template <typename WT, typename XT>
static void launch_typed(const void* w, int ldw, const void* x, int ldx, const float* bias, void* y, int y_f16,
                         int ldy, int batch, int h_out, int w_in, int act, cudaStream_t s) {
  constexpr int V = Vec16<WT>::N;
  const int threads = 256;
  const int warps = threads / 32;
  const unsigned grid = static_cast<unsigned>((h_out + warps - 1) / warps);
  const bool vec_ok = (w_in % V == 0) && (ldw % V == 0) && (ldx % V == 0) &&
                      (reinterpret_cast<uintptr_t>(w) % 16 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
  const WT* wt = static_cast<const WT*>(w);
  const XT* xt = static_cast<const XT*>(x);
  if (!vec_ok) {
    gemv_scalar_kernel<WT, XT><<<grid, threads, 0, s>>>(wt, ldw, xt, ldx, bias, y, y_f16, ldy, batch, h_out, w_in, act);
  } else if (batch == 1) {
    gemv_vec_kernel<WT, XT, 1><<<grid, threads, 0, s>>>(wt, ldw, xt, ldx, bias, y, y_f16, ldy, batch, h_out, w_in, act);
  } else if (batch == 2) {
    gemv_vec_kernel<WT, XT, 2><<<grid, threads, 0, s>>>(wt, ldw, xt, ldx, bias, y, y_f16, ldy, batch, h_out, w_in, act);
  } else if (batch <= 4) {
    gemv_vec_kernel<WT, XT, 4><<<grid, threads, 0, s>>>(wt, ldw, xt, ldx, bias, y, y_f16, ldy, batch, h_out, w_in, act);
  } else {
    gemv_vec_kernel<WT, XT, 8><<<grid, threads, 0, s>>>(wt, ldw, xt, ldx, bias, y, y_f16, ldy, batch, h_out, w_in, act);
  }
  note_launch();
}

cudaError_t launch_gemv(const void* w, int w_f16, int ldw, const void* x, int x_f16, int ldx, const float* bias,
                        void* y, int y_f16, int ldy, int batch, int h_out, int w_in, int act, cudaStream_t s) {
  if (w_f16) {
    if (x_f16)
      launch_typed<__half, __half>(w, ldw, x, ldx, bias, y, y_f16, ldy, batch, h_out, w_in, act, s);
    else
      launch_typed<__half, float>(w, ldw, x, ldx, bias, y, y_f16, ldy, batch, h_out, w_in, act, s);
  } else {
    if (x_f16)
      launch_typed<float, __half>(w, ldw, x, ldx, bias, y, y_f16, ldy, batch, h_out, w_in, act, s);
    else
      launch_typed<float, float>(w, ldw, x, ldx, bias, y, y_f16, ldy, batch, h_out, w_in, act, s);
  }
  return cudaGetLastError();
}

}  // namespace lotus_impl
