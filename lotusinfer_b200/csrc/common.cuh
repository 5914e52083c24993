// Small device helpers shared by the bandwidth-bound kernels.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace lotus_dev {

// Activation with the values of the reference's ActivationFunction enum
// (include/lotus_utils.hpp:44-48): 0 none, 1 ReLU, 2 sigmoid 1/(1+exp(-x)).
__device__ __forceinline__ float act_fn(float v, int act) {
  if (act == 1) return fmaxf(v, 0.0f);
  if (act == 2) return 1.0f / (1.0f + expf(-v));
  return v;
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while the kernel before it is still running; it
// calls griddep_wait() before its first access to memory an earlier kernel
// writes or reads (activations, workspaces), which returns once every
// prerequisite grid has completed and its memory is visible.  Reads of
// weights and biases, shared-memory and TMEM set-up may come before it.
// griddep_launch() lets this grid's own dependents start being scheduled
// (they are, once every CTA of this grid has issued it or exited).  Both are
// no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Grid size for a grid-stride loop: enough CTAs to fill 148 SMs several
// times over, never more than the work needs.
__host__ __forceinline__ unsigned grid_for(size_t work, int block, int per_sm_ctas = 8) {
  const size_t need = (work + block - 1) / block;
  const size_t cap = static_cast<size_t>(148) * per_sm_ctas;
  return static_cast<unsigned>(need < cap ? (need == 0 ? 1 : need) : cap);
}

}  // namespace lotus_dev
