// Shared device helpers for the actkv sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/actkv_b200.h"

namespace actkv {

constexpr float kLog2e = 1.4426950408889634f;

// ------------------------------------------------------------------ element loads as fp32
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

__device__ __forceinline__ void flag(int32_t* status, int bit) {
  if (status) atomicOr(status, bit);
}

// Programmatic dependent launch.  A kernel launched by launch_pdl may be scheduled while the kernel
// before it in the stream is still finishing: pdl_wait() returns once that kernel has completed and
// its memory is visible (at once for an ordinary launch), so such a kernel calls it before its first
// access to global memory; pdl_trigger() lets the next launch_pdl kernel be scheduled as soon as
// every CTA of this one has called it or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Orderable key of a float: larger float -> larger unsigned key.  -0.0 is folded onto +0.0 so that
// the two compare equal, as they do in torch.
__device__ __forceinline__ uint32_t order_key(float x) {
  uint32_t b = __float_as_uint(x + 0.0f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// ------------------------------------------------------------------ block-wide reductions
// All threads of the block must call these; `red` is shared scratch of >= 32 entries.
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ T block_sum(T v, T* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  T r = 0;
  if (warp == 0) {
    r = lane < nw ? red[lane] : T(0);
    r = warp_sum(r);
    if (lane == 0) red[0] = r;
  }
  __syncthreads();
  r = red[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float r = lane < nw ? red[lane] : -INFINITY;
    r = warp_max(r);
    if (lane == 0) red[0] = r;
  }
  __syncthreads();
  float r = red[0];
  __syncthreads();
  return r;
}

// Exclusive prefix count of `pred` over the block in thread order; returns the block total in
// *total.  `red` needs >= 33 ints of shared scratch.
__device__ __forceinline__ int block_excl_count(bool pred, int* red, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  const unsigned ball = __ballot_sync(0xffffffffu, pred);
  const int in_warp = __popc(ball & ((1u << lane) - 1u));
  __syncthreads();
  if (lane == 0) red[warp] = __popc(ball);
  __syncthreads();
  if (warp == 0) {
    int c = lane < nw ? red[lane] : 0;
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane < nw) red[lane] = incl - c;
    if (lane == 31) red[32] = incl;
  }
  __syncthreads();
  const int base = red[warp];
  *total = red[32];
  __syncthreads();
  return base + in_warp;
}

// Exclusive prefix sum of v over the block in thread order; the block total goes to *total.
// All threads must call it; `red` needs >= 33 ints of shared scratch.
__device__ __forceinline__ int block_excl_sum(int v, int* red, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int c = lane < nw ? red[lane] : 0;
    int ci = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, ci, o);
      if (lane >= o) ci += y;
    }
    if (lane < nw) red[lane] = ci - c;
    if (lane == 31) red[32] = ci;
  }
  __syncthreads();
  const int base = red[warp];
  *total = red[32];
  __syncthreads();
  return base + incl - v;
}

}  // namespace actkv
