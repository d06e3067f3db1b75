// Shared device helpers for the sampler kernels: float bit views, IEEE
// single-rounding arithmetic, warp/block scans and reductions.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define PESTI_FULL_MASK 0xffffffffu

__device__ __forceinline__ uint32_t fbits(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float bitsf(uint32_t u) { return __uint_as_float(u); }

// One IEEE round-to-nearest f32 operation each; never contracted into FMA.
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

__device__ __forceinline__ bool is_nan(float x) { return x != x; }

template <typename T>
__device__ __forceinline__ T warp_incl_scan_add(T v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_up_sync(PESTI_FULL_MASK, v, o);
    if (lane >= o) v += y;
  }
  return v;
}

template <typename T>
__device__ __forceinline__ T warp_reduce_add(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(PESTI_FULL_MASK, v, o);
  return v;
}

__device__ __forceinline__ float warp_reduce_fmax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(PESTI_FULL_MASK, v, o));
  return v;
}

template <typename T>
__device__ __forceinline__ T warp_reduce_max(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    T y = __shfl_xor_sync(PESTI_FULL_MASK, v, o);
    v = y > v ? y : v;
  }
  return v;
}

template <typename T>
__device__ __forceinline__ T warp_reduce_min(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    T y = __shfl_xor_sync(PESTI_FULL_MASK, v, o);
    v = y < v ? y : v;
  }
  return v;
}

// Block-wide exclusive prefix sum; `scratch` holds >= 33 T in shared memory.
// Every thread of the block must call it.  Returns the exclusive prefix of v
// in thread order and writes the block total to `total`.
template <typename T>
__device__ __forceinline__ T block_excl_scan_add(T v, T* scratch, T& total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const T inc = warp_incl_scan_add(v);
  if (lane == 31) scratch[wid] = inc;
  __syncthreads();
  if (wid == 0) {
    const T w = lane < nw ? scratch[lane] : T(0);
    const T wi = warp_incl_scan_add(w);
    if (lane < nw) scratch[lane] = wi - w;
    if (lane == nw - 1) scratch[32] = wi;
  }
  __syncthreads();
  const T res = scratch[wid] + inc - v;
  total = scratch[32];
  __syncthreads();
  return res;
}

template <typename T>
__device__ __forceinline__ T block_reduce_add(T v, T* scratch) {
  T total;
  (void)block_excl_scan_add(v, scratch, total);
  return total;
}

template <typename T>
__device__ __forceinline__ T block_reduce_max(T v, T* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_reduce_max(v);
  if (lane == 0) scratch[wid] = v;
  __syncthreads();
  if (wid == 0) {
    T w = lane < nw ? scratch[lane] : scratch[0];
    w = warp_reduce_max(w);
    if (lane == 0) scratch[32] = w;
  }
  __syncthreads();
  const T r = scratch[32];
  __syncthreads();
  return r;
}

template <typename T>
__device__ __forceinline__ T block_reduce_min(T v, T* scratch) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_reduce_min(v);
  if (lane == 0) scratch[wid] = v;
  __syncthreads();
  if (wid == 0) {
    T w = lane < nw ? scratch[lane] : scratch[0];
    w = warp_reduce_min(w);
    if (lane == 0) scratch[32] = w;
  }
  __syncthreads();
  const T r = scratch[32];
  __syncthreads();
  return r;
}
