// Per-row draws on the device: one PCG32 generator per row (O'Neill 2014,
// XSH-RR 64->32), the same generator as the host Pcg32 of pesti_sampler.py.
// A row's draw is (next_u32 >> 8) * 2^-24, the [0, 1) 24-bit grid of the f32
// draw the reference takes once per sample() call (sampling.rs:98).
#pragma once
#include <stdint.h>

namespace pesti {

constexpr uint64_t PCG_MULT = 6364136223846793005ull;

__device__ __forceinline__ uint32_t pcg32_next(uint64_t& state, uint64_t inc) {
  const uint64_t old = state;
  state = old * PCG_MULT + inc;
  const uint32_t xs = (uint32_t)(((old >> 18) ^ old) >> 27);
  const uint32_t rot = (uint32_t)(old >> 59);
  return (xs >> rot) | (xs << ((32u - rot) & 31u));
}

// Row b: stream first_stream + b, seeded with `seed` (state and increment at
// state[2b], state[2b+1]).
__global__ void pcg32_seed_kernel(uint64_t* state, long long B, uint64_t seed, uint64_t first_stream) {
  const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const uint64_t inc = ((first_stream + (uint64_t)b) << 1) | 1ull;
  uint64_t st = 0ull;
  (void)pcg32_next(st, inc);
  st += seed;
  (void)pcg32_next(st, inc);
  state[2 * b] = st;
  state[2 * b + 1] = inc;
}

// One draw per row into u[b]; the row's state advances by one step.
__global__ void pcg32_draw_kernel(uint64_t* state, long long B, float* u) {
  const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  uint64_t st = state[2 * b];
  const uint64_t inc = state[2 * b + 1];
  const uint32_t v = pcg32_next(st, inc);
  state[2 * b] = st;
  u[b] = (float)(v >> 8) * 0x1p-24f;
}

}  // namespace pesti
