// The loop control of generate() (transformer/model.rs:508-531) on the
// device, for B sequences decoded together: after each step's sample, the
// token goes to the next step's input and into the row's output, and the row
// stops on a stop token, after max_tokens tokens, or when its position
// reaches max_seq_len, without a read back to the host per step.
#pragma once
#include <stdint.h>

namespace pesti {

// One block; rows tid, tid + blockDim.x, ...  done codes: 1 stop token,
// 2 max_tokens, 3 max_seq_len.
__global__ void __launch_bounds__(256) generate_advance_kernel(const uint32_t* __restrict__ next, long long B,
                                                               const uint32_t* __restrict__ stop, long long n_stop,
                                                               long long max_tokens, long long max_seq_len,
                                                               uint32_t* __restrict__ generated, long long cap,
                                                               int32_t* __restrict__ count, uint8_t* __restrict__ done,
                                                               uint32_t* __restrict__ last, int32_t* active) {
  int live = 0;
  for (long long b = threadIdx.x; b < B; b += blockDim.x) {
    uint8_t d = done[b];
    if (d == 0) {
      long long c = count[b];
      if (c >= max_tokens) {  // the loop's bound (for _ in 0..max_tokens), already reached
        d = 2;
      } else {
        const uint32_t t = next[b];
        bool is_stop = false;
        for (long long j = 0; j < n_stop; ++j) is_stop = is_stop || stop[j] == t;  // stop_tokens.contains
        if (is_stop) {
          d = 1;  // break before the push
        } else {
          generated[b * cap + c] = t;  // generated.push(next_token)
          last[b] = t;                 // context.push(next_token): the next forward's input
          ++c;                         // pos += 1
          count[b] = (int32_t)c;
          if (c >= max_seq_len) d = 3;     // if pos >= max_seq_len { break }
          else if (c >= max_tokens) d = 2;  // the loop ends
        }
      }
      done[b] = d;
    }
    live += d == 0 ? 1 : 0;
  }
  __shared__ int total;
  if (threadIdx.x == 0) total = 0;
  __syncthreads();
  if (live) atomicAdd(&total, live);
  __syncthreads();
  if (threadIdx.x == 0 && active) *active = total;
}

}  // namespace pesti
