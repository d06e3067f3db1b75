// The llama.cpp sampler chain of PESTI's llama.cpp backend
// (llm-runner/src/llama.rs:465-508, `build_sampler`) on the GPU, one thread
// block of 1024 per row:
//
//   temperature (T > 0) -> top-k (k > 0) -> top-p (p > 0) -> min-p (> 0,
//   at least 256 kept) -> top-n-sigma (n = tfs, 0 < tfs < 1) -> typical
//   (0 < p < 1) -> repetition / frequency / presence penalties (penalty != 1)
//   -> inverse-CDF draw with the caller's u.
//
// The stages are the published filters (llama.cpp, wrapped by the
// llama-cpp-2 crate, is not part of the reference tree).  The row's candidate
// list is kept in index order in a per-row scratch array (logit, index, f64
// probability weight).  Every cut is a radix select over 8-bit digits of a
// sort key (the ordered bits of the f32 logit, or of the f64 typical
// deviation), by count (top-k, min-p's min_keep) or by probability mass
// (top-p, typical, the draw), followed by an ordered compaction in place.
// Masses are summed in f64 in a fixed order (per-warp histograms, warp
// butterflies, warps in order), so a row gives the same result on every run.
//
// Conventions shared with the CPU restatement of the chain: NaN logits count
// as -inf; the weight of a candidate is exp(l - max) in f64 (1 when l == max);
// ties in a sort key keep index order; a mass cut keeps the shortest prefix
// whose running mass reaches target * S, or the whole list when rounding
// leaves the target unreached.
#pragma once
#include <math.h>
#include <stdint.h>

#include "pesti_common.cuh"

namespace pesti {

constexpr int CH_THREADS = 1024;
constexpr int CH_WARPS = CH_THREADS / 32;
constexpr int CH_WINDOW = 8192;  // repetition window tokens held in shared memory
constexpr int CH_MIN_P_KEEP = 256;
constexpr int CH_Q = 4;     // 1024-element sub-tiles per chunk, loaded together
constexpr int CH_QRAW = 8;  // the same for the two passes over the raw row

// Mirrors pesti_llama_chain_params (the fields of llm-runner/src/llama/sampler.rs
// that build_sampler reads).
struct ChainArgs {
  float temperature;
  int32_t top_k;
  float top_p;
  float min_p;
  float tfs;
  float typical_p;
  float repetition_penalty;
  int32_t repeat_last_n;
  float frequency_penalty;
  float presence_penalty;
};

// Dynamic shared memory of the chain kernel.
struct ChainShared {
  double whist[CH_WARPS][256];  // per-warp mass histograms
  double mass[256];
  uint32_t cnt[256];
  double wd[CH_WARPS];
  uint32_t wu[CH_WARPS];
  uint32_t wu2[CH_WARPS];
  float wf[CH_WARPS];
  unsigned long long prefix;
  long long rem_cnt;
  double rem_mass;
  int all;  // the target was not reached: take every element of the bucket
  int pos;
  int take_eq;
  uint32_t h12[4096];  // top-k prefilter: counts of the top 12 key bits
  uint8_t wkeep[128];  // one-warp path: kept flags by list position
  int wn;              // one-warp path: the new list length
  uint32_t cq[CH_QRAW][CH_WARPS];
  uint32_t cq2[CH_QRAW][CH_WARPS];
  double dq[CH_Q][CH_WARPS];
  int window[CH_WINDOW];
};

__device__ __forceinline__ uint32_t ch_desc_key(float l) {
  const uint32_t u = __float_as_uint(l);
  const uint32_t asc = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ~asc;
}

// Candidate sources: the raw row (widened, NaN -> -inf, divided by T) or the
// scratch list.
template <typename TIn>
struct ChRaw {
  const TIn* row;
  float T;
  __device__ __forceinline__ float logit(int j) const {
    float x = load_logit<TIn>(row, j);
    if (x != x) x = -INFINITY;
    return T > 0.0f ? fdiv(x, T) : x;
  }
  __device__ __forceinline__ int index(int j) const { return j; }
};
struct ChList {
  float* l;
  int* i;
  __device__ __forceinline__ float logit(int j) const { return l[j]; }
  __device__ __forceinline__ int index(int j) const { return i[j]; }
};

// ---- block helpers (every thread calls them; each starts with a barrier) ----

__device__ __forceinline__ double ch_sum_d(ChainShared& sh, double v) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_reduce_add(v);
  __syncthreads();
  if (lane == 0) sh.wd[w] = v;
  __syncthreads();
  return warp_reduce_add(sh.wd[lane]);
}

__device__ __forceinline__ float ch_max_f(ChainShared& sh, float v) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_reduce_fmax(v);
  __syncthreads();
  if (lane == 0) sh.wf[w] = v;
  __syncthreads();
  return warp_reduce_fmax(sh.wf[lane]);
}

__device__ __forceinline__ uint32_t ch_sum_u(ChainShared& sh, uint32_t v) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_reduce_add(v);
  __syncthreads();
  if (lane == 0) sh.wu[w] = v;
  __syncthreads();
  return warp_reduce_add(sh.wu[lane]);
}

__device__ __forceinline__ int ch_max_i(ChainShared& sh, int v) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_reduce_max(v);
  __syncthreads();
  if (lane == 0) sh.wu[w] = (uint32_t)v;
  __syncthreads();
  return warp_reduce_max((int)sh.wu[lane]);
}

// One warp's contribution to the digit histograms.  By count: a shared
// atomic per element.  By mass: one group of equal digits at a time, its
// f64 sum by a warp butterfly into the warp's own histogram (a fixed order,
// so the sums do not depend on timing).
__device__ __forceinline__ void ch_hist_add(ChainShared& sh, bool act, uint32_t d, double w, bool by_mass) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (!by_mass) {  // counts are exact in any order: one atomic per element
    if (act) atomicAdd(&sh.cnt[d], 1u);
    return;
  }
  uint32_t rem = __ballot_sync(PESTI_FULL_MASK, act);
  while (rem) {
    const int L = __ffs(rem) - 1;
    const uint32_t d0 = __shfl_sync(PESTI_FULL_MASK, d, L);
    const bool in = act && d == d0;
    const uint32_t g = __ballot_sync(PESTI_FULL_MASK, in);
    const double s = warp_reduce_add(in ? w : 0.0);
    if (lane == L) {
      sh.whist[wid][d0] += s;
      atomicAdd(&sh.cnt[d0], (uint32_t)__popc(g));
    }
    rem &= ~g;
  }
}

// Top-k prefilter over a source: counts the top 12 bits of every key, and
// returns the largest 12-bit bucket b such that the buckets up to b hold at
// least k elements (the k-th smallest key lies in bucket b).
template <int Q, class Src, class KeyF>
__device__ uint32_t ch_bucket12(ChainShared& sh, const Src& src, int n, KeyF key, long long k) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  __syncthreads();
  for (int t = tid; t < 4096; t += CH_THREADS) sh.h12[t] = 0u;
  __syncthreads();
  for (int j0 = 0; j0 < n; j0 += CH_THREADS * Q) {
    uint32_t dq[Q];
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int j = j0 + q * CH_THREADS + tid;
      dq[q] = j < n ? key(src.logit(j)) >> 20 : 0xffffffffu;
    }
#pragma unroll
    for (int q = 0; q < Q; ++q)
      if (dq[q] != 0xffffffffu) atomicAdd(&sh.h12[dq[q]], 1u);
  }
  __syncthreads();
  // thread t: bins 4t .. 4t+3; block prefix of their counts
  uint32_t c[4], c4 = 0u;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    c[q] = sh.h12[tid * 4 + q];
    c4 += c[q];
  }
  const uint32_t ic = warp_incl_scan_add(c4);
  if (lane == 31) sh.wu[w] = ic;
  __syncthreads();
  const uint32_t vw = sh.wu[lane];
  const uint32_t iw = warp_incl_scan_add(vw);
  long long cum = (long long)__shfl_sync(PESTI_FULL_MASK, iw - vw, w) + (ic - c4);
  if (tid == 0) sh.prefix = 4095ull;
  __syncthreads();
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (cum < k && cum + c[q] >= k) sh.prefix = (unsigned long long)(tid * 4 + q);
    cum += c[q];
  }
  __syncthreads();
  return (uint32_t)sh.prefix;
}

// Radix select over the n elements of a source; key(l) maps a logit to its
// sort key.  By count: the want_cnt smallest keys (ties in list order).  By
// mass: the shortest prefix in key order whose running mass reaches
// want_mass.  Leaves in shared memory the boundary key (sh.prefix) and, by
// count, how many elements equal to it are kept (sh.rem_cnt); by mass the
// walk below finds that.  Each chunk loads CH_Q sub-tiles of 1024 elements
// before it adds them up, so their loads are in flight together.
template <typename K, class Src, class KeyF, class WF>
__device__ void ch_radix(ChainShared& sh, const Src& src, int n, KeyF key, WF wt, bool by_mass, long long want_cnt,
                         double want_mass) {
  constexpr int NB = (int)sizeof(K) * 8;
  const int tid = threadIdx.x, lane = tid & 31;
  __syncthreads();
  if (tid == 0) {
    sh.prefix = 0ull;
    sh.rem_cnt = want_cnt;
    sh.rem_mass = want_mass;
    sh.all = 0;
  }
  for (int shift = NB - 8; shift >= 0; shift -= 8) {
    __syncthreads();
    for (int t = tid; t < 256; t += CH_THREADS) sh.cnt[t] = 0u;
    if (by_mass)
      for (int t = tid; t < CH_WARPS * 256; t += CH_THREADS) (&sh.whist[0][0])[t] = 0.0;
    __syncthreads();
    const K pre = (K)sh.prefix;
    const int hs = shift + 8;
    for (int j0 = 0; j0 < n; j0 += CH_THREADS * CH_Q) {
      K kq[CH_Q];
      double wq[CH_Q];
      bool aq[CH_Q];
#pragma unroll
      for (int q = 0; q < CH_Q; ++q) {
        const int j = j0 + q * CH_THREADS + tid;
        kq[q] = j < n ? key(src.logit(j)) : (K)0;
        aq[q] = j < n && (hs >= NB || (kq[q] >> hs) == (pre >> hs));
      }
      // weights only of the elements inside the prefix found so far
#pragma unroll
      for (int q = 0; q < CH_Q; ++q) wq[q] = (by_mass && aq[q]) ? wt(j0 + q * CH_THREADS + tid) : 0.0;
#pragma unroll
      for (int q = 0; q < CH_Q; ++q) ch_hist_add(sh, aq[q], (uint32_t)(kq[q] >> shift) & 255u, wq[q], by_mass);
    }
    __syncthreads();
    if (by_mass && tid < 256) {
      double m = 0.0;
      for (int q = 0; q < CH_WARPS; ++q) m += sh.whist[q][tid];
      sh.mass[tid] = m;
    }
    __syncthreads();
    if (tid < 32) {
      // lane: bins 8*lane .. 8*lane+7
      uint32_t c8 = 0u;
      double m8 = 0.0;
      for (int q = 0; q < 8; ++q) {
        c8 += sh.cnt[lane * 8 + q];
        if (by_mass) m8 += sh.mass[lane * 8 + q];
      }
      const uint32_t ic = warp_incl_scan_add(c8);
      const double im = warp_incl_scan_add(m8);
      long long cc = (long long)(ic - c8);
      double cm = im - m8;
      const long long rc = sh.rem_cnt;
      const double rm = sh.rem_mass;
      const bool all = sh.all != 0;
      int hit = -1, last = -1;
      long long hc = 0;
      double hm = 0.0;
      for (int q = 0; q < 8; ++q) {
        const int b = lane * 8 + q;
        const uint32_t c = sh.cnt[b];
        if (c == 0u) continue;
        last = b;
        const double m = by_mass ? sh.mass[b] : 0.0;
        if (hit < 0 && !all && (by_mass ? cm + m >= rm : cc + (long long)c >= rc)) {
          hit = b;
          hc = cc;
          hm = cm;
        }
        cc += c;
        cm += m;
      }
      const uint32_t hb = __ballot_sync(PESTI_FULL_MASK, hit >= 0);
      if (hb) {
        const int L = __ffs(hb) - 1;
        if (lane == L) {
          sh.prefix |= (unsigned long long)hit << shift;
          sh.rem_cnt = rc - hc;
          sh.rem_mass = rm - hm;
        }
      } else {
        // unreached (or already taking everything): the highest bucket, whole
        const uint32_t lb = __ballot_sync(PESTI_FULL_MASK, last >= 0);
        if (lb) {
          const int L = 31 - __clz(lb);
          if (lane == L) {
            sh.prefix |= (unsigned long long)last << shift;
            sh.rem_cnt = (long long)sh.cnt[last];
            sh.rem_mass = INFINITY;
            sh.all = 1;
          }
        }
      }
    }
  }
  __syncthreads();
}

// After ch_radix: the elements equal to the boundary key, in list order,
// until the kept count (by count) or the running mass (by mass) is reached.
// Sets sh.take_eq (kept elements equal to the boundary key) and sh.pos (the
// list position of the last kept one); when the target stays unreached,
// every equal element is kept and sh.pos is the last of them.  The running
// mass is summed in list order: sub-tile, then warp, then lane.
template <typename K, class Src, class KeyF, class WF>
__device__ void ch_walk(ChainShared& sh, const Src& src, int n, KeyF key, WF wt, bool by_mass) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const uint32_t lt = (1u << lane) - 1u;
  __syncthreads();
  const K bk = (K)sh.prefix;
  const long long rc = sh.rem_cnt;
  const double rm = sh.rem_mass;
  __syncthreads();
  if (tid == 0) sh.pos = 0x7fffffff;
  long long base_c = 0;
  double base_m = 0.0;
  int last_eq = -1;
  for (int j0 = 0; j0 < n; j0 += CH_THREADS * CH_Q) {
    bool eq[CH_Q];
    double wv[CH_Q];
#pragma unroll
    for (int q = 0; q < CH_Q; ++q) {
      const int j = j0 + q * CH_THREADS + tid;
      eq[q] = j < n && key(src.logit(j)) == bk;
    }
#pragma unroll
    for (int q = 0; q < CH_Q; ++q) wv[q] = (by_mass && eq[q]) ? wt(j0 + q * CH_THREADS + tid) : 0.0;
    uint32_t be[CH_Q];
    double iw[CH_Q];
#pragma unroll
    for (int q = 0; q < CH_Q; ++q) {
      be[q] = __ballot_sync(PESTI_FULL_MASK, eq[q]);
      iw[q] = by_mass ? warp_incl_scan_add(wv[q]) : 0.0;
      if (lane == 31) {
        sh.cq[q][w] = __popc(be[q]);
        sh.dq[q][w] = iw[q];
      }
    }
    __syncthreads();
    long long run_c = base_c;
    double run_m = base_m;
    bool hit = false;
    int hitj = 0;
    long long hit_rank = 0;
#pragma unroll
    for (int q = 0; q < CH_Q; ++q) {
      const uint32_t vc = sh.cq[q][lane];
      const uint32_t ic = warp_incl_scan_add(vc);
      const long long ex_c = run_c + __shfl_sync(PESTI_FULL_MASK, ic - vc, w) + __popc(be[q] & lt);
      double ex_m = run_m, tot_m = 0.0;
      if (by_mass) {
        const double vm = sh.dq[q][lane];
        const double im = warp_incl_scan_add(vm);
        ex_m += __shfl_sync(PESTI_FULL_MASK, im - vm, w);
        tot_m = __shfl_sync(PESTI_FULL_MASK, im, 31);
      }
      const bool h = eq[q] && (by_mass ? ex_m + iw[q] >= rm : ex_c + 1 >= rc);
      if (h && !hit) {
        hit = true;
        hitj = j0 + q * CH_THREADS + tid;
        hit_rank = ex_c + 1;
      }
      if (eq[q]) last_eq = j0 + q * CH_THREADS + tid;
      run_c += __shfl_sync(PESTI_FULL_MASK, ic, 31);
      run_m += tot_m;
    }
    if (hit) atomicMin(&sh.pos, hitj);
    __syncthreads();
    const int p = sh.pos;
    if (hit && p == hitj) sh.take_eq = (int)hit_rank;
    base_c = run_c;
    base_m = run_m;
    if (p != 0x7fffffff) break;
  }
  const int lastj = ch_max_i(sh, last_eq);
  if (tid == 0 && sh.pos == 0x7fffffff) {
    sh.pos = lastj;
    sh.take_eq = (int)base_c;
  }
  __syncthreads();
}

// Ordered compaction of a source into the list (in place when the source is
// the list).  SEL: keeps key < bk and the first take_eq elements equal to bk;
// otherwise keeps the elements whose logit satisfies pred.  Returns the new
// length.  Each chunk's elements are read before its first barrier and
// written after it, to positions below the chunk's end.
template <bool SEL, typename K, int Q = CH_Q, class Src, class KeyF, class Pred>
__device__ int ch_compact(ChainShared& sh, const Src& src, int n, KeyF key, K bk, long long take_eq, Pred pred,
                          float* ol, int* oi) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const uint32_t lt = (1u << lane) - 1u;
  long long base_eq = 0;
  int base_out = 0;
  __syncthreads();
  for (int j0 = 0; j0 < n; j0 += CH_THREADS * Q) {
    float lv[Q];
    int iv[Q];
    bool kp[Q], eq[Q];
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const int j = j0 + q * CH_THREADS + tid;
      const bool have = j < n;
      lv[q] = have ? src.logit(j) : 0.0f;
      iv[q] = have ? src.index(j) : 0;
      if (SEL) {
        const K k = key(lv[q]);
        kp[q] = have && k < bk;
        eq[q] = have && k == bk;
      } else {
        kp[q] = have && pred(lv[q]);
        eq[q] = false;
      }
    }
    if (SEL) {
      uint32_t be[Q];
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        be[q] = __ballot_sync(PESTI_FULL_MASK, eq[q]);
        if (lane == 0) sh.cq[q][w] = __popc(be[q]);
      }
      __syncthreads();
      long long run = base_eq;
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        const uint32_t v = sh.cq[q][lane];
        const uint32_t ic = warp_incl_scan_add(v);
        const long long r = run + __shfl_sync(PESTI_FULL_MASK, ic - v, w) + __popc(be[q] & lt);
        kp[q] = kp[q] || (eq[q] && r < take_eq);
        run += __shfl_sync(PESTI_FULL_MASK, ic, 31);
      }
      base_eq = run;
    }
    uint32_t bo[Q];
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      bo[q] = __ballot_sync(PESTI_FULL_MASK, kp[q]);
      if (lane == 0) sh.cq2[q][w] = __popc(bo[q]);
    }
    __syncthreads();
    int run = base_out;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
      const uint32_t v = sh.cq2[q][lane];
      const uint32_t ic = warp_incl_scan_add(v);
      const int pos = run + (int)__shfl_sync(PESTI_FULL_MASK, ic - v, w) + __popc(bo[q] & lt);
      if (kp[q]) {
        ol[pos] = lv[q];
        oi[pos] = iv[q];
      }
      run += (int)__shfl_sync(PESTI_FULL_MASK, ic, 31);
    }
    base_out = run;
    __syncthreads();
  }
  return base_out;
}

// ---- one-warp path for short lists (at most 128 candidates) ----
// A stage on a short list runs in warp 0 alone: a bitonic sort in registers
// by (key, list position), an f64 prefix in sorted order, and an ordered
// compaction, with no block-wide barrier inside.

constexpr int CH_WE = 4;             // list elements per lane
constexpr int CH_WN = 32 * CH_WE;    // 128

template <typename K>
__device__ __forceinline__ bool ch_pair_less(K ka, int ja, K kb, int jb) {
  return ka < kb || (ka == kb && ja < jb);
}

// Orders two registers of one lane: ascending when up.
template <typename K>
__device__ __forceinline__ void ch_cex(K& ka, int& ja, K& kb, int& jb, bool up) {
  const bool sw = up ? ch_pair_less(kb, jb, ka, ja) : ch_pair_less(ka, ja, kb, jb);
  if (sw) {
    const K tk = ka;
    ka = kb;
    kb = tk;
    const int tj = ja;
    ja = jb;
    jb = tj;
  }
}

// Warp 0 sorts the first n (<= 128) list elements by (key, position): lane
// l ends with sorted positions h*32 + l in kk[h], jj[h] (padding: the
// largest key, position 0x7fffffff).
template <typename K, class KeyF>
__device__ __forceinline__ void ch_warp_sort(const float* l, int n, KeyF key, K (&kk)[CH_WE], int (&jj)[CH_WE]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int h = 0; h < CH_WE; ++h) {
    const int j = h * 32 + lane;
    if (j < n) {
      kk[h] = key(l[j]);
      jj[h] = j;
    } else {
      kk[h] = ~(K)0;
      jj[h] = 0x7fffffff;
    }
  }
#pragma unroll
  for (int k = 2; k <= CH_WN; k <<= 1) {
#pragma unroll
    for (int js = k >> 1; js > 0; js >>= 1) {
      if (js == 64) {
        ch_cex(kk[0], jj[0], kk[2], jj[2], (lane & k) == 0);
        ch_cex(kk[1], jj[1], kk[3], jj[3], ((32 + lane) & k) == 0);
      } else if (js == 32) {
        ch_cex(kk[0], jj[0], kk[1], jj[1], (lane & k) == 0);
        ch_cex(kk[2], jj[2], kk[3], jj[3], ((64 + lane) & k) == 0);
      } else {
        const bool lower = (lane & js) == 0;
#pragma unroll
        for (int h = 0; h < CH_WE; ++h) {
          const K ok = __shfl_xor_sync(PESTI_FULL_MASK, kk[h], js);
          const int oj = __shfl_xor_sync(PESTI_FULL_MASK, jj[h], js);
          const bool up = ((h * 32 + lane) & k) == 0;
          const bool oless = ch_pair_less(ok, oj, kk[h], jj[h]);
          const bool same = ok == kk[h] && oj == jj[h];
          // ascending pairs: the lower position keeps the smaller
          const bool take = (lower == up) ? oless : (!oless && !same);
          if (take) {
            kk[h] = ok;
            jj[h] = oj;
          }
        }
      }
    }
  }
}

// Warp 0: max, weights into cw and their sum (lane order, then a butterfly).
__device__ __forceinline__ double ch_warp_weights(const float* l, double* cw, int n, float& mx_out) {
  const int lane = threadIdx.x & 31;
  float mx = -INFINITY;
#pragma unroll
  for (int h = 0; h < CH_WE; ++h) {
    const int j = h * 32 + lane;
    if (j < n) mx = fmaxf(mx, l[j]);
  }
  mx = warp_reduce_fmax(mx);
  double s = 0.0;
#pragma unroll
  for (int h = 0; h < CH_WE; ++h) {
    const int j = h * 32 + lane;
    if (j < n) {
      const float x = l[j];
      const double w = x == mx ? 1.0 : exp((double)x - (double)mx);
      cw[j] = w;
      s += w;
    }
  }
  __syncwarp();
  mx_out = mx;
  return warp_reduce_add(s);
}

// Warp 0: the cut on a short list, by count (the want_cnt first in key
// order) or by mass (the shortest prefix in key order whose running mass
// reaches target, or all).  Marks the kept list positions in sh.wkeep and
// returns the list position of the last kept element.
template <typename K, class KeyF>
__device__ __forceinline__ int ch_warp_select(ChainShared& sh, const float* l, const double* cw, int n, KeyF key,
                                              bool by_mass, int want_cnt, double target) {
  const int lane = threadIdx.x & 31;
  K kk[CH_WE];
  int jj[CH_WE];
  ch_warp_sort<K>(l, n, key, kk, jj);
  int pstar = -1;
  if (by_mass) {
    double run = 0.0;
#pragma unroll
    for (int h = 0; h < CH_WE; ++h) {
      const bool v = jj[h] < n;
      const double w = v ? cw[jj[h]] : 0.0;
      const double c = run + warp_incl_scan_add(w);
      const uint32_t hb = __ballot_sync(PESTI_FULL_MASK, v && c >= target);
      if (pstar < 0 && hb) pstar = h * 32 + __ffs(hb) - 1;
      run = __shfl_sync(PESTI_FULL_MASK, c, 31);
    }
    if (pstar < 0) pstar = n - 1;
  } else {
    pstar = min(want_cnt, n) - 1;
  }
#pragma unroll
  for (int h = 0; h < CH_WE; ++h)
    if (jj[h] < n) sh.wkeep[jj[h]] = (h * 32 + lane) <= pstar ? 1 : 0;
  const int hq = pstar >> 5;
  int mine = jj[0];
#pragma unroll
  for (int h = 1; h < CH_WE; ++h)
    if (hq == h) mine = jj[h];
  const int bj = __shfl_sync(PESTI_FULL_MASK, mine, pstar & 31);
  __syncwarp();
  return bj;
}

// Warp 0: ordered compaction of a short list in place by sh.wkeep.
__device__ __forceinline__ int ch_warp_compact(ChainShared& sh, float* l, int* ix, int n) {
  const int lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  float lv[CH_WE];
  int iv[CH_WE];
  bool kp[CH_WE];
  __syncwarp();
#pragma unroll
  for (int h = 0; h < CH_WE; ++h) {
    const int j = h * 32 + lane;
    kp[h] = j < n && sh.wkeep[j] != 0;
    lv[h] = j < n ? l[j] : 0.0f;
    iv[h] = j < n ? ix[j] : 0;
  }
  __syncwarp();
  int run = 0;
#pragma unroll
  for (int h = 0; h < CH_WE; ++h) {
    const uint32_t b = __ballot_sync(PESTI_FULL_MASK, kp[h]);
    if (kp[h]) {
      const int pos = run + __popc(b & lt);
      l[pos] = lv[h];
      ix[pos] = iv[h];
    }
    run += __popc(b);
  }
  __syncwarp();
  return run;
}

// f64 weights exp(l - max) of the list into cw; returns their sum (fixed
// order).  mx: the list's largest logit.
__device__ __forceinline__ double ch_weights(ChainShared& sh, const float* l, double* cw, int n, float mx) {
  double s = 0.0;
#pragma unroll 4
  for (int j = threadIdx.x; j < n; j += CH_THREADS) {
    const float x = l[j];
    const double w = x == mx ? 1.0 : exp((double)x - (double)mx);
    cw[j] = w;
    s += w;
  }
  return ch_sum_d(sh, s);
}

__device__ __forceinline__ float ch_list_max(ChainShared& sh, const float* l, int n) {
  float m = -INFINITY;
#pragma unroll 4
  for (int j = threadIdx.x; j < n; j += CH_THREADS) m = fmaxf(m, l[j]);
  return ch_max_f(sh, m);
}

// TIn: float (f32 logits), uint16_t (bf16 bits) or __half.
template <typename TIn>
__global__ void __launch_bounds__(CH_THREADS, 1)
    llama_chain_kernel(const TIn* __restrict__ logits, int V, long long ld, ChainArgs a,
                       const int32_t* __restrict__ hist, const int32_t* __restrict__ hist_len, long long hist_ld,
                       const float* __restrict__ u, int32_t* __restrict__ out_tok, int32_t* __restrict__ out_kept,
                       float* __restrict__ sl, int* __restrict__ si, double* __restrict__ sw) {
  extern __shared__ __align__(16) unsigned char ch_smem[];
  ChainShared& sh = *reinterpret_cast<ChainShared*>(ch_smem);
  const int tid = threadIdx.x;
  const long long b = blockIdx.x;
  const ChRaw<TIn> raw{logits + b * ld, a.temperature};
  float* l = sl + b * (long long)V;
  int* ix = si + b * (long long)V;
  double* cw = sw + b * (long long)V;
  const ChList list{l, ix};
  auto dkey = [](float x) -> uint32_t { return ch_desc_key(x); };
  auto wlist = [&](int j) -> double { return cw[j]; };
  auto wnone = [](int) -> double { return 0.0; };
  auto every = [](float) { return true; };
  int n = V;

  // temperature + top-k, from the raw row into the list
  if (a.top_k > 0 && a.top_k < n) {
    // two passes over the row: the 12-bit bucket of the k-th largest logit,
    // then every element up to that bucket into the list; the exact select
    // runs on the list
    const uint32_t b12 = ch_bucket12<CH_QRAW>(sh, raw, n, dkey, a.top_k);
    n = ch_compact<false, uint32_t, CH_QRAW>(sh, raw, n, dkey, 0u, 0,
                                             [b12](float x) { return (ch_desc_key(x) >> 20) <= b12; }, l, ix);
    if (a.top_k < n && n <= CH_WN) {
      if (tid < 32) {
        ch_warp_select<uint32_t>(sh, l, cw, n, dkey, false, a.top_k, 0.0);
        const int m = ch_warp_compact(sh, l, ix, n);
        if (tid == 0) sh.wn = m;
      }
      __syncthreads();
      n = sh.wn;
    } else if (a.top_k < n) {
      ch_radix<uint32_t>(sh, list, n, dkey, wnone, false, a.top_k, 0.0);
      const uint32_t bk = (uint32_t)sh.prefix;
      const long long te = sh.rem_cnt;
      n = ch_compact<true, uint32_t>(sh, list, n, dkey, bk, te, every, l, ix);
    }
  } else {
    n = ch_compact<false, uint32_t, CH_QRAW>(sh, raw, n, dkey, 0u, 0, every, l, ix);
  }

  // top-p
  if (a.top_p > 0.0f && a.top_p < 1.0f && n <= CH_WN) {
    if (tid < 32) {
      float mx;
      const double S = ch_warp_weights(l, cw, n, mx);
      ch_warp_select<uint32_t>(sh, l, cw, n, dkey, true, 0, (double)a.top_p * S);
      const int m = ch_warp_compact(sh, l, ix, n);
      if (tid == 0) sh.wn = m;
    }
    __syncthreads();
    n = sh.wn;
  } else if (a.top_p > 0.0f && a.top_p < 1.0f) {
    const float mx = ch_list_max(sh, l, n);
    const double S = ch_weights(sh, l, cw, n, mx);
    ch_radix<uint32_t>(sh, list, n, dkey, wlist, true, 0, (double)a.top_p * S);
    ch_walk<uint32_t>(sh, list, n, dkey, wlist, true);
    const uint32_t bk = (uint32_t)sh.prefix;
    const long long te = sh.take_eq;
    n = ch_compact<true, uint32_t>(sh, list, n, dkey, bk, te, every, l, ix);
  }

  // min-p, at least 256 kept
  if (a.min_p > 0.0f) {
    const float mx = ch_list_max(sh, l, n);
    const double thr = log((double)a.min_p);
    uint32_t c = 0u;
#pragma unroll 4
    for (int j = tid; j < n; j += CH_THREADS) {
      const float x = l[j];
      const double d = x == mx ? 0.0 : (double)x - (double)mx;
      c += d >= thr ? 1u : 0u;
    }
    c = ch_sum_u(sh, c);
    const int keep = max((int)c, min(CH_MIN_P_KEEP, n));
    if (keep < n) {
      ch_radix<uint32_t>(sh, list, n, dkey, wnone, false, keep, 0.0);
      const uint32_t bk = (uint32_t)sh.prefix;
      const long long te = sh.rem_cnt;
      n = ch_compact<true, uint32_t>(sh, list, n, dkey, bk, te, every, l, ix);
    }
  }

  // top-n-sigma (the config's tfs)
  if (a.tfs > 0.0f && a.tfs < 1.0f) {
    const float mx = ch_list_max(sh, l, n);
    double s = 0.0;
    uint32_t c = 0u;
    for (int j = tid; j < n; j += CH_THREADS) {
      const float x = l[j];
      if (isfinite(x)) {
        s += (double)x;
        ++c;
      }
    }
    s = ch_sum_d(sh, s);
    c = ch_sum_u(sh, c);
    if (c > 0u) {
      const double mu = s / (double)c;
      double q = 0.0;
      for (int j = tid; j < n; j += CH_THREADS) {
        const float x = l[j];
        if (isfinite(x)) {
          const double e = (double)x - mu;
          q += e * e;
        }
      }
      q = ch_sum_d(sh, q);
      const double sigma = sqrt(q / (double)c);
      const double thr = (double)mx - (double)a.tfs * sigma;
      n = ch_compact<false, uint32_t>(sh, list, n, dkey, 0u, 0, [thr](float x) { return (double)x >= thr; }, l, ix);
    }
  }

  // typical
  if (a.typical_p > 0.0f && a.typical_p < 1.0f && n <= CH_WN) {
    if (tid < 32) {
      float mx;
      const double S = ch_warp_weights(l, cw, n, mx);
      double e = 0.0;
#pragma unroll
      for (int h = 0; h < CH_WE; ++h) {
        const int j = h * 32 + tid;
        if (j < n) {
          const float x = l[j];
          const double w = cw[j];
          if (w > 0.0) e += w * (x == mx ? 0.0 : (double)x - (double)mx);
        }
      }
      e = warp_reduce_add(e);
      const double lnS = log(S);
      const double H = lnS - e / S;
      auto tkey = [&](float x) -> unsigned long long {
        const double d = x == mx ? 0.0 : (double)x - (double)mx;
        return (unsigned long long)__double_as_longlong(fabs(lnS - d - H));
      };
      ch_warp_select<unsigned long long>(sh, l, cw, n, tkey, true, 0, (double)a.typical_p * S);
      const int m = ch_warp_compact(sh, l, ix, n);
      if (tid == 0) sh.wn = m;
    }
    __syncthreads();
    n = sh.wn;
  } else if (a.typical_p > 0.0f && a.typical_p < 1.0f) {
    const float mx = ch_list_max(sh, l, n);
    const double S = ch_weights(sh, l, cw, n, mx);
    double e = 0.0;
    for (int j = tid; j < n; j += CH_THREADS) {
      const float x = l[j];
      const double w = cw[j];
      if (w > 0.0) e += w * (x == mx ? 0.0 : (double)x - (double)mx);
    }
    e = ch_sum_d(sh, e);
    const double lnS = log(S);
    const double H = lnS - e / S;
    auto tkey = [&](float x) -> unsigned long long {
      const double d = x == mx ? 0.0 : (double)x - (double)mx;
      return (unsigned long long)__double_as_longlong(fabs(lnS - d - H));
    };
    ch_radix<unsigned long long>(sh, list, n, tkey, wlist, true, 0, (double)a.typical_p * S);
    ch_walk<unsigned long long>(sh, list, n, tkey, wlist, true);
    const unsigned long long bk = sh.prefix;
    const long long te = sh.take_eq;
    n = ch_compact<true, unsigned long long>(sh, list, n, tkey, bk, te, every, l, ix);
  }

  // penalties over the last repeat_last_n tokens of the row's history
  if (a.repetition_penalty != 1.0f && a.repeat_last_n != 0 && hist != nullptr) {
    const long long hl = hist_len ? min(max((long long)hist_len[b], 0ll), hist_ld) : hist_ld;
    const long long w = a.repeat_last_n < 0 ? hl : min(hl, (long long)a.repeat_last_n);
    const int32_t* h = hist + b * hist_ld + (hl - w);
    // the window padded to a power of two (at least 2, at most CH_WINDOW)
    int wp = 2;
    while (wp < w) wp <<= 1;
    __syncthreads();
    for (int t = tid; t < wp; t += CH_THREADS) {
      const int32_t v = t < w ? h[t] : -1;
      sh.window[t] = (v >= 0 && v < V) ? v : 0x7fffffff;
    }
    __syncthreads();
    // bitonic sort of the window (ascending)
    for (int k = 2; k <= wp; k <<= 1) {
      for (int jj = k >> 1; jj > 0; jj >>= 1) {
        for (int t = tid; t < wp; t += CH_THREADS) {
          const int p = t ^ jj;
          if (p > t) {
            const int x = sh.window[t], y = sh.window[p];
            const bool up = (t & k) == 0;
            if ((x > y) == up) {
              sh.window[t] = y;
              sh.window[p] = x;
            }
          }
        }
        __syncthreads();
      }
    }
    const float rp = a.repetition_penalty;
    for (int t = tid; t < wp; t += CH_THREADS) {
      const int tok = sh.window[t];
      if (tok == 0x7fffffff || (t > 0 && sh.window[t - 1] == tok)) continue;
      int e2 = t + 1;
      while (e2 < wp && sh.window[e2] == tok) ++e2;
      const int c = e2 - t;
      // the candidate list is in index order
      int lo = 0, hi = n;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (ix[mid] < tok) lo = mid + 1; else hi = mid;
      }
      if (lo < n && ix[lo] == tok) {
        float v = l[lo];
        v = v <= 0.0f ? __fmul_rn(v, rp) : fdiv(v, rp);
        const float sub = fadd(__fmul_rn((float)c, a.frequency_penalty), c > 0 ? a.presence_penalty : 0.0f);
        l[lo] = fsub(v, sub);
      }
    }
    __syncthreads();
  }

  // the draw
  if (n <= CH_WN) {
    if (tid < 32) {
      float mx;
      const double S = ch_warp_weights(l, cw, n, mx);
      const int bj = ch_warp_select<uint32_t>(sh, l, cw, n, dkey, true, 0, (double)u[b] * S);
      if (tid == 0) {
        out_tok[b] = (n > 0 && bj >= 0 && bj < n) ? ix[bj] : -1;
        if (out_kept) out_kept[b] = n;
      }
    }
  } else {
    const float mx = ch_list_max(sh, l, n);
    const double S = ch_weights(sh, l, cw, n, mx);
    ch_radix<uint32_t>(sh, list, n, dkey, wlist, true, 0, (double)u[b] * S);
    ch_walk<uint32_t>(sh, list, n, dkey, wlist, true);
    if (tid == 0) {
      // every stage keeps at least one candidate; -1 would mark an empty list
      out_tok[b] = (n > 0 && sh.pos >= 0 && sh.pos < n) ? ix[sh.pos] : -1;
      if (out_kept) out_kept[b] = n;
    }
  }
}

}  // namespace pesti
