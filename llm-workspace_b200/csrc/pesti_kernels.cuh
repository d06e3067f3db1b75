// Kernels of the sampler.  Semantics follow llm-runner/src/transformer/sampling.rs
// line by line; every f32 operation the reference performs is performed here
// as the same single IEEE operation on the same operands, and every f32 sum
// is the reference's sequential fold, emulated exactly (pesti_fold.cuh).
//
// Three kernels per batch:
//   slice_stats_kernel  the one HBM pass: per sub-slice (one warp each) the max
//                       and argmax of the raw logits, NaN/inf flags, an
//                       approximate partial softmax sum and per-segment maxima;
//   survivor_kernel     re-reads each sub-slice (from L2) knowing the row max:
//                       drops the elements that provably do not change any
//                       fold, computes exp exactly for the rest, summarises
//                       each sub-slice's part of the softmax fold and lists
//                       the top-k candidates;
//   row_kernel          one block per row: resolves the softmax fold from the
//                       summaries, then top-k / top-p / draw.
#pragma once
#include <stdint.h>
#include <cuda_bf16.h>
#include "pesti_common.cuh"
#include "pesti_exp.cuh"
#include "pesti_fold.cuh"
#include "../../include/pesti_sampler.h"

namespace pesti {

constexpr int K1_WARPS = 8;  // warps (= sub-slices) per slice block
constexpr int K1_NT = K1_WARPS * 32;
constexpr int K2_NT = 512;
constexpr int MAX_SUBS = 512;     // sub-slices per row
constexpr int TOPK_SMALL = 1024;  // top-k values handled by the generic candidate path
constexpr int CAND_MAX = 2048;    // candidate buffer of that path
constexpr int FAST_K = 256;       // top-k values handled by the fast path
constexpr int CAND_CAP = 2048;    // candidates listed per row by the survivor kernel
constexpr int TAU_BINS = 4096;    // 12-bit histogram used to place the candidate threshold
constexpr uint32_t TR_SAT = 0x40000000u;  // saturation of fold increments (>= any binade)

// An element more than ABSORB scaled units below an EARLIER element of the
// row is added as an exact no-op by the index-order folds and by the sorted
// folds (derivation at survivor_kernel).
constexpr float ABSORB = 17.35f;
// Prefix-max pruning is used only while the prefix max is within this many
// scaled units of the row max (keeps the values involved far from subnormal).
constexpr float PRUNE_FLOOR = 60.0f;

enum : uint32_t { MF_NAN = 1u, MF_POSINF = 2u, MF_NEGINF = 4u };

struct SubStat {      // slice_stats_kernel, one per sub-slice
  float max_raw;      // max of the raw logits, NaN ignored (the f32::max fold, sampling.rs:126)
  float sum_rel;      // sum of 2^(y - y_max), y = raw*log2(e)/T_eff (float, approximate)
  uint32_t last_max;  // last index holding max_raw (0xffffffff if none)
  uint32_t first_max; // first index holding max_raw
  int32_t last_nan;   // last NaN index or -1
  uint32_t flags;     // MF_*
  uint32_t pad[2];
};

struct SubSurv {      // survivor_kernel, one per sub-slice
  int32_t count;      // survivors stored (exact exp, logit index) at the sub-slice's own start
  uint32_t lo_bits;   // binade the softmax fold is in when it enters the sub-slice
                      // (speculated); fold::SPECIAL: replay the survivors one by one
  uint32_t k0, k1;    // total fold increment (ulps of that binade) for an even / odd entry state
  float pruned_max;   // largest raw logit dropped (-inf if none)
  uint32_t pad[3];
};

struct SliceArgs {
  const void* logits;
  long long B, V, ld;
  pesti_sampling_params uni;
  const pesti_sampling_params* per_row;
  int P;            // slice blocks per row
  long long SL;     // elements per sub-slice (one warp each)
  long long nseg;   // 32*VE-element segments per row
  SubStat* stats;   // [B][P*K1_WARPS]
  SubSurv* surv;    // [B][P*K1_WARPS]
  float* seg_max;   // [B][nseg]
  float* surv_e;    // [B][V]: survivors of sub-slice s compacted at its own start
  uint32_t* surv_idx;
  int* cand_count;  // [B]
  float* cand_e;    // [B][CAND_CAP]
  uint32_t* cand_idx;
  float* row_tau;   // [B] candidate threshold (raw units)
};

struct RowArgs {
  const void* logits;
  int dtype;
  long long B, V, ld;
  pesti_sampling_params uni;
  const pesti_sampling_params* per_row;
  int P;
  long long SL;
  const SubStat* stats;
  const SubSurv* surv;
  const float* surv_e;
  const uint32_t* surv_idx;
  const int* cand_count;
  const float* cand_e;
  const uint32_t* cand_idx;
  const float* row_tau;
  float* E;       // [B][V] sequence built by the generic path
  uint32_t* I;
  uint32_t* SK0;  // [B][V] sort buffers (null when no row needs them)
  uint32_t* SV0;
  uint32_t* SK1;
  uint32_t* SV1;
  float* Q;       // [B][V]
  const float* u;
  uint32_t* out;
  float* kept_p;
  uint32_t* kept_idx;
  long long kept_width;
  int64_t* kept_count;
  int* status;    // bit 0: a row needed sort buffers that were not provided
};

__device__ __forceinline__ pesti_sampling_params row_params(const pesti_sampling_params& uni,
                                                            const pesti_sampling_params* per_row,
                                                            long long b) {
  return per_row ? per_row[b] : uni;
}

__device__ __forceinline__ bool is_greedy(const pesti_sampling_params& p) {
  return (p.flags & PESTI_FLAG_GREEDY_IF_ZERO_T) && p.temperature == 0.0f;
}

// Rows whose kept list is an explicit top-k of at most FAST_K entries.
__device__ __forceinline__ bool fast_topk(const pesti_sampling_params& p, long long V) {
  const long long k = (long long)p.top_k;
  return !is_greedy(p) && k >= 1 && (k < V ? k : V) <= FAST_K;
}

// Rows whose folds run only in index order or over an explicit top-k list:
// pruning against a lower bound of the running softmax sum is valid for them.
__device__ __forceinline__ bool sum_pruning_ok(const pesti_sampling_params& p) {
  return p.top_k >= 1u || !(p.top_p > 0.0f);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }

template <typename TIn>
__device__ __forceinline__ float load_logit(const TIn* row, long long j);
template <>
__device__ __forceinline__ float load_logit<float>(const float* row, long long j) { return __ldg(row + j); }
template <>
__device__ __forceinline__ float load_logit<uint16_t>(const uint16_t* row, long long j) {
  return bf16_bits_to_f32(__ldg(row + j));
}
__device__ __forceinline__ float load_logit_dyn(const void* row, int dtype, long long j) {
  return dtype == PESTI_BF16 ? load_logit<uint16_t>((const uint16_t*)row, j)
                             : load_logit<float>((const float*)row, j);
}

// Order-preserving u32 key of a float (for selection over signed values).
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = fbits(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  return bitsf((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// ---------------------------------------------------------------------------
// Fold transducers: the effect of a run of elements on the fold state while
// it stays in one binade, as a pair of bit-increments for an even / odd entry
// state (the parity only matters for elements exactly halfway between two
// multiples of the ulp).  Increments saturate at TR_SAT, which no binade fits.
// ---------------------------------------------------------------------------
struct Tr {
  uint32_t a0, a1;
};
__device__ __forceinline__ uint32_t tr_sat(uint32_t x) { return x > TR_SAT ? TR_SAT : x; }
// f first, then g
__device__ __forceinline__ Tr tr_compose(Tr f, Tr g) {
  Tr r;
  r.a0 = tr_sat(f.a0 + ((f.a0 & 1u) ? g.a1 : g.a0));
  r.a1 = tr_sat(f.a1 + (((f.a1 + 1u) & 1u) ? g.a1 : g.a0));
  return r;
}
// Composition over the warp's lanes in lane order; the result is in lane 0.
__device__ __forceinline__ Tr tr_warp_reduce(Tr t) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    Tr o;
    o.a0 = __shfl_down_sync(PESTI_FULL_MASK, t.a0, off);
    o.a1 = __shfl_down_sync(PESTI_FULL_MASK, t.a1, off);
    if ((lane & (2 * off - 1)) == 0) t = tr_compose(t, o);
  }
  return t;
}
// Inclusive composition over lanes 0..lane (in lane order).
__device__ __forceinline__ Tr tr_warp_incl_scan(Tr t) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    Tr o;
    o.a0 = __shfl_up_sync(PESTI_FULL_MASK, t.a0, off);
    o.a1 = __shfl_up_sync(PESTI_FULL_MASK, t.a1, off);
    if (lane >= off) t = tr_compose(o, t);
  }
  return t;
}

// ---------------------------------------------------------------------------
// Streaming of one warp's contiguous sub-slice [start, end) of a row: 16-byte
// loads (U of them in flight per lane) when the row is 16-byte aligned, scalar
// loads for the tail.  f(x, pos0, nv) receives a lane's VE consecutive values
// (nv valid) at positions pos0..; a call covers one 32*VE-element segment per
// warp, and within a warp the calls run in row order.
// ---------------------------------------------------------------------------
template <typename TIn, int VE, int U, bool VEC, typename F>
__device__ __forceinline__ void stream_subslice(const TIn* row, long long start, long long end, F&& f) {
  const int lane = threadIdx.x & 31;
  const long long CH = 32LL * VE * U;
  long long pos = start;
  if (VEC) {
    for (; pos + CH <= end; pos += CH) {
      float4 raw[U];
#pragma unroll
      for (int uu = 0; uu < U; ++uu) {
        const TIn* p = row + pos + (long long)uu * 32 * VE + (long long)lane * VE;
        raw[uu] = __ldg(reinterpret_cast<const float4*>(p));
      }
#pragma unroll
      for (int uu = 0; uu < U; ++uu) {
        float x[VE];
        if (sizeof(TIn) == 4) {
          x[0] = raw[uu].x; x[1] = raw[uu].y; x[2] = raw[uu].z; x[3] = raw[uu].w;
        } else {
          const uint32_t wds[4] = {__float_as_uint(raw[uu].x), __float_as_uint(raw[uu].y),
                                   __float_as_uint(raw[uu].z), __float_as_uint(raw[uu].w)};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            x[2 * q] = __uint_as_float(wds[q] << 16);
            x[2 * q + 1] = __uint_as_float(wds[q] & 0xffff0000u);
          }
        }
        f(x, pos + (long long)uu * 32 * VE + (long long)lane * VE, VE);
      }
    }
  }
  for (; pos < end; pos += 32LL * VE) {
    float x[VE];
    const long long p0 = pos + (long long)lane * VE;
    int nv = 0;
#pragma unroll
    for (int e = 0; e < VE; ++e) {
      const long long j = p0 + e;
      if (j < end) {
        x[e] = load_logit<TIn>(row, j);
        nv = e + 1;
      } else {
        x[e] = 0.0f;
      }
    }
    f(x, p0, nv);
  }
}

// ---------------------------------------------------------------------------
// Pass 1, the HBM pass.
// ---------------------------------------------------------------------------
template <typename TIn, int VE, int U, bool VEC>
__global__ void __launch_bounds__(K1_NT) slice_stats_kernel(SliceArgs a) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const long long b = blockIdx.x / a.P;
  const int slice = (int)(blockIdx.x % a.P);
  const long long sub = (long long)slice * K1_WARPS + w;
  const long long start = sub * a.SL;
  long long end = start + a.SL;
  if (end > a.V) end = a.V;
  if (slice == 0 && w == 0 && lane == 0) a.cand_count[b] = 0;
  const TIn* row = (const TIn*)a.logits + b * a.ld;
  const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
  const float c2 = 1.4426950408889634f / (prm.temperature > 0.0f ? prm.temperature : 1.0f);
  const float NEG_INF = -__int_as_float(0x7f800000);
  float best_v = NEG_INF, fbest_v = NEG_INF;
  long long best_i = -1, fbest_i = -1, last_nan = -1;
  uint32_t flags = 0;
  float run_m = NEG_INF, run_s = 0.0f;  // online partial sum, log2 units
  float* segmax = a.seg_max + b * a.nseg;
  stream_subslice<TIn, VE, U, VEC>(row, start, end, [&](const float* x, long long pos0, int nv) {
    float lm = NEG_INF;
#pragma unroll
    for (int e = 0; e < VE; ++e) {
      if (e >= nv) continue;
      const float xv = x[e];
      const long long pos = pos0 + e;
      if (is_nan(xv)) {
        last_nan = pos;
        flags |= MF_NAN;
        continue;
      }
      lm = fmaxf(lm, xv);
      if (best_i < 0 || xv >= best_v) { best_v = xv; best_i = pos; }
      if (fbest_i < 0 || xv > fbest_v) { fbest_v = xv; fbest_i = pos; }
      if (xv == -NEG_INF) flags |= MF_POSINF;
      if (xv == NEG_INF) flags |= MF_NEGINF;
    }
    // approximate partial softmax sum (guides the fold speculation only)
    const float nm = fmaxf(run_m, lm * c2);
    if (nm > NEG_INF) {
      float acc = run_s * exp2f(run_m - nm);
#pragma unroll
      for (int e = 0; e < VE; ++e)
        if (e < nv && !is_nan(x[e])) acc += exp2f(x[e] * c2 - nm);
      run_s = acc;
      run_m = nm;
    }
    const float sm = warp_reduce_fmax(lm);
    if (lane == 0) segmax[(pos0 - (long long)lane * VE) / (32LL * VE)] = sm;
  });
  const float mx = warp_reduce_fmax(best_i >= 0 ? best_v : NEG_INF);
  long long li = (best_i >= 0 && best_v == mx) ? best_i : -1;
  long long fi = (fbest_i >= 0 && fbest_v == mx) ? fbest_i : (1LL << 62);
  li = warp_reduce_max(li);
  fi = warp_reduce_min(fi);
  const long long ln = warp_reduce_max(last_nan);
  uint32_t fl = flags;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) fl |= __shfl_xor_sync(PESTI_FULL_MASK, fl, o);
  const float wm = warp_reduce_fmax(run_m);
  float ws = (run_m > NEG_INF && wm > NEG_INF) ? run_s * exp2f(run_m - wm) : 0.0f;
  ws = warp_reduce_add(ws);
  if (lane == 0) {
    SubStat m;
    m.max_raw = mx;
    m.sum_rel = ws;  // relative to 2^(mx*c2) (wm == mx*c2: the same float product)
    m.last_max = li >= 0 ? (uint32_t)li : 0xffffffffu;
    m.first_max = fi < (1LL << 62) ? (uint32_t)fi : 0xffffffffu;
    m.last_nan = (int32_t)ln;
    m.flags = fl;
    m.pad[0] = m.pad[1] = 0;
    a.stats[b * (long long)a.P * K1_WARPS + sub] = m;
  }
}

// ---------------------------------------------------------------------------
// Pass 2: survivors, exact exp, fold summaries, top-k candidates.
//
// Which elements may be dropped (x_i = raw_i/T is the scaled logit):
//  (a) prefix max: an EARLIER element j with x_j >= x_i + 17.34 gives
//      e_i <= 0.989*2^-25*e_j; the running softmax sum s_{i-1} >= e_j and
//      ulp(s)/2 > s*2^-25, so fl(s + e_i) returns s.  The same ratio makes i a
//      no-op in the sorted folds (they start at p_max >= p_j) and in the
//      index-order folds of p and q.  Tested on raw values as
//      raw_i < P - (17.35*T*(1+2^-20) + 2^-21*|P|), P = prefix max; the slack
//      covers the rounding of raw/T, of x - m (<= 2^-24*104 wherever exp is
//      not 0) and of exp.  Used while P/T >= m - 60.
//  (b) running sum: each step of a fold of non-negative terms has relative
//      error <= 2^-24, so s_{i-1} >= (sum_{j<i} e_j)*(1 - V*2^-24).  With the
//      approximate prefix sum A of the earlier sub-slices (pass 1),
//      L = A*(1 - V*2^-24)*(1 - 2^-10) <= s_{i-1}, and e_i < 0.99*2^-25*L makes
//      i a no-op in the index-order folds (also for p = e/S and q = p/total,
//      whose running sums are bounded the same way).  It does NOT bound the
//      sorted folds, so it is used only for top-k rows (whose kept list is
//      explicit and checked) and unfiltered rows (index order only).
// ---------------------------------------------------------------------------
struct SurvShared {
  float mraw[MAX_SUBS];
  float srel[MAX_SUBS];
  double apre[MAX_SUBS];
  float ppre[MAX_SUBS];
  uint32_t hist[TAU_BINS];
  double dscr[34];
  float fscr[34];
  int iscr[34];
  uint32_t uscr[34];
  float tau;
  int flags;
};

template <typename TIn, int VE, int U, bool VEC>
__global__ void __launch_bounds__(K1_NT) survivor_kernel(SliceArgs a) {
  __shared__ SurvShared sh;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const long long b = blockIdx.x / a.P;
  const int slice = (int)(blockIdx.x % a.P);
  const int nsub = a.P * K1_WARPS;
  const long long sub = (long long)slice * K1_WARPS + w;
  const long long V = a.V;
  const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
  const float T = prm.temperature;
  const bool scale = T > 0.0f;
  const float t_eff = scale ? T : 1.0f;
  const float NEG_INF = -__int_as_float(0x7f800000), INF = __int_as_float(0x7f800000);
  SubSurv* so = a.surv + b * nsub + sub;
  // ---- row prologue (every block of the row computes the same values) ----
  float mx = NEG_INF;
  int f = 0;
  for (int s = tid; s < MAX_SUBS; s += K1_NT) {
    const bool has = s < nsub && (long long)s * a.SL < V;
    SubStat st;
    if (has) st = a.stats[b * nsub + s];
    sh.mraw[s] = has ? st.max_raw : NEG_INF;
    sh.srel[s] = has ? st.sum_rel : 0.0f;
    if (has) {
      mx = fmaxf(mx, st.max_raw);
      f |= (int)st.flags;
    }
  }
  mx = -block_reduce_min(-mx, sh.fscr);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) f |= __shfl_xor_sync(PESTI_FULL_MASK, f, o);
  if (lane == 0) sh.iscr[w] = f;
  __syncthreads();
  if (tid == 0) {
    int g = 0;
    for (int q = 0; q < K1_WARPS; ++q) g |= sh.iscr[q];
    sh.flags = g;
  }
  __syncthreads();
  const uint32_t fl = (uint32_t)sh.flags;
  const float m = scale ? fdiv(mx, T) : mx;
  const bool uniform = (fl & MF_NAN) || (scale && T == INF && (fl & (MF_POSINF | MF_NEGINF))) || !(fabsf(m) < INF);
  if (is_greedy(prm) || uniform || V <= 0) {
    if (lane == 0) {
      so->count = 0;
      so->lo_bits = fold::SPECIAL;
      so->k0 = so->k1 = 0;
      so->pruned_max = NEG_INF;
    }
    return;
  }
  const float c2 = 1.4426950408889634f / t_eff;
  const float ym = mx * c2;
  // exclusive prefix sums (approximate softmax mass) and prefix maxima over sub-slices
  {
    constexpr int PER = MAX_SUBS / K1_NT;
    double loc[PER];
    float lmx[PER];
    double lsum = 0.0;
    float run = NEG_INF;
#pragma unroll
    for (int r = 0; r < PER; ++r) {
      const int s = tid * PER + r;
      const float mm = sh.mraw[s];
      loc[r] = mm > NEG_INF ? (double)exp2f(mm * c2 - ym) * (double)sh.srel[s] : 0.0;
      lmx[r] = mm;
      lsum += loc[r];
      run = fmaxf(run, mm);
    }
    double dt;
    double ex = block_excl_scan_add(lsum, sh.dscr, dt);
    float inc = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(PESTI_FULL_MASK, inc, o);
      if (lane >= o) inc = fmaxf(inc, y);
    }
    if (lane == 31) sh.fscr[w] = inc;
    __syncthreads();
    float wpre = NEG_INF;
    for (int q = 0; q < w; ++q) wpre = fmaxf(wpre, sh.fscr[q]);
    float exc = __shfl_up_sync(PESTI_FULL_MASK, inc, 1);
    if (lane == 0) exc = NEG_INF;
    float pmax = fmaxf(wpre, exc);
#pragma unroll
    for (int r = 0; r < PER; ++r) {
      const int s = tid * PER + r;
      sh.apre[s] = ex;
      sh.ppre[s] = pmax;
      ex += loc[r];
      pmax = fmaxf(pmax, lmx[r]);
    }
    __syncthreads();
  }
  // candidate threshold: a lower bound of the k-th largest raw logit, from the
  // segment maxima (maxima of disjoint segments are distinct elements),
  // rounded down to the start of its 12-bit key bin
  const long long k = (long long)prm.top_k;
  if (fast_topk(prm, V)) {
    const long long keff = k < V ? k : V;
    for (int i = tid; i < TAU_BINS; i += K1_NT) sh.hist[i] = 0u;
    __syncthreads();
    const float* segm = a.seg_max + b * a.nseg;
    for (long long j0 = 0; j0 < a.nseg; j0 += K1_NT) {
      const long long j = j0 + tid;
      const float v = j < a.nseg ? segm[j] : NEG_INF;
      const bool ok = j < a.nseg && !is_nan(v) && v > NEG_INF;
      const uint32_t d = ok ? (fkey(v) >> 20) : (uint32_t)(TAU_BINS + lane);
      const uint32_t peers = __match_any_sync(PESTI_FULL_MASK, d);
      if (ok && (peers & ((1u << lane) - 1u)) == 0u) atomicAdd(&sh.hist[d], (uint32_t)__popc(peers));
    }
    __syncthreads();
    // top-down scan over the bins: thread t owns bins [TAU_BINS-16(t+1), TAU_BINS-16t)
    constexpr int BPT = TAU_BINS / K1_NT;
    uint32_t loc = 0;
#pragma unroll
    for (int q = 0; q < BPT; ++q) loc += sh.hist[TAU_BINS - 1 - BPT * tid - q];
    uint32_t tot;
    const uint32_t ex = block_excl_scan_add(loc, sh.uscr, tot);
    if ((long long)ex < keff && (long long)(ex + loc) >= keff) {
      uint32_t cum = ex;
      for (int q = 0; q < BPT; ++q) {
        const int bin = TAU_BINS - 1 - BPT * tid - q;
        cum += sh.hist[bin];
        if ((long long)cum >= keff) {
          sh.tau = fkey_inv((uint32_t)bin << 20);
          break;
        }
      }
    }
    if (tid == 0 && (long long)tot < keff) sh.tau = NEG_INF;
    __syncthreads();
    if (tid == 0 && slice == 0) a.row_tau[b] = sh.tau;
  } else {
    if (tid == 0) {
      sh.tau = INF;
      if (slice == 0) a.row_tau[b] = INF;
    }
    __syncthreads();
  }
  const float tau = sh.tau;

  // ---- this warp's sub-slice ----
  const long long start = sub * a.SL;
  long long end = start + a.SL;
  if (end > V) end = V;
  const TIn* row = (const TIn*)a.logits + b * a.ld;
  const long long out_base = b * V + start;
  const float c1 = ABSORB * t_eff * (1.0f + 0x1p-20f);
  const float pf = (m - PRUNE_FLOOR) * t_eff;
  const float p_floor = pf + 0x1p-20f * fabsf(pf);
  const float invT = 1.0f / t_eff;
  float run_max = sh.ppre[sub];
  const double A = sh.apre[sub];
  // A is built from float products raw*c2 whose rounding grows with |y|:
  // widen the margin with the magnitude of the scaled logits
  const double mag = 0x1p-20 * ((double)fabsf(ym) + 64.0);
  const double L = A * (1.0 - (double)V * 0x1p-24) * (1.0 - 0x1p-10) * exp2(-mag);
  const bool use_L = sum_pruning_ok(prm) && L >= 0x1p-60;
  const float thrL = use_L ? m + (float)log(L) - 17.36f : NEG_INF;
  // fold speculation: the softmax fold enters this sub-slice near A and
  // leaves near A + own (a guess: the row kernel verifies it against the exact state)
  const double own = sh.mraw[sub] > NEG_INF ? (double)exp2f(sh.mraw[sub] * c2 - ym) * (double)sh.srel[sub] : 0.0;
  uint32_t lo = fold::SPECIAL;
  if (A >= 0x1p-100) {
    const uint32_t l = fbits(__double2float_rz(A)) & 0x7f800000u;
    const double lov = (double)bitsf(l);
    if (A >= lov * (1.0 + fold::MU) && A + own * (1.0 + 0x1p-8) <= 2.0 * lov * (1.0 - fold::MU)) lo = l;
  }
  const float lo_half = lo == fold::SPECIAL ? 0.0f : bitsf(lo - 0x00800000u);
  Tr acc{0u, 0u};
  bool complex_sub = lo == fold::SPECIAL;
  long long total = 0;
  float pruned_max = NEG_INF;
  int* ccount = a.cand_count + b;

  stream_subslice<TIn, VE, U, VEC>(row, start, end, [&](const float* x, long long pos0, int nv) {
    float pre[VE];
    float lm = NEG_INF;
#pragma unroll
    for (int e = 0; e < VE; ++e) {
      pre[e] = lm;
      if (e < nv) lm = fmaxf(lm, x[e]);
    }
    float inc = lm;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(PESTI_FULL_MASK, inc, o);
      if (lane >= o) inc = fmaxf(inc, y);
    }
    float exc = __shfl_up_sync(PESTI_FULL_MASK, inc, 1);
    if (lane == 0) exc = NEG_INF;
    const float seg_max = __shfl_sync(PESTI_FULL_MASK, inc, 31);
    const float p0 = fmaxf(run_max, exc);
    bool sv[VE], cd[VE];
    float ev[VE];
    int cnt = 0, ccnt = 0;
    Tr lt{0u, 0u};
    bool big = false;
#pragma unroll
    for (int e = 0; e < VE; ++e) {
      const float xv = x[e];
      const bool valid = e < nv && !is_nan(xv);
      const float P = fmaxf(p0, pre[e]);
      const bool pruneP = P >= p_floor && xv < fsub(P, fadd(c1, 0x1p-21f * fabsf(P)));
      const float xa = xv * invT;
      const bool pruneL = xa < thrL - 0x1p-19f * (fabsf(xa) + fabsf(thrL));
      sv[e] = valid && !(pruneP || pruneL);
      cd[e] = valid && xv >= tau;
      ev[e] = 0.0f;
      if (sv[e] || cd[e]) {
        const float xs = scale ? fdiv(xv, T) : xv;  // sampling.rs:46
        ev[e] = pesti_expf(fsub(xs, m));            // sampling.rs:127
      }
      if (valid && !sv[e]) pruned_max = fmaxf(pruned_max, xv);
      if (sv[e]) {
        ++cnt;
        if (!complex_sub) {
          if (ev[e] >= lo_half) big = true;
          const uint32_t k0 = fbits(fadd(bitsf(lo), ev[e])) - lo;
          const uint32_t k1 = fbits(fadd(bitsf(lo + 1u), ev[e])) - (lo + 1u);
          lt = tr_compose(lt, Tr{k0, k1});
        }
      }
      ccnt += cd[e] ? 1 : 0;
    }
    run_max = fmaxf(run_max, seg_max);
    // survivors, compacted in row order
    const int cinc = warp_incl_scan_add(cnt);
    const int wsum = __shfl_sync(PESTI_FULL_MASK, cinc, 31);
    long long o = out_base + total + (cinc - cnt);
#pragma unroll
    for (int e = 0; e < VE; ++e) {
      if (sv[e]) {
        a.surv_e[o] = ev[e];
        a.surv_idx[o] = (uint32_t)(pos0 + e);
        ++o;
      }
    }
    total += wsum;
    // fold summary of this segment, composed in row order
    if (__any_sync(PESTI_FULL_MASK, big)) complex_sub = true;
    if (!complex_sub && wsum > 0) {
      const Tr seg = tr_warp_reduce(lt);
      if (lane == 0) acc = tr_compose(acc, seg);
    }
    // top-k candidates (one atomic per warp per segment)
    const int ctot = warp_reduce_add(ccnt);
    if (ctot > 0) {
      int basec = 0;
      if (lane == 0) basec = atomicAdd(ccount, ctot);
      basec = __shfl_sync(PESTI_FULL_MASK, basec, 0);
      int cex = warp_incl_scan_add(ccnt) - ccnt;
#pragma unroll
      for (int e = 0; e < VE; ++e) {
        if (cd[e]) {
          const int slot = basec + cex;
          if (slot < CAND_CAP) {
            a.cand_e[b * CAND_CAP + slot] = ev[e];
            a.cand_idx[b * CAND_CAP + slot] = (uint32_t)(pos0 + e);
          }
          ++cex;
        }
      }
    }
  });
  const float pm = warp_reduce_fmax(pruned_max);
  if (lane == 0) {
    so->count = (int32_t)total;
    so->lo_bits = complex_sub ? fold::SPECIAL : lo;
    so->k0 = acc.a0;
    so->k1 = acc.a1;
    so->pruned_max = pm;
  }
}

// ---------------------------------------------------------------------------
// Row kernel: one block per row.
// ---------------------------------------------------------------------------
struct SubInfo {
  long long start;
  long long cnt;    // sequence elements the sub-slice contributes
  long long base;   // their first position in the row's sequence
  int dense;
};

struct RowShared {
  union {
    fold::Smem f;
    sort::Smem s;
    struct {
      unsigned long long key[CAND_MAX];
      float q[CAND_MAX];
      uint32_t hist[256];
      uint32_t sel_prefix;
      long long sel_k;
      int cand_n;
    } c;
  } u;
  SubInfo sub[MAX_SUBS];
  long long lscr[34];
  float fscr[34];
  int iscr[34];
  long long n;
  uint32_t flags;
  uint32_t s_bits;
  uint32_t e_star;
  int need_dense;
  int fallback;
};

// Rust's Iterator::max_by over the raw logits with partial_cmp (sampling.rs:115-122)
// when the row holds NaN: the scan adopts every NaN and then the element right
// after it, so the result is the last maximum after the last NaN (or that NaN
// itself when it is the final element).
__device__ uint32_t nan_argmax(const void* row, int dtype, long long V, long long last_nan, RowShared& sh) {
  if (last_nan == V - 1) return (uint32_t)last_nan;
  float mx = -__int_as_float(0x7f800000);
  for (long long j = last_nan + 1 + threadIdx.x; j < V; j += K2_NT) mx = fmaxf(mx, load_logit_dyn(row, dtype, j));
  mx = -block_reduce_min(-mx, sh.fscr);
  long long li = -1;
  for (long long j = last_nan + 1 + threadIdx.x; j < V; j += K2_NT)
    if (load_logit_dyn(row, dtype, j) == mx) li = j;
  li = block_reduce_max(li, sh.lscr);
  return (uint32_t)(li < 0 ? last_nan + 1 : li);
}

__device__ void write_kept_pad(const RowArgs& a, long long b, long long from) {
  if (!a.kept_p && !a.kept_idx) return;
  for (long long j = from + threadIdx.x; j < a.kept_width; j += K2_NT) {
    if (a.kept_p) a.kept_p[b * a.kept_width + j] = 0.0f;
    if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = 0xffffffffu;
  }
}

// k-th largest (1-based) bit pattern among E[0..n) (non-negative floats).
__device__ uint32_t select_kth_largest(const float* E, long long n, long long k, RowShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (tid == 0) {
    sh.u.c.sel_prefix = 0u;
    sh.u.c.sel_k = k;
  }
  uint32_t mask = 0u;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += K2_NT) sh.u.c.hist[i] = 0u;
    __syncthreads();
    const uint32_t prefix = sh.u.c.sel_prefix;
    for (long long j0 = 0; j0 < n; j0 += K2_NT) {
      const long long j = j0 + tid;
      const uint32_t x = j < n ? fbits(E[j]) : 0u;
      const bool match = j < n && (x & mask) == prefix;
      const uint32_t d = match ? ((x >> shift) & 255u) : 256u + (uint32_t)lane;
      const uint32_t peers = __match_any_sync(PESTI_FULL_MASK, d);  // one atomic per digit per warp
      if (match && (peers & ((1u << lane) - 1u)) == 0u) atomicAdd(&sh.u.c.hist[d], (uint32_t)__popc(peers));
    }
    __syncthreads();
    if (tid < 32) {
      // the digit holding the k-th largest: warp scan over the 256 bins, top down
      const long long kk = sh.u.c.sel_k;
      uint32_t c8[8];
      uint32_t lsum = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        c8[q] = sh.u.c.hist[255 - (lane * 8 + q)];
        lsum += c8[q];
      }
      const uint32_t incl = warp_incl_scan_add(lsum);
      const uint32_t excl = incl - lsum;
      const bool here = (long long)excl < kk && (long long)incl >= kk;
      __syncwarp();
      if (here) {
        uint32_t cum = excl;
        int q = 0;
        for (; q < 7; ++q) {
          if ((long long)(cum + c8[q]) >= kk) break;
          cum += c8[q];
        }
        sh.u.c.sel_k = kk - cum;
        sh.u.c.sel_prefix = prefix | ((uint32_t)(255 - (lane * 8 + q)) << shift);
      }
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  return sh.u.c.sel_prefix;
}

// Bitonic sort of key[0..m), m a power of two, descending; whole block.
__device__ void bitonic_desc(unsigned long long* key, int m) {
  for (int kk = 2; kk <= m; kk <<= 1) {
    for (int j = kk >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < m; i += K2_NT) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long x = key[i], y = key[ixj];
          const bool desc = (i & kk) == 0;
          if (desc ? (x < y) : (x > y)) {
            key[i] = y;
            key[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Fold of n values from global memory by one warp, starting from state s
// (bits), 32 elements per step: a transducer scan over the lanes gives every
// lane's state under the current binade; the first element that would leave
// the binade (or is large next to s) is added directly, and the step resumes
// after it.  Returns the final state.  All 32 lanes must call it.
__device__ uint32_t warp_fold(const float* v, long long n, uint32_t s) {
  const int lane = threadIdx.x & 31;
  long long j = 0;
  while (j < n) {
    const long long idx = j + lane;
    const bool valid = idx < n;
    const float x = valid ? v[idx] : 0.0f;
    const uint32_t lo = fold::binade_lo_bits(s);
    const uint32_t hi = fold::binade_hi_bits(lo);
    const bool big = valid && (lo == 0u ? x >= 0x1p-127f : fbits(x) >= lo - 0x00800000u);
    Tr t{0u, 0u};
    if (valid && !big) {
      t.a0 = fbits(fadd(bitsf(lo), x)) - lo;
      t.a1 = fbits(fadd(bitsf(lo + 1u), x)) - (lo + 1u);
    }
    const Tr incl = tr_warp_incl_scan(t);
    const unsigned long long sum = (unsigned long long)s + ((s & 1u) ? incl.a1 : incl.a0);
    const uint32_t after = sum > 0xffffffffull ? 0xffffffffu : (uint32_t)sum;
    const bool bad = valid && (big || after >= hi);
    const uint32_t badm = __ballot_sync(PESTI_FULL_MASK, bad);
    const int nvalid = (int)(n - j < 32 ? n - j : 32);
    if (badm == 0u) {
      s = __shfl_sync(PESTI_FULL_MASK, after, nvalid - 1);
      j += nvalid;
    } else {
      const int f0 = __ffs(badm) - 1;
      const uint32_t prev = __shfl_sync(PESTI_FULL_MASK, after, f0 > 0 ? f0 - 1 : 0);
      const uint32_t before = f0 > 0 ? prev : s;  // lanes < f0 are exact
      const float xf = __shfl_sync(PESTI_FULL_MASK, x, f0);
      s = fbits(fadd(bitsf(before), xf));
      j += f0 + 1;
    }
  }
  return s;
}

__global__ void __launch_bounds__(K2_NT) row_kernel(RowArgs a) {
  extern __shared__ __align__(16) unsigned char row_smem[];
  RowShared& sh = *reinterpret_cast<RowShared*>(row_smem);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const long long b = blockIdx.x;
  const long long V = a.V;
  const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
  const float T = prm.temperature;
  const int nsub = a.P * K1_WARPS;
  const void* row = a.dtype == PESTI_BF16 ? (const void*)((const uint16_t*)a.logits + b * a.ld)
                                          : (const void*)((const float*)a.logits + b * a.ld);
  float* E = a.E + b * V;
  uint32_t* I = a.I + b * V;
  const float r = a.u ? a.u[b] : 0.0f;
  const float INF = __int_as_float(0x7f800000);
  const SubStat* stats = a.stats + b * nsub;
  const SubSurv* survs = a.surv + b * nsub;

  // ---- row summary from the sub-slice statistics ----
  float mx = -INF;
  long long li = -1, fi = 1LL << 62, ln = -1;
  int f = 0;
  for (int s = tid; s < nsub; s += K2_NT) {
    if ((long long)s * a.SL >= V) continue;
    const SubStat st = stats[s];
    mx = fmaxf(mx, st.max_raw);
    ln = ln > st.last_nan ? ln : st.last_nan;
    f |= (int)st.flags;
  }
  mx = -block_reduce_min(-mx, sh.fscr);
  for (int s = tid; s < nsub; s += K2_NT) {
    if ((long long)s * a.SL >= V) continue;
    const SubStat st = stats[s];
    if (st.max_raw == mx) {
      if (st.last_max != 0xffffffffu) li = li > (long long)st.last_max ? li : (long long)st.last_max;
      if (st.first_max != 0xffffffffu) fi = fi < (long long)st.first_max ? fi : (long long)st.first_max;
    }
  }
  li = block_reduce_max(li, sh.lscr);
  fi = block_reduce_min(fi, sh.lscr);
  ln = block_reduce_max(ln, sh.lscr);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) f |= __shfl_xor_sync(PESTI_FULL_MASK, f, o);
  if (lane == 0) sh.iscr[wid] = f;
  __syncthreads();
  if (tid == 0) {
    int g = 0;
    for (int q = 0; q < K2_NT / 32; ++q) g |= sh.iscr[q];
    sh.flags = (uint32_t)g;
  }
  __syncthreads();
  const uint32_t fl = sh.flags;
  const long long last_max = li, first_max = fi < (1LL << 62) ? fi : -1, last_nan = ln;

  if (V <= 0) {  // empty slice: sample() and argmax() return 0
    if (tid == 0) {
      a.out[b] = 0u;
      if (a.kept_count) a.kept_count[b] = 0;
    }
    write_kept_pad(a, b, 0);
    return;
  }

  if (is_greedy(prm)) {  // generate(): temperature == 0 -> argmax (model.rs:517-521)
    uint32_t tok;
    if (prm.flags & PESTI_FLAG_ARGMAX_FIRST) tok = first_max >= 0 ? (uint32_t)first_max : 0u;
    else if (fl & MF_NAN) tok = nan_argmax(row, a.dtype, V, last_nan, sh);
    else tok = last_max >= 0 ? (uint32_t)last_max : 0u;
    if (tid == 0) {
      a.out[b] = tok;
      if (a.kept_count) a.kept_count[b] = 0;
    }
    write_kept_pad(a, b, 0);
    return;
  }

  // sampling.rs:43-50 temperature; the max of x/T is RN(max(raw)/T) (monotone)
  const bool scale = T > 0.0f;
  const float m = scale ? fdiv(mx, T) : mx;
  const bool nanx = (fl & MF_NAN) || (scale && T == INF && (fl & (MF_POSINF | MF_NEGINF)));
  const long long k = (long long)prm.top_k;
  const bool topp = prm.top_p > 0.0f && k == 0;
  const uint32_t r_tau = fold::tau_bits_of(r);

  if (nanx || !(fabsf(m) < INF)) {
    // softmax sum is NaN or not > 0: every probability is 1/V (sampling.rs:129-133).
    // All entries are equal, so both stable sorts keep index order.
    if (tid == 0) {
      const float pv = fdiv(1.0f, (float)__ll2float_rn(V));
      long long K;
      fold::Result tr;
      if (k > 0) {
        K = k < V ? k : V;
        tr = fold::repeat_fold(pv, K, 0u, fold::NO_QUERY, false);
      } else if (topp) {
        tr = fold::repeat_fold(pv, V, 0u, fold::tau_bits_of(prm.top_p), true);
        K = tr.hit >= 0 ? tr.hit + 1 : V;
        if (tr.hit >= 0) tr.s_bits = tr.hit_s_bits;
      } else {
        K = V;
        tr = fold::repeat_fold(pv, V, 0u, fold::NO_QUERY, false);
      }
      const float total = bitsf(tr.s_bits);
      uint32_t tok;
      if (!(total > 0.0f)) {
        tok = 0u;  // unreachable: 1/V > 0
      } else {
        const float q = fdiv(pv, total);
        const fold::Result dr = fold::repeat_fold(q, K, 0u, r_tau, true);
        tok = (uint32_t)(dr.hit >= 0 ? dr.hit : K - 1);
      }
      a.out[b] = tok;
      if (a.kept_count) a.kept_count[b] = K;
      sh.n = K;
    }
    __syncthreads();
    const long long K = sh.n;
    const float pv = fdiv(1.0f, (float)__ll2float_rn(V));
    for (long long j = tid; j < a.kept_width; j += K2_NT) {
      const bool in = j < K;
      if (a.kept_p) a.kept_p[b * a.kept_width + j] = in ? pv : 0.0f;
      if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = in ? (uint32_t)j : 0xffffffffu;
    }
    return;
  }

  // largest dropped logit -> an upper bound of the exp of every dropped element
  float pm = -INF;
  for (int s = tid; s < nsub; s += K2_NT)
    if ((long long)s * a.SL < V) pm = fmaxf(pm, survs[s].pruned_max);
  pm = -block_reduce_min(-pm, sh.fscr);
  const float e_pruned = pm > -INF ? pesti_expf(fsub(scale ? fdiv(pm, T) : pm, m)) : 0.0f;

  // ---------------- fast path: explicit top-k of at most FAST_K ----------------
  if (fast_topk(prm, V)) {
    const long long keff = k < V ? k : V;
    // softmax denominator (sampling.rs:128): resolve the index-order fold from
    // the sub-slice summaries; replay a sub-slice element by element whenever
    // its summary does not apply to the exact state.
    if (wid == 0) {
      uint32_t s = 0u;
      for (int q = 0; q < nsub; ++q) {
        const long long st = (long long)q * a.SL;
        if (st >= V) break;
        const SubSurv sv = survs[q];
        if (sv.count <= 0) continue;
        bool applied = false;
        if (sv.lo_bits != fold::SPECIAL && fold::binade_lo_bits(s) == sv.lo_bits) {
          const uint32_t inc = (s & 1u) ? sv.k1 : sv.k0;
          const unsigned long long ns = (unsigned long long)s + inc;
          if (ns < (unsigned long long)fold::binade_hi_bits(sv.lo_bits)) {
            s = (uint32_t)ns;
            applied = true;
          }
        }
        if (!applied) s = warp_fold(a.surv_e + b * V + st, sv.count, s);
      }
      if (lane == 0) sh.s_bits = s;
    }
    __syncthreads();
    const float S = bitsf(sh.s_bits);
    const int C = a.cand_count[b];
    const float tau = a.row_tau[b];
    bool ok = C >= keff && C <= CAND_CAP && C <= CAND_MAX;
    if (ok) {
      int mm2 = 1;
      while (mm2 < C) mm2 <<= 1;
      for (int j = tid; j < mm2; j += K2_NT) {
        unsigned long long key = 0ull;
        if (j < C) {
          const float p = fdiv(a.cand_e[b * CAND_CAP + j], S);  // sampling.rs:130
          key = ((unsigned long long)fbits(p) << 32) | (unsigned long long)(~a.cand_idx[b * CAND_CAP + j]);
        }
        sh.u.c.key[j] = key;
      }
      __syncthreads();
      bitonic_desc(sh.u.c.key, mm2);  // (p desc, index asc): the stable sort of sampling.rs:60
      // every element outside the candidates (raw < tau) must rank below the keff-th
      const float pk = bitsf((uint32_t)(sh.u.c.key[keff - 1] >> 32));
      const float e_tau = tau > -INF ? pesti_expf(fsub(scale ? fdiv(tau, T) : tau, m)) : 0.0f;
      ok = fdiv(e_tau, S) < pk;
    }
    if (ok) {
      if (tid == 0) {
        uint32_t s = 0u;  // total over the kept list (sampling.rs:81)
        for (long long j = 0; j < keff; ++j) s = fbits(fadd(bitsf(s), bitsf((uint32_t)(sh.u.c.key[j] >> 32))));
        sh.e_star = s;
      }
      __syncthreads();
      const float total = bitsf(sh.e_star);
      for (long long j = tid; j < keff; j += K2_NT)
        sh.u.c.q[j] = fdiv(bitsf((uint32_t)(sh.u.c.key[j] >> 32)), total);  // sampling.rs:94
      __syncthreads();
      if (tid == 0) {
        const fold::Result dr = fold::thread_fold(sh.u.c.q, keff, 0u, r_tau, true);  // sampling.rs:99-105
        const long long at = dr.hit >= 0 ? dr.hit : keff - 1;                     // sampling.rs:108-111
        a.out[b] = ~(uint32_t)(sh.u.c.key[at] & 0xffffffffull);
        if (a.kept_count) a.kept_count[b] = keff;
      }
      for (long long j = tid; j < a.kept_width; j += K2_NT) {
        const bool in = j < keff;
        const unsigned long long kv = in ? sh.u.c.key[j] : 0ull;
        if (a.kept_p) a.kept_p[b * a.kept_width + j] = in ? bitsf((uint32_t)(kv >> 32)) : 0.0f;
        if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = in ? ~(uint32_t)(kv & 0xffffffffull) : 0xffffffffu;
      }
      return;
    }
    __syncthreads();
    // otherwise: the generic path below
  }

  // ---------------- generic path ----------------
  bool dense_all = false;
  for (int attempt = 0; attempt < 2; ++attempt) {
    for (int s = tid; s < nsub; s += K2_NT) {
      const long long st = (long long)s * a.SL;
      long long len = V - st;
      len = len < 0 ? 0 : (len > a.SL ? a.SL : len);
      sh.sub[s].start = st;
      sh.sub[s].dense = dense_all;
      sh.sub[s].cnt = dense_all ? len : (long long)(survs[s].count > 0 ? survs[s].count : 0);
    }
    __syncthreads();
    {
      long long c = tid < nsub ? sh.sub[tid].cnt : 0;
      long long tot;
      long long ex = block_excl_scan_add(c, sh.lscr, tot);
      if (tid < nsub) sh.sub[tid].base = ex;
      if (tid == 0) sh.n = tot;
    }
    __syncthreads();
    const long long n = sh.n;
    long long above = 0;  // elements whose exp exceeds that of every dropped one
    for (int s = 0; s < nsub; ++s) {
      const SubInfo si = sh.sub[s];
      for (long long jj = tid; jj < si.cnt; jj += K2_NT) {
        float e;
        uint32_t idx;
        if (si.dense) {
          idx = (uint32_t)(si.start + jj);
          const float raw = load_logit_dyn(row, a.dtype, si.start + jj);
          const float x = scale ? fdiv(raw, T) : raw;  // sampling.rs:46
          e = pesti_expf(fsub(x, m));                  // sampling.rs:127
        } else {
          e = a.surv_e[b * V + si.start + jj];
          idx = a.surv_idx[b * V + si.start + jj];
        }
        E[si.base + jj] = e;
        I[si.base + jj] = idx;
        above += (dense_all || e > e_pruned) ? 1 : 0;
      }
    }
    above = block_reduce_add(above, sh.lscr);  // also orders the E/I writes
    const float e_lim = dense_all ? -1.0f : e_pruned;
    // softmax denominator: sequential fold in index order (sampling.rs:128)
    const fold::Result sr = fold::block_fold(E, n, 0u, fold::NO_QUERY, false, sh.u.f);
    const float S = bitsf(sr.s_bits);

    int need_dense = 0;
    if (k > 0) {
      const long long keff = k < V ? k : V;
      if (!dense_all && above < keff) { dense_all = true; continue; }
      if (keff <= TOPK_SMALL) {
        // ---- top-k by candidates (sampling.rs:59-63) ----
        const uint32_t ek = select_kth_largest(E, n, keff, sh);
        if (tid == 0) {
          const float pk = fdiv(bitsf(ek), S);
          uint32_t e = ek;
          int it = 0;
          while (e > 0u && it < 64 && fdiv(bitsf(e - 1u), S) == pk) { --e; ++it; }
          sh.e_star = e;
          sh.fallback = it >= 64;
        }
        __syncthreads();
        const uint32_t estar = sh.e_star;
        long long cc = 0;
        for (long long j = tid; j < n; j += K2_NT) cc += fbits(E[j]) >= estar ? 1 : 0;
        cc = block_reduce_add(cc, sh.lscr);
        if (!sh.fallback && cc <= CAND_MAX) {
          int mm2 = 1;
          while (mm2 < (int)cc) mm2 <<= 1;
          for (int j = tid; j < mm2; j += K2_NT) sh.u.c.key[j] = 0ull;
          if (tid == 0) sh.u.c.cand_n = 0;
          __syncthreads();
          for (long long j = tid; j < n; j += K2_NT) {
            const float e = E[j];
            if (fbits(e) >= estar) {
              const int slot = atomicAdd(&sh.u.c.cand_n, 1);
              const float p = fdiv(e, S);  // sampling.rs:130
              sh.u.c.key[slot] = ((unsigned long long)fbits(p) << 32) | (unsigned long long)(~I[j]);
            }
          }
          __syncthreads();
          bitonic_desc(sh.u.c.key, mm2);  // (p desc, index asc) == the stable sort of sampling.rs:60
          if (tid == 0) {
            uint32_t s = 0u;  // sampling.rs:81
            for (long long j = 0; j < keff; ++j) s = fbits(fadd(bitsf(s), bitsf((uint32_t)(sh.u.c.key[j] >> 32))));
            sh.e_star = s;
          }
          __syncthreads();
          const float total = bitsf(sh.e_star);
          for (long long j = tid; j < keff; j += K2_NT)
            sh.u.c.q[j] = fdiv(bitsf((uint32_t)(sh.u.c.key[j] >> 32)), total);  // sampling.rs:94
          __syncthreads();
          if (tid == 0) {
            const fold::Result dr = fold::thread_fold(sh.u.c.q, keff, 0u, r_tau, true);  // sampling.rs:99-105
            const long long at = dr.hit >= 0 ? dr.hit : keff - 1;                     // sampling.rs:108-111
            a.out[b] = ~(uint32_t)(sh.u.c.key[at] & 0xffffffffull);
            if (a.kept_count) a.kept_count[b] = keff;
          }
          for (long long j = tid; j < a.kept_width; j += K2_NT) {
            const bool in = j < keff;
            const unsigned long long kv = in ? sh.u.c.key[j] : 0ull;
            if (a.kept_p) a.kept_p[b * a.kept_width + j] = in ? bitsf((uint32_t)(kv >> 32)) : 0.0f;
            if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = in ? ~(uint32_t)(kv & 0xffffffffull) : 0xffffffffu;
          }
          return;
        }
        // too many equal candidates: the sorted path below
      }
    }

    if (!a.SK0 || !a.Q) {
      if (tid == 0) {
        atomicOr(a.status, 1);
        a.out[b] = 0xffffffffu;
      }
      return;
    }
    uint32_t* SK0 = a.SK0 + b * V;
    uint32_t* SV0 = a.SV0 + b * V;
    uint32_t* SK1 = a.SK1 + b * V;
    uint32_t* SV1 = a.SV1 + b * V;
    float* Q = a.Q + b * V;

    if (k == 0 && !topp) {
      // ---- no filter: kept list = all V in index order (sampling.rs:92-111) ----
      for (long long j = tid; j < n; j += K2_NT) Q[j] = fdiv(E[j], S);
      __syncthreads();
      const fold::Result tr = fold::block_fold(Q, n, 0u, fold::NO_QUERY, false, sh.u.f);
      const float total = bitsf(tr.s_bits);
      for (long long j = tid; j < n; j += K2_NT) Q[j] = fdiv(Q[j], total);
      __syncthreads();
      const fold::Result dr = fold::block_fold(Q, n, 0u, r_tau, true, sh.u.f);
      if (tid == 0) {
        a.out[b] = dr.hit >= 0 ? I[dr.hit] : (uint32_t)(V - 1);
        if (a.kept_count) a.kept_count[b] = V;
      }
      for (long long j = tid; j < a.kept_width; j += K2_NT) {
        const bool in = j < V;
        float p = 0.0f;
        if (in) {
          const float raw = load_logit_dyn(row, a.dtype, j);
          const float x = scale ? fdiv(raw, T) : raw;
          p = fdiv(pesti_expf(fsub(x, m)), S);
        }
        if (a.kept_p) a.kept_p[b * a.kept_width + j] = p;
        if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = in ? (uint32_t)j : 0xffffffffu;
      }
      return;
    }

    // ---- sorted path: top-p (sampling.rs:65-78) or a large top-k ----
    for (long long j = tid; j < n; j += K2_NT) {
      SK0[j] = ~fbits(fdiv(E[j], S));
      SV0[j] = (uint32_t)j;
    }
    __syncthreads();
    const int which = sort::block_radix_sort(SK0, SV0, SK1, SV1, n, sh.u.s);
    const uint32_t* SK = which ? SK1 : SK0;
    const uint32_t* SV = which ? SV1 : SV0;
    for (long long j = tid; j < n; j += K2_NT) Q[j] = bitsf(~SK[j]);
    __syncthreads();
    long long c;
    long long kept_total;
    float total;
    if (topp) {
      const fold::Result pr = fold::block_fold(Q, n, 0u, fold::tau_bits_of(prm.top_p), true, sh.u.f);
      if (pr.hit >= 0) {
        c = pr.hit + 1;
        kept_total = c;
        total = bitsf(pr.hit_s_bits);
        if (!(E[SV[pr.hit]] > e_lim)) need_dense = 1;
      } else {
        c = n;
        kept_total = V;
        total = bitsf(pr.s_bits);
        if (!dense_all && n < V && a.kept_width > above) need_dense = 1;
      }
    } else {
      const long long keff = k < V ? k : V;
      c = keff;  // survivors hold the top keff (above >= keff or dense)
      kept_total = keff;
      const fold::Result pr = fold::block_fold(Q, c, 0u, fold::NO_QUERY, false, sh.u.f);
      total = bitsf(pr.s_bits);
    }
    if (need_dense) { dense_all = true; continue; }
    for (long long j = tid; j < a.kept_width; j += K2_NT) {
      const bool in = j < c;
      if (a.kept_p) a.kept_p[b * a.kept_width + j] = in ? Q[j] : 0.0f;
      if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = in ? I[SV[j]] : 0xffffffffu;
    }
    __syncthreads();
    for (long long j = tid; j < c; j += K2_NT) Q[j] = fdiv(Q[j], total);
    __syncthreads();
    const fold::Result dr = fold::block_fold(Q, c, 0u, r_tau, true, sh.u.f);
    if (tid == 0) {
      int nd = 0;
      uint32_t tok = 0;
      if (dr.hit >= 0) {
        const uint32_t pos = SV[dr.hit];
        if (!(E[pos] > e_lim)) nd = 1;
        tok = I[pos];
      } else {
        if (!dense_all && kept_total > c) nd = 1;  // last element of the full list is a dropped one
        tok = I[SV[c - 1]];
      }
      sh.need_dense = nd;
      if (!nd) {
        a.out[b] = tok;
        if (a.kept_count) a.kept_count[b] = kept_total;
      }
    }
    __syncthreads();
    if (sh.need_dense) { dense_all = true; continue; }
    return;
  }
}

}  // namespace pesti
