// Kernels of the sampler: the slice scan (one HBM pass over the logits) and
// the per-row sampler.  Semantics follow llm-runner/src/transformer/sampling.rs
// line by line; every f32 operation the reference performs is performed here
// as the same single IEEE operation on the same operands.
#pragma once
#include <stdint.h>
#include <cuda_bf16.h>
#include "pesti_common.cuh"
#include "pesti_exp.cuh"
#include "pesti_fold.cuh"
#include "../../include/pesti_sampler.h"

namespace pesti {

constexpr int K1_WARPS = 8;  // warps (= sub-slices) per slice-scan block
constexpr int K1_NT = K1_WARPS * 32;
constexpr int K2_NT = 512;
constexpr int MAX_SUBS = 512;    // sub-slices per row handled by the row kernel
constexpr int TOPK_SMALL = 1024; // top-k values handled by the candidate path
constexpr int CAND_MAX = 2048;   // candidate buffer of that path

// Absorption distance, in scaled-logit units: an element more than this below
// an earlier element of the same row is added as an exact no-op by every fold
// (e_i < 2^-25 * e_j <= ulp(s)/2).  25*ln2 = 17.3287; the margin absorbs the
// rounding of x/T, x-m and exp.  Derivation is in the slice-scan kernel.
constexpr float ABSORB = 17.35f;
// Survivors of the slice scan cover every element with d = x - m >= -NEAR_D.
constexpr float NEAR_D = 17.33f;
// Pruning is trusted only if the prefix maximum it used was within this many
// scaled units of the row maximum (keeps the pruned values' neighbours normal).
constexpr float PRUNE_FLOOR = 60.0f;

enum : uint32_t { MF_NAN = 1u, MF_POSINF = 2u, MF_NEGINF = 4u };

// Per sub-slice summary written by the slice scan.
struct WarpMeta {
  float max_raw;         // max of the raw logits, NaN ignored (f32::max fold, sampling.rs:126)
  uint32_t last_max;     // last index holding max_raw (0xffffffff if none)
  uint32_t first_max;    // first index holding max_raw
  int32_t last_nan;      // last NaN index or -1
  int32_t count;         // survivors written, or -1: too many, read the raw logits
  uint32_t flags;        // MF_*
  float prune_floor;     // smallest prefix max that pruned an element (+inf if none)
  uint32_t pad;
};

struct SliceArgs {
  const void* logits;
  long long B, V, ld;
  pesti_sampling_params uni;
  const pesti_sampling_params* per_row;
  int P;           // slices per row (blocks per row)
  long long SL;    // elements per sub-slice (one warp each)
  WarpMeta* meta;  // [B][P*K1_WARPS]
  float* surv_raw; // [B][V]: survivors of sub-slice s compacted at its own start
  uint32_t* surv_idx;
};

struct RowArgs {
  const void* logits;
  int dtype;
  long long B, V, ld;
  pesti_sampling_params uni;
  const pesti_sampling_params* per_row;
  int P;
  long long SL;
  const WarpMeta* meta;
  const float* surv_raw;
  const uint32_t* surv_idx;
  float* E;       // [B][V] exp values of the row's sequence
  uint32_t* I;    // [B][V] their logit indices
  uint32_t* SK0;  // [B][V] sort buffers (may be null when no row needs them)
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
  int* status;    // bit 0: a row needed buffers that were not provided
};

__device__ __forceinline__ pesti_sampling_params row_params(const pesti_sampling_params& uni,
                                                            const pesti_sampling_params* per_row,
                                                            long long b) {
  return per_row ? per_row[b] : uni;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
  return __uint_as_float(((uint32_t)h) << 16);
}

template <typename TIn>
__device__ __forceinline__ float load_logit(const TIn* row, long long j);
template <>
__device__ __forceinline__ float load_logit<float>(const float* row, long long j) {
  return __ldg(row + j);
}
template <>
__device__ __forceinline__ float load_logit<uint16_t>(const uint16_t* row, long long j) {
  return bf16_bits_to_f32(__ldg(row + j));
}

__device__ __forceinline__ float load_logit_dyn(const void* row, int dtype, long long j) {
  return dtype == PESTI_BF16 ? load_logit<uint16_t>((const uint16_t*)row, j)
                             : load_logit<float>((const float*)row, j);
}

// ---------------------------------------------------------------------------
// Slice scan.  One warp streams one contiguous sub-slice of a row, with 16-byte
// loads, and produces (a) the row-max / argmax / NaN summary and (b) the
// survivors: every element that is not provably absorbed by the index-order
// softmax fold.  Element i (scaled x_i = raw_i/T) is dropped when an EARLIER
// element j of the same row has x_j >= x_i + 17.34: then e_i <= 0.989*2^-25*e_j
// and, since the running sum s_{i-1} >= e_j and ulp(s)/2 > s*2^-25, the add
// fl(s + e_i) returns s.  The same ratio bound makes i a no-op in the top-p,
// total and draw folds (sorted order starts at p_max >= p_j; index order has
// p_j before i), so the folds over the survivors equal the folds over the row.
// The test is done on raw values: raw_i < P - (17.35*T*(1+2^-20) + 2^-21*|P|),
// P = prefix max; the slack covers the rounding of raw/T (2^-24 relative),
// x - m (<= 2^-24*104 for elements whose exp is not 0) and of exp itself.
// ---------------------------------------------------------------------------
template <typename TIn, int VE, int U, bool VEC>
__global__ void __launch_bounds__(K1_NT) slice_scan_kernel(SliceArgs a) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const long long b = blockIdx.x / a.P;
  const int slice = (int)(blockIdx.x % a.P);
  const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
  const bool greedy = (prm.flags & PESTI_FLAG_GREEDY_IF_ZERO_T) && prm.temperature == 0.0f;
  const float t_eff = prm.temperature > 0.0f ? prm.temperature : 1.0f;
  const float c1 = ABSORB * t_eff * (1.0f + 0x1p-20f);
  const long long sub = (long long)slice * K1_WARPS + w;
  const long long start = sub * a.SL;
  long long end = start + a.SL;
  if (end > a.V) end = a.V;
  const TIn* row = (const TIn*)a.logits + b * a.ld;
  const long long out_base = b * a.V + start;
  const long long cap = a.SL / 4;

  float run_max = -__int_as_float(0x7f800000);
  float best_v = run_max, fbest_v = run_max;
  long long best_i = -1, fbest_i = -1, last_nan = -1;
  uint32_t flags = 0;
  long long total = 0;
  bool dense = false;
  float floor_p = __int_as_float(0x7f800000);

  auto process = [&](const float* x, long long pos0, int nv) {
    // exclusive prefix maxima inside the lane, then across lanes
    float pre[VE];
    float lm = -__int_as_float(0x7f800000);
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
    if (lane == 0) exc = -__int_as_float(0x7f800000);
    const float seg_max = __shfl_sync(PESTI_FULL_MASK, inc, 31);
    const float p0 = fmaxf(run_max, exc);
    int cnt = 0;
    bool sv[VE];
#pragma unroll
    for (int e = 0; e < VE; ++e) {
      const float P = fmaxf(p0, pre[e]);
      const float thr = fsub(P, fadd(c1, 0x1p-21f * fabsf(P)));
      const bool valid = e < nv;
      sv[e] = valid && !greedy && x[e] >= thr;
      if (valid && !greedy && !sv[e] && !is_nan(x[e])) floor_p = fminf(floor_p, P);
      cnt += sv[e] ? 1 : 0;
      if (valid) {
        const float xv = x[e];
        const long long pos = pos0 + e;
        if (is_nan(xv)) {
          last_nan = pos;
          flags |= MF_NAN;
        } else {
          if (best_i < 0 || xv >= best_v) { best_v = xv; best_i = pos; }
          if (fbest_i < 0 || xv > fbest_v) { fbest_v = xv; fbest_i = pos; }
          if (xv == __int_as_float(0x7f800000)) flags |= MF_POSINF;
          if (xv == -__int_as_float(0x7f800000)) flags |= MF_NEGINF;
        }
      }
    }
    run_max = fmaxf(run_max, seg_max);
    const int cinc = warp_incl_scan_add(cnt);
    const int wsum = __shfl_sync(PESTI_FULL_MASK, cinc, 31);
    if (!dense) {
      if (total + wsum > cap) {
        dense = true;
      } else {
        long long o = out_base + total + (cinc - cnt);
#pragma unroll
        for (int e = 0; e < VE; ++e) {
          if (sv[e]) {
            a.surv_raw[o] = x[e];
            a.surv_idx[o] = (uint32_t)(pos0 + e);
            ++o;
          }
        }
      }
    }
    total += wsum;
  };

  const long long CH = 32LL * VE * U;  // elements per warp iteration
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
        process(x, pos + (long long)uu * 32 * VE + (long long)lane * VE, VE);
      }
    }
  }
  // tail (and the whole sub-slice when rows are not 16-byte aligned)
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
    process(x, p0, nv);
  }

  // warp summary
  const float mx = warp_reduce_fmax(best_i >= 0 ? best_v : -__int_as_float(0x7f800000));
  long long li = (best_i >= 0 && best_v == mx) ? best_i : -1;
  long long fi = (fbest_i >= 0 && fbest_v == mx) ? fbest_i : (1LL << 62);
  li = warp_reduce_max(li);
  fi = warp_reduce_min(fi);
  const long long ln = warp_reduce_max(last_nan);
  uint32_t fl = flags;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) fl |= __shfl_xor_sync(PESTI_FULL_MASK, fl, o);
  const float fp = -warp_reduce_fmax(-floor_p);
  if (lane == 0) {
    WarpMeta m;
    m.max_raw = mx;
    m.last_max = li >= 0 ? (uint32_t)li : 0xffffffffu;
    m.first_max = fi < (1LL << 62) ? (uint32_t)fi : 0xffffffffu;
    m.last_nan = (int32_t)ln;
    m.count = dense ? -1 : (int32_t)total;
    m.flags = fl;
    m.prune_floor = fp;
    m.pad = 0;
    a.meta[b * (long long)a.P * K1_WARPS + sub] = m;
  }
}

// ---------------------------------------------------------------------------
// Row sampler: one block per row.
// ---------------------------------------------------------------------------
struct SubInfo {
  long long start;
  long long len;    // elements of the sub-slice inside the row
  long long cnt;    // sequence elements it contributes
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
      uint32_t iscr[34];
      long long lscr[34];
      uint32_t sel_prefix;
      long long sel_k;
      int cand_n;
    } c;
  } u;
  SubInfo sub[MAX_SUBS];
  long long lscr[34];
  float fscr[34];
  int iscr[34];
  uint32_t uscr[34];
  // row state
  float max_raw;
  long long last_max, first_max, last_nan;
  uint32_t flags;
  long long n;
  long long near_cnt;
  int need_dense;
  uint32_t e_star;
  int fallback;
};

// Rust's Iterator::max_by over the raw logits with partial_cmp (sampling.rs:115-122)
// when the row holds NaN: the scan adopts every NaN and then the element right
// after it, so the result is the last maximum after the last NaN (or that NaN
// itself when it is the final element).
__device__ uint32_t nan_argmax(const void* row, int dtype, long long V, long long last_nan,
                               RowShared& sh) {
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
  const int tid = threadIdx.x;
  if (tid == 0) {
    sh.u.c.sel_prefix = 0u;
    sh.u.c.sel_k = k;
  }
  uint32_t mask = 0u;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += K2_NT) sh.u.c.hist[i] = 0u;
    __syncthreads();
    const uint32_t prefix = sh.u.c.sel_prefix;
    for (long long j = tid; j < n; j += K2_NT) {
      const uint32_t x = fbits(E[j]);
      if ((x & mask) == prefix) atomicAdd(&sh.u.c.hist[(x >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      long long kk = sh.u.c.sel_k;
      uint32_t cum = 0;
      int d = 255;
      for (; d > 0; --d) {
        if ((long long)(cum + sh.u.c.hist[d]) >= kk) break;
        cum += sh.u.c.hist[d];
      }
      sh.u.c.sel_k = kk - cum;
      sh.u.c.sel_prefix = prefix | ((uint32_t)d << shift);
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  return sh.u.c.sel_prefix;
}

// Bitonic sort of sh.u.c.key[0..m), m a power of two, descending.
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

__global__ void __launch_bounds__(K2_NT) row_kernel(RowArgs a) {
  extern __shared__ __align__(16) unsigned char row_smem[];
  RowShared& sh = *reinterpret_cast<RowShared*>(row_smem);
  const int tid = threadIdx.x;
  const long long b = blockIdx.x;
  const long long V = a.V;
  const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
  const float T = prm.temperature;
  const bool greedy = (prm.flags & PESTI_FLAG_GREEDY_IF_ZERO_T) && T == 0.0f;
  const int nsub = a.P * K1_WARPS;
  const void* row = a.dtype == PESTI_BF16 ? (const void*)((const uint16_t*)a.logits + b * a.ld)
                                          : (const void*)((const float*)a.logits + b * a.ld);
  float* E = a.E + b * V;
  uint32_t* I = a.I + b * V;
  const float r = a.u ? a.u[b] : 0.0f;
  const float INF = __int_as_float(0x7f800000);

  // ---- row summary from the sub-slice metadata ----
  float mx = -INF;
  long long li = -1, fi = 1LL << 62, ln = -1;
  uint32_t fl = 0;
  for (int s = tid; s < nsub; s += K2_NT) {
    const WarpMeta m = a.meta[b * nsub + s];
    const long long st = (long long)s * a.SL;
    long long len = V - st;
    len = len < 0 ? 0 : (len > a.SL ? a.SL : len);
    if (len > 0) {
      mx = fmaxf(mx, m.max_raw);
      ln = ln > m.last_nan ? ln : m.last_nan;
      fl |= m.flags;
    }
  }
  mx = -block_reduce_min(-mx, sh.fscr);
  for (int s = tid; s < nsub; s += K2_NT) {
    const WarpMeta m = a.meta[b * nsub + s];
    const long long st = (long long)s * a.SL;
    if (st < V && m.max_raw == mx) {
      if (m.last_max != 0xffffffffu) li = li > (long long)m.last_max ? li : (long long)m.last_max;
      if (m.first_max != 0xffffffffu) fi = fi < (long long)m.first_max ? fi : (long long)m.first_max;
    }
  }
  li = block_reduce_max(li, sh.lscr);
  fi = block_reduce_min(fi, sh.lscr);
  ln = block_reduce_max(ln, sh.lscr);
  {
    // OR-reduce of flags
    int f = 0;
    for (int s = tid; s < nsub; s += K2_NT) {
      const long long st = (long long)s * a.SL;
      if (st < V) f |= (int)a.meta[b * nsub + s].flags;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) f |= __shfl_xor_sync(PESTI_FULL_MASK, f, o);
    if ((tid & 31) == 0) sh.iscr[tid >> 5] = f;
    __syncthreads();
    if (tid == 0) {
      int g = 0;
      for (int q = 0; q < K2_NT / 32; ++q) g |= sh.iscr[q];
      sh.flags = (uint32_t)g;
    }
    __syncthreads();
    fl = sh.flags;
    __syncthreads();
  }
  const long long last_max = li, first_max = fi < (1LL << 62) ? fi : -1, last_nan = ln;

  if (V <= 0) {  // empty slice: sample() and argmax() return 0
    if (tid == 0) {
      a.out[b] = 0u;
      if (a.kept_count) a.kept_count[b] = 0;
    }
    write_kept_pad(a, b, 0);
    return;
  }

  if (greedy) {  // generate(): temperature == 0 -> argmax (model.rs:517-521)
    uint32_t tok;
    if (prm.flags & PESTI_FLAG_ARGMAX_FIRST) {
      tok = first_max >= 0 ? (uint32_t)first_max : 0u;
    } else if (fl & MF_NAN) {
      tok = nan_argmax(row, a.dtype, V, last_nan, sh);
    } else {
      tok = last_max >= 0 ? (uint32_t)last_max : 0u;
    }
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
        tok = (uint32_t)((fl & MF_NAN) ? 0 : (last_max >= 0 ? last_max : 0));
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

  // ---- sequence of survivors (index order) ----
  const float m_scaled = m;
  bool dense_all = false;
  for (int attempt = 0; attempt < 2; ++attempt) {
    // sub-slice layout and offsets
    for (int s = tid; s < nsub; s += K2_NT) {
      const WarpMeta mm = a.meta[b * nsub + s];
      const long long st = (long long)s * a.SL;
      long long len = V - st;
      len = len < 0 ? 0 : (len > a.SL ? a.SL : len);
      int dn = dense_all || mm.count < 0;
      if (!dn && len > 0 && mm.prune_floor < INF) {
        // pruning against a prefix max far below the row max is not trusted
        const float fs = scale ? fdiv(mm.prune_floor, T) : mm.prune_floor;
        if (!(fsub(m_scaled, fs) <= PRUNE_FLOOR)) dn = 1;
      }
      sh.sub[s].start = st;
      sh.sub[s].len = len;
      sh.sub[s].dense = dn;
      sh.sub[s].cnt = dn ? len : (long long)(mm.count > 0 ? mm.count : 0);
    }
    __syncthreads();
    // exclusive offsets (nsub <= MAX_SUBS)
    {
      long long c = tid < nsub ? sh.sub[tid].cnt : 0;
      long long tot;
      long long ex = block_excl_scan_add(c, sh.lscr, tot);
      if (tid < nsub) sh.sub[tid].base = ex;
      if (tid == 0) sh.n = tot;
    }
    __syncthreads();
    const long long n = sh.n;
    long long near = 0;
    for (int s = 0; s < nsub; ++s) {
      const SubInfo si = sh.sub[s];
      for (long long jj = tid; jj < si.cnt; jj += K2_NT) {
        float raw;
        uint32_t idx;
        if (si.dense) {
          idx = (uint32_t)(si.start + jj);
          raw = load_logit_dyn(row, a.dtype, si.start + jj);
        } else {
          raw = a.surv_raw[b * V + si.start + jj];
          idx = a.surv_idx[b * V + si.start + jj];
        }
        const float x = scale ? fdiv(raw, T) : raw;  // sampling.rs:46
        const float d = fsub(x, m_scaled);           // sampling.rs:127
        const float e = pesti_expf(d);
        E[si.base + jj] = e;
        I[si.base + jj] = idx;
        near += d >= -NEAR_D ? 1 : 0;
      }
    }
    near = block_reduce_add(near, sh.lscr);  // also orders the E/I writes
    // softmax denominator: sequential fold in index order (sampling.rs:128)
    const fold::Result sr = fold::block_fold(E, n, 0u, fold::NO_QUERY, false, sh.u.f);
    const float S = bitsf(sr.s_bits);

    int need_dense = 0;
    if (k > 0) {
      const long long keff = k < V ? k : V;
      if (!dense_all && near < keff) { dense_all = true; continue; }
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
          // (p desc, index asc) == the stable sort of sampling.rs:60
          bitonic_desc(sh.u.c.key, mm2);
          if (tid == 0) {
            // total over the kept list (sampling.rs:81)
            uint32_t s = 0u;
            for (long long j = 0; j < keff; ++j) s = fbits(fadd(bitsf(s), bitsf((uint32_t)(sh.u.c.key[j] >> 32))));
            sh.e_star = s;
          }
          __syncthreads();
          const float total = bitsf(sh.e_star);
          for (long long j = tid; j < keff; j += K2_NT)
            sh.u.c.q[j] = fdiv(bitsf((uint32_t)(sh.u.c.key[j] >> 32)), total);  // sampling.rs:94
          __syncthreads();
          if (tid == 0) {
            uint32_t tok;
            if (!(total > 0.0f)) {
              tok = (uint32_t)last_max;
            } else {
              const fold::Result dr = fold::thread_fold(sh.u.c.q, keff, 0u, r_tau, true);  // sampling.rs:99-105
              const long long at = dr.hit >= 0 ? dr.hit : keff - 1;                     // sampling.rs:108-111
              tok = ~(uint32_t)(sh.u.c.key[at] & 0xffffffffull);
            }
            a.out[b] = tok;
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
        // too many equal candidates: fall through to the sorted path
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
          p = fdiv(pesti_expf(fsub(x, m_scaled)), S);
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
        if (!dense_all && E[SV[pr.hit]] < 4.2e-8f) need_dense = 1;
      } else {
        c = n;
        kept_total = V;
        total = bitsf(pr.s_bits);
        if (!dense_all && n < V && a.kept_width > near) need_dense = 1;
      }
    } else {
      const long long keff = k < V ? k : V;
      c = keff;  // survivors hold the top keff (near >= keff or dense)
      kept_total = keff;
      const fold::Result pr = fold::block_fold(Q, c, 0u, fold::NO_QUERY, false, sh.u.f);
      total = bitsf(pr.s_bits);
    }
    if (need_dense) { dense_all = true; continue; }
    // kept list (p before normalisation)
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
        if (!dense_all && E[pos] < 4.2e-8f) nd = 1;
        tok = I[pos];
      } else {
        if (!dense_all && kept_total > c) nd = 1;  // last element of the full list is a pruned one
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
