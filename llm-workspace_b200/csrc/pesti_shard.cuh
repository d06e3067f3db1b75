// Vocabulary-sharded sampling: the kernels that run once every shard's
// exchange record is in place.
//
// Each rank holds one contiguous, equally wide column range (a "shard") of
// every row.  The softmax denominator of sampling.rs:128 is one sequential
// f32 fold over the WHOLE row in index order, so shard r's part of it is a
// function F_r of the fold state s_r at its first column:
//     s_0 = 0,   s_{r+1} = F_r(s_r),   S = s_G.
// The ranks evaluate the chain without moving logits:
//  1. every shard folds its terms exactly (the fold entries of the survivor
//     and classification passes, walked by the row kernel) from an
//     approximate start, the earlier shards' approximate mass, and records
//     the increment delta_r = F_r(start) - start together with its top
//     candidates;
//  2. after those records are exchanged, the chained increments estimate
//     s_r within a few ulps; shard r tabulates F_r exactly at TAB_W
//     consecutive floats around that estimate (shard_table_kernel);
//  3. after the tables are exchanged, every rank chains them from s_0 = 0
//     (shard_finish_kernel): each s_r is looked up exactly, so S is the
//     reference's fold bit for bit.  The global top-k is the top-k of the
//     merged shard candidates (each shard lists its own top ksh by exp, and
//     a bound on the rest), then total, normalisation and draw follow the
//     single-device fast path.
// A row whose chain leaves a table, whose candidates cannot prove the top-k,
// or that is not a top-k row (greedy rows with NaN, top-p, no filter, large
// top-k) is listed for the gathered path: its shards are all-gathered into
// whole rows and sampled by the single-device kernels.
#pragma once
#include "pesti_kernels.cuh"

namespace pesti {

constexpr int TAB_W = 32;      // start states tabulated per shard and row (one per lane)
constexpr int TAB_BELOW = 16;  // of them below the chained estimate

struct ShardTab {
  uint32_t base;          // bits of the first tabulated start state
  uint32_t status;        // SH_OK, or SH_SKIP / SH_FAIL
  uint32_t tab[TAB_W];    // tab[j]: the shard's exact fold from the state with bits base + j
};
static_assert(sizeof(ShardTab) == 136, "tables are exchanged as raw bytes");

__host__ __device__ inline const ShardRec* shard_rec(const unsigned char* recs, long long stride, long long B,
                                                     int r, long long b) {
  return reinterpret_cast<const ShardRec*>(recs + ((long long)r * B + b) * stride);
}

struct TabArgs {
  const void* logits;  // this shard's columns, [B, ld]
  int dtype;
  long long B, ld;
  pesti_sampling_params uni;
  const pesti_sampling_params* per_row;
  const RowInfo* info;
  const unsigned char* recs;  // [G][B] exchange records
  long long rec_stride;
  int rank;
  const FoldEnt* ment_g;      // [B][FAST_ENTS] this shard's merged fold entries
  const int* nment_g;
  ShardTab* tab_out;          // [B]
};

// One warp per row: lane j folds the shard's merged entries from the state
// with bits base + j.  A run the state does not fit (or a replay marker) is
// folded from the raw logits of its column range, one lane at a time.
// Dynamic shared memory: TAB_SMEM bytes.
constexpr size_t TAB_SMEM = FAST_ENTS * sizeof(FoldEnt) + STAGE * sizeof(float);
__global__ void __launch_bounds__(32) shard_table_kernel(TabArgs a) {
  extern __shared__ __align__(16) unsigned char tab_smem[];
  FoldEnt* ent = reinterpret_cast<FoldEnt*>(tab_smem);
  float* stage = reinterpret_cast<float*>(ent + FAST_ENTS);
  const int lane = threadIdx.x;
  const long long b = blockIdx.x;
  ShardTab* out = a.tab_out + b;
  const int nm = a.nment_g[b];
  // the state at the shard's first column, estimated by chaining the earlier
  // shards' increments (each exact for its own approximate start)
  double est = 0.0;
  bool ok = nm >= 0;
  for (int r = 0; r < a.rank && ok; ++r) {
    const ShardRec* rc = shard_rec(a.recs, a.rec_stride, a.B, r, b);
    ok = rc->status == SH_OK;
    est += rc->delta;
  }
  if (!ok) {
    if (lane == 0) {
      out->base = 0u;
      out->status = nm < 0 ? SH_SKIP : SH_FAIL;
    }
    return;
  }
  for (int i = lane; i < nm; i += 32) ent[i] = a.ment_g[b * FAST_ENTS + i];
  __syncwarp();
  const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
  const float T = prm.temperature;
  const bool scale = T > 0.0f;
  const float m = a.info[b].m;
  const void* row = a.dtype != PESTI_F32 ? (const void*)((const uint16_t*)a.logits + b * a.ld)
                                          : (const void*)((const float*)a.logits + b * a.ld);
  const uint32_t eb = fbits(__double2float_rn(est));
  const uint32_t base = eb >= (uint32_t)TAB_BELOW ? eb - (uint32_t)TAB_BELOW : 0u;
  uint32_t s = base + (uint32_t)lane;
  for (int i = 0; i < nm; ++i) {
    const FoldEnt en = ent[i];
    bool fits = true;
    if (en.lo == fold::SPECIAL) {
      s = fbits(fadd(bitsf(s), bitsf(en.a0)));
    } else {
      const uint32_t ns = s + ((s & 1u) ? en.a1 : en.a0);  // < 2^31 + 2^30: no wrap
      // also false for every replay marker (no binade has its bits)
      fits = fold::binade_lo_bits(s) == en.lo && ns < fold::binade_hi_bits(en.lo);
      if (fits) s = ns;
    }
    uint32_t bad = __ballot_sync(PESTI_FULL_MASK, !fits);
    if (bad) {
      const uint32_t from = i > 0 ? ent[i - 1].end : 0u;
      const void* src = a.dtype != PESTI_F32 ? (const void*)((const uint16_t*)row + from)
                                              : (const void*)((const float*)row + from);
      while (bad) {
        const int l = __ffs(bad) - 1;
        bad &= bad - 1u;
        const uint32_t s0 = __shfl_sync(PESTI_FULL_MASK, s, l);
        const uint32_t s1 = warp_fold(src, a.dtype, (long long)en.end - from, s0, stage, scale, T, m);
        if (lane == l) s = s1;
      }
    }
  }
  out->tab[lane] = s;
  if (lane == 0) {
    out->base = base;
    out->status = SH_OK;
  }
}

struct FinishArgs {
  long long B, V_total;
  int G;
  pesti_sampling_params uni;
  const pesti_sampling_params* per_row;
  const RowInfo* info;        // any shard's (their whole-row fields agree)
  const unsigned char* recs;  // [G][B]
  long long rec_stride;
  int ksh;
  const ShardTab* tabs;       // [G][B]
  const float* u;
  uint32_t* out;
  float* kept_p;
  uint32_t* kept_idx;
  long long kept_width;
  int64_t* kept_count;
  int* nflag;                 // rows listed for the gathered path
  int* flag_rows;             // row | reason (GR_*) << 28
};

constexpr int FIN_KEYS = 4096;  // merged candidates a row may hold
constexpr int FIN_MAXG = 64;    // shards

struct FinishShared {
  unsigned long long key[FIN_KEYS];
  float q[FAST_K];
  int off[FIN_MAXG + 1];
  uint32_t s;
  int bad;
};

// One block (K2_NT threads) per row, on every rank: chain the tables to the
// exact softmax sum, merge the candidates, then top-k / total / draw as the
// single-device fast path does.  Greedy rows take the argmax from the shard
// summaries (via RowInfo).
__global__ void __launch_bounds__(K2_NT) shard_finish_kernel(FinishArgs a) {
  __shared__ FinishShared sh;
  const int tid = threadIdx.x;
  const long long b = blockIdx.x;
  const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
  const RowInfo ri = a.info[b];
  const long long VT = a.V_total;
  auto pad_kept = [&](long long from) {
    for (long long j = from + tid; j < a.kept_width; j += K2_NT) {
      if (a.kept_p) a.kept_p[b * a.kept_width + j] = 0.0f;
      if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = 0xffffffffu;
    }
  };
  auto gather_row = [&](uint32_t why) {  // the row goes to the gathered path
    if (tid == 0) {
      const int slot = atomicAdd(a.nflag, 1);
      a.flag_rows[slot] = (int)((uint32_t)b | (why << 28));
      a.out[b] = 0xffffffffu;
    }
  };
  if (is_greedy(prm)) {  // generate(): temperature == 0 -> argmax (model.rs:517-521)
    if (ri.flags & MF_NAN) {  // Iterator::max_by over NaN: on whole rows
      gather_row(GR_ROW);
      return;
    }
    const long long t = (prm.flags & PESTI_FLAG_ARGMAX_FIRST) ? ri.first_max : ri.last_max;
    if (tid == 0) {
      a.out[b] = t >= 0 ? (uint32_t)t : 0u;
      if (a.kept_count) a.kept_count[b] = 0;
    }
    pad_kept(0);
    return;
  }
  if (ri.uniform || !fast_topk(prm, VT)) {
    gather_row(GR_ROW);
    return;
  }
  const long long k = (long long)prm.top_k;
  const long long keff = k < VT ? k : VT;
  if (tid == 0) {
    // s_{r+1} = F_r(s_r), each F_r read exactly from its table
    uint32_t s = 0u, bad = 0u;
    int n = 0;
    for (int r = 0; r < a.G && !bad; ++r) {
      const ShardRec* rc = shard_rec(a.recs, a.rec_stride, a.B, r, b);
      const ShardTab* tb = a.tabs + (long long)r * a.B + b;
      if (rc->status != SH_OK || tb->status != SH_OK) {
        bad = rc->status != SH_OK ? rc->why : GR_CHAIN;
        break;
      }
      const uint32_t j = s - tb->base;
      if (j >= (uint32_t)TAB_W) {
        bad = GR_CHAIN;
        break;
      }
      s = tb->tab[j];
      sh.off[r] = n;
      n += rc->n;
    }
    sh.off[a.G] = n;
    sh.s = s;
    if (!bad && (n > FIN_KEYS || (long long)n < keff)) bad = GR_BOUND;
    if (!bad && !(bitsf(s) > 0.0f)) bad = GR_CHAIN;
    sh.bad = (int)bad;
  }
  __syncthreads();
  if (sh.bad) {
    gather_row((uint32_t)sh.bad);
    return;
  }
  const float S = bitsf(sh.s);
  const int n = sh.off[a.G];
  int mm2 = 1;
  while (mm2 < n) mm2 <<= 1;
  // keys (p desc, column asc) with p = e/S (sampling.rs:130): the stable sort of sampling.rs:60
  for (int r = 0; r < a.G; ++r) {
    const ShardRec* rc = shard_rec(a.recs, a.rec_stride, a.B, r, b);
    const ShardCand* cd = reinterpret_cast<const ShardCand*>(rc + 1);
    const int o = sh.off[r], c = sh.off[r + 1] - o;
    for (int i = tid; i < c; i += K2_NT)
      sh.key[o + i] = ((unsigned long long)fbits(fdiv(bitsf(cd[i].e_bits), S)) << 32) | (unsigned long long)(~cd[i].col);
  }
  for (int j = n + tid; j < mm2; j += K2_NT) sh.key[j] = 0ull;
  __syncthreads();
  bitonic_desc(sh.key, mm2);
  // every element a shard did not list must rank below the keff-th
  const float pk = bitsf((uint32_t)(sh.key[keff - 1] >> 32));
  if (tid == 0) sh.bad = 0;
  __syncthreads();
  for (int r = tid; r < a.G; r += K2_NT)
    if (!(fdiv(shard_rec(a.recs, a.rec_stride, a.B, r, b)->bound, S) < pk)) sh.bad = 1;
  __syncthreads();
  if (sh.bad) {
    gather_row(GR_BOUND);
    return;
  }
  if (tid == 0) {  // total over the kept list (sampling.rs:81)
    uint32_t tb = 0u;
    for (long long j = 0; j < keff; ++j) tb = fbits(fadd(bitsf(tb), bitsf((uint32_t)(sh.key[j] >> 32))));
    sh.s = tb;
  }
  __syncthreads();
  const float total = bitsf(sh.s);
  for (long long j = tid; j < keff; j += K2_NT) sh.q[j] = fdiv(bitsf((uint32_t)(sh.key[j] >> 32)), total);  // sampling.rs:94
  __syncthreads();
  if (tid == 0) {
    const float r = a.u[b];
    const fold::Result dr = fold::thread_fold(sh.q, keff, 0u, fold::tau_bits_of(r), true);  // sampling.rs:99-105
    const long long at = dr.hit >= 0 ? dr.hit : keff - 1;                                  // sampling.rs:108-111
    a.out[b] = ~(uint32_t)(sh.key[at] & 0xffffffffull);
    if (a.kept_count) a.kept_count[b] = keff;
  }
  for (long long j = tid; j < a.kept_width; j += K2_NT) {
    const bool in = j < keff;
    const unsigned long long kv = in ? sh.key[j] : 0ull;
    if (a.kept_p) a.kept_p[b * a.kept_width + j] = in ? bitsf((uint32_t)(kv >> 32)) : 0.0f;
    if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = in ? ~(uint32_t)(kv & 0xffffffffull) : 0xffffffffu;
  }
}

// Gathered path: row rows[i] of a matrix with src_pitch bytes per row copied
// (width bytes) to row i of a buffer with dst_pitch bytes per row; 16-byte
// words when every address and length allows, bytes otherwise.
__global__ void gather_rows_kernel(const unsigned char* src, long long src_pitch, const int* rows, int n,
                                   long long width, unsigned char* dst, long long dst_pitch) {
  const int i = blockIdx.y;
  if (i >= n) return;
  const unsigned char* s = src + (long long)rows[i] * src_pitch;
  unsigned char* d = dst + (long long)i * dst_pitch;
  const long long t0 = (long long)blockIdx.x * blockDim.x + threadIdx.x, step = (long long)gridDim.x * blockDim.x;
  if ((((uintptr_t)s | (uintptr_t)d | (uintptr_t)width) & 15u) == 0u) {
    const uint4* s4 = reinterpret_cast<const uint4*>(s);
    uint4* d4 = reinterpret_cast<uint4*>(d);
    for (long long j = t0; j < width / 16; j += step) d4[j] = s4[j];
  } else {
    for (long long j = t0; j < width; j += step) d[j] = s[j];
  }
}

// Results of the gathered rows (compact [n] / [n, W]) written to their rows.
__global__ void scatter_results_kernel(const int* rows, int n, const uint32_t* tok, const float* kp,
                                       const uint32_t* ki, const int64_t* kc, long long W, uint32_t* out,
                                       float* kept_p, uint32_t* kept_idx, int64_t* kept_count) {
  const int i = blockIdx.x;
  if (i >= n) return;
  const long long b = rows[i];
  if (threadIdx.x == 0) {
    out[b] = tok[i];
    if (kept_count) kept_count[b] = kc[i];
  }
  for (long long j = threadIdx.x; j < W; j += blockDim.x) {
    if (kept_p) kept_p[b * W + j] = kp[(long long)i * W + j];
    if (kept_idx) kept_idx[b * W + j] = ki[(long long)i * W + j];
  }
}

// Per-row values of the gathered rows: u and (device) parameters.
__global__ void gather_row_values_kernel(const int* rows, int n, const float* u, float* u_out,
                                         const pesti_sampling_params* prm, pesti_sampling_params* prm_out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    u_out[i] = u[rows[i]];
    if (prm) prm_out[i] = prm[rows[i]];
  }
}

}  // namespace pesti

namespace pesti {

// Test support: the largest relative error of the hardware 2^y approximation
// (ex2.approx.ftz.f32) against exp2 in double, over every float y in
// [-200, 0] and y = -inf, as the bits of a non-negative double (which order
// as unsigned integers).  Below y = -126 (results under 2^-126) a result of 0
// is allowed (flushed); any other result counts with its error, and a
// non-zero result for -inf counts as error 1.  The bound the classification's
// cheap exp relies on is checked against it.
__global__ void ex2_approx_error_kernel(unsigned long long* max_bits) {
  const uint32_t n = 0x43480000u + 1u;  // bit patterns 0x80000000 (-0) .. 0xC3480000 (-200)
  unsigned long long best = 0ull;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float y = __uint_as_float(0x80000000u + i);
    const float r = ex2_approx(y);
    const double ref = exp2((double)y);
    double rel = fabs((double)r - ref) / ref;
    if (y < -126.0f && r == 0.0f) rel = 0.0;
    const unsigned long long b = (unsigned long long)__double_as_longlong(rel);
    best = b > best ? b : best;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && ex2_approx(-__int_as_float(0x7f800000)) != 0.0f)
    best = (unsigned long long)__double_as_longlong(1.0);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(PESTI_FULL_MASK, best, o);
    best = t > best ? t : best;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(max_bits, best);
}

}  // namespace pesti
