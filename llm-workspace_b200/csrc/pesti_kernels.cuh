// Kernels of the sampler.  Semantics follow llm-runner/src/transformer/sampling.rs
// line by line; every f32 operation the reference performs is performed here
// as the same single IEEE operation on the same operands, and every f32 sum
// is the reference's sequential fold, emulated exactly (pesti_fold.cuh).
//
// Three kernels per batch:
//   slice_stats_kernel  the one HBM pass: per sub-slice (one warp each) the max
//                       of the raw logits, NaN/inf flags, an approximate
//                       partial softmax sum and per-segment maxima.  The last
//                       block of each row to finish turns these into the row
//                       prologue (row max and argmax, candidate threshold,
//                       per-sub-slice prefix mass and prefix max).
//   survivor_kernel     re-reads each sub-slice (from L2): drops the elements
//                       that provably do not change any fold, classifies the
//                       rest into the sub-slice's part of the softmax fold
//                       (runs of plain integer increments and single elements
//                       to add directly) and lists the top-k candidates;
//   row_kernel          one block per row: walks the fold entries to the exact
//                       softmax sum, then top-k / top-p / draw.
#pragma once
#include <stdint.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
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
constexpr int FAST_CAND = 1024;   // candidates the fast path sorts
constexpr int TAU_BINS = 4096;    // 12-bit histogram used to place the candidate threshold
constexpr int MAX_MATCH = 64;     // segments holding the row max re-scanned for its indices
constexpr int QCAP = 512;         // survivor queue per warp (power of two)
constexpr int GR = 8;             // survivors per lane in one classification task
constexpr int GROUP = 32 * GR;    // survivors per classification task
constexpr int POOL_CAP = 4096;    // fold entries per row (all its classification tasks)
constexpr int UNIT = 256;         // elements of one classification unit of the fused pass
constexpr int STAGE = 256;        // values staged per round trip by warp_fold
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
  float sum_rel;      // sum of 2^(y - y_max), y = raw*log2(e)/T_eff (approximate)
  int32_t last_nan;   // last NaN index or -1
  uint32_t flags;     // MF_*
};

struct RowInfo {      // row prologue, written by the last slice_stats block of the row
  float max_raw;      // row max of the raw logits (NaN ignored)
  float m;            // max of the scaled logits: RN(max_raw/T) when T > 0 (division is monotone)
  float tau;          // candidate threshold (raw units); +inf when no candidates are needed
  uint32_t flags;     // MF_* over the row
  long long last_max, first_max, last_nan;  // argmax indices: greedy rows only
  int uniform;        // the softmax sum is NaN or not > 0: all probabilities are 1/V
  float e_tau;        // exact exp(RN(tau/T) - m) when tau is finite, else 0
  float s_start;      // vocabulary shard: approximate softmax fold state at the shard's first
                      // column (the mass of the earlier shards); 0 for whole rows
  float S;            // the cluster pass's exact softmax sum (rows it leaves with only[b] == 2)
  float min_raw;      // the smallest raw logit (NaN ignored; the cluster pass only)
};

// One vocabulary shard of a row, summarised before the shards are combined
// (first phase of the sharded path).  Every rank holds one contiguous,
// equally wide column range; the summaries of all ranks are all-gathered.
struct ShardSum {
  float max_raw;          // max of the shard's raw logits (NaN ignored)
  uint32_t flags;         // MF_* over the shard
  float tau;              // lower bound of the shard's k-th largest raw logit (-inf: none;
                          // +inf: not a top-k row)
  int32_t last_nan;       // shard column of its last NaN, -1
  double mass;            // approximate softmax mass of the shard relative to 2^(max_raw*c2)
  long long last_max, first_max;  // shard columns holding its max (greedy rows), -1
};
static_assert(sizeof(ShardSum) == 40, "ShardSum is exchanged as raw bytes");

// The pass over HBM's running state of a sub-slice at the start of each
// UNIT-element unit, for the fused pass: the approximate mass of the
// sub-slice's elements before the unit, relative to 2^mlog, and their max.
struct UnitPre {
  float mass;   // sum of 2^(x*c2 - mlog) over the sub-slice's elements before the unit
  float mlog;   // log2-unit max those sums are relative to (-inf: none)
  float pmax;   // max raw logit of the sub-slice before the unit (-inf: none)
  float pad;
};

struct SubPre {       // per sub-slice, from the row prologue
  double A;           // approximate softmax mass of the earlier sub-slices
  float P;            // max raw logit of the earlier sub-slices
  float thrL;         // raw logits below it are absorbed by the running sum (bound (b)), or -inf
};

struct FoldEnt {      // one entry of a sub-slice's part of the softmax fold
  uint32_t lo;        // binade (bits of its lowest value) of a run; fold::SPECIAL: one element
  uint32_t a0, a1;    // run: increments for an even / odd entry state; special: bits of the value
  uint32_t end;       // row index just past the entry's last element: the entry covers the
                      // row from the previous entry's end (the elements between are no-ops)
};

struct SubSurv {      // one per sub-slice: survivor_kernel, or the fused pass (fast-path rows)
  int32_t count;      // survivors stored at the sub-slice's own start (survivor_kernel)
  int32_t ngroups;    // classification groups of the sub-slice (tasks, or the fused pass's units)
  int32_t pad;        // survivor_kernel: the classification tasks list the candidates;
                      // row_kernel scratch: the sub-slice is replayed
  float pruned_max;   // largest raw logit dropped (-inf if none)
};


struct ClassTask {    // one group of GROUP survivors of a sub-slice (task-queue classification)
  int32_t b;          // row
  int32_t qj;         // sub-slice * jmax + group
};

struct GroupEnt {     // one per classification group (task or fused unit): its fold entries
  uint32_t ent[4];    // inl: the unit's only entry (a FoldEnt), kept here instead of the pool
  int32_t off;        // first entry in the row's pool
  int32_t nent;       // entries (0 with replay)
  int32_t replay;     // the pool was full: the row kernel replays the sub-slice
  int32_t inl;
};

struct SliceArgs {
  const void* logits;
  int dtype;        // pesti_dtype of the logits
  long long B, V, ld;
  pesti_sampling_params uni;
  const pesti_sampling_params* per_row;
  int P;            // slice blocks per row
  long long SL;     // elements per sub-slice (one warp each)
  long long nseg;   // 32*VE-element segments per row
  SubStat* stats;   // [B][P*K1_WARPS]
  SubPre* pre;      // [B][P*K1_WARPS]
  RowInfo* info;    // [B]
  int* row_ctr;     // [B] blocks of the row finished (reset by the last one)
  SubSurv* surv;    // [B][P*K1_WARPS]
  float* seg_max;   // [B][nseg]
  UnitPre* unit_pre;  // [B][nunit], nunit = ceil(V / UNIT)
  float* surv_raw;  // [B][V]: raw logits of the survivors of sub-slice s, compacted at its own start
  uint32_t* surv_idx;
  int jmax;         // classification groups per sub-slice (ceil(SL / UNIT) = ceil(SL / GROUP))
  int* item_next;   // items of the fused pass taken from the counter
  int fused;        // the rows of the fast path take the fused pass (else: survivors + task queue)
  ClassTask* tasks; // [B*P*K1_WARPS*jmax] task-queue classification
  int* task_count;  // tasks queued
  int* task_next;   // tasks taken
  int* task_count_h;  // tasks of the rows' first sub-slices (the slowest), queued from the top of the list
  GroupEnt* gsurv;  // [B][P*K1_WARPS][jmax]
  FoldEnt* pool;    // [B][POOL_CAP] fold entries
  int* pool_ctr;    // [B]
  int* cand_count;  // [B]
  float* cand_e;    // [B][CAND_CAP] exact exps of the top-k candidates (sampling.rs:127)
  uint32_t* cand_idx;
  int fast_enabled; // rows of the fast path keep no survivors (see survivor_kernel)
  long long V_total;      // length of the whole row (V unless the call is one vocabulary shard)
  float band;             // relative guard band of the fold classification around binade edges
  // vocabulary shards (all null / 0 for whole rows)
  ShardSum* shard_out;        // first phase: the row's shard summary instead of its prologue
  const ShardSum* shard_all;  // second phase: [G][B] summaries of every shard
  int shard_G, shard_rank;
};

struct RowArgs {
  const void* logits;
  int dtype;
  long long B, V, ld;
  pesti_sampling_params uni;
  const pesti_sampling_params* per_row;
  int P;
  long long SL;
  const RowInfo* info;
  const SubSurv* surv;
  int jmax;
  const GroupEnt* gsurv;
  const FoldEnt* pool;
  const float* surv_raw;
  const uint32_t* surv_idx;
  const int* cand_count;
  const float* cand_e;
  const uint32_t* cand_idx;
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
  int* status;       // bit 0: a row needed sort buffers that were not provided
  int fast_enabled;  // the launch provides the fast path's shared memory
  int fast_ents;     // and stages this many fold entries per row (<= FAST_ENTS)
  long long V_total;   // length of the whole row (V unless the call is one vocabulary shard)
  // vocabulary shard (shard = 1): instead of sampling, each row's fold from
  // the shard's approximate start state and its top candidates go to an
  // exchange record, and its merged fold entries are kept for the table walks
  int shard;
  long long col0;          // the shard's first column in the whole row
  unsigned char* rec;      // [B] records of rec_stride bytes: ShardRec + ksh ShardCand
  long long rec_stride;
  int ksh;
  FoldEnt* ment_g;         // [B][FAST_ENTS] merged fold entries
  int* nment_g;            // [B] their count (-1: the row is not sampled from shards)
  // rows left by the cluster pass (only != null): a block samples its row only
  // when only[b] != 0, from the whole row (no survivor lists) on the generic
  // path, or (only[b] == 2, nucleus != 0) a bf16 top-p row by distinct values
  const int* only;
  int nucleus;  // the launch provides the nucleus rows' shared memory
};

// Exchange record of one row of one vocabulary shard (second phase).
enum : uint32_t { SH_OK = 0u, SH_SKIP = 1u, SH_FAIL = 2u };
// Why a row took the gathered path (top 4 bits of its entry in the list).
enum : uint32_t { GR_ROW = 1u, GR_ENTRIES = 2u, GR_CANDS = 3u, GR_CHAIN = 4u, GR_BOUND = 5u, GR_KINDS = 6u };
struct ShardRec {
  double delta;     // exact fold of the shard's softmax terms from s_start, minus s_start
  float s_start;    // the approximate state the fold started from
  uint32_t status;  // SH_OK; SH_SKIP: not a sharded row; SH_FAIL: the row needs the gathered path
  float bound;      // every element of the shard not listed has an exp <= bound
  int32_t n;        // candidates listed (at most ksh), by (exp desc, column asc)
  uint32_t why;     // SH_FAIL: GR_ENTRIES (fold entries overflow) or GR_CANDS (candidates)
  uint32_t pad;
};
struct ShardCand {
  uint32_t e_bits;  // exact exp (sampling.rs:127)
  uint32_t col;     // column in the whole row
};
static_assert(sizeof(ShardRec) == 32 && sizeof(ShardCand) == 8, "records are exchanged as raw bytes");

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

// Logit element types of the kernels: float (PESTI_F32), uint16_t (the bits
// of a bf16, PESTI_BF16) and __half (PESTI_F16).  Every one widens to f32
// exactly, which is what the reference's &[f32] would hold.
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

template <typename TIn>
__device__ __forceinline__ float load_logit(const TIn* row, long long j);
template <>
__device__ __forceinline__ float load_logit<float>(const float* row, long long j) { return __ldg(row + j); }
template <>
__device__ __forceinline__ float load_logit<uint16_t>(const uint16_t* row, long long j) {
  return bf16_bits_to_f32(__ldg(row + j));
}
template <>
__device__ __forceinline__ float load_logit<__half>(const __half* row, long long j) {
  return f16_bits_to_f32(__ldg(reinterpret_cast<const unsigned short*>(row) + j));
}
__device__ __forceinline__ float load_logit_dyn(const void* row, int dtype, long long j) {
  return dtype == PESTI_BF16  ? load_logit<uint16_t>((const uint16_t*)row, j)
         : dtype == PESTI_F16 ? load_logit<__half>((const __half*)row, j)
                              : load_logit<float>((const float*)row, j);
}
// The two 16-bit logits of a 32-bit word (the lower address first), widened.
template <typename TIn>
__device__ __forceinline__ void unpack2(uint32_t w, float& lo, float& hi);
template <>
__device__ __forceinline__ void unpack2<uint16_t>(uint32_t w, float& lo, float& hi) {
  lo = __uint_as_float(w << 16);
  hi = __uint_as_float(w & 0xffff0000u);
}
template <>
__device__ __forceinline__ void unpack2<__half>(uint32_t w, float& lo, float& hi) {
  lo = f16_bits_to_f32((uint16_t)(w & 0xffffu));
  hi = f16_bits_to_f32((uint16_t)(w >> 16));
}
template <>
__device__ __forceinline__ void unpack2<float>(uint32_t, float& lo, float& hi) {  // never called
  lo = hi = 0.0f;
}

// Order-preserving u32 key of a float (for selection over signed values).
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = fbits(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  return bitsf((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// 2^x by the hardware approximation (ex2.approx.ftz.f32, relative error about
// 2^-22); used only for the approximate sums that steer the speculation.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// exp(z) for z <= 0 by the hardware 2^y, y = z log2 e with log2 e split in two
// floats (LH + LL, their sum within 3e-16 of it) and one rounding, so that
// |y - z log2 e| <= |z| log2 e 2^-24 (1 + 2^-23) and 2^y is within
// |z| 2^-24 * 1.0001 of exp(z).  Against the correctly rounded f32 exp (within
// 2^-24 of exp(z)) the relative error is below
// PESTI_EX2_APPROX_RELERR + (|z| + 1) 2^-24 * 1.001 whenever it is not 0; it is
// 0 only when exp(z) < 2^-126 (y below -126, where subnormal results flush).
// rint(t) for 0 <= t < 2^23 (round to nearest even, as rintf) and its
// integer k, by one float addition of 2^23: in [2^23, 2^24) the floats are
// the integers, and k is the distance of the sum's bits from 2^23's.  This
// keeps the rounding and the conversion off the special-function pipe.
__device__ __forceinline__ float rint_small(float t, uint32_t& k) {
  const float r = __fadd_rn(t, 0x1p23f);
  k = __float_as_uint(r) - 0x4b000000u;
  return __fsub_rn(r, 0x1p23f);
}

__device__ __forceinline__ float exp_hw(float z) {
  return ex2_approx(__fmaf_rn(z, 0x1.715476p+0f, __fmul_rn(z, 0x1.4ae0c0p-26f)));
}
// Twice that bound (the margin the decisions below keep), as DE_0 + |z| DE_Z.
// From the approximate argument z' = fl(x*rT - m) (rT = fl(1/T)) instead of
// the reference's z = fl(fl(x/T) - m), z' - z is within (|x*rT| + |z'|) 2^-23
// (1 + 2^-20), so exp_hw(z') is within DE_0/2 + DE_Z (|x*rT| + 1.5 |z'|) of
// exp(z) relative, and the decisions keep DE_0 + DE_Z * arg_margin.
constexpr float DE_Z = 0x1.01p-23f;  // >= 2 * 1.001 * 2^-24
constexpr float DE_0 = 2.0f * PESTI_EX2_APPROX_RELERR + DE_Z;
// (rT = 1 for unscaled rows, where fmaf(x, 1, -m) is exactly fl(x - m); the
// scaled rows' margin is valid, and larger, there too.)
__device__ __forceinline__ float arg_margin(float x, float rT, float zq) {
  return fmaf(2.0f, fabsf(x * rT), 3.0f * fabsf(zq));
}

// Programmatic dependent launch: a kernel lets the next one in the stream be
// scheduled early (launch_dependents) and the next one waits for the
// previous grid's completion and memory (wait) before it touches its inputs.
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch_next() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Out-of-line copy of the exact exp for the kernels whose code size matters.
__device__ __noinline__ float pesti_expf_call(float x) { return pesti_expf(x); }

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
// warp, and within a warp the calls run in row order.  g() runs after every
// chunk of U segments (and after every tail segment).
// ---------------------------------------------------------------------------
struct NoChunkHook {
  __device__ __forceinline__ void operator()() const {}
};

template <typename TIn, int VE, int U, bool VEC, typename F, typename G = NoChunkHook>
__device__ __forceinline__ void stream_subslice(const TIn* row, long long start, long long end, F&& f,
                                                G&& g = G()) {
  const int lane = threadIdx.x & 31;
  const long long CH = 32LL * VE * U;
  long long pos = start;
  if (VEC) {
    for (; pos + CH <= end; pos += CH, g()) {
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
          for (int q = 0; q < 4; ++q) unpack2<TIn>(wds[q], x[2 * q], x[2 * q + 1]);
        }
        f(x, pos + (long long)uu * 32 * VE + (long long)lane * VE, VE);
      }
    }
  }
  for (; pos < end; pos += 32LL * VE, g()) {
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
// Pass 1, the HBM pass, and the row prologue.
// ---------------------------------------------------------------------------
struct StatsShared {
  uint32_t hist[TAU_BINS];
  uint32_t hist2[256];  // the candidate threshold's second level
  float mraw[MAX_SUBS];
  float srel[MAX_SUBS];
  double dscr[34];
  float fscr[34];
  long long lscr[34];
  uint32_t uscr[34];
  int iscr[34];
  int match[MAX_MATCH];
  int nmatch;
  float tau;
  uint32_t tbin, tabove;  // the candidate threshold's 12-bit bin and the count above it
  int last;
};

// Candidate threshold: a lower bound of the k-th largest raw logit among the
// call's columns, from the segment maxima (maxima of disjoint segments are
// distinct elements): the k-th largest segment max rounded down to the start
// of its 20-bit key bin (a 12-bit histogram, then 8 more bits inside the bin
// that holds it); -inf when there are fewer than k segments.  Every thread of
// the block calls it.
template <int SEG_REG>
__device__ float kth_lower_bound(const SliceArgs& a, const float* segm, const float (&segr)[SEG_REG],
                                 bool seg_in_regs, long long keff, StatsShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31;
  const float NEG_INF = -__int_as_float(0x7f800000);
  for (int i = tid; i < TAU_BINS; i += K1_NT) sh.hist[i] = 0u;
  for (int i = tid; i < 256; i += K1_NT) sh.hist2[i] = 0u;
  if (tid == 0) {
    sh.tau = NEG_INF;
    sh.tbin = 0xffffffffu;
  }
  __syncthreads();
  auto add = [&](float v) {  // -inf (also padding) and NaN are not counted
    const bool ok = !is_nan(v) && v > NEG_INF;
    const uint32_t d = ok ? (fkey(v) >> 20) : (uint32_t)(TAU_BINS + lane);
    const uint32_t peers = __match_any_sync(PESTI_FULL_MASK, d);
    if (ok && (peers & ((1u << lane) - 1u)) == 0u) atomicAdd(&sh.hist[d], (uint32_t)__popc(peers));
  };
  if (seg_in_regs) {
#pragma unroll
    for (int r = 0; r < SEG_REG; ++r) add(segr[r]);
  } else {
    for (long long j0 = 0; j0 < a.nseg; j0 += K1_NT) {
      const long long j = j0 + tid;
      add(j < a.nseg ? segm[j] : NEG_INF);
    }
  }
  __syncthreads();
  constexpr int BPT = TAU_BINS / K1_NT;  // top-down: thread t owns bins [4096-16(t+1), 4096-16t)
  uint32_t loc = 0;
#pragma unroll
  for (int q = 0; q < BPT; ++q)  // in an order rotated by the thread: 2-way bank conflicts, not 16
    loc += sh.hist[TAU_BINS - 1 - BPT * tid - ((q + tid) & (BPT - 1))];
  uint32_t tot;
  const uint32_t ex = block_excl_scan_add(loc, sh.uscr, tot);  // ends with a barrier
  if ((long long)ex < keff && (long long)(ex + loc) >= keff) {
    uint32_t cum = ex;
    for (int q = 0; q < BPT; ++q) {
      const int bin = TAU_BINS - 1 - BPT * tid - q;
      if ((long long)(cum + sh.hist[bin]) >= keff) {
        sh.tbin = (uint32_t)bin;
        sh.tabove = cum;
        break;
      }
      cum += sh.hist[bin];
    }
  }
  __syncthreads();
  const uint32_t tb = sh.tbin;
  if (tb == 0xffffffffu) return NEG_INF;  // fewer than k segments
  // the second level: 8 more key bits of the segment maxima inside bin tb
  auto add2 = [&](float v) {
    const bool ok = !is_nan(v) && v > NEG_INF && (fkey(v) >> 20) == tb;
    if (ok) atomicAdd(&sh.hist2[(fkey(v) >> 12) & 255u], 1u);
  };
  if (seg_in_regs) {
#pragma unroll
    for (int r = 0; r < SEG_REG; ++r) add2(segr[r]);
  } else {
    for (long long j = tid; j < a.nseg; j += K1_NT) add2(segm[j]);
  }
  __syncthreads();
  if (tid < 32) {  // top-down over the 256 sub-bins, 8 per lane
    uint32_t c8[8], lsum = 0u;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      c8[q] = sh.hist2[255 - (lane * 8 + q)];
      lsum += c8[q];
    }
    const uint32_t incl = warp_incl_scan_add(lsum) + sh.tabove;
    const uint32_t excl = incl - lsum;
    if ((long long)excl < keff && (long long)incl >= keff) {
      uint32_t cum = excl;
      int q = 0;
      for (; q < 7; ++q) {
        if ((long long)(cum + c8[q]) >= keff) break;
        cum += c8[q];
      }
      sh.tau = fkey_inv((tb << 20) | ((uint32_t)(255 - (lane * 8 + q)) << 12));
    }
  }
  __syncthreads();
  return sh.tau;
}

// Everything that needs every sub-slice of the row: run by the last block.
// Three forms:
//  - whole rows: the row prologue (RowInfo and the per-sub-slice SubPre);
//  - first phase of a vocabulary shard (a.shard_out): the shard's summary
//    (its max, flags, approximate mass, candidate threshold and, for greedy
//    rows, the columns of its max) instead;
//  - second phase (a.shard_all): the row prologue of this shard with the row
//    max, flags, candidate threshold and argmax taken over every shard's
//    summary, and the prefix mass and prefix max of every sub-slice starting
//    from those of the earlier shards.
template <typename TIn, int VE>
__device__ void row_prologue(const SliceArgs& a, long long b, StatsShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int nsub = a.P * K1_WARPS;
  const long long V = a.V;         // columns of this call (one shard's, when sharded)
  const long long VT = a.V_total;  // length of the whole row
  const bool summary = a.shard_out != nullptr;
  const bool sharded = a.shard_all != nullptr;
  const float NEG_INF = -__int_as_float(0x7f800000), INF = __int_as_float(0x7f800000);
  const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
  const float T = prm.temperature;
  const bool scale = T > 0.0f;
  const float t_eff = scale ? T : 1.0f;
  const SubStat* st = a.stats + b * nsub;
  // the table of the exact exp that one thread takes at the end (the
  // candidate threshold's) is brought into this SM's L1 now
  if (tid < 4) {
    const char* tab = reinterpret_cast<const char*>(tid < 2 ? pesti_exp_t_hi_d : pesti_exp_t_lo_d);
    asm volatile("prefetch.global.L1 [%0];" ::"l"(tab + (tid & 1) * 128));
  }
  // the segment maxima (for the candidate threshold) are fetched now, while
  // the sub-slice statistics are combined
  constexpr int SEG_REG = 4;
  const float* segm = a.seg_max + b * a.nseg;
  const bool seg_in_regs = a.nseg <= (long long)SEG_REG * K1_NT;
  float segr[SEG_REG];
#pragma unroll
  for (int r = 0; r < SEG_REG; ++r) {
    const long long j = (long long)r * K1_NT + tid;
    segr[r] = !sharded && seg_in_regs && j < a.nseg ? segm[j] : NEG_INF;
  }
  float mx = NEG_INF;
  int ln = -1;
  int f = 0;
  constexpr int PERS = MAX_SUBS / K1_NT;
#pragma unroll
  for (int r = 0; r < PERS; ++r) {
    const int s = r * K1_NT + tid;
    const bool has = s < nsub && (long long)s * a.SL < V;
    float mr = NEG_INF, sr = 0.0f;
    if (has) {
      const SubStat x = st[s];
      mr = x.max_raw;
      sr = x.sum_rel;
      mx = fmaxf(mx, mr);
      ln = ln > x.last_nan ? ln : x.last_nan;
      f |= (int)x.flags;
    }
    sh.mraw[s] = mr;
    sh.srel[s] = sr;
  }
  // row max, last NaN and flags in one reduction
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(PESTI_FULL_MASK, mx, o));
    const int lo2 = __shfl_xor_sync(PESTI_FULL_MASK, ln, o);
    ln = ln > lo2 ? ln : lo2;
    f |= __shfl_xor_sync(PESTI_FULL_MASK, f, o);
  }
  if (lane == 0) {
    sh.fscr[w] = mx;
    sh.iscr[w] = f;
    sh.lscr[w] = ln;
  }
  __syncthreads();
  int fl = 0;
  for (int q = 0; q < K1_WARPS; ++q) {
    mx = fmaxf(mx, sh.fscr[q]);
    fl |= sh.iscr[q];
    ln = ln > (int)sh.lscr[q] ? ln : (int)sh.lscr[q];
  }
  __syncthreads();
  long long li = -1, fi = 1LL << 62;
  long long lnl = ln;   // last NaN (row index)
  double ex0 = 0.0;     // approximate mass of the earlier shards
  float pmax0 = NEG_INF;  // their max
  float tau_all = INF;    // the candidate threshold over every shard
  if (sharded) {
    // combine the shards' summaries (each thread reads all of them)
    const float c2 = 1.4426950408889634f / t_eff;
    float gmx = NEG_INF, tmax = NEG_INF;
    uint32_t gfl = 0u;
    lnl = -1;
    for (int r = 0; r < a.shard_G; ++r) {
      const ShardSum q = a.shard_all[(long long)r * a.B + b];
      gmx = fmaxf(gmx, q.max_raw);
      gfl |= q.flags;
      tmax = fmaxf(tmax, q.tau);
      if (q.last_nan >= 0) lnl = (long long)r * V + q.last_nan;
    }
    for (int r = 0; r < a.shard_G; ++r) {
      const ShardSum q = a.shard_all[(long long)r * a.B + b];
      if (q.max_raw == gmx) {  // greedy rows: the columns of the row max
        if (q.first_max >= 0 && fi == (1LL << 62)) fi = (long long)r * V + q.first_max;
        if (q.last_max >= 0) li = (long long)r * V + q.last_max;
      }
      if (r < a.shard_rank) {
        pmax0 = fmaxf(pmax0, q.max_raw);
        if (q.max_raw > NEG_INF) ex0 += exp2((double)(q.max_raw * c2) - (double)(gmx * c2)) * q.mass;
      }
    }
    mx = gmx;
    fl = (int)gfl;
    tau_all = tmax;
  } else if (is_greedy(prm)) {
    // first and last index holding the row max: re-scan only the segments
    // whose max it is (usually one)
    if (tid == 0) sh.nmatch = 0;
    __syncthreads();
    for (long long j = tid; j < a.nseg; j += K1_NT) {
      if (segm[j] == mx) {
        const int slot = atomicAdd(&sh.nmatch, 1);
        if (slot < MAX_MATCH) sh.match[slot] = (int)j;
      }
    }
    __syncthreads();
    const int nmatch = sh.nmatch;
    const TIn* row = (const TIn*)a.logits + b * a.ld;
    if (nmatch <= MAX_MATCH) {
      for (int q = 0; q < nmatch; ++q) {
        const long long p = (long long)sh.match[q] * (32LL * VE) + tid;
        if (tid < 32 * VE && p < V && load_logit<TIn>(row, p) == mx) {
          li = li > p ? li : p;
          fi = fi < p ? fi : p;
        }
      }
    } else {  // many segments share the max (e.g. a constant row): scan the row
      for (long long p = tid; p < V; p += K1_NT) {
        if (load_logit<TIn>(row, p) == mx) {
          li = li > p ? li : p;
          fi = fi < p ? fi : p;
        }
      }
    }
    li = block_reduce_max(li, sh.lscr);
    fi = block_reduce_min(fi, sh.lscr);
  }
  const long long k = (long long)prm.top_k;
  const long long keff = k < VT ? k : VT;
  if (summary) {
    // the shard's approximate mass relative to its own max, and its candidate threshold
    const float c2 = 1.4426950408889634f / t_eff;
    const float ym = mx * c2;
    constexpr int PER = MAX_SUBS / K1_NT;
    double lsum = 0.0;
#pragma unroll
    for (int r = 0; r < PER; ++r) {
      const float mm = sh.mraw[tid * PER + r];
      lsum += mm > NEG_INF ? (double)exp2f(mm * c2 - ym) * (double)sh.srel[tid * PER + r] : 0.0;
    }
    const double mass = block_reduce_add(lsum, sh.dscr);
    float tau = INF;
    if (!is_greedy(prm) && fast_topk(prm, VT)) tau = kth_lower_bound<SEG_REG>(a, segm, segr, seg_in_regs, keff, sh);
    if (tid == 0) {
      ShardSum q;
      q.max_raw = mx;
      q.flags = (uint32_t)fl;
      q.tau = tau;
      q.last_nan = ln;
      q.mass = mass;
      q.last_max = li;
      q.first_max = fi < (1LL << 62) ? fi : -1;
      a.shard_out[b] = q;
    }
    return;
  }
  const float m = scale ? fdiv(mx, T) : mx;  // sampling.rs:46 on the max element
  const bool uniform = (fl & MF_NAN) || (scale && T == INF && (fl & (MF_POSINF | MF_NEGINF))) ||
                       !(fabsf(m) < INF) || VT <= 0;
  const bool need_pre = !is_greedy(prm) && !uniform;
  // with at most 32*PER sub-slices only warp 0 holds any: it computes the
  // prefix alone (the same values, without block barriers), and the other
  // warps go on to the candidate threshold
  const bool warp0_only = nsub <= 32 * (MAX_SUBS / K1_NT);
  if (need_pre && (!warp0_only || w == 0)) {
    // exclusive prefix of the approximate softmax mass and of the max, per sub-slice
    const float c2 = 1.4426950408889634f / t_eff;
    const float ym = mx * c2;
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
    double ex = ex0 + (warp0_only ? warp_incl_scan_add(lsum) - lsum : block_excl_scan_add(lsum, sh.dscr, dt));
    float inc = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(PESTI_FULL_MASK, inc, o);
      if (lane >= o) inc = fmaxf(inc, y);
    }
    float wpre = pmax0;
    if (!warp0_only) {
      if (lane == 31) sh.fscr[w] = inc;
      __syncthreads();
      for (int q = 0; q < w; ++q) wpre = fmaxf(wpre, sh.fscr[q]);
    }
    float exc = __shfl_up_sync(PESTI_FULL_MASK, inc, 1);
    if (lane == 0) exc = NEG_INF;
    float pmax = fmaxf(wpre, exc);
    // bound (b) of the survivor pass, in raw units: with
    // L = A (1 - V 2^-24)(1 - 2^-10) 2^-(2^-20 (|y_max| + 64)) <= the running
    // sum (A was built from float products raw*c2 whose rounding grows with
    // |y|), t = m + ln(L) - 17.36 and eta = 2^-20 (|t| + |m| + 1),
    // x < (t - eta) T implies fl(fl(x/T) - m) < t - m - eta/2 (the roundings
    // of x/T and of the difference are below eta/8), so the exact exp is below
    // e^-17.36 L (1 + 2^-24) < 0.99 * 2^-25 L.  Rounded toward -inf.
    const bool sum_ok = sum_pruning_ok(prm);
    const double lfac = (1.0 - (double)VT * 0x1p-24) * (1.0 - 0x1p-10) * exp2(-0x1p-20 * ((double)fabsf(ym) + 64.0));
#pragma unroll
    for (int r = 0; r < PER; ++r) {
      const int s = tid * PER + r;
      if (s < nsub) {
        SubPre p;
        p.A = ex;
        p.P = pmax;
        p.thrL = -INF;
        const double L = ex * lfac;
        if (sum_ok && L >= 0x1p-60) {
          const double tL = (double)m + log(L) - 17.36;
          const double eta = 0x1p-20 * (fabs(tL) + fabs((double)m) + 1.0);
          p.thrL = __double2float_rd((tL - eta) * (double)t_eff);
        }
        a.pre[b * nsub + s] = p;
      }
      ex += loc[r];
      pmax = fmaxf(pmax, lmx[r]);
    }
  }
  float tau = INF;
  if (need_pre && fast_topk(prm, VT))
    tau = sharded ? tau_all : kth_lower_bound<SEG_REG>(a, segm, segr, seg_in_regs, keff, sh);
  if (tid == 0) {
    RowInfo ri;
    ri.max_raw = mx;
    ri.m = m;
    ri.tau = tau;
    ri.flags = (uint32_t)fl;
    ri.last_max = li;
    ri.first_max = fi < (1LL << 62) ? fi : -1;
    ri.last_nan = lnl;
    ri.uniform = uniform ? 1 : 0;
    ri.e_tau = tau > NEG_INF && tau < INF ? pesti_expf_call(fsub(scale ? fdiv(tau, T) : tau, m)) : 0.0f;
    ri.s_start = (float)ex0;
    ri.S = 0.0f;
    ri.min_raw = 0.0f;
    a.info[b] = ri;
  }
}

template <typename TIn, int VE, int U, bool VEC>
__global__ void __launch_bounds__(K1_NT) slice_stats_kernel(SliceArgs a) {
  __shared__ StatsShared sh;
  grid_dep_launch_next();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const long long b = blockIdx.x / a.P;
  const int slice = (int)(blockIdx.x % a.P);
  const long long sub = (long long)slice * K1_WARPS + w;
  const long long start = sub * a.SL;
  long long end = start + a.SL;
  if (end > a.V) end = a.V;
  if (slice == 0 && w == 0 && lane == 0) {
    a.cand_count[b] = 0;
    a.pool_ctr[b] = 0;
    if (b == 0) {
      *a.item_next = 0;
      *a.task_count = 0;
      *a.task_next = 0;
      *a.task_count_h = 0;
    }
  }
  const TIn* row = (const TIn*)a.logits + b * a.ld;
  const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
  const float c2 = 1.4426950408889634f / (prm.temperature > 0.0f ? prm.temperature : 1.0f);
  const float NEG_INF = -__int_as_float(0x7f800000), INF = __int_as_float(0x7f800000);
  int last_nan = -1;
  uint32_t flags = 0;
  uint32_t sub_key = fkey(NEG_INF);     // max over the sub-slice, as an ordered key
  float run_m = NEG_INF, run_s = 0.0f;  // online partial sum, log2 units (per lane; fused: of the warp)
  float* segmax = a.seg_max + b * a.nseg;
  stream_subslice<TIn, VE, U, VEC>(row, start, end, [&](const float* x, long long pos0, int nv) {
    float lm = NEG_INF;
    bool odd = false;
#pragma unroll
    for (int e = 0; e < VE; ++e) {
      if (e < nv) {
        lm = fmaxf(lm, x[e]);  // fmaxf skips NaN, as f32::max does
        odd |= !(fabsf(x[e]) < INF);
      }
    }
    if (odd) {  // NaN or +-inf: rare
#pragma unroll
      for (int e = 0; e < VE; ++e) {
        if (e >= nv) continue;
        if (is_nan(x[e])) {
          last_nan = (int)(pos0 + e);
          flags |= MF_NAN;
        } else if (!(fabsf(x[e]) < INF)) {
          flags |= x[e] > 0.0f ? MF_POSINF : MF_NEGINF;
        }
      }
    }
    const long long seg = (pos0 - (long long)lane * VE) / (32LL * VE);
    const uint32_t sk = __reduce_max_sync(PESTI_FULL_MASK, fkey(lm));
    // approximate partial softmax sum (steers the fold speculation only)
    if (a.fused) {
      // warp-uniform running sum of the sub-slice, recorded at every unit start
      constexpr int SPU = UNIT / (32 * VE);  // segments per unit
      if (seg % SPU == 0 && lane == 0)
        a.unit_pre[b * ((a.V + UNIT - 1) / UNIT) + seg / SPU] = UnitPre{run_s, run_m, fkey_inv(sub_key), 0.0f};
      const float smax = fkey_inv(sk);
      if (smax > NEG_INF) {
        const float sc = smax * c2;
        float ls = 0.0f;
#pragma unroll
        for (int e = 0; e < VE; ++e)
          if (e < nv && !is_nan(x[e])) ls += ex2_approx(fmaf(x[e], c2, -sc));
        ls = warp_reduce_add(ls);
        const float nm = fmaxf(run_m, sc);
        run_s = (run_m > NEG_INF ? run_s * ex2_approx(run_m - nm) : 0.0f) + ls * ex2_approx(sc - nm);
        run_m = nm;
      }
    } else {
      // per lane, combined at the end
      const float nm = fmaxf(run_m, lm * c2);
      if (nm > NEG_INF) {
        float acc = run_s * ex2_approx(run_m - nm);
#pragma unroll
        for (int e = 0; e < VE; ++e)
          if (e < nv && !is_nan(x[e])) acc += ex2_approx(fmaf(x[e], c2, -nm));
        run_s = acc;
        run_m = nm;
      }
    }
    sub_key = sk > sub_key ? sk : sub_key;
    if (lane == 0) segmax[seg] = fkey_inv(sk);
  });
  const float mx = fkey_inv(sub_key);
  const int ln = (int)__reduce_max_sync(PESTI_FULL_MASK, (unsigned)(last_nan + 1)) - 1;
  const uint32_t fl = __reduce_or_sync(PESTI_FULL_MASK, flags);
  float ws = run_s;  // fused: already the warp's
  if (!a.fused) {
    const float wm = warp_reduce_fmax(run_m);
    ws = (run_m > NEG_INF && wm > NEG_INF) ? run_s * ex2_approx(run_m - wm) : 0.0f;
    ws = warp_reduce_add(ws);
  }
  if (lane == 0) {
    SubStat m;
    m.max_raw = mx;
    m.sum_rel = ws;  // relative to 2^(mx*c2) (the warp's max of run_m == mx*c2: the same float product)
    m.last_nan = ln;
    m.flags = fl;
    a.stats[b * (long long)a.P * K1_WARPS + sub] = m;
  }
  // the last block of the row to finish computes the row prologue (no waiting:
  // the other blocks simply exit)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(&a.row_ctr[b], 1);
    sh.last = prev == a.P - 1;
  }
  __syncthreads();
  if (!sh.last) return;
  __threadfence();
  row_prologue<TIn, VE>(a, b, sh);
  if (threadIdx.x == 0) a.row_ctr[b] = 0;
}

// Second phase of a vocabulary shard: the row prologue of the shard once the
// summaries of every shard are in a.shard_all (one block per row).
template <typename TIn, int VE>
__global__ void __launch_bounds__(K1_NT) shard_prologue_kernel(SliceArgs a) {
  __shared__ StatsShared sh;
  grid_dep_launch_next();
  row_prologue<TIn, VE>(a, (long long)blockIdx.x, sh);
}

// ---------------------------------------------------------------------------
// Pass 2: survivors, fold entries, top-k candidates.
//
// Which elements may be dropped (x_i = raw_i/T is the scaled logit):
//  (a) prefix max: an EARLIER element j with x_j >= x_i + 17.34 gives
//      e_i <= 0.989*2^-25*e_j; the running softmax sum s_{i-1} >= e_j and
//      ulp(s)/2 > s*2^-25, so fl(s + e_i) returns s.  The same ratio makes i a
//      no-op in the sorted folds (they start at p_max >= p_j) and in the
//      index-order folds of p and q.  Tested on raw values as
//      raw_i < P - (17.35*T*(1+2^-20) + 2^-21*|P|), P = the max of the row
//      before the element's segment; the slack covers the rounding of raw/T,
//      of x - m (<= 2^-24*104 wherever exp is not 0) and of exp.  Used while
//      P/T >= m - 60.
//  (b) running sum: each step of a fold of non-negative terms has relative
//      error <= 2^-24, so s_{i-1} >= (sum_{j<i} e_j)*(1 - V*2^-24).  With the
//      approximate prefix mass A of the earlier sub-slices (pass 1, margin
//      for its own error), L <= s_{i-1}, and e_i < 0.99*2^-25*L makes i a
//      no-op in the index-order folds (also for p = e/S and q = p/total,
//      whose running sums are bounded the same way).  It does NOT bound the
//      sorted folds, so it is used only for top-k rows (whose kept list is
//      explicit and checked) and unfiltered rows (index order only).
//
// Fold entries: the survivors of a sub-slice, in row order, are classified
// against an approximate running sum (A plus the sum of the earlier
// survivors).  An element that is large next to the state (>= half its
// binade's bottom) or may carry the state across a binade edge (within a
// relative 2^-10 of it) is SPECIAL: the row kernel adds it with a real f32
// add.  Maximal runs of the others in one binade become one entry holding the
// run's integer increments for an even and an odd entry state.  An increment
// is e/w rounded to an integer; it is taken from an approximation of e
// (exp_hw, with its error bound) whenever e/w is farther than that bound
// from a rounding boundary, and from the exact exp otherwise.  The row kernel
// checks every run against the exact state (right binade at entry, still
// inside it at exit) and replays the run element by element when the check
// fails, so the classification never decides a result.
// ---------------------------------------------------------------------------
constexpr uint32_t KEY_NONE = 0xfffffffeu;  // no open run
static_assert(QCAP >= 32 + 256, "a chunk may add 256 survivors to a queue holding up to 31");

// The open run of a group's fold while its survivors are classified: the
// composed increments, how many survivors it covers, and its binade
// (KEY_NONE when there is no open run).
struct Seg {
  uint32_t a0, a1, cnt, key;
};
// Segmented composition: `b` follows `a`; a flagged `b` starts a new run.
__device__ __forceinline__ Seg seg_join(Seg a, Seg b, bool b_starts) {
  if (b_starts) return b;
  const Tr t = tr_compose(Tr{a.a0, a.a1}, Tr{b.a0, b.a1});
  return Seg{t.a0, t.a1, a.cnt + b.cnt, a.key};
}
__device__ __forceinline__ Seg seg_shfl_up(Seg s, int off) {
  return Seg{__shfl_up_sync(PESTI_FULL_MASK, s.a0, off), __shfl_up_sync(PESTI_FULL_MASK, s.a1, off),
             __shfl_up_sync(PESTI_FULL_MASK, s.cnt, off), __shfl_up_sync(PESTI_FULL_MASK, s.key, off)};
}
__device__ __forceinline__ Seg seg_shfl(Seg s, int src) {
  return Seg{__shfl_sync(PESTI_FULL_MASK, s.a0, src), __shfl_sync(PESTI_FULL_MASK, s.a1, src),
             __shfl_sync(PESTI_FULL_MASK, s.cnt, src), __shfl_sync(PESTI_FULL_MASK, s.key, src)};
}

constexpr int K1_STAGES = 4;  // 16-byte loads in flight per lane in the survivor pass

constexpr int K1_LOADS = 2;  // 16-byte loads per lane per chunk of the survivor pass

struct SurvShared {
  float4 stage[K1_WARPS][K1_STAGES][K1_LOADS][32];  // chunks on their way from L2 (cp.async)
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One warp per sub-slice (with the fused pass: of a row NOT on the fast
// path).  The sub-slice is read from L2 in 32*VE-element
// chunks (one 16-byte load per lane) with K1_STAGES chunks in flight; every
// element either provably leaves every fold unchanged (derivation above) or
// survives, and survivors are stored (raw logit and index) in row order at the
// sub-slice's start.  For rows of the fast path the sub-slice then becomes
// ceil(count / GROUP) classification tasks; their candidates for the top-k are
// taken from the survivors by the classification pass whenever tau lies above
// every threshold the sub-slice can use (SubSurv::cand_here = 0), else here.
template <typename TIn, int VE, bool VEC>
__global__ void __launch_bounds__(K1_NT, 4) survivor_kernel(SliceArgs a) {
  __shared__ __align__(16) SurvShared sh;
  grid_dep_launch_next();
  grid_dep_wait();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const long long b = blockIdx.x / a.P;
  const int slice = (int)(blockIdx.x % a.P);
  const int nsub = a.P * K1_WARPS;
  const long long sub = (long long)slice * K1_WARPS + w;
  const long long V = a.V;
  const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
  const RowInfo ri = a.info[b];
  const float T = prm.temperature;
  const bool scale = T > 0.0f;
  const float t_eff = scale ? T : 1.0f;
  const float NEG_INF = -__int_as_float(0x7f800000);
  SubSurv* so = a.surv + b * nsub + sub;
  // with the fused pass, the rows of the fast path are its alone
  if (a.fused && a.fast_enabled && fast_topk(prm, a.V_total) && !is_greedy(prm) && !ri.uniform) return;
  if (is_greedy(prm) || ri.uniform) {
    if (lane == 0) *so = SubSurv{0, 0, 0, NEG_INF};
    return;
  }
  const float m = ri.m;
  const float tau = ri.tau;
  const SubPre pr = a.pre[b * nsub + sub];
  const long long start = sub * a.SL;
  long long end = start + a.SL;
  if (end > V) end = V;
  const TIn* row = (const TIn*)a.logits + b * a.ld;
  float* sraw = a.surv_raw + b * V + start;
  uint32_t* sidx = a.surv_idx + b * V + start;
  const float c1 = ABSORB * t_eff * (1.0f + 0x1p-20f);
  const float pf = (m - PRUNE_FLOOR) * t_eff;
  const float p_floor = pf + 0x1p-20f * fabsf(pf);
  const float thrLr = pr.thrL;  // bound (b), from the row prologue
  auto bound_a = [&](float P) { return P >= p_floor ? fsub(P, fadd(c1, 0x1p-21f * fabsf(P))) : NEG_INF; };
  // bound (a) uses the max of the row before each chunk: the maxima of the
  // earlier sub-slices, then this sub-slice's segment maxima from the first pass
  const float* segm = a.seg_max + b * a.nseg + start / (32LL * VE);
  float run_max = pr.P;
  float pruned_max = NEG_INF;
  const bool fast = a.fast_enabled && fast_topk(prm, a.V_total);
  // the largest threshold any chunk can use is that of the row max: with tau
  // above it every candidate (raw >= tau) survives
  const bool cand_here = fast && !(tau >= fmaxf(bound_a(ri.max_raw), thrLr));
  int* ccount = a.cand_count + b;
  float4* stg = &sh.stage[w][0][0][0];
  long long sins = 0;  // survivors stored so far

  // a chunk is K1_LOADS segments of 32*VE elements, one 16-byte load per lane
  // each; segment q of chunk c starts at c*CHV + q*SEG, lane l holds its
  // elements l*VE .. l*VE + VE-1
  constexpr int SEG = 32 * VE;
  constexpr int CHV = K1_LOADS * SEG;
  const int len = (int)(end - start);
  const int nchunk = (len + CHV - 1) / CHV;
  const int nfull = VEC ? len / CHV : 0;  // chunks read through the pipeline
  const TIn* rsub = row + start;
  if (VEC) {
#pragma unroll
    for (int st = 0; st < K1_STAGES; ++st) {
      if (st < nfull)
#pragma unroll
        for (int q = 0; q < K1_LOADS; ++q) cp_async16(&stg[(st * K1_LOADS + q) * 32 + lane], rsub + st * CHV + q * SEG + lane * VE);
      cp_async_commit();
    }
  }
  float segv = NEG_INF;  // segment maxima of segments s0 + lane, 32 at a time
  uint32_t sins32 = 0u;  // survivors stored so far (< SL)
  for (int c = 0; c < nchunk; ++c) {
    if (((c * K1_LOADS) & 31) == 0) {
      const int s0 = c * K1_LOADS + lane;
      segv = s0 < (len + SEG - 1) / SEG ? segm[s0] : NEG_INF;
    }
    float x[K1_LOADS][VE];
    int nv[K1_LOADS];
    const bool piped = VEC && c < nfull;
    if (piped) {
      cp_async_wait<K1_STAGES - 1>();  // chunk c has arrived (each lane reads its own bytes)
#pragma unroll
      for (int q = 0; q < K1_LOADS; ++q) {
        const float4 r4 = stg[((c % K1_STAGES) * K1_LOADS + q) * 32 + lane];
        if (sizeof(TIn) == 4) {
          x[q][0] = r4.x; x[q][1] = r4.y; x[q][2] = r4.z; x[q][3] = r4.w;
        } else {
          const uint32_t wds[4] = {__float_as_uint(r4.x), __float_as_uint(r4.y), __float_as_uint(r4.z),
                                   __float_as_uint(r4.w)};
#pragma unroll
          for (int h = 0; h < 4; ++h) unpack2<TIn>(wds[h], x[q][2 * h], x[q][2 * h + 1]);
        }
        nv[q] = VE;
      }
    } else {
#pragma unroll
      for (int q = 0; q < K1_LOADS; ++q) {
        const int p0 = c * CHV + q * SEG + lane * VE;
        nv[q] = 0;
#pragma unroll
        for (int e = 0; e < VE; ++e) {
          x[q][e] = p0 + e < len ? load_logit<TIn>(rsub, p0 + e) : 0.0f;
          nv[q] = p0 + e < len ? e + 1 : nv[q];
        }
      }
    }
    // per segment one threshold for both bounds (NaN fails it): bound (a)
    // with the max of the row before the segment (exact), bound (b)
    bool sv[K1_LOADS][VE];
    uint32_t packed = 0u;
    float thr_lo = __int_as_float(0x7f800000);
#pragma unroll
    for (int q = 0; q < K1_LOADS; ++q) {
      const float thr = fmaxf(bound_a(run_max), thrLr);
      thr_lo = fminf(thr_lo, thr);
      run_max = fmaxf(run_max, __shfl_sync(PESTI_FULL_MASK, segv, (c * K1_LOADS + q) & 31));
      uint32_t n = 0u;
#pragma unroll
      for (int e = 0; e < VE; ++e) {
        sv[q][e] = e < nv[q] && x[q][e] >= thr;
        n += sv[q][e] ? 1u : 0u;
      }
      packed |= n << (16 * q);
    }
    static_assert(K1_LOADS == 2, "segment counts are packed in 16-bit halves");
    // survivors are stored in row order (segment by segment, lane by lane)
    const uint32_t incl = warp_incl_scan_add(packed);
    const uint32_t tot = __shfl_sync(PESTI_FULL_MASK, incl, 31);
    const uint32_t excl = incl - packed;
#pragma unroll
    for (int q = 0; q < K1_LOADS; ++q) {
      uint32_t o = sins32 + ((excl >> (16 * q)) & 0xffffu) + (q == 1 ? (tot & 0xffffu) : 0u);
      const uint32_t p0 = (uint32_t)(start + c * CHV + q * SEG + lane * VE);
#pragma unroll
      for (int e = 0; e < VE; ++e) {
        if (sv[q][e]) {
          sraw[o] = x[q][e];
          sidx[o] = p0 + (uint32_t)e;
          ++o;
        }
      }
    }
    sins32 += (tot & 0xffffu) + (tot >> 16);
    if (!fast) {  // the largest dropped logit (fmaxf skips NaN)
#pragma unroll
      for (int q = 0; q < K1_LOADS; ++q)
#pragma unroll
        for (int e = 0; e < VE; ++e)
          if (e < nv[q] && !sv[q][e]) pruned_max = fmaxf(pruned_max, x[q][e]);
    }
    if (cand_here) {  // top-k candidates (their exact exps are taken by the row kernel)
#pragma unroll
      for (int q = 0; q < K1_LOADS; ++q) {
        int ccnt = 0;
#pragma unroll
        for (int e = 0; e < VE; ++e) ccnt += (e < nv[q] && x[q][e] >= tau) ? 1 : 0;
        if (__any_sync(PESTI_FULL_MASK, ccnt > 0)) {
          const int cex0 = warp_incl_scan_add(ccnt);
          const int ctot = __shfl_sync(PESTI_FULL_MASK, cex0, 31);
          int basec = 0;
          if (lane == 0) basec = atomicAdd(ccount, ctot);
          basec = __shfl_sync(PESTI_FULL_MASK, basec, 0);
          int slot = basec + cex0 - ccnt;
          const uint32_t p0 = (uint32_t)(start + c * CHV + q * SEG + lane * VE);
#pragma unroll
          for (int e = 0; e < VE; ++e) {
            if (e < nv[q] && x[q][e] >= tau) {
              if (slot < CAND_CAP) {
                a.cand_e[b * CAND_CAP + slot] = pesti_expf_call(fsub(scale ? fdiv(x[q][e], T) : x[q][e], m));
                a.cand_idx[b * CAND_CAP + slot] = p0 + (uint32_t)e;
              }
              ++slot;
            }
          }
        }
      }
    }
    (void)thr_lo;
    if (piped) {  // the stage just read (its values are used above) takes chunk c + K1_STAGES
      const int cn = c + K1_STAGES;
      if (cn < nfull)
#pragma unroll
        for (int q = 0; q < K1_LOADS; ++q)
          cp_async16(&stg[((c % K1_STAGES) * K1_LOADS + q) * 32 + lane], rsub + cn * CHV + q * SEG + lane * VE);
      cp_async_commit();
    }
  }
  sins = sins32;
  if (VEC) cp_async_wait<0>();
  const float pm = warp_reduce_fmax(pruned_max);
  const int ngroups = fast ? (int)((sins + GROUP - 1) / GROUP) : 0;
  if (ngroups > 0 && lane == 0) {
    // a row's first sub-slice, where the running sum is small and most
    // elements need the general classification, has the slowest tasks: they
    // go to the top of the list, which the classification takes first
    const bool heavy = sub == 0;
    const long long cap = a.B * (long long)nsub * a.jmax;
    const int t0 = atomicAdd(heavy ? a.task_count_h : a.task_count, ngroups);
    for (int j = 0; j < ngroups; ++j)
      a.tasks[heavy ? cap - 1 - (t0 + j) : t0 + j] = ClassTask{(int)b, (int)(sub * a.jmax + j)};
  }
  if (lane == 0) *so = SubSurv{(int32_t)sins, ngroups, cand_here ? 0 : 1, pm};
}

// ---------------------------------------------------------------------------
// Classification of survivors into fold entries (rows of the fast path).
//
// A group is up to GROUP consecutive survivors of one sub-slice, classified
// against an approximate fold state at its first survivor.  Lane l takes
// survivors [l*g, l*g + g), g = ceil(n/32): one warp scan gives every element
// its approximate running state and a segmented scan over the lanes joins the
// runs that cross lane boundaries.  The per-element loops are kept rolled (the
// values wait in shared memory between the passes): this code runs out of
// instruction cache long before it runs out of issue slots.
// ---------------------------------------------------------------------------

struct ClassShared {
  float raw[K1_WARPS][GROUP];     // the group's survivors (raw logit, row index)
  uint32_t idx[K1_WARPS][GROUP];
  float ea[K1_WARPS][GROUP];
  uint32_t ck[K1_WARPS][GROUP];
  uint32_t c0[K1_WARPS][GROUP];
  uint32_t c1[K1_WARPS][GROUP];
};

// Group j of sub-slice `sub` of row b: n (1..GROUP) survivors in graw/gidx
// (this warp's shared arrays), s_approx the approximate fold state before the
// first of them.  Writes the group's GroupEnt and, unless it is one clean
// run, its entries in the row's pool; returns the group's approximate mass
// (the sum of the approximate exps).  try_clean = false skips the clean case
// (a caller that has tried it already).  All 32 lanes call it.
__device__ __forceinline__ float classify_group(const SliceArgs& a, long long b, long long sub, int j, int n,
                                            bool try_clean,
                                            double s_approx, bool scale, float T, float m, float* graw,
                                            uint32_t* gidx, float* eas, uint32_t* cks, uint32_t* c0s,
                                            uint32_t* c1s) {
  const int lane = threadIdx.x & 31;
  const int nsub = a.P * K1_WARPS;
  // e_exact lies within a relative DE of the approximation (twice its error
  // bound: margin for the float arithmetic of the bounds below); DE grows with
  // |z| (see exp_hw) and is set after pass A from the group's largest |z|
  float DE = 0.0f;
  // Guard band around binade edges (2^-12 for whole rows).  The approximate
  // state tracks the fold within about 1.2e-4 on a row of 128k (its bias is
  // the mass that the fold absorbs, and it grows along the row); a run
  // predicted in the wrong binade fails its check in the row kernel and is
  // replayed there, so the band trades entries for replays and never decides
  // a result.
  const float BAND = a.band;
  // element i of the group: its run key (binade or SPECIAL) and increments
  auto classify = [&](int i, float ea, float av, float bv, uint32_t& key, uint32_t& k0, uint32_t& k1) {
    uint32_t lo = 0u;
    bool special;
    const float eu = ea * (1.0f + DE);  // upper bound of the exact value
    if (av < 0x1p-126f) {
      special = eu >= 0x1p-127f || bv > 0x1p-126f * (1.0f - BAND);
    } else {
      lo = fbits(av) & 0x7f800000u;
      const float lov = bitsf(lo);
      special = eu >= bitsf(lo - 0x00800000u) || av < lov * (1.0f + BAND) || bv > 2.0f * lov * (1.0f - BAND);
    }
    bool need_exact = special;
    k0 = k1 = 0u;
    if (!special) {
      const uint32_t E = lo >> 23;  // w = 2^(E-150) (E = 0: the subnormal grid 2^-149)
      const int sh2 = 150 - (int)(E == 0u ? 1u : E);
      if (ea == 0.0f) {
        need_exact = E < 40u;  // exact e < 4.5e-38: rounds to 0 on any grid >= 2^-110
      } else {
        const float tt = __uint_as_float(fbits(ea) + ((uint32_t)sh2 << 23));  // ea/w, exact scaling
        uint32_t kq;
        const float kr = rint_small(tt, kq);
        const float slack = 0.5f - fabsf(tt - kr);
        if (!(tt < 0x1p22f) || slack <= tt * DE + 0x1p-24f) need_exact = true;
        else k0 = k1 = kq;
      }
    }
    if (need_exact) {
      const float raw = graw[i];
      const float ex = pesti_expf_call(fsub(scale ? fdiv(raw, T) : raw, m));  // sampling.rs:46,127, exact
      if (special) {
        k0 = fbits(ex);
      } else {
        k0 = fbits(fadd(bitsf(lo), ex)) - lo;
        k1 = fbits(fadd(bitsf(lo + 1u), ex)) - (lo + 1u);
      }
    }
    key = special ? fold::SPECIAL : lo;
  };

  const int g = (n + 31) >> 5;  // elements per lane: the group's fill decides the loop length
  const int i0 = lane * g;
  const int nl = n - i0 < 0 ? 0 : (n - i0 > g ? g : n - i0);  // valid elements of the lane
  __syncwarp();
  // approximate states as floats relative to the carried double (the guard
  // band is 2^-12; float rounding is 2^-24)
  const float sb = (float)s_approx;
  // A clean group: the whole range of its approximate states lies inside one
  // binade (within the guard band), so every element is a plain increment
  // k = rint(e/w) of one run (e < lo there, so k is in the binade's units).
  // k comes from the approximation where it decides it and from the exact
  // exp otherwise; unless some element is a tie (its k depends on the
  // parity of the state), the group's fold is that run with the sum of the
  // increments: one entry, no segmentation.  The binade is that of the
  // start, so the increments are formed in pass A itself, speculatively; the
  // group's end state decides, and only then are the exact exps of the
  // elements the approximation leaves undecided taken.
  uint32_t clo = 0u;
  bool possible = false;
  if (try_clean && sb >= 0x1p-126f) {
    clo = fbits(sb) & 0x7f800000u;
    possible = sb >= bitsf(clo) * (1.0f + BAND);
  }
  const int sh2 = 150 - (int)(clo >> 23);  // w = 2^(E-150) (E = 0: the subnormal grid 2^-149)
  uint32_t ksum = 0u, undecided = 0u;  // undecided: bit jj, element jj of the lane
  // pass A: approximate exps of the reference's arguments z = x/T - m
  // (sampling.rs:46,127), from the approximate argument x*rT - m: within
  // (DE_0 + arg_margin * DE_Z) / 2 of the exact exp
  const float rT = scale ? 1.0f / T : 1.0f;
  float ltot = 0.0f;
  float zmax = 0.0f;  // the largest arg_margin of the lane's elements with e > 0
#pragma unroll 1
  for (int jj = 0; jj < nl; ++jj) {
    const float raw = graw[i0 + jj];
    const float zq = fmaf(raw, rT, -m);
    const float e = exp_hw(zq);
    const float q = arg_margin(raw, rT, zq);
    eas[jj * 32 + lane] = e;
    ltot += e;
    if (e > 0.0f) zmax = fmaxf(zmax, q);
    if (possible) {
      bool exact;
      if (e == 0.0f) {
        exact = (clo >> 23) < 40u;  // else: exact e < 1.2e-38 rounds to 0 on this grid
      } else {
        const float tt = __uint_as_float(fbits(e) + ((uint32_t)sh2 << 23));  // e/w, exact scaling
        uint32_t kq;
        const float kr = rint_small(tt, kq);
        const float slack = 0.5f - fabsf(tt - kr);
        exact = !(tt < 0x1p22f && slack > tt * fmaf(q, DE_Z, DE_0) + 0x1p-24f);
        if (!exact) ksum += kq;
      }
      if (exact) undecided |= 1u << jj;
    }
  }
  // the group's margin (zmax >= 0: its bits order as unsigned integers)
  DE = fmaf(__uint_as_float(__reduce_max_sync(PESTI_FULL_MASK, __float_as_uint(zmax))), DE_Z, DE_0);
  const float lincl = warp_incl_scan_add(ltot);
  const float gtot = __shfl_sync(PESTI_FULL_MASK, lincl, 31);
  const float lbase = lincl - ltot;
  if (possible && sb + gtot <= 2.0f * bitsf(clo) * (1.0f - BAND)) {
    bool decided = true;
    for (uint32_t um = undecided; um != 0u; um &= um - 1u) {
      const int jj = __ffs(um) - 1;
      const float raw = graw[i0 + jj];
      const float ex = pesti_expf_call(fsub(scale ? fdiv(raw, T) : raw, m));  // sampling.rs:46,127, exact
      const uint32_t k0 = fbits(fadd(bitsf(clo), ex)) - clo;
      const uint32_t k1 = fbits(fadd(bitsf(clo + 1u), ex)) - (clo + 1u);
      decided = decided && k0 == k1;
      ksum += k0;
    }
    if (__all_sync(PESTI_FULL_MASK, decided)) {
      const uint32_t inc = tr_sat(warp_reduce_add(ksum));  // each < 2^22, at most 256 of them
      if (lane == 0)
        a.gsurv[(b * nsub + sub) * a.jmax + j] = GroupEnt{{clo, inc, inc, gidx[n - 1] + 1u}, 0, 1, 0, 1};
      return gtot;
    }
  }
  // the key of the lane's last element decides whether the next lane's first
  // element continues its run
  uint32_t last_key = KEY_NONE;
  if (nl > 0) {
    const float el = eas[(nl - 1) * 32 + lane];
    uint32_t k0, k1;
    classify(i0 + nl - 1, el, sb + (lbase + (ltot - el)), sb + (lbase + ltot), last_key, k0, k1);
  }
  uint32_t prev_key = __shfl_up_sync(PESTI_FULL_MASK, last_key, 1);
  if (lane == 0) prev_key = KEY_NONE;
  // pass B: lane summary; `lead` continues the run open before the lane,
  // `trail` is the run open after it (hh: the lane starts at least one run)
  bool hh = false;
  Seg lead{0u, 0u, 0u, KEY_NONE}, trail{0u, 0u, 0u, KEY_NONE};
  int n_int = 0;  // entries closed inside the lane after its first run start
  {
    uint32_t cur = prev_key;
    float runf = lbase;
#pragma unroll 1
    for (int jj = 0; jj < nl; ++jj) {
      const float ea = eas[jj * 32 + lane];
      const float av = sb + runf;
      runf += ea;
      uint32_t k, k0, k1;
      classify(i0 + jj, ea, av, sb + runf, k, k0, k1);
      cks[jj * 32 + lane] = k;
      c0s[jj * 32 + lane] = k0;
      c1s[jj * 32 + lane] = k1;
      const bool head = k == fold::SPECIAL || cur == fold::SPECIAL || cur == KEY_NONE || k != cur;
      if (head) {
        if (hh && trail.cnt > 0u) ++n_int;
        hh = true;
        if (k == fold::SPECIAL) {
          ++n_int;
          trail = Seg{0u, 0u, 0u, KEY_NONE};
        } else {
          trail = Seg{k0, k1, 1u, k};
        }
      } else if (!hh) {
        const Tr tt = tr_compose(Tr{lead.a0, lead.a1}, Tr{k0, k1});
        lead = Seg{tt.a0, tt.a1, lead.cnt + 1u, KEY_NONE};
      } else {
        const Tr tt = tr_compose(Tr{trail.a0, trail.a1}, Tr{k0, k1});
        trail = Seg{tt.a0, tt.a1, trail.cnt + 1u, trail.key};
      }
      cur = k;
    }
  }
  // segmented inclusive scan over the lanes
  Seg inc = hh ? trail : lead;
  bool fl = hh;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const Seg o = seg_shfl_up(inc, off);
    const bool of = __shfl_up_sync(PESTI_FULL_MASK, fl, off);
    if (lane >= off) {
      inc = seg_join(o, inc, fl);
      fl = fl || of;
    }
  }
  // the run open before the lane
  const Seg none{0u, 0u, 0u, KEY_NONE};
  Seg xin = seg_shfl_up(inc, 1);
  const bool xfl = __shfl_up_sync(PESTI_FULL_MASK, fl, 1);
  xin = lane == 0 ? none : seg_join(none, xin, xfl);
  const Seg last = seg_shfl(inc, 31);
  // entries, in row order: the run closed by the lane's first start, then
  // the ones closed inside the lane; the run still open at the group's end
  // closes it
  const Seg first = seg_join(xin, lead, false);
  const int ne = n_int + ((hh && first.cnt > 0u) ? 1 : 0);
  const int neincl = warp_incl_scan_add(ne);
  const int nclosed = __shfl_sync(PESTI_FULL_MASK, neincl, 31);
  const int netot = nclosed + (last.cnt > 0u ? 1 : 0);
  // the entries' place in the row's pool: one atomic, whose latency pass C
  // overlaps when the entries fit in the warp's approximate-exp array (no
  // longer read): pass C writes them there and they are copied once the
  // place is known
  constexpr int STAGED = GROUP * (int)sizeof(float) / (int)sizeof(FoldEnt);
  const bool staged = netot <= STAGED;
  int off0 = 0;
  if (lane == 0) off0 = atomicAdd(a.pool_ctr + b, netot);
  if (!staged) off0 = __shfl_sync(PESTI_FULL_MASK, off0, 0);
  const bool replay_known = !staged && off0 + netot > POOL_CAP;
  if (!replay_known) {
    FoldEnt* ent = staged ? reinterpret_cast<FoldEnt*>(eas) : a.pool + b * POOL_CAP + off0;
    __syncwarp();  // every lane is done reading eas
    int slot = neincl - ne;
    if (hh) {  // pass C: the same walk, writing the entries
      uint32_t cur = prev_key;
      bool started = false;
      Seg tr{0u, 0u, 0u, KEY_NONE};
      auto rend = [&](int i) { return gidx[i] + 1u; };  // past survivor i
#pragma unroll 1
      for (int jj = 0; jj < nl; ++jj) {
        const uint32_t k = cks[jj * 32 + lane], k0 = c0s[jj * 32 + lane], k1 = c1s[jj * 32 + lane];
        const bool head = k == fold::SPECIAL || cur == fold::SPECIAL || cur == KEY_NONE || k != cur;
        if (head) {
          if (!started) {
            if (first.cnt > 0u) ent[slot++] = FoldEnt{first.key, first.a0, first.a1, rend(i0 + jj - 1)};
            started = true;
          } else if (tr.cnt > 0u) {
            ent[slot++] = FoldEnt{tr.key, tr.a0, tr.a1, rend(i0 + jj - 1)};
          }
          if (k == fold::SPECIAL) {
            ent[slot++] = FoldEnt{fold::SPECIAL, k0, 0u, rend(i0 + jj)};
            tr = Seg{0u, 0u, 0u, KEY_NONE};
          } else {
            tr = Seg{k0, k1, 1u, k};
          }
        } else if (started) {
          const Tr tt = tr_compose(Tr{tr.a0, tr.a1}, Tr{k0, k1});
          tr = Seg{tt.a0, tt.a1, tr.cnt + 1u, tr.key};
        }
        cur = k;
      }
    }
    if (lane == 0 && last.cnt > 0u) ent[nclosed] = FoldEnt{last.key, last.a0, last.a1, gidx[n - 1] + 1u};
  }
  if (staged) {
    off0 = __shfl_sync(PESTI_FULL_MASK, off0, 0);
    __syncwarp();  // the staged entries of every lane are visible
    if (off0 + netot <= POOL_CAP) {
      const FoldEnt* sent = reinterpret_cast<const FoldEnt*>(eas);
      FoldEnt* ent = a.pool + b * POOL_CAP + off0;
      for (int e = lane; e < netot; e += 32) ent[e] = sent[e];
    }
  }
  const bool replay = off0 + netot > POOL_CAP;
  if (lane == 0)
    a.gsurv[(b * nsub + sub) * a.jmax + j] = GroupEnt{{0u, 0u, 0u, 0u}, off0, replay ? 0 : netot, replay ? 1 : 0, 0};
  return gtot;
}

// The task-queue classification (rows of the fast path when the fused pass
// is not used): each task is GROUP consecutive survivors of one sub-slice
// stored by the survivor pass.  Its approximate starting state is the
// sub-slice's prefix mass A plus the masses of the sub-slice's earlier
// survivors, so the tasks are independent and a persistent grid of warps
// takes them: each warp's first task is its own index (a burst of thousands
// of atomics on one counter would serialise the start), later ones come from
// the counter, claimed when a task is done (a claim made earlier would tie
// the next task to a warp whose current one runs long, while other warps
// idle).  The tasks of every row's first sub-slice, which cost the most, are
// taken first; then the others from the end of their list (the survivor pass
// queues the tasks of its slowest warps last).
__global__ void __launch_bounds__(K1_NT) classify_kernel(SliceArgs a) {
  __shared__ ClassShared sh;
  grid_dep_launch_next();
  grid_dep_wait();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int nsub = a.P * K1_WARPS;
  const long long V = a.V;
  const int nlow = *a.task_count, nhigh = *a.task_count_h;
  const int ntasks = nlow + nhigh;
  const long long cap = a.B * (long long)nsub * a.jmax;  // the list's slots
  auto task_at = [&](int i) { return i < nhigh ? a.tasks[cap - 1 - i] : a.tasks[nlow - 1 - (i - nhigh)]; };
  float* graw = sh.raw[w];
  uint32_t* gidx = sh.idx[w];
  const int nwarps = (int)gridDim.x * K1_WARPS;
  int t = (int)blockIdx.x * K1_WARPS + w;
  ClassTask tk_next = t < ntasks ? task_at(t) : ClassTask{0, 0};
  for (;;) {
    if (t >= ntasks) break;
    const ClassTask tk = tk_next;
    const long long b = tk.b;
    const long long sub = tk.qj / a.jmax;
    const int j = tk.qj - (int)sub * a.jmax;
    const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
    const RowInfo ri = a.info[b];
    const float T = prm.temperature;
    const bool scale = T > 0.0f;
    const float m = ri.m;
    const SubSurv ssv = a.surv[b * nsub + sub];
    const long long gbase = b * V + sub * a.SL + (long long)j * GROUP;  // first survivor of the group
    const int n = ssv.count - j * GROUP < GROUP ? ssv.count - j * GROUP : GROUP;
    const float* sraw = a.surv_raw + b * V + sub * a.SL;
    __syncwarp();  // the previous task is done with the shared arrays
#pragma unroll 8
    for (int i = lane; i < n; i += 32) {  // the group's survivors, in one coalesced pass
      graw[i] = a.surv_raw[gbase + i];
      gidx[i] = a.surv_idx[gbase + i];
    }
    // approximate state at the group's start: the prefix mass of the earlier
    // sub-slices plus that of the sub-slice's earlier survivors
    // (exp(x/T - m) = 2^(x c2 - m log2 e); a relative 2^-12 is all it needs)
    double s_approx = a.pre[b * nsub + sub].A;
    if (j > 0) {
      const float c2 = 1.4426950408889634f / (scale ? T : 1.0f);
      const float mc = m * 1.4426950408889634f;
      float acc = 0.0f;
#pragma unroll 8
      for (int i = lane; i < j * GROUP; i += 32) acc += ex2_approx(fmaf(sraw[i], c2, -mc));
      s_approx += (double)warp_reduce_add(acc);
    }
    __syncwarp();
    // the group's top-k candidates (all of them survived): counted first and
    // their slots reserved with one atomic, whose latency the classification
    // overlaps; written after it (the row kernel sorts the candidates, so
    // their order in the list is free)
    const float tau = ri.tau;
    int ccount = 0, cbase = 0;
    if (ssv.pad) {
      for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        ccount += __popc(__ballot_sync(PESTI_FULL_MASK, i < n && graw[i] >= tau));
      }
      if (ccount > 0 && lane == 0) cbase = atomicAdd(a.cand_count + b, ccount);
    }
    (void)classify_group(a, b, sub, j, n, true, s_approx, scale, T, m, graw, gidx, sh.ea[w], sh.ck[w], sh.c0[w],
                         sh.c1[w]);
    int claim = 0;
    if (lane == 0) claim = atomicAdd(a.task_next, 1);  // its latency overlaps the candidate writes
    if (ccount > 0) {
      int slot0 = __shfl_sync(PESTI_FULL_MASK, cbase, 0);
      for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        const float raw = i < n ? graw[i] : 0.0f;
        const bool cand = i < n && raw >= tau;
        const uint32_t bal = __ballot_sync(PESTI_FULL_MASK, cand);
        const int slot = slot0 + __popc(bal & ((1u << lane) - 1u));
        if (cand && slot < CAND_CAP) {
          a.cand_e[b * CAND_CAP + slot] = pesti_expf_call(fsub(scale ? fdiv(raw, T) : raw, m));  // sampling.rs:46,127
          a.cand_idx[b * CAND_CAP + slot] = gidx[i];
        }
        slot0 += __popc(bal);
      }
    }
    t = nwarps + __shfl_sync(PESTI_FULL_MASK, claim, 0);
    if (t < ntasks) tk_next = task_at(t);
  }
}

// The fused pass over the rows of the fast path: a persistent grid of warps
// takes items (each warp its own index first, then from a counter, claimed
// one item ahead): first every row's HEAD first units one at a time
// (where the running sum is small, most elements survive and the general
// classification is the rule, so they are spread over many warps), then
// items of RUN consecutive UNIT-element units of one row.  Per item: the approximate fold state at its first
// unit (the sub-slice's prefix mass plus the per-segment masses of the pass
// over HBM) and the prefix max; per unit: the drop test of the survivor pass
// (bound (a) with the prefix max up to each segment, bound (b)), the top-k
// candidates (raw >= tau, exact exps), the survivors compacted in row order
// into shared memory and classified as one group, whose approximate mass
// advances the state.  The next unit's elements are fetched (cp.async) while
// a unit is classified.
constexpr int RUN = 4;    // units per item past the head: a sub-slice (a multiple of 1024 elements) holds whole items
constexpr int HEAD = 16;  // units of each row taken one per item (a multiple of RUN)

struct FusedShared {
  ClassShared c;
  float4 stage[K1_WARPS][2][2][32];  // per warp: two units' elements, at most 2 16-byte loads per lane
};

template <typename TIn, int VE, bool VEC>
__global__ void __launch_bounds__(K1_NT, 3) fused_classify_kernel(SliceArgs a) {
  extern __shared__ __align__(16) unsigned char fused_smem[];
  FusedShared& fsh = *reinterpret_cast<FusedShared*>(fused_smem);
  ClassShared& sh = fsh.c;
  constexpr int LOADS = UNIT / (32 * VE);  // 16-byte loads per lane per unit
  constexpr int SEGW = 32 * VE;            // elements of one segment
  static_assert(LOADS <= 2, "stage holds two loads per lane");
  grid_dep_launch_next();
  grid_dep_wait();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int nsub = a.P * K1_WARPS;
  const long long V = a.V;
  const float NEG_INF = -__int_as_float(0x7f800000);
  float* graw = sh.raw[w];
  uint32_t* gidx = sh.idx[w];
  float4 (*stage)[2][32] = fsh.stage[w];
  const int B = (int)a.B;
  const int nchunk = (int)((V + UNIT - 1) / UNIT);
  const int head = nchunk < HEAD ? nchunk : HEAD;
  const int nhead = B * head;
  const int nitem = nhead + B * ((nchunk - head + RUN - 1) / RUN);
  const int nw = (int)gridDim.x * K1_WARPS;
  const int ups = (int)(a.SL / UNIT);  // units per sub-slice
  const int jmax_row = a.jmax;
  // item it: row b, units [c0, cend)
  auto coords = [&](int itm, int& bb, int& cc0, int& ccend) {
    if (itm < nhead) {
      bb = itm % B;
      cc0 = itm / B;
      ccend = cc0 + 1;
    } else {
      const int t = itm - nhead;
      bb = t % B;
      cc0 = head + (t / B) * RUN;
      ccend = cc0 + RUN < nchunk ? cc0 + RUN : nchunk;
    }
  };
  auto fetch = [&](int bb, int cc, int buf) {  // unit cc of row bb into stage[buf]
    if (VEC && (long long)(cc + 1) * UNIT <= V) {
      const TIn* row = (const TIn*)a.logits + (long long)bb * a.ld + (long long)cc * UNIT;
#pragma unroll
      for (int q = 0; q < LOADS; ++q) cp_async16(&stage[buf][q][lane], row + q * SEGW + lane * VE);
    }
  };
  int it = (int)blockIdx.x * K1_WARPS + w;
  int b = 0, c0 = 0, cend = 0;
  if (it < nitem) coords(it, b, c0, cend);
  int buf = 0;
  if (it < nitem) fetch(b, c0, 0);
  cp_async_commit();
  int claim = 0;
  if (lane == 0 && it < nitem) claim = atomicAdd(a.item_next, 1);
  // an item's records: its row's parameters and prologue, its sub-slice's
  // prefix, the state of the pass over HBM at its first unit; loaded one item
  // ahead (their latency hides behind the current item)
  struct ItemRec {
    pesti_sampling_params prm;
    RowInfo ri;
    SubPre pr;
    UnitPre up;
  };
  auto load_rec = [&](int bb, int cc0) {
    ItemRec q;
    q.prm = row_params(a.uni, a.per_row, bb);
    q.ri = a.info[bb];
    q.pr = a.pre[(long long)bb * nsub + cc0 / ups];
    q.up = a.unit_pre[(long long)bb * nchunk + cc0];
    return q;
  };
  ItemRec cur;
  if (it < nitem) cur = load_rec(b, c0);
  while (it < nitem) {
    const int nit = nw + __shfl_sync(PESTI_FULL_MASK, claim, 0);  // the next item
    int nb = 0, nc0 = 0, ncend = 0;
    ItemRec nxt;
    if (nit < nitem) {
      coords(nit, nb, nc0, ncend);
      if (lane == 0) claim = atomicAdd(a.item_next, 1);
      nxt = load_rec(nb, nc0);
    }
    const pesti_sampling_params prm = cur.prm;
    const RowInfo& ri = cur.ri;
    const bool take = !is_greedy(prm) && !ri.uniform && a.fast_enabled && fast_topk(prm, a.V_total);
    const float T = prm.temperature;
    const bool scale = T > 0.0f;
    const float t_eff = scale ? T : 1.0f;
    const float rT = scale ? 1.0f / T : 1.0f;  // the approximate argument x*rT - m of the clean units
    const float m = ri.m;
    const int sub = c0 / ups;
    const long long sub0 = (long long)sub * a.SL;
    const SubPre pr = cur.pr;
    double s_est = 0.0;
    float run_max = NEG_INF;
    if (take) {
      // the approximate state and the max before the item: the earlier
      // sub-slices' (prologue) plus this sub-slice's up to the item (pass over HBM)
      const float ym = ri.max_raw * (1.4426950408889634f / t_eff);
      s_est = pr.A + (cur.up.mlog > NEG_INF ? (double)(cur.up.mass * ex2_approx(cur.up.mlog - ym)) : 0.0);
      run_max = fmaxf(pr.P, cur.up.pmax);
    }
    const float c1 = ABSORB * t_eff * (1.0f + 0x1p-20f);
    const float pf = (m - PRUNE_FLOOR) * t_eff;
    const float p_floor = pf + 0x1p-20f * fabsf(pf);
    auto bound_a = [&](float P) { return P >= p_floor ? fsub(P, fadd(c1, 0x1p-21f * fabsf(P))) : NEG_INF; };
    for (int c = c0; c < cend; ++c, buf ^= 1) {
      // the next unit's elements, while this one is classified
      if (c + 1 < cend) fetch(b, c + 1, buf ^ 1);
      else if (nit < nitem) fetch(nb, nc0, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
      __syncwarp();
      if (!take) continue;
      const long long start = (long long)c * UNIT;
      const int j = c - sub * ups;
      const int len = (int)(V - start < UNIT ? V - start : UNIT);
      // the unit's elements
      float x[LOADS][VE];
      int nv[LOADS];
      if (VEC && len == UNIT) {
#pragma unroll
        for (int q = 0; q < LOADS; ++q) {
          const float4 r4 = stage[buf][q][lane];
          if (sizeof(TIn) == 4) {
            x[q][0] = r4.x; x[q][1] = r4.y; x[q][2] = r4.z; x[q][3] = r4.w;
          } else {
            const uint32_t wds[4] = {__float_as_uint(r4.x), __float_as_uint(r4.y), __float_as_uint(r4.z),
                                     __float_as_uint(r4.w)};
#pragma unroll
            for (int h = 0; h < 4; ++h) unpack2<TIn>(wds[h], x[q][2 * h], x[q][2 * h + 1]);
          }
          nv[q] = VE;
        }
      } else {
        const TIn* row = (const TIn*)a.logits + (long long)b * a.ld + start;
#pragma unroll
        for (int q = 0; q < LOADS; ++q) {
          const int p0 = q * SEGW + lane * VE;
          nv[q] = 0;
#pragma unroll
          for (int e = 0; e < VE; ++e) {
            x[q][e] = p0 + e < len ? load_logit<TIn>(row, p0 + e) : 0.0f;
            nv[q] = p0 + e < len ? e + 1 : nv[q];
          }
        }
      }
      // drop test per segment (bound (a) with the max of the row before the
      // segment, bound (b)); NaN fails it.  svm: the lane's survivors, bit q*VE + e
      uint32_t svm = 0u;
#pragma unroll
      for (int q = 0; q < LOADS; ++q) {
        const float thr = fmaxf(bound_a(run_max), pr.thrL);
        float lm = NEG_INF;  // the segment's max (fmaxf skips NaN, as the pass over HBM)
#pragma unroll
        for (int e = 0; e < VE; ++e) {
          if (e < nv[q]) lm = fmaxf(lm, x[q][e]);
          if (e < nv[q] && x[q][e] >= thr) svm |= 1u << (q * VE + e);
        }
        run_max = fmaxf(run_max, fkey_inv(__reduce_max_sync(PESTI_FULL_MASK, fkey(lm))));
      }
      // top-k candidates (sampling.rs:46,127 exactly)
      {
        const float tau = ri.tau;
#pragma unroll
        for (int q = 0; q < LOADS; ++q) {
          int cc = 0;
#pragma unroll
          for (int e = 0; e < VE; ++e) cc += (e < nv[q] && x[q][e] >= tau) ? 1 : 0;
          if (__any_sync(PESTI_FULL_MASK, cc > 0)) {
            const int ci = warp_incl_scan_add(cc);
            const int ctot = __shfl_sync(PESTI_FULL_MASK, ci, 31);
            int basec = 0;
            if (lane == 0) basec = atomicAdd(a.cand_count + b, ctot);
            basec = __shfl_sync(PESTI_FULL_MASK, basec, 0);
            int slot = basec + ci - cc;
            const uint32_t p0 = (uint32_t)(start + q * SEGW + lane * VE);
#pragma unroll
            for (int e = 0; e < VE; ++e) {
              if (e < nv[q] && x[q][e] >= tau) {
                if (slot < CAND_CAP) {
                  a.cand_e[(long long)b * CAND_CAP + slot] = pesti_expf_call(fsub(scale ? fdiv(x[q][e], T) : x[q][e], m));
                  a.cand_idx[(long long)b * CAND_CAP + slot] = p0 + (uint32_t)e;
                }
                ++slot;
              }
            }
          }
        }
      }
      if (j == 0) {
        // the sub-slice's record; the last sub-slice holding columns also writes
        // those of the sub-slices past the row's end (no units, no entries)
        long long slen = V - sub0;
        slen = slen > a.SL ? a.SL : slen;
        if (lane == 0) a.surv[(long long)b * nsub + sub] = SubSurv{0, (int32_t)((slen + UNIT - 1) / UNIT), 0, NEG_INF};
        if (sub0 + a.SL >= V)
          for (int q = sub + 1 + lane; q < nsub; q += 32) a.surv[(long long)b * nsub + q] = SubSurv{0, 0, 0, NEG_INF};
      }
      // the survivors in row order (segment by segment, lane by lane)
      int n = 0;
#pragma unroll
      for (int q = 0; q < LOADS; ++q) {
        const uint32_t mq = (svm >> (q * VE)) & ((1u << VE) - 1u);
        const int cq = __popc(mq);
        const int iq = warp_incl_scan_add(cq);
        int oq = n + iq - cq;
        const uint32_t p0 = (uint32_t)(start + q * SEGW + lane * VE);
#pragma unroll
        for (int e = 0; e < VE; ++e) {
          if ((mq >> e) & 1u) {
            graw[oq] = x[q][e];
            gidx[oq] = p0 + (uint32_t)e;
            ++oq;
          }
        }
        n += __shfl_sync(PESTI_FULL_MASK, iq, 31);
      }
      GroupEnt* ge = a.gsurv + ((long long)b * nsub + sub) * jmax_row + j;
      if (n == 0) {
        if (lane == 0) *ge = GroupEnt{{0u, 0u, 0u, 0u}, 0, 0, 0, 0};
        continue;
      }
      __syncwarp();
      // A clean unit (one pass per survivor): the range of its approximate
      // states lies inside the binade of its start (within the guard band),
      // so every survivor is a plain increment k = rint(e/w) of one run; k
      // comes from the approximation (exp_hw of the exact argument,
      // sampling.rs:46,127, with its error bound as margin) where it decides
      // it and from the exact exp otherwise (taken once the unit is known to
      // be clean), and no survivor may be a tie.  Anything else goes to the
      // general classification.
      {
        const float BAND = a.band;
        const float sb = (float)s_est;
        const uint32_t clo = fbits(sb) & 0x7f800000u;
        const float lov = bitsf(clo);
        const bool possible = sb >= 0x1p-126f && sb >= lov * (1.0f + BAND);
        const int sh2 = 150 - (int)(clo >> 23);  // w = 2^(E-150)
        const int g = (n + 31) >> 5;
        const int i0 = lane * g;
        const int nl = n - i0 < 0 ? 0 : (n - i0 > g ? g : n - i0);
        float ltot = 0.0f;
        uint32_t ksum = 0u, undecided = 0u;  // undecided: bit jj, element jj of the lane
#pragma unroll 2
        for (int jj = 0; jj < nl; ++jj) {
          const float raw = graw[i0 + jj];
          const float zq = fmaf(raw, rT, -m);  // approximate x/T - m (rT = 1: exactly x - m)
          const float ea = exp_hw(zq);
          ltot += ea;
          if (!possible) continue;
          bool exact;
          if (ea == 0.0f) {
            exact = (clo >> 23) < 40u;  // else: exact e < 1.2e-38 rounds to 0 on this grid
          } else {
            const float tt = __uint_as_float(fbits(ea) + ((uint32_t)sh2 << 23));  // ea/w, exact scaling
            uint32_t kq;
            const float kr = rint_small(tt, kq);
            const float slack = 0.5f - fabsf(tt - kr);
            exact = !(tt < 0x1p22f && slack > tt * fmaf(arg_margin(raw, rT, zq), DE_Z, DE_0) + 0x1p-24f);
            if (!exact) ksum += kq;
          }
          if (exact) undecided |= 1u << jj;
        }
        const float usum = warp_reduce_add(ltot);
        if (possible && sb + usum <= 2.0f * lov * (1.0f - BAND)) {
          bool decided = true;
          for (uint32_t um = undecided; um != 0u; um &= um - 1u) {
            const int jj = __ffs(um) - 1;
            const float raw = graw[i0 + jj];
            const float ex = pesti_expf_call(fsub(scale ? fdiv(raw, T) : raw, m));  // sampling.rs:127, exact
            const uint32_t k0 = fbits(fadd(lov, ex)) - clo;
            const uint32_t k1 = fbits(fadd(bitsf(clo + 1u), ex)) - (clo + 1u);
            decided = decided && k0 == k1;
            ksum += k0;
          }
          if (__all_sync(PESTI_FULL_MASK, decided)) {
            const uint32_t inc = tr_sat(__reduce_add_sync(PESTI_FULL_MASK, ksum));  // each < 2^22, at most 256
            if (lane == 0) *ge = GroupEnt{{clo, inc, inc, gidx[n - 1] + 1u}, 0, 1, 0, 1};
            s_est += (double)usum;
            continue;
          }
        }
      }
      // (its clean case was tried above)
      s_est += (double)classify_group(a, b, sub, j, n, false, s_est, scale, T, m, graw, gidx, sh.ea[w], sh.ck[w],
                                      sh.c0[w], sh.c1[w]);
      __syncwarp();
    }
    it = nit;
    b = nb;
    c0 = nc0;
    cend = ncend;
    cur = nxt;
  }
  cp_async_wait<0>();
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
  uint32_t e_star;
  int need_dense;
  int fallback;
  int fast_ok;
};

// Fast-path arrays, placed after RowShared in dynamic shared memory.
constexpr int FAST_ENTS = 4096;  // fold entries of a row the fast path can stage
constexpr int FAST_ENTS_SHORT = 1024;  // the staging a launch over short rows provides
constexpr int MERGE_EPT = FAST_ENTS / K2_NT;  // of them per thread in the merge
constexpr int FAST_PAIRS = 2048; // (sub-slice, group) pairs of a row the fast path stages
constexpr uint32_t ENT_REPLAY = 0xfffffffdu;  // staged entry: replay the whole sub-slice
struct FastSmem {
  unsigned long long key[FAST_CAND];
  float q[FAST_K];
  float stage[STAGE];
  Seg wseg[K2_NT / 32];        // block-wide segmented scan: per-warp totals and prefixes
  Seg wpre[K2_NT / 32];
  int wfl[K2_NT / 32];
  int pstart[FAST_PAIRS];      // staging: each pair's first entry in the row and in the pool
  int poff[FAST_PAIRS];
  int total;                   // entries of the row (> the launch's capacity: not staged)
  int nment;                   // merged entries
  // followed by FoldEnt ent[cap] (the row's entries in row order; after the
  // merge, in place, the same with consecutive runs of one binade merged),
  // uint16_t owner[cap] (staging: the pair each entry comes from),
  // SubSurv[nsub] and int eoff[nsub] (scratch); cap = RowArgs::fast_ents
};
__host__ __device__ inline size_t fast_smem_bytes(int nsub, int cap) {
  return sizeof(FastSmem) + (size_t)cap * (sizeof(FoldEnt) + sizeof(uint16_t)) +
         (size_t)nsub * (sizeof(SubSurv) + sizeof(int));
}

// Merge of a row's staged fold entries ent[0..total): consecutive runs of
// one binade become one run (their increments compose; the merged run covers
// the row up to the last one's end), so that the walk takes one step per
// binade change or special.  A block-wide segmented scan with EPT consecutive
// entries per thread (EPT * K2_NT >= total), written back in place (every
// thread has read its entries before the first barrier); sets fs.nment.
template <int EPT>
__device__ __forceinline__ void merge_runs(FastSmem& fs, FoldEnt* ent, int total, RowShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  auto single = [](uint32_t key) { return key == fold::SPECIAL || key == ENT_REPLAY; };
  const FoldEnt none{KEY_NONE, 0u, 0u, 0u};
  const int e0 = tid * EPT;
  FoldEnt x[EPT];
#pragma unroll
  for (int i = 0; i < EPT; ++i) x[i] = e0 + i < total ? ent[e0 + i] : none;
  const uint32_t kp = e0 > 0 && e0 < total ? ent[e0 - 1].lo : KEY_NONE;
  const uint32_t kn = e0 + EPT < total ? ent[e0 + EPT].lo : KEY_NONE;
  // h[i]: entry i starts a run; hn: the entry after the thread's last one does
  bool h[EPT];
  Seg agg{0u, 0u, 0u, KEY_NONE};
  bool aflag = false;
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const uint32_t pk = i == 0 ? kp : x[i - 1].lo;
    h[i] = e0 + i < total && (e0 + i == 0 || single(x[i].lo) || single(pk) || x[i].lo != pk);
    const Seg v{x[i].a0, x[i].a1, 0u, x[i].lo};
    if (e0 + i < total) {
      agg = i == 0 ? v : seg_join(agg, v, h[i]);
      aflag = aflag || h[i];
    }
  }
  const bool hn = e0 + EPT < total && (single(kn) || single(x[EPT - 1].lo) || kn != x[EPT - 1].lo);
  Seg inc = agg;
  bool fl = aflag;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const Seg o = seg_shfl_up(inc, off);
    const bool of = __shfl_up_sync(PESTI_FULL_MASK, fl, off);
    if (lane >= off) {
      inc = seg_join(o, inc, fl);
      fl = fl || of;
    }
  }
  if (lane == 31) {
    fs.wseg[wid] = inc;
    fs.wfl[wid] = fl ? 1 : 0;
  }
  __syncthreads();
  if (wid == 0) {  // exclusive segmented scan over the warps' totals
    constexpr int NW = K2_NT / 32;
    const Seg idn{0u, 0u, 0u, KEY_NONE};
    Seg wi = lane < NW ? fs.wseg[lane] : idn;
    bool wf = lane < NW ? fs.wfl[lane] != 0 : false;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const Seg o = seg_shfl_up(wi, off);
      const bool of = __shfl_up_sync(PESTI_FULL_MASK, wf, off);
      if (lane >= off) {
        wi = seg_join(o, wi, wf);
        wf = wf || of;
      }
    }
    const Seg we = seg_shfl_up(wi, 1);
    if (lane < NW) fs.wpre[lane] = lane == 0 ? idn : we;
  }
  __syncthreads();
  Seg pre = fs.wpre[wid];
  const Seg ex = seg_shfl_up(inc, 1);
  const bool exf = __shfl_up_sync(PESTI_FULL_MASK, fl, 1);
  if (lane > 0) pre = seg_join(pre, ex, exf);
  // an entry ends a merged run when the next one starts a run (or none follows)
  bool end[EPT];
  int nend = 0;
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    end[i] = e0 + i < total && (i + 1 < EPT ? (e0 + i + 1 >= total || h[i + 1]) : (e0 + EPT >= total || hn));
    nend += end[i] ? 1 : 0;
  }
  int tot;
  int o = block_excl_scan_add(nend, sh.iscr, tot);
  Seg cur = pre;
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    if (e0 + i < total) {
      cur = seg_join(cur, Seg{x[i].a0, x[i].a1, 0u, x[i].lo}, h[i]);
      if (end[i]) ent[o++] = FoldEnt{single(x[i].lo) ? x[i].lo : cur.key, cur.a0, cur.a1, x[i].end};
    }
  }
  if (tid == 0) fs.nment = tot;
  __syncthreads();
}

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

// The same, by one warp.
__device__ void warp_bitonic_desc(unsigned long long* key, int m) {
  const int lane = threadIdx.x & 31;
  for (int kk = 2; kk <= m; kk <<= 1) {
    for (int j = kk >> 1; j > 0; j >>= 1) {
      for (int i = lane; i < m; i += 32) {
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
      __syncwarp();
    }
  }
}

// Bitonic sort, descending, of 32*R keys held R per lane (element r*32 + lane),
// by one warp in registers.
template <int R>
__device__ __forceinline__ void warp_sort_desc_regs(unsigned long long (&v)[R]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32 * R; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= 32) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int rp = r ^ (j >> 5);
          if (rp > r) {
            const bool desc = ((r * 32 + lane) & k) == 0;
            const unsigned long long x = v[r], y = v[rp];
            if (desc ? (x < y) : (x > y)) {
              v[r] = y;
              v[rp] = x;
            }
          }
        }
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const unsigned long long y = __shfl_xor_sync(PESTI_FULL_MASK, v[r], j);
          const bool desc = ((r * 32 + lane) & k) == 0;
          const bool keep_max = desc == ((lane & j) == 0);
          v[r] = keep_max ? (v[r] > y ? v[r] : y) : (v[r] < y ? v[r] : y);
        }
      }
    }
  }
}

template <int R>
__device__ void warp_sort_keys(unsigned long long* key, int n) {
  const int lane = threadIdx.x & 31;
  unsigned long long v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = r * 32 + lane < n ? key[r * 32 + lane] : 0ull;
  warp_sort_desc_regs<R>(v);
#pragma unroll
  for (int r = 0; r < R; ++r)
    if (r * 32 + lane < n) key[r * 32 + lane] = v[r];
  __syncwarp();
}

// The sequential f32 fold s = s0; s = s + v[j] over n values in shared
// memory by one thread, with the query of fold::thread_fold (first j with
// bits(s) >= tau_bits); the loads go out eight at a time ahead of the
// dependent adds.
__device__ __forceinline__ fold::Result serial_fold8(const float* v, long long n, uint32_t s0_bits,
                                                     uint32_t tau_bits, bool stop_at_hit) {
  fold::Result r;
  uint32_t s = s0_bits & 0x7fffffffu;
  r.hit = -1;
  r.hit_s_bits = 0;
  for (long long j0 = 0; j0 < n; j0 += 8) {
    float x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) x[u] = j0 + u < n ? v[j0 + u] : 0.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (j0 + u < n) {
        s = fbits(fadd(bitsf(s), x[u]));
        if (r.hit < 0 && s >= tau_bits) {
          r.hit = j0 + u;
          r.hit_s_bits = s;
        }
      }
    }
    if (stop_at_hit && r.hit >= 0) break;
  }
  r.s_bits = s;
  return r;
}

// Fold of len values in shared memory, in order, by one warp from state s
// (bits): each step takes 32 of them with a transducer scan over the lanes,
// adds the first one that would leave the binade (or is large next to s)
// directly, and resumes after it.  All 32 lanes must call it; the result is
// warp-uniform.
__device__ __forceinline__ uint32_t warp_fold_staged(const float* stage, int len, uint32_t s) {
  const int lane = threadIdx.x & 31;
  int j = 0;
  while (j < len) {
    const int idx = j + lane;
    const bool valid = idx < len;
    const float x = valid ? stage[idx] : 0.0f;
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
    const int nvalid = len - j < 32 ? len - j : 32;
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

// Fold of the exps of n raw logits (f32 or bf16, in global memory) by one
// warp, starting from state s (bits).  The exact exps are staged STAGE at a
// time in shared memory and folded by warp_fold_staged.  All 32 lanes must
// call it.
__device__ uint32_t warp_fold(const void* raw, int dtype, long long n, uint32_t s, float* stage, bool scale,
                              float T, float m) {
  const int lane = threadIdx.x & 31;
  for (long long base = 0; base < n; base += STAGE) {
    const int len = (int)(n - base < STAGE ? n - base : STAGE);
    __syncwarp();
    for (int i = lane; i < len; i += 32) {
      const float xr = load_logit_dyn(raw, dtype, base + i);
      stage[i] = pesti_expf_call(fsub(scale ? fdiv(xr, T) : xr, m));  // sampling.rs:46,127
    }
    __syncwarp();
    s = warp_fold_staged(stage, len, s);
  }
  __syncwarp();
  return s;
}

}  // namespace pesti
#include "pesti_nucleus.cuh"
namespace pesti {

__global__ void __launch_bounds__(K2_NT) row_kernel(RowArgs a) {
  grid_dep_wait();
  extern __shared__ __align__(16) unsigned char row_smem[];
  RowShared& sh = *reinterpret_cast<RowShared*>(row_smem);
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const long long b = blockIdx.x;
  if (a.only && a.only[b] == 0) return;  // the cluster pass sampled the row
  const long long V = a.V;
  const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
  const RowInfo ri = a.info[b];
  const float T = prm.temperature;
  const int nsub = a.P * K1_WARPS;
  const void* row = a.dtype != PESTI_F32 ? (const void*)((const uint16_t*)a.logits + b * a.ld)
                                          : (const void*)((const float*)a.logits + b * a.ld);
  float* E = a.E + b * V;
  uint32_t* I = a.I + b * V;
  const float r = a.u ? a.u[b] : 0.0f;
  const float INF = __int_as_float(0x7f800000);
  const SubSurv* survs = a.surv + b * nsub;
  const uint32_t fl = ri.flags;

  const long long VT = a.V_total;
  if (a.shard) {
    // of a vocabulary shard, only rows of the fast top-k path are sampled
    // through exchange records; the others are marked for the gathered path
    const bool ok = V > 0 && !is_greedy(prm) && !ri.uniform && a.fast_enabled && fast_topk(prm, VT);
    if (!ok) {
      if (tid == 0) {
        ShardRec* rc = reinterpret_cast<ShardRec*>(a.rec + b * a.rec_stride);
        *rc = ShardRec{0.0, 0.0f, SH_SKIP, 0.0f, 0, GR_ROW, 0u};
        a.nment_g[b] = -1;
      }
      return;
    }
  }

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
    if (prm.flags & PESTI_FLAG_ARGMAX_FIRST) tok = ri.first_max >= 0 ? (uint32_t)ri.first_max : 0u;
    else if (fl & MF_NAN) tok = nan_argmax(row, a.dtype, V, ri.last_nan, sh);
    else tok = ri.last_max >= 0 ? (uint32_t)ri.last_max : 0u;
    if (tid == 0) {
      a.out[b] = tok;
      if (a.kept_count) a.kept_count[b] = 0;
    }
    write_kept_pad(a, b, 0);
    return;
  }

  const bool scale = T > 0.0f;
  const float m = ri.m;
  const long long k = (long long)prm.top_k;
  const bool topp = prm.top_p > 0.0f && k == 0;
  const uint32_t r_tau = fold::tau_bits_of(r);

  // top-p rows of bf16 logits whose softmax sum the cluster pass has folded:
  // by distinct values (pesti_nucleus.cuh); the generic path if that fails
  if (a.only && a.nucleus && a.only[b] == 2 && a.dtype == PESTI_BF16 && !ri.uniform) {
    NucSmem& ns = *reinterpret_cast<NucSmem*>(row_smem + sizeof(RowShared));
    if (nucleus_rows(a, b, ri, prm, (const uint16_t*)row, sh, ns)) return;
    __syncthreads();
  }

  if (ri.uniform) {
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

  // ---------------- fast path: explicit top-k of at most FAST_K (one warp) ----------------
  if (a.fast_enabled && fast_topk(prm, VT)) {
    FastSmem& fs = *reinterpret_cast<FastSmem*>(row_smem + sizeof(RowShared));
    const int cap = a.fast_ents;
    FoldEnt* fent = reinterpret_cast<FoldEnt*>(row_smem + sizeof(RowShared) + sizeof(FastSmem));
    uint16_t* fown = reinterpret_cast<uint16_t*>(fent + cap);
    SubSurv* ss = reinterpret_cast<SubSurv*>(fown + cap);
    int* eoff = reinterpret_cast<int*>(ss + nsub);
    // warp 1 fetches the candidates now (they are sorted after the staging)
    int C = 0;
    unsigned long long ck[2] = {0ull, 0ull};
    if (wid == 1) {
      C = a.cand_count[b];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int j = r * 32 + lane;
        if (j < C && j < CAND_CAP)
          ck[r] = ((unsigned long long)fbits(a.cand_e[b * CAND_CAP + j]) << 32) |
                  (unsigned long long)(~a.cand_idx[b * CAND_CAP + j]);
      }
    }
    // stage the row's fold entries, compacted, with the whole block: one
    // thread per (sub-slice, group) pair in row order; a sub-slice with an
    // overflowed group stages a single replay marker
    const long long keff = k < VT ? k : VT;
    {
      const GroupEnt* gs = a.gsurv + b * nsub * a.jmax;
      const FoldEnt* pool = a.pool + b * POOL_CAP;
      int* rep = eoff;  // per sub-slice: a group overflowed
      const int npair = nsub * a.jmax;
      // with at most one pair per thread, its record is read once (here)
      const bool one = npair <= K2_NT;
      GroupEnt ge1{{0u, 0u, 0u, 0u}, 0, 0, 0, 0};
      if (one && tid < npair) ge1 = gs[tid];
      for (int q = tid; q < nsub; q += K2_NT) {
        ss[q] = survs[q];
        if ((long long)q * a.SL >= V) ss[q].ngroups = 0;  // past the row's end: no units
        rep[q] = 0;
      }
      __syncthreads();
      for (int t = tid; t < npair; t += K2_NT) {
        const int q = t / a.jmax, j = t - q * a.jmax;
        if (j < ss[q].ngroups && (one ? ge1.replay : gs[t].replay)) rep[q] = 1;
      }
      __syncthreads();
      // each pair's place in the row (a block scan), then every entry copied
      // by its own thread: the loads from the pool are all in flight at once
      int base = 0;
      for (int t0 = 0; t0 < npair; t0 += K2_NT) {
        const int t = t0 + tid;
        int ne = 0, off = 0;
        bool inl = false;
        FoldEnt ient{0u, 0u, 0u, 0u};
        if (t < npair) {
          const int q = t / a.jmax;
          const int j = t - q * a.jmax;
          if (j < ss[q].ngroups) {
            if (rep[q]) {
              ne = j == 0 ? 1 : 0;
              off = -1 - q;  // replay marker of sub-slice q
            } else {
              const GroupEnt ge = one ? ge1 : gs[t];
              ne = ge.nent;
              off = ge.off;
              inl = ge.inl != 0;
              ient = FoldEnt{ge.ent[0], ge.ent[1], ge.ent[2], ge.ent[3]};
            }
          }
        }
        int tot;
        const int ex = base + block_excl_scan_add(ne, sh.iscr, tot);
        if (t < FAST_PAIRS) {
          fs.pstart[t] = ex;
          fs.poff[t] = off;
        }
        if (t < FAST_PAIRS && ex + ne <= cap) {
          if (inl) {  // a one-entry task keeps its entry in its record
            fent[ex] = ient;
            fown[ex] = 0xffffu;
          } else {
            for (int i = 0; i < ne; ++i) fown[ex + i] = (uint16_t)t;
          }
        }
        base += tot;
      }
      if (npair > FAST_PAIRS) base = cap + 1;  // too many pairs to stage: the generic path
      __syncthreads();
      if (base <= cap) {
        for (int e = tid; e < base; e += K2_NT) {
          const int t = fown[e];
          if (t == 0xffff) continue;  // staged already
          const int off = fs.poff[t];
          if (off < 0) {
            const long long qend = ((long long)(-1 - off) + 1) * a.SL;
            fent[e] = FoldEnt{ENT_REPLAY, 0u, 0u, (uint32_t)(qend < V ? qend : V)};
          } else {
            fent[e] = pool[off + (e - fs.pstart[t])];
          }
        }
      }
      if (tid == 0) fs.total = base;
      __syncthreads();
    }
    // merge consecutive runs of one binade (fewer steps for the walk below)
    if (fs.total <= 2 * K2_NT) merge_runs<2>(fs, fent, fs.total, sh);
    else if (fs.total <= cap) merge_runs<MERGE_EPT>(fs, fent, fs.total, sh);
    if (wid != 1) C = a.cand_count[b];
    // a shard lists any number of candidates up to FAST_CAND (the row's k-th
    // largest may lie in another shard)
    const bool cand_ok = (a.shard || C >= keff) && C <= FAST_CAND;
    if (wid == 1 && fs.total <= cap && cand_ok) {
      // candidates by (e desc, index asc) while warp 0 folds; the order by p
      // = e/S differs only inside groups of equal p (fixed up below)
#pragma unroll
      for (int r = 0; r < 2; ++r)
        if (r * 32 + lane < C) fs.key[r * 32 + lane] = ck[r];
      for (int j = 64 + lane; j < C; j += 32)
        fs.key[j] = ((unsigned long long)fbits(a.cand_e[b * CAND_CAP + j]) << 32) |
                    (unsigned long long)(~a.cand_idx[b * CAND_CAP + j]);
      __syncwarp();
      if (C <= 32) warp_sort_keys<1>(fs.key, C);
      else if (C <= 64) warp_sort_keys<2>(fs.key, C);
      else if (C <= 128) warp_sort_keys<4>(fs.key, C);
      else {
        int mm2 = 1;
        while (mm2 < C) mm2 <<= 1;
        for (int j = C + lane; j < mm2; j += 32) fs.key[j] = 0ull;
        __syncwarp();
        warp_bitonic_desc(fs.key, mm2);
      }

    }
    uint32_t s = a.shard ? fbits(ri.s_start) : 0u;
    if (wid == 0 && fs.total <= cap) {
      // softmax denominator (sampling.rs:128): walk the merged entries with the
      // exact state.  An entry the state does not fit (or a replay marker) is folded from
      // the raw logits of the row range it covers, from the state before it
      // (the dropped elements in the range are exact no-ops).
      const int nm = fs.nment;
      constexpr int WB = 8;  // entries per batch; the next batch is loaded while one is walked
      int i = 0;
      while (i < nm) {
        int fi = -1;  // first entry the state does not fit
        FoldEnt nx[WB];
#pragma unroll
        for (int u = 0; u < WB; ++u) nx[u] = fent[i + u < nm ? i + u : nm - 1];
        for (; i < nm; i += WB) {
          FoldEnt en[WB];
#pragma unroll
          for (int u = 0; u < WB; ++u) {
            en[u] = nx[u];
            const int k = i + WB + u;
            nx[u] = fent[k < nm ? k : nm - 1];
          }
          // branch-free: the state stops at the first entry it does not fit
#pragma unroll
          for (int u = 0; u < WB; ++u) {
            const bool live = fi < 0 && i + u < nm;
            const bool sp = en[u].lo == fold::SPECIAL;
            const uint32_t s_sp = fbits(fadd(bitsf(s), bitsf(en[u].a0)));
            const uint32_t ns = s + ((s & 1u) ? en[u].a1 : en[u].a0);  // < 2^31 + 2^30: no wrap
            // also false for every replay marker (no binade has its bits)
            const bool fits = fold::binade_lo_bits(s) == en[u].lo && ns < fold::binade_hi_bits(en[u].lo);
            fi = live && !sp && !fits ? i + u : fi;
            s = live && (sp || fits) ? (sp ? s_sp : ns) : s;
          }
          if (fi >= 0) break;
        }
        if (fi < 0) break;
        const uint32_t from = fi > 0 ? fent[fi - 1].end : 0u;
        const uint32_t to = fent[fi].end;
        const void* src = a.dtype != PESTI_F32 ? (const void*)((const uint16_t*)row + from)
                                                : (const void*)((const float*)row + from);
        s = warp_fold(src, a.dtype, (long long)to - from, s, fs.stage, scale, T, m);
        i = fi + 1;
      }
    }
    __syncthreads();
    if (a.shard) {
      // exchange record: the exact fold from the approximate start, the top
      // ksh candidates with their columns in the whole row, and a bound on
      // every element not listed (the next candidate's exp, or exp(tau) above
      // every non-candidate)
      if (wid == 0) {
        ShardRec* rc = reinterpret_cast<ShardRec*>(a.rec + b * a.rec_stride);
        ShardCand* cd = reinterpret_cast<ShardCand*>(rc + 1);
        const bool ok = fs.total <= cap && cand_ok;
        const int nl = ok ? (C < a.ksh ? C : a.ksh) : 0;
        for (int j = lane; j < nl; j += 32) {
          const unsigned long long kv = fs.key[j];
          cd[j] = ShardCand{(uint32_t)(kv >> 32), ~(uint32_t)(kv & 0xffffffffull) + (uint32_t)a.col0};
        }
        if (ok)
          for (int i = lane; i < fs.nment; i += 32) a.ment_g[b * FAST_ENTS + i] = fent[i];
        if (lane == 0) {
          ShardRec r;
          r.delta = ok ? (double)bitsf(s) - (double)ri.s_start : 0.0;
          r.s_start = ri.s_start;
          r.status = ok ? SH_OK : SH_FAIL;
          r.bound = ok && C > a.ksh ? bitsf((uint32_t)(fs.key[a.ksh] >> 32)) : ri.e_tau;
          r.n = nl;
          r.why = fs.total > cap ? GR_ENTRIES : (ok ? 0u : GR_CANDS);
          r.pad = 0u;
          *rc = r;
          a.nment_g[b] = ok ? fs.nment : -1;
        }
      }
      return;
    }
    if (wid == 0 && fs.total <= cap) {
      const float S = bitsf(s);
      bool ok = cand_ok;
      if (ok) {
        // p = e/S (sampling.rs:130); the list stays sorted by p except inside
        // groups of equal p, which the stable sort (sampling.rs:60) orders by index
        for (int j = lane; j < C; j += 32) {
          const unsigned long long kv = fs.key[j];
          fs.key[j] = ((unsigned long long)fbits(fdiv(bitsf((uint32_t)(kv >> 32)), S)) << 32) | (kv & 0xffffffffull);
        }
        __syncwarp();
        bool viol = false;
        for (int j = lane; j + 1 < C; j += 32) viol |= fs.key[j] < fs.key[j + 1];
        if (__any_sync(PESTI_FULL_MASK, viol)) {
          if (lane == 0) {  // insertion sort: only equal-p groups are out of order
            for (int j = 1; j < C; ++j) {
              const unsigned long long kv = fs.key[j];
              int t = j - 1;
              while (t >= 0 && fs.key[t] < kv) {
                fs.key[t + 1] = fs.key[t];
                --t;
              }
              fs.key[t + 1] = kv;
            }
          }
          __syncwarp();
        }
        // every element outside the candidates (raw < tau) must rank below the keff-th
        const float pk = bitsf((uint32_t)(fs.key[keff - 1] >> 32));
        ok = fdiv(ri.e_tau, S) < pk;
      }
      if (ok) {
        // total over the kept list (sampling.rs:81), normalisation (:94), draw (:99-111)
        for (long long j = lane; j < keff; j += 32) fs.q[j] = bitsf((uint32_t)(fs.key[j] >> 32));
        __syncwarp();
        uint32_t tb = 0u;
        if (lane == 0) tb = serial_fold8(fs.q, keff, 0u, fold::NO_QUERY, false).s_bits;
        const float total = bitsf(__shfl_sync(PESTI_FULL_MASK, tb, 0));
        for (long long j = lane; j < keff; j += 32) fs.q[j] = fdiv(fs.q[j], total);
        __syncwarp();
        if (lane == 0) {
          const fold::Result dr = serial_fold8(fs.q, keff, 0u, r_tau, true);
          const long long at = dr.hit >= 0 ? dr.hit : keff - 1;
          a.out[b] = ~(uint32_t)(fs.key[at] & 0xffffffffull);
          if (a.kept_count) a.kept_count[b] = keff;
        }
        for (long long j = lane; j < a.kept_width; j += 32) {
          const bool in = j < keff;
          const unsigned long long kv = in ? fs.key[j] : 0ull;
          if (a.kept_p) a.kept_p[b * a.kept_width + j] = in ? bitsf((uint32_t)(kv >> 32)) : 0.0f;
          if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = in ? ~(uint32_t)(kv & 0xffffffffull) : 0xffffffffu;
        }
      }
      if (lane == 0) sh.fast_ok = ok ? 1 : 0;
    } else if (tid == 0 && fs.total > cap) {
      sh.fast_ok = 0;
    }
    __syncthreads();
    if (sh.fast_ok) return;
    // otherwise: the generic path below
  }

  // largest dropped logit -> an upper bound of the exp of every dropped element
  float pm = -INF;
  if (!a.only)
    for (int s = tid; s < nsub; s += K2_NT)
      if ((long long)s * a.SL < V) pm = fmaxf(pm, survs[s].pruned_max);
  pm = -block_reduce_min(-pm, sh.fscr);
  const float e_pruned = pm > -INF ? pesti_expf(fsub(scale ? fdiv(pm, T) : pm, m)) : 0.0f;

  // ---------------- generic path ----------------
  // rows of the fast path have no survivor list: all their elements
  bool dense_all = a.only != nullptr || (a.fast_enabled && fast_topk(prm, V));
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
    constexpr int REB = 8;  // loads issued per thread before their stores (key and cut loops)
    for (int s = 0; s < nsub; ++s) {
      const SubInfo si = sh.sub[s];
      // the next step's load is issued before this step's exp
      float raw_n = 0.0f;
      uint32_t idx_n = 0u;
      if (tid < si.cnt) {
        if (si.dense) {
          idx_n = (uint32_t)(si.start + tid);
          raw_n = load_logit_dyn(row, a.dtype, si.start + tid);
        } else {
          raw_n = a.surv_raw[b * V + si.start + tid];
          idx_n = a.surv_idx[b * V + si.start + tid];
        }
      }
      for (long long jj = tid; jj < si.cnt; jj += K2_NT) {
        const float raw = raw_n;
        const uint32_t idx = idx_n;
        const long long jn = jj + K2_NT;
        if (jn < si.cnt) {
          if (si.dense) {
            idx_n = (uint32_t)(si.start + jn);
            raw_n = load_logit_dyn(row, a.dtype, si.start + jn);
          } else {
            raw_n = a.surv_raw[b * V + si.start + jn];
            idx_n = a.surv_idx[b * V + si.start + jn];
          }
        }
        const float x = scale ? fdiv(raw, T) : raw;  // sampling.rs:46
        const float e = pesti_expf(fsub(x, m));      // sampling.rs:127
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

    // top-p rows whose largest probability already reaches top_p: the
    // sorted cumulative sum stops after its first element (sampling.rs:66-78),
    // total is that probability, normalised it is 1 and the draw takes it
    // (sampling.rs:81-105).  The row's largest exp is exp(0) = 1, and the
    // first element of the stable sort is the lowest index among the
    // elements of that probability.  No sort needed.
    if (k == 0 && prm.top_p > 0.0f) {
      const float p0 = fdiv(1.0f, S);  // sampling.rs:130 on the row's maximum
      if (p0 >= prm.top_p) {
        if (tid == 0) sh.e_star = 0xffffffffu;
        __syncthreads();
        uint32_t best = 0xffffffffu;
        for (long long j = tid; j < n; j += K2_NT)
          if (fdiv(E[j], S) == p0) best = I[j] < best ? I[j] : best;
        if (best != 0xffffffffu) atomicMin(&sh.e_star, best);
        __syncthreads();
        const uint32_t idx0 = sh.e_star;
        if (tid == 0) {
          a.out[b] = idx0;
          if (a.kept_count) a.kept_count[b] = 1;
        }
        for (long long j = tid; j < a.kept_width; j += K2_NT) {
          if (a.kept_p) a.kept_p[b * a.kept_width + j] = j == 0 ? p0 : 0.0f;
          if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = j == 0 ? idx0 : 0xffffffffu;
        }
        return;
      }
    }

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
    for (long long j0 = tid; j0 < n; j0 += (long long)K2_NT * REB) {
      float ev[REB];
#pragma unroll
      for (int r = 0; r < REB; ++r) {
        const long long j = j0 + (long long)r * K2_NT;
        ev[r] = j < n ? E[j] : 0.0f;
      }
#pragma unroll
      for (int r = 0; r < REB; ++r) {
        const long long j = j0 + (long long)r * K2_NT;
        if (j < n) {
          SK0[j] = ~fbits(fdiv(ev[r], S));
          SV0[j] = (uint32_t)j;
        }
      }
    }
    __syncthreads();
    const int which = sort::block_radix_sort(SK0, SV0, SK1, SV1, n, sh.u.s);
    const uint32_t* SK = which ? SK1 : SK0;
    const uint32_t* SV = which ? SV1 : SV0;
    for (long long j0 = tid; j0 < n; j0 += (long long)K2_NT * REB) {
      uint32_t kv[REB];
#pragma unroll
      for (int r = 0; r < REB; ++r) {
        const long long j = j0 + (long long)r * K2_NT;
        kv[r] = j < n ? SK[j] : 0u;
      }
#pragma unroll
      for (int r = 0; r < REB; ++r) {
        const long long j = j0 + (long long)r * K2_NT;
        if (j < n) Q[j] = bitsf(~kv[r]);
      }
    }
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
    for (long long j0 = tid; j0 < c; j0 += (long long)K2_NT * REB) {
      float qv[REB];
#pragma unroll
      for (int r = 0; r < REB; ++r) {
        const long long j = j0 + (long long)r * K2_NT;
        qv[r] = j < c ? Q[j] : 0.0f;
      }
#pragma unroll
      for (int r = 0; r < REB; ++r) {
        const long long j = j0 + (long long)r * K2_NT;
        if (j < c) Q[j] = fdiv(qv[r], total);
      }
    }
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
