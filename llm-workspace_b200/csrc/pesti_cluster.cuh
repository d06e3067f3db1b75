// One thread-block cluster per row: the whole sampling step of a row in one
// launch (sampling.rs:39-111 for top-k rows, and the argmax branch of
// generate, transformer/model.rs:517-521).
//
// The row is split over the cluster's CTAs and their warps; warp g (in row
// order, over the CTAs by rank) owns the contiguous range [wstart[g], wstart[g+1]).
// The first warps of a row get shorter ranges: there the running sum is small,
// most elements survive the pruning and the state crosses binades often.
// The CTAs exchange their partial results through distributed shared memory
// and cluster barriers, so nothing crosses a kernel boundary:
//
//   pass 1   each warp streams its range from HBM: maximum (NaN ignored, as
//            the f32::max fold of sampling.rs:126 does), NaN/inf flags, an
//            approximate softmax mass relative to its own maximum, and the
//            maximum of every 32*VE-element segment;
//   combine  every CTA reads every warp's summary from the cluster: the row
//            maximum m, each warp's approximate fold state at its start (the
//            mass of the earlier warps) and prefix maximum, the pruning
//            thresholds, and the candidate threshold tau (a lower bound of
//            the k-th largest logit, from the segment maxima);
//   pass 2   each warp re-reads its range (from L2): elements that provably
//            leave the softmax fold unchanged are dropped; every survivor
//            gets its exact exp and its approximate fold state, and becomes
//            either part of a run (a plain integer increment of the state's
//            bits inside one binade, as a transducer for an even and an odd
//            entry state) or an explicit element (added with a real f32 add);
//            elements at or above tau are the top-k candidates;
//   walk     the leader CTA gathers every CTA's entries and candidates, walks
//            the entries with the exact state (the softmax sum S bit for bit,
//            sampling.rs:128), sorts the candidates by (p desc, index asc),
//            and folds total, normalises and draws (sampling.rs:81-111).
//
// A run whose binade the approximate state predicted wrongly fails its check
// in the walk and is folded again from the raw logits of its range, so the
// approximation never decides a result.  Rows the cluster cannot finish
// exactly (NaN or infinite rows, rows that are not top-k <= 256, too many
// candidates, a probability tie at the candidate threshold) get their row
// prologue written and a flag set; the row kernel's generic path samples them
// in the launch that follows.
#pragma once
#include <cooperative_groups.h>
#include "pesti_kernels.cuh"

namespace pesti {
namespace cg = cooperative_groups;

constexpr int CL_WARPS = 8;             // warps per CTA
constexpr int CL_NT = CL_WARPS * 32;
constexpr int CL_MAXC = 16;             // CTAs per cluster (row)
constexpr int CL_SEGS = 20;             // 32*VE-element segments per warp at most
constexpr int CL_U = 4;                 // segments loaded at once per warp (pass 1)
constexpr int CL_STAGES = 4;            // segments in flight per warp through shared memory (pass 2)
constexpr int CL_P1S = 8;               // segments in flight per warp through shared memory (pass 1)
constexpr int CL_R = 4;                 // survivors per lane in one classification batch
constexpr int CL_BATCH = 32 * CL_R;     // survivors classified together
constexpr int CL_RING = 256;            // survivor ring per warp (power of two)
constexpr int CL_EW = 48;               // fold entries per warp (beyond: its range is replayed)
constexpr int CL_LIST = 128;            // merged fold entries per CTA (beyond: its range is replayed)
constexpr int CL_CCAP = 256;            // top-k candidates per CTA
constexpr int CL_LOCAL = 512;           // fold entries of a row the leader gathers
constexpr int CL_RGRP = CL_NT - 32;     // the leader's replay group: every warp but warp 1
constexpr int CL_RPT = 4;               // replayed elements per thread and chunk
constexpr int CL_RCH = CL_RGRP * CL_RPT;  // replayed elements per chunk
constexpr long long CL_MAX_V = 131072;  // longest row of the cluster path (f32)
constexpr long long CL_MAX_V16 = 262144;  // the same for 16-bit logits
static_assert(CL_SEGS <= 32, "one lane per segment in the warp summary");

struct ClusterArgs {
  const void* logits;
  int dtype;
  long long B, V, ld;
  pesti_sampling_params uni;
  const pesti_sampling_params* per_row;
  // warp g of the row owns [wstart[g], wstart[g+1]): multiples of 32*VE (the
  // last end is V), at most CL_SEGS*32*VE long, C*CL_WARPS + 1 entries
  int wstart[CL_MAXC * CL_WARPS + 1];
  const float* u;
  uint32_t* out;
  float* kept_p;
  uint32_t* kept_idx;
  long long kept_width;
  int64_t* kept_count;
  int* fb;            // [B]: 1 when the row is left to the row kernel's generic path
  RowInfo* info;      // [B]: those rows' prologue
  float band;         // relative guard band around binade edges
  int early_dependents;  // let the row kernel launch at once (its blocks then wait for this grid)
  int nucleus;          // bf16 top-p rows are folded here and finished by the row kernel
};

struct ClWarp {       // one warp's pass-1 summary, read by every CTA of the cluster
  float max_raw;      // max of its raw logits, NaN ignored (-inf: none)
  float sum_rel;      // sum of 2^(raw*c2 - max_raw*c2), c2 = log2(e)/T_eff (approximate)
  int32_t last_nan;   // last NaN index, -1
  uint32_t flags;     // MF_*
  int32_t first_max, last_max;  // first / last index holding max_raw (greedy rows), -1
  float min_raw;      // min of its raw logits, NaN ignored (+inf: none)
  int32_t pad1;
};

struct ClShared {
  ClWarp wst[CL_WARPS];
  float segmax[CL_WARPS][CL_SEGS];
  float segmass[CL_WARPS][CL_SEGS];  // approximate mass of each segment relative to its max
  double A[CL_WARPS];         // approximate fold state at each warp's start
  float P[CL_WARPS];          // max raw logit before each warp
  float thrL[CL_WARPS];       // raw logits below it are absorbed by the running sum (or -inf)
  int wn[CL_WARPS];           // fold entries of each warp (-1: overflow, replay its range)
  float cand_e[CL_CCAP];      // the CTA's top-k candidates: exact exp, row index
  uint32_t cand_i[CL_CCAP];
  int ncand;                  // candidates found (may exceed CL_CCAP)
  int nlist;                  // merged fold entries of the CTA
  FoldEnt list[CL_LIST];
  // row state, computed by every CTA
  float max_raw, m, tau, e_tau, min_raw;
  uint32_t flags;
  int last_nan, first_max, last_max;
  int status;                 // leader: 0 sampled, 1 fallback
  double dscr[34];
  float fscr[34];
  int iscr[34];
  uint32_t uscr[34];
  union {
    struct {                  // pass 1: the HBM stream's ring of segments per warp
      float4 ring[CL_WARPS][CL_P1S * 32];
    } r;
    struct {                  // the candidate threshold (combine)
      uint32_t hist[256];
      float tau;
    } t;
    struct {                  // pass 2: staged segments, survivor rings and fold entries per warp
      float4 stg[CL_WARPS][CL_STAGES * 32];
      float qraw[CL_WARPS][CL_RING];
      uint32_t qidx[CL_WARPS][CL_RING];
      FoldEnt went[CL_WARPS][CL_EW];
    } c;
    struct {                  // leader: the row's entries and candidates
      FoldEnt ent[CL_LOCAL];
      unsigned long long key[FAST_CAND];
      float q[FAST_K];
      float stage[STAGE];
      int coff[CL_MAXC + 1];
      int ccnt[CL_MAXC + 1];
      int nent, ncand;
      int rep_fi[2];            // walk -> replay group: the entry to replay (-1: done), by parity
      uint32_t rep_s;           // the exact state at the start of a replay chunk
      int rcnt[CL_RPT * (CL_WARPS - 1)];  // kept elements per (element slot, group warp)
      float rstage[CL_RCH];     // a replay chunk's kept exps, in row order
    } f;
  } u;
};

// Named barrier of the leader's replay group (warps 0 and 2..7).
__device__ __forceinline__ void cl_rbar() { asm volatile("bar.sync 1, %0;" ::"n"(CL_RGRP) : "memory"); }

// Fold of the exps of the row's elements [from, to) from the exact state s
// (held by warp 0) by the replay group; the result is warp 0's.  Per chunk of
// CL_RCH elements every thread takes the exact exps of its elements.  An
// element whose addition leaves both an even and an odd state of the chunk's
// starting binade unchanged (its exp is below half that binade's ulp) is
// dropped: the state never decreases, so the exp stays below half the ulp
// of every binade the state can reach.  Warp 0 folds the rest in row order.
__device__ uint32_t cl_replay(const void* row, int dtype, uint32_t from, uint32_t to, uint32_t s, bool scale,
                              float T, float m, ClShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int gt = w == 0 ? lane : tid - 32;  // 0 .. CL_RGRP-1 in row order
  const int gw = gt >> 5;
  const uint32_t lt = (1u << lane) - 1u;
  for (uint32_t base = from; base < to; base += CL_RCH) {
    if (tid == 0) sh.u.f.rep_s = s;
    cl_rbar();
    const uint32_t lo = fold::binade_lo_bits(sh.u.f.rep_s);
    float e[CL_RPT];
    uint32_t bm[CL_RPT];
#pragma unroll
    for (int k = 0; k < CL_RPT; ++k) {
      const uint32_t idx = base + (uint32_t)(k * CL_RGRP + gt);
      const bool valid = idx < to;
      e[k] = 0.0f;
      if (valid) {
        const float xr = load_logit_dyn(row, dtype, (long long)idx);
        e[k] = pesti_expf_call(fsub(scale ? fdiv(xr, T) : xr, m));  // sampling.rs:46,127
      }
      const bool kept = valid && (fbits(fadd(bitsf(lo), e[k])) != lo || fbits(fadd(bitsf(lo + 1u), e[k])) != lo + 1u);
      bm[k] = __ballot_sync(PESTI_FULL_MASK, kept);
      if (lane == 0) sh.u.f.rcnt[k * (CL_WARPS - 1) + gw] = __popc(bm[k]);
    }
    cl_rbar();
    int off[CL_RPT], tot = 0;
#pragma unroll
    for (int k = 0; k < CL_RPT; ++k) off[k] = 0;
    for (int j = 0; j < CL_RPT * (CL_WARPS - 1); ++j) {
      const int c = sh.u.f.rcnt[j];
#pragma unroll
      for (int k = 0; k < CL_RPT; ++k) off[k] += j < k * (CL_WARPS - 1) + gw ? c : 0;
      tot += c;
    }
#pragma unroll
    for (int k = 0; k < CL_RPT; ++k)
      if ((bm[k] >> lane) & 1u) sh.u.f.rstage[off[k] + __popc(bm[k] & lt)] = e[k];
    cl_rbar();
    if (w == 0) s = warp_fold_staged(sh.u.f.rstage, tot, s);
  }
  return s;
}

// Candidate threshold: a lower bound of the keff-th largest raw logit, from
// the row's segment maxima (vals, NV per thread, -inf where none; maxima of
// disjoint segments are distinct elements).  A 256-bin histogram of their
// distance below the row max mx in units of t_eff/8 places the keff-th
// largest; the threshold lies two bins further down (one bin for the
// rounding of the distances), rounded toward -inf.  -inf when the first 255
// bins hold fewer than keff maxima.  Every thread calls it.
template <int NV>
__device__ float cl_tau(const float (&vals)[NV], float mx, float t_eff, long long keff, ClShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31;
  const float NEG_INF = -__int_as_float(0x7f800000);
  uint32_t* hist = sh.u.t.hist;
  for (int i = tid; i < 256; i += CL_NT) hist[i] = 0u;
  __syncthreads();
  const float inv = 8.0f / t_eff;
#pragma unroll
  for (int r = 0; r < NV; ++r) {
    const float v = vals[r];
    if (v > NEG_INF) {  // also false for NaN
      const float d = (mx - v) * inv;
      const uint32_t bin = d < 255.0f ? (uint32_t)d : 255u;
      atomicAdd(&hist[bin], 1u);
    }
  }
  __syncthreads();
  if (tid < 32) {
    uint32_t c8[8], lsum = 0u;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      c8[q] = lane * 8 + q < 255 ? hist[lane * 8 + q] : 0u;
      lsum += c8[q];
    }
    const uint32_t incl = warp_incl_scan_add(lsum);
    const uint32_t excl = incl - lsum;
    int bin = 1 << 30;
    if ((long long)excl < keff && (long long)incl >= keff) {
      uint32_t cum = excl;
      int q = 0;
      for (; q < 7; ++q) {
        if ((long long)(cum + c8[q]) >= keff) break;
        cum += c8[q];
      }
      bin = lane * 8 + q;
    }
    bin = __reduce_min_sync(PESTI_FULL_MASK, (uint32_t)bin);
    if (lane == 0)
      sh.u.t.tau = bin < 255 ? __fsub_rd(mx, __fmul_ru(t_eff, (float)(bin + 2) * 0.125f)) : NEG_INF;
  }
  __syncthreads();
  return sh.u.t.tau;
}

// Loads segment q of a warp's range (32*VE elements, VE per lane, in row
// order): one 16-byte load per lane when the segment is whole and the rows are
// 16-byte aligned, scalar loads otherwise (0 beyond the range, nv valid).
template <typename TIn, int VE, bool VEC>
__device__ __forceinline__ void cl_load(const TIn* row, long long pos0, long long end, float (&x)[VE], int& nv) {
  if (VEC && pos0 + VE <= end) {
    const float4 r4 = __ldg(reinterpret_cast<const float4*>(row + pos0));
    if (sizeof(TIn) == 4) {
      x[0] = r4.x; x[1] = r4.y; x[2] = r4.z; x[3] = r4.w;
    } else {
      const uint32_t wds[4] = {__float_as_uint(r4.x), __float_as_uint(r4.y), __float_as_uint(r4.z),
                               __float_as_uint(r4.w)};
#pragma unroll
      for (int h = 0; h < 4; ++h) unpack2<TIn>(wds[h], x[2 * h], x[2 * h + 1]);
    }
    nv = VE;
    return;
  }
  nv = 0;
#pragma unroll
  for (int e = 0; e < VE; ++e) {
    const bool in = pos0 + e < end;
    x[e] = in ? load_logit<TIn>(row, pos0 + e) : 0.0f;
    nv = in ? e + 1 : nv;
  }
}

__device__ __forceinline__ void cl_write_pad(const ClusterArgs& a, long long b, long long from) {
  for (long long j = from + (threadIdx.x & 31); j < a.kept_width; j += 32) {
    if (a.kept_p) a.kept_p[b * a.kept_width + j] = 0.0f;
    if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = 0xffffffffu;
  }
}

template <typename TIn, int VE, bool VEC>
__global__ void __launch_bounds__(CL_NT, 4) row_cluster_kernel(ClusterArgs a) {
  __shared__ __align__(16) ClShared sh;
  cg::cluster_group cl = cg::this_cluster();
  const int C = (int)cl.num_blocks();
  const int cr = (int)cl.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const long long b = blockIdx.x / C;
  if (a.early_dependents) grid_dep_launch_next();
  const long long V = a.V;
  const pesti_sampling_params prm = row_params(a.uni, a.per_row, b);
  const float T = prm.temperature;
  const bool scale = T > 0.0f;
  const float t_eff = scale ? T : 1.0f;
  const float NEG_INF = -__int_as_float(0x7f800000), INF = __int_as_float(0x7f800000);
  const bool greedy = is_greedy(prm);
  const TIn* row = (const TIn*)a.logits + b * a.ld;
  constexpr int SEG = 32 * VE;
  const int g = cr * CL_WARPS + w;  // the warp's place in the row
  const long long s0 = a.wstart[g];
  const long long s1 = a.wstart[g + 1];
  const int nseg = s0 < V ? (int)((s1 - s0 + SEG - 1) / SEG) : 0;
  const float c2 = 1.4426950408889634f / t_eff;

  // ---------------- pass 1: the HBM stream ----------------
  {
    float lmax = NEG_INF;   // lane: max of its elements
    float lmin = INF;       // and min
    float gmax = NEG_INF;   // greedy rows: the lane's max, with its indices
    uint32_t lflags = 0u;
    int lnan = -1, lfirst = -1, llast = -1;
    // whole segments of aligned rows stream through a ring of CL_P1S
    // segments per warp (cp.async, each lane its own 16 bytes), so that the
    // next segments' loads are in flight while one is processed
    const int nfull1 = VEC ? (int)((s1 - s0) / SEG) : 0;
    float4* ring = sh.u.r.ring[w];
    if (VEC) {
#pragma unroll
      for (int st = 0; st < CL_P1S; ++st) {
        if (st < nfull1) cp_async16(&ring[st * 32 + lane], row + s0 + (long long)st * SEG + lane * VE);
        cp_async_commit();
      }
    }
    for (int q0 = 0; q0 < nseg; q0 += CL_U) {
      float x[CL_U][VE];
      int nv[CL_U];
#pragma unroll
      for (int uu = 0; uu < CL_U; ++uu) {
        const int q = q0 + uu;
        nv[uu] = 0;
        if (VEC && q < nfull1) {
          cp_async_wait<CL_P1S - 1>();  // segment q has arrived
          const float4 r4 = ring[(q % CL_P1S) * 32 + lane];
          if (sizeof(TIn) == 4) {
            x[uu][0] = r4.x; x[uu][1] = r4.y; x[uu][2] = r4.z; x[uu][3] = r4.w;
          } else {
            const uint32_t wds[4] = {__float_as_uint(r4.x), __float_as_uint(r4.y), __float_as_uint(r4.z),
                                     __float_as_uint(r4.w)};
#pragma unroll
            for (int h = 0; h < 4; ++h) unpack2<TIn>(wds[h], x[uu][2 * h], x[uu][2 * h + 1]);
          }
          nv[uu] = VE;
          const int qn = q + CL_P1S;  // the slot just read takes segment q + CL_P1S
          if (qn < nfull1) cp_async16(&ring[(q % CL_P1S) * 32 + lane], row + s0 + (long long)qn * SEG + lane * VE);
          cp_async_commit();
        } else if (q < nseg) {
          cl_load<TIn, VE, VEC>(row, s0 + (long long)q * SEG + lane * VE, s1, x[uu], nv[uu]);
        }
      }
      float lsu[CL_U];  // the lane's part of each segment's mass
#pragma unroll
      for (int uu = 0; uu < CL_U; ++uu) {
        lsu[uu] = 0.0f;
        if (q0 + uu >= nseg) continue;
        const long long p0 = s0 + (long long)(q0 + uu) * SEG + lane * VE;
        float smax = NEG_INF;
        if (nv[uu] == VE) {
          // a whole lane: fmaxf/fminf skip NaN (as f32::max does), the
          // infinities show in the lane's max and min, NaN in one flag
          float smin = INF;
          bool nan = false;
#pragma unroll
          for (int e = 0; e < VE; ++e) {
            const float v = x[uu][e];
            smax = fmaxf(smax, v);
            smin = fminf(smin, v);
            nan = nan || is_nan(v);
          }
          lmin = fminf(lmin, smin);
          lflags |= (smax == INF ? MF_POSINF : 0u) | (smin == NEG_INF ? MF_NEGINF : 0u);
          if (nan) {  // rare: the flag and the last NaN's index
            lflags |= MF_NAN;
#pragma unroll
            for (int e = 0; e < VE; ++e) lnan = is_nan(x[uu][e]) ? (int)(p0 + e) : lnan;
          }
        } else {
#pragma unroll
          for (int e = 0; e < VE; ++e) {
            const float v = x[uu][e];
            const bool in = e < nv[uu];
            const bool nan = in && is_nan(v);
            const bool ok = in && !nan;
            lflags |= (nan ? MF_NAN : 0u) | (ok && v == INF ? MF_POSINF : 0u) | (ok && v == NEG_INF ? MF_NEGINF : 0u);
            lnan = nan ? (int)(p0 + e) : lnan;
            smax = fmaxf(smax, ok ? v : NEG_INF);
            lmin = fminf(lmin, ok ? v : INF);
          }
        }
        if (greedy) {  // first and last index of the lane's max so far (greedy is row-uniform)
#pragma unroll
          for (int e = 0; e < VE; ++e) {
            const float v = x[uu][e];
            if (e < nv[uu] && !is_nan(v)) {
              if (lfirst < 0 || v > gmax) {
                gmax = v;
                lfirst = (int)(p0 + e);
                llast = lfirst;
              } else if (v == gmax) {
                llast = (int)(p0 + e);
              }
            }
          }
        }
        // the segment's max (every lane's keys; NaN never reaches smax) and
        // its approximate mass relative to that max: sum of 2^(x*c2 - max*c2)
        const float segm = fkey_inv(__reduce_max_sync(PESTI_FULL_MASK, fkey(smax)));
        lmax = fmaxf(lmax, smax);
        float ls = 0.0f;
        if (segm > NEG_INF && segm < INF) {
          const float ym = segm * c2;
#pragma unroll
          for (int e = 0; e < VE; ++e)
            if (e < nv[uu] && !is_nan(x[uu][e])) ls += ex2_approx(fmaf(x[uu][e], c2, -ym));
        }
        lsu[uu] = ls;
        if (lane == 0) sh.segmax[w][q0 + uu] = segm;
      }
      // the CL_U masses summed over the lanes together: halves of the values
      // are exchanged (lane bit 4, then bit 3), then each lane's one value is
      // reduced over the 8 lanes that share it; lane 8*uu ends with mass uu
      static_assert(CL_U == 4, "the transposed reduction takes four values");
      {
        const bool h16 = (lane & 16) != 0, h8 = (lane & 8) != 0;
        const float k0 = h16 ? lsu[2] : lsu[0], k1 = h16 ? lsu[3] : lsu[1];
        const float s0v = h16 ? lsu[0] : lsu[2], s1v = h16 ? lsu[1] : lsu[3];
        const float b0 = k0 + __shfl_xor_sync(PESTI_FULL_MASK, s0v, 16);
        const float b1 = k1 + __shfl_xor_sync(PESTI_FULL_MASK, s1v, 16);
        float c = (h8 ? b1 : b0) + __shfl_xor_sync(PESTI_FULL_MASK, h8 ? b0 : b1, 8);
        c += __shfl_xor_sync(PESTI_FULL_MASK, c, 4);
        c += __shfl_xor_sync(PESTI_FULL_MASK, c, 2);
        c += __shfl_xor_sync(PESTI_FULL_MASK, c, 1);
        const int uu = lane >> 3;  // (bit 4, bit 3) = the value's index
        if ((lane & 7) == 0 && q0 + uu < nseg) sh.segmass[w][q0 + uu] = c;
      }
    }
    if (VEC) cp_async_wait<0>();  // the ring's last (empty) groups; its space is reused after pass 1
    for (int q = nseg + lane; q < CL_SEGS; q += 32) {
      sh.segmax[w][q] = NEG_INF;
      sh.segmass[w][q] = 0.0f;
    }
    __syncwarp();
    // the warp's summary: its max, and its mass relative to it (an infinite
    // row is uniform, its mass is never used)
    const float wmax = fkey_inv(__reduce_max_sync(PESTI_FULL_MASK, fkey(lmax)));
    float part = 0.0f;
    if (lane < nseg && wmax < INF) {
      const float sq = sh.segmax[w][lane];
      if (sq > NEG_INF) part = sh.segmass[w][lane] * ex2_approx(fmaf(sq, c2, -wmax * c2));
    }
    const float wsum = warp_reduce_add(part);
    const uint32_t wfl = __reduce_or_sync(PESTI_FULL_MASK, lflags);
    const int wnan = (int)__reduce_max_sync(PESTI_FULL_MASK, (uint32_t)(lnan + 1)) - 1;
    int wfirst = -1, wlast = -1;
    if (greedy) {
      // first / last index of the warp's max (the lanes' own maxima may be lower)
      const bool mine = gmax == wmax && lfirst >= 0;
      wfirst = (int)__reduce_min_sync(PESTI_FULL_MASK, mine ? (uint32_t)lfirst : 0xffffffffu);
      wlast = (int)__reduce_max_sync(PESTI_FULL_MASK, mine ? (uint32_t)(llast + 1) : 0u) - 1;
      if (wfirst == (int)0xffffffff) wfirst = -1;
    }
    const float wmin = -fkey_inv(__reduce_max_sync(PESTI_FULL_MASK, fkey(-lmin)));
    if (lane == 0) sh.wst[w] = ClWarp{wmax, wsum, wnan, wfl, wfirst, wlast, wmin, 0};
  }
  cl.sync();

  // ---------------- combine: the row prologue, in every CTA ----------------
  const int NWR = C * CL_WARPS;
  ClWarp rw{NEG_INF, 0.0f, -1, 0u, -1, -1, INF, 0};
  if (tid < NWR) rw = *cl.map_shared_rank(&sh.wst[tid % CL_WARPS], tid / CL_WARPS);
  // every segment max of the row (for the candidate threshold), fetched now
  constexpr int NV = CL_MAXC * CL_WARPS * CL_SEGS / CL_NT;
  float vals[NV];
#pragma unroll
  for (int r = 0; r < NV; ++r) {
    const int i = r * CL_NT + tid;
    const int wi = i / CL_SEGS;
    vals[r] = wi < NWR ? *cl.map_shared_rank(&sh.segmax[wi % CL_WARPS][i % CL_SEGS], wi / CL_WARPS) : NEG_INF;
  }
  // row max, flags, last NaN
  uint32_t mk = __reduce_max_sync(PESTI_FULL_MASK, fkey(rw.max_raw));
  uint32_t fo = __reduce_or_sync(PESTI_FULL_MASK, rw.flags);
  uint32_t ln = __reduce_max_sync(PESTI_FULL_MASK, (uint32_t)(rw.last_nan + 1));
  uint32_t mn = __reduce_max_sync(PESTI_FULL_MASK, fkey(-rw.min_raw));
  if (lane == 0) {
    sh.uscr[w] = mk;
    sh.uscr[16 + w] = mn;
    sh.iscr[w] = (int)fo;
    sh.iscr[8 + w] = (int)ln;
  }
  __syncthreads();
  mk = 0u;
  fo = 0u;
  ln = 0u;
  mn = 0u;
  for (int q = 0; q < CL_WARPS; ++q) {
    mk = mk > sh.uscr[q] ? mk : sh.uscr[q];
    mn = mn > sh.uscr[16 + q] ? mn : sh.uscr[16 + q];
    fo |= (uint32_t)sh.iscr[q];
    ln = ln > (uint32_t)sh.iscr[8 + q] ? ln : (uint32_t)sh.iscr[8 + q];
  }
  const float mnv = -fkey_inv(mn);  // row min (NaN ignored)
  const float mx = fkey_inv(mk);
  const uint32_t fl = fo;
  const int last_nan = (int)ln - 1;
  int first_max = -1, last_max = -1;
  if (greedy) {
    const bool hold = tid < NWR && rw.max_raw == mx && rw.first_max >= 0;
    uint32_t fm = __reduce_min_sync(PESTI_FULL_MASK, hold ? (uint32_t)rw.first_max : 0xffffffffu);
    uint32_t lm = __reduce_max_sync(PESTI_FULL_MASK, hold ? (uint32_t)(rw.last_max + 1) : 0u);
    __syncthreads();
    if (lane == 0) {
      sh.uscr[w] = fm;
      sh.uscr[8 + w] = lm;
    }
    __syncthreads();
    fm = 0xffffffffu;
    lm = 0u;
    for (int q = 0; q < CL_WARPS; ++q) {
      fm = fm < sh.uscr[q] ? fm : sh.uscr[q];
      lm = lm > sh.uscr[8 + q] ? lm : sh.uscr[8 + q];
    }
    first_max = fm == 0xffffffffu ? -1 : (int)fm;
    last_max = (int)lm - 1;
  }
  const float m = scale ? fdiv(mx, T) : mx;  // sampling.rs:46 on the max element
  const bool uniform = (fl & MF_NAN) || (scale && T == INF && (fl & (MF_POSINF | MF_NEGINF))) ||
                       !(fabsf(m) < INF);
  const long long k = (long long)prm.top_k;
  const long long keff = k < V ? k : V;
  const bool fast = !greedy && !uniform && fast_topk(prm, V);
  // top-p rows of bf16 logits: the cluster folds S exactly, the row kernel
  // takes their sorted folds by distinct values (pesti_nucleus.cuh)
  const bool nuc = a.nucleus && !greedy && !uniform && a.dtype == PESTI_BF16 && prm.top_k == 0u && prm.top_p > 0.0f;
  // greedy rows are finished here (NaN rows with the last-index rule go to
  // the row kernel, which re-scans after the last NaN as max_by does)
  int decided = -1;  // 0: sampled here, 1: fallback
  if (greedy) decided = ((fl & MF_NAN) && !(prm.flags & PESTI_FLAG_ARGMAX_FIRST)) ? 1 : 0;
  else if (!fast && !nuc) decided = 1;

  float tau = INF;
  if (decided < 0) {
    // prefix mass and prefix max of the warps (exclusive, in row order)
    const float ym = mx * c2;
    // (float exp2 within 2 ulp: the pruning's lower bound keeps a 2^-10 slack)
    const double mass = (tid < NWR && rw.max_raw > NEG_INF) ? (double)(exp2f(rw.max_raw * c2 - ym) * rw.sum_rel) : 0.0;
    double tot;
    const double A = block_excl_scan_add(mass, sh.dscr, tot);
    float inc = tid < NWR ? rw.max_raw : NEG_INF;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(PESTI_FULL_MASK, inc, o);
      if (lane >= o) inc = fmaxf(inc, y);
    }
    if (lane == 31) sh.fscr[w] = inc;
    __syncthreads();
    float pm = NEG_INF;
    for (int q = 0; q < w; ++q) pm = fmaxf(pm, sh.fscr[q]);
    float exc = __shfl_up_sync(PESTI_FULL_MASK, inc, 1);
    if (lane == 0) exc = NEG_INF;
    pm = fmaxf(pm, exc);
    if (tid < NWR && tid / CL_WARPS == cr) {
      const int wl = tid % CL_WARPS;
      sh.A[wl] = A;
      sh.P[wl] = pm;
      // bound (b) of the pruning, in raw units (derivation at row_prologue):
      // L <= the running sum, t = m + ln(L) - 17.36, rounded toward -inf
      const double lfac = (1.0 - (double)V * 0x1p-24) * (1.0 - 0x1p-10) * exp2(-0x1p-20 * ((double)fabsf(ym) + 64.0));
      const double L = A * lfac;
      float thr = NEG_INF;
      if (L >= 0x1p-60) {
        const double tL = (double)m + log(L) - 17.36;
        const double eta = 0x1p-20 * (fabs(tL) + fabs((double)m) + 1.0);
        thr = __double2float_rd((tL - eta) * (double)t_eff);
      }
      sh.thrL[wl] = thr;
    }
    // candidate threshold from every segment max of the row (none for top-p rows)
    tau = nuc ? INF : cl_tau<NV>(vals, mx, t_eff, keff, sh);
    if (tid == 0) {
      sh.tau = tau;
      sh.e_tau = tau > NEG_INF && tau < INF ? pesti_expf_call(fsub(scale ? fdiv(tau, T) : tau, m)) : 0.0f;
      sh.ncand = 0;
    }
    __syncthreads();  // the histogram's space becomes the survivor rings
  }
  if (cr == 0 && tid == 0) {
    sh.max_raw = mx;
    sh.m = m;
    sh.flags = fl;
    sh.last_nan = last_nan;
    sh.first_max = first_max;
    sh.last_max = last_max;
    sh.min_raw = mnv;
  }

  // ---------------- pass 2: fold entries and candidates ----------------
  // Segment by segment in row order, with the approximate fold state s_run
  // (the mass of the row before the segment, from pass 1).  A segment whose
  // whole state range lies inside one binade, away from its edges, with no
  // element large next to the state, adds rint(e/w) per element (w the
  // binade's ulp): the approximate exps decide those increments with a proven
  // margin, the exact exp is taken where they do not, and consecutive such
  // segments of one binade form one run.  Any other segment goes element by
  // element (its survivors of the pruning, with their own approximate states).
  if (decided < 0) {
    const float c1 = ABSORB * t_eff * (1.0f + 0x1p-20f);
    const float pf = (m - PRUNE_FLOOR) * t_eff;
    const float p_floor = pf + 0x1p-20f * fabsf(pf);
    auto bound_a = [&](float Pv) { return Pv >= p_floor ? fsub(Pv, fadd(c1, 0x1p-21f * fabsf(Pv))) : NEG_INF; };
    const float ym = mx * c2;
    const double lfac = (1.0 - (double)V * 0x1p-24) * (1.0 - 0x1p-10) * exp2(-0x1p-20 * ((double)fabsf(ym) + 64.0));
    // bound (b) from a lower bound L of the running sum (derivation at
    // row_prologue): raw logits below it leave every later state unchanged
    auto bound_b = [&](double L) {
      float thr = NEG_INF;
      if (L >= 0x1p-60) {
        const double tL = (double)m + log(L) - 17.36;
        const double eta = 0x1p-20 * (fabs(tL) + fabs((double)m) + 1.0);
        thr = __double2float_rd((tL - eta) * (double)t_eff);
      }
      return thr;
    };
    const float rT = scale ? 1.0f / T : 1.0f;  // the approximate argument x*rT - m (margins below)
    float thr_b = sh.thrL[w];
    float run_max = sh.P[w];
    const float BAND = a.band;
    float* qraw = sh.u.c.qraw[w];
    uint32_t* qidx = sh.u.c.qidx[w];
    FoldEnt* went = sh.u.c.went[w];
    float4* stg = sh.u.c.stg[w];
    double s_run = sh.A[w];       // approximate fold state before the next segment
    double s_thr = s_run;         // the state bound (b) was last taken at
    int wn = 0;                   // entries written
    bool over = false;            // entries overflowed: the walk replays the range
    uint32_t lkey = KEY_NONE;     // key of the last entry written
    uint32_t pkey = KEY_NONE;     // the open run of whole segments (its binade), not yet written
    uint32_t pk = 0u;             // its increment, this lane's part
    uint32_t pend = 0u;           // the row index past its last element

    // the open run becomes an entry (or extends the last one, of the same binade)
    auto flush = [&]() {
      if (pkey == KEY_NONE) return;
      const uint32_t ks = tr_sat(warp_reduce_add(pk));
      if (lkey == pkey) {
        if (lane == 0) {
          const FoldEnt pe = went[wn - 1];
          went[wn - 1] = FoldEnt{pkey, tr_sat(pe.a0 + ks), tr_sat(pe.a1 + ks), pend};
        }
      } else {
        if (lane == 0 && wn < CL_EW) went[wn] = FoldEnt{pkey, ks, ks, pend};
        ++wn;
        if (wn > CL_EW) over = true;
      }
      lkey = pkey;
      pkey = KEY_NONE;
      pk = 0u;
    };

    const int nfull = VEC ? (int)((s1 - s0) / SEG) : 0;  // whole segments, staged through shared memory
    if (VEC) {
#pragma unroll
      for (int st = 0; st < CL_STAGES; ++st) {
        if (st < nfull) cp_async16(&stg[st * 32 + lane], row + s0 + (long long)st * SEG + lane * VE);
        cp_async_commit();
      }
    }
#pragma unroll 1
    for (int q = 0; q < nseg; ++q) {
      float x[VE];
      int nv;
      const long long p0 = s0 + (long long)q * SEG + lane * VE;
      const bool piped = VEC && q < nfull;
      if (piped) {
        cp_async_wait<CL_STAGES - 1>();  // segment q has arrived (each lane reads its own bytes)
        const float4 r4 = stg[(q % CL_STAGES) * 32 + lane];
        if (sizeof(TIn) == 4) {
          x[0] = r4.x; x[1] = r4.y; x[2] = r4.z; x[3] = r4.w;
        } else {
          const uint32_t wds[4] = {__float_as_uint(r4.x), __float_as_uint(r4.y), __float_as_uint(r4.z),
                                   __float_as_uint(r4.w)};
#pragma unroll
          for (int h = 0; h < 4; ++h) unpack2<TIn>(wds[h], x[2 * h], x[2 * h + 1]);
        }
        nv = VE;
      } else {
        cl_load<TIn, VE, false>(row, p0, s1, x, nv);
      }
      if (piped) {  // the stage just read takes segment q + CL_STAGES
        const int qn = q + CL_STAGES;
        if (qn < nfull) cp_async16(&stg[(q % CL_STAGES) * 32 + lane], row + s0 + (long long)qn * SEG + lane * VE);
        cp_async_commit();
      }
      const float segm = sh.segmax[w][q];
      // top-k candidates (raw >= tau; their exact exps, sampling.rs:127)
      int nc = 0;
#pragma unroll
      for (int e = 0; e < VE; ++e) nc += (e < nv && x[e] >= tau) ? 1 : 0;
      if (__any_sync(PESTI_FULL_MASK, nc > 0)) {
        const int cin = warp_incl_scan_add(nc);
        int cb = 0;
        if (lane == 31) cb = atomicAdd(&sh.ncand, cin);
        cb = __shfl_sync(PESTI_FULL_MASK, cb, 31) + cin - nc;
        uint32_t cm = 0u;
#pragma unroll
        for (int e = 0; e < VE; ++e) cm |= (e < nv && x[e] >= tau) ? (1u << e) : 0u;
#pragma unroll 1
        for (; cm != 0u; cm &= cm - 1u, ++cb) {
          const int e = __ffs(cm) - 1;
          float xv = x[0];
#pragma unroll
          for (int r2 = 1; r2 < VE; ++r2) xv = e == r2 ? x[r2] : xv;
          if (cb < CL_CCAP) {
            sh.cand_e[cb] = pesti_expf_call(fsub(scale ? fdiv(xv, T) : xv, m));
            sh.cand_i[cb] = (uint32_t)(p0 + e);
          }
        }
      }
      // the segment's largest exp and its mass, relative to the row max
      const float emx = segm > NEG_INF ? ex2_approx(fmaf(segm, c2, -ym)) : 0.0f;
      const float smass = emx * sh.segmass[w][q];
      if (over) {
        s_run += (double)smass;
        continue;
      }
      const float sb = (float)s_run;
      bool done = false;
      if (sb >= 0x1p-126f) {
        const uint32_t lo = fbits(sb) & 0x7f800000u;
        const float lov = bitsf(lo);
        if (sb >= lov * (1.0f + BAND) && sb + smass * (1.0f + 0x1p-14f) <= 2.0f * lov * (1.0f - BAND) &&
            emx * (1.0f + 0x1p-14f) < 0.5f * lov) {
          // plain increments: rint(e/w) from the approximate exp where its
          // margin decides it.  Against the exact exp of the reference's
          // argument z = fl(fl(x/T) - m), exp_hw(fl(x*rT - m)) is within
          // DE_0/2 + DE_Z*(|x*rT| + 1.5|z'|) relative; the test keeps twice that.
          const uint32_t E = lo >> 23;
          const uint32_t sc = (uint32_t)(150 - (int)E) << 23;  // e/w = e * 2^(150-E)
          uint32_t kseg = 0u, und = 0u;  // und: elements the approximation leaves undecided
          // branch-free per element: an exp that flushed to 0 is an exact
          // value below 2^-126, which rounds to 0 on a grid of E >= 40
#pragma unroll
          for (int e = 0; e < VE; ++e) {
            const float xv = x[e];
            const float zq = fmaf(xv, rT, -m);  // rT = 1 for unscaled rows: exactly fl(x - m)
            const float ea = exp_hw(zq);
            const float tt = __uint_as_float(fbits(ea) + sc);
            uint32_t kd;
            const float kr = rint_small(tt, kd);
            const float de = fmaf(arg_margin(xv, rT, zq), DE_Z, DE_0);
            const bool in = e < nv;
            const bool dec = ea != 0.0f && tt < 0x1p22f && 0.5f - fabsf(tt - kr) > tt * de + 0x1p-24f;
            const bool zero = ea == 0.0f && E >= 40u;
            kseg += in && dec ? kd : 0u;
            und |= in && !dec && !zero ? (1u << e) : 0u;
          }
          bool tie = false;
#pragma unroll 1
          for (uint32_t mm = und; mm != 0u; mm &= mm - 1u) {
            const int e = __ffs(mm) - 1;
            float xv = x[0];
#pragma unroll
            for (int r2 = 1; r2 < VE; ++r2) xv = e == r2 ? x[r2] : xv;
            const float ex = pesti_expf_call(fsub(scale ? fdiv(xv, T) : xv, m));  // sampling.rs:46,127
            const uint32_t k0 = fbits(fadd(lov, ex)) - lo;
            const uint32_t k1 = fbits(fadd(bitsf(lo + 1u), ex)) - (lo + 1u);
            tie = tie || k0 != k1;
            kseg += k0;
          }
          if (!__any_sync(PESTI_FULL_MASK, tie)) {
            if (pkey != lo) {
              flush();
              pkey = lo;
            }
            pk += kseg;
            pend = (uint32_t)(s0 + (long long)q * SEG + SEG < s1 ? s0 + (long long)q * SEG + SEG : s1);
            done = true;
          }
        }
      }
      if (!done) {
        flush();
        // a segment whose entries would overflow the warp's list (explicit
        // elements near a binade edge) is rolled back and refolded by the walk
        // from its raw logits instead: its entries, and the last entry before
        // it (which its first run may extend), are kept aside
        const int wn0 = wn;
        const uint32_t lkey0 = lkey;
        FoldEnt prev0{0u, 0u, 0u, 0u};
        if (wn0 > 0 && wn0 <= CL_EW) prev0 = went[wn0 - 1];
        // element by element: the survivors of the pruning, in row order
        if (s_run >= 2.0 * s_thr && s_run > 0.0) {  // bound (b) again once the state has doubled
          float tb = 0.0f;
          if (lane == 0) tb = bound_b(s_run * lfac);
          thr_b = fmaxf(thr_b, __shfl_sync(PESTI_FULL_MASK, tb, 0));
          s_thr = s_run;
        }
        const float thr = fmaxf(bound_a(run_max), thr_b);
        // survivors into the ring in row order: parts of 128 elements (all
        // of the lanes [ph*LPP, (ph+1)*LPP))
        constexpr int NPART = VE / 4;
        constexpr int LPP = 32 / NPART;
        uint32_t sv = 0u;
#pragma unroll
        for (int e = 0; e < VE; ++e) sv |= (e < nv && x[e] >= thr) ? (1u << e) : 0u;
        uint32_t tail = 0u;
#pragma unroll
        for (int ph = 0; ph < NPART; ++ph) {
          const bool mine = lane / LPP == ph;
          const int cnt = mine ? __popc(sv) : 0;
          const int sin = warp_incl_scan_add(cnt);
          const int tot = __shfl_sync(PESTI_FULL_MASK, sin, 31);
          uint32_t o = tail + (uint32_t)(sin - cnt);
          if (mine) {
#pragma unroll
            for (int e = 0; e < VE; ++e) {
              if (sv & (1u << e)) {
                qraw[o] = x[e];
                qidx[o] = (uint32_t)(p0 + e);
                ++o;
              }
            }
          }
          tail += (uint32_t)tot;
        }
        __syncwarp();
        // 32 survivors at a time: each element's approximate state decides a
        // run of its binade or an explicit element (near a binade edge, or
        // large next to the state); runs are summed over the lanes (composed
        // when some element is a tie)
        float sbj = sb;
        const int n = (int)tail;
#pragma unroll 1
        for (int j = 0; j * 32 < n && !over; ++j) {
          const int i = j * 32 + lane;
          const int nj = n - j * 32 < 32 ? n - j * 32 : 32;
          const bool valid = i < n;
          const float raw = valid ? qraw[i] : 0.0f;
          const uint32_t idx = valid ? qidx[i] : 0u;
          // the approximate argument x*rT - m (its margin in dej); the exact
          // z = fl(fl(x/T) - m) (sampling.rs:46,127) only where an exact exp is taken
          const float zq = valid ? fmaf(raw, rT, -m) : 0.0f;  // rT = 1 for unscaled rows: exactly fl(x - m)
          const float eaj = valid ? exp_hw(zq) : 0.0f;
          const float incl = warp_incl_scan_add(eaj);
          float excl = __shfl_up_sync(PESTI_FULL_MASK, incl, 1);
          if (lane == 0) excl = 0.0f;
          const float av = sbj + excl;  // approximate state before the element
          const float bv = av + eaj;    // and after it
          const float dej = fmaf(arg_margin(raw, rT, zq), DE_Z, DE_0);
          uint32_t key = KEY_NONE, k0 = 0u, k1 = 0u;
          if (valid) {
            bool special = !(av >= 0x1p-126f);
            uint32_t lo = 0u;
            float lov = 0.0f;
            if (!special) {
              lo = fbits(av) & 0x7f800000u;
              lov = bitsf(lo);
              special = eaj * (1.0f + dej) >= 0.5f * lov || av < lov * (1.0f + BAND) ||
                        bv > 2.0f * lov * (1.0f - BAND);
            }
            bool need = special;
            if (!special) {
              const uint32_t E = lo >> 23;
              if (eaj == 0.0f) {
                need = E < 40u;  // else the exact value (< 2^-126) rounds to 0 on this grid
              } else {
                const float tt = __uint_as_float(fbits(eaj) + ((uint32_t)(150 - (int)E) << 23));  // ea/w
                uint32_t kq;
                const float kr = rint_small(tt, kq);
                need = !(tt < 0x1p22f && 0.5f - fabsf(tt - kr) > tt * dej + 0x1p-24f);
                k0 = k1 = kq;
              }
            }
            if (need) {
              const float zj = fsub(scale ? fdiv(raw, T) : raw, m);  // sampling.rs:46,127
              const float ex = pesti_expf_call(zj);                   // exact
              if (special) {
                k0 = fbits(ex);
              } else {
                k0 = fbits(fadd(lov, ex)) - lo;
                k1 = fbits(fadd(bitsf(lo + 1u), ex)) - (lo + 1u);
              }
            }
            key = special ? fold::SPECIAL : lo;
          }
          uint32_t pky = __shfl_up_sync(PESTI_FULL_MASK, key, 1);
          if (lane == 0) pky = lkey;
          const bool hd = valid && (key == fold::SPECIAL || pky == fold::SPECIAL || pky == KEY_NONE || key != pky);
          // lane 0 may continue the warp's last entry (a run of the same binade)
          const bool cont = __shfl_sync(PESTI_FULL_MASK, valid && !hd, 0);
          const bool nhd = __shfl_down_sync(PESTI_FULL_MASK, hd, 1);
          const bool is_end = valid && (lane == nj - 1 || nhd);
          const uint32_t ends = __ballot_sync(PESTI_FULL_MASK, is_end);
          const int base = cont ? wn - 1 : wn;
          const int slot = base + __popc(ends & ((1u << lane) - 1u));
          const bool tie = valid && key != fold::SPECIAL && k0 != k1;
          if (!__any_sync(PESTI_FULL_MASK, tie)) {
            // plain integer increments: a run is a difference of prefix sums
            const uint32_t H = __ballot_sync(PESTI_FULL_MASK, hd || lane == 0);
            const uint32_t kk = valid && key != fold::SPECIAL ? k0 : 0u;
            const uint32_t scn = warp_incl_scan_add(kk);
            const int st = 31 - __clz(H & (0xffffffffu >> (31 - lane)));  // the run's first lane
            const uint32_t pre = __shfl_sync(PESTI_FULL_MASK, scn, st > 0 ? st - 1 : 0);
            const uint32_t run = tr_sat(scn - (st > 0 ? pre : 0u));
            if (is_end && slot < CL_EW) {
              if (key == fold::SPECIAL) {
                went[slot] = FoldEnt{key, k0, 0u, idx + 1u};
              } else if (st == 0 && cont) {
                const FoldEnt pe = went[slot];
                went[slot] = FoldEnt{key, tr_sat(pe.a0 + run), tr_sat(pe.a1 + run), idx + 1u};
              } else {
                went[slot] = FoldEnt{key, run, run, idx + 1u};
              }
            }
          } else {
            // some element is a tie: compose the (even, odd) increments
            Seg v{k0, k1, 1u, key};
            if (cont && lane == 0) {
              const FoldEnt pe = went[wn - 1];
              const Tr t = tr_compose(Tr{pe.a0, pe.a1}, Tr{k0, k1});
              v = Seg{t.a0, t.a1, 1u, key};
            }
            Seg inc = v;
            bool flg = hd || lane == 0;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
              const Seg o2 = seg_shfl_up(inc, off);
              const bool of = __shfl_up_sync(PESTI_FULL_MASK, flg, off);
              if (lane >= off) {
                inc = seg_join(o2, inc, flg);
                flg = flg || of;
              }
            }
            if (is_end && slot < CL_EW) went[slot] = FoldEnt{key, inc.a0, inc.a1, idx + 1u};
          }
          wn = base + __popc(ends);
          if (wn > CL_EW) over = true;
          lkey = __shfl_sync(PESTI_FULL_MASK, key, nj - 1);
          sbj += __shfl_sync(PESTI_FULL_MASK, incl, 31);
          __syncwarp();
        }
        if (over && wn0 < CL_EW) {
          const uint32_t seg_end = (uint32_t)(s0 + (long long)q * SEG + SEG < s1 ? s0 + (long long)q * SEG + SEG : s1);
          if (lane == 0) {
            if (wn0 > 0) went[wn0 - 1] = prev0;
            went[wn0] = FoldEnt{ENT_REPLAY, 0u, 0u, seg_end};
          }
          __syncwarp();
          wn = wn0 + 1;
          lkey = ENT_REPLAY;
          over = false;
        }
        (void)lkey0;
      }
      run_max = fmaxf(run_max, segm);
      s_run += (double)smass;
    }
    if (!over) flush();
    if (VEC) cp_async_wait<0>();
    if (lane == 0) sh.wn[w] = over ? -1 : wn;
  }
  __syncthreads();

  // ---------------- the CTA's entries, merged, in row order ----------------
  if (decided < 0 && tid == 0) {
    // the warps of repl (a bit mask) and the warps that overflowed become one
    // replay marker each; false when the merged list does not fit
    int nl = 0;
    auto merge = [&](uint32_t repl) -> bool {
      nl = 0;
      uint32_t last = KEY_NONE;
      for (int q = 0; q < CL_WARPS; ++q) {
        const long long ws0 = a.wstart[cr * CL_WARPS + q];
        if (ws0 >= V) break;
        const int n = sh.wn[q];
        if (n < 0 || ((repl >> q) & 1u)) {
          const long long we = a.wstart[cr * CL_WARPS + q + 1];
          if (last == ENT_REPLAY) {
            sh.list[nl - 1].end = (uint32_t)we;
          } else {
            if (nl >= CL_LIST) return false;
            sh.list[nl++] = FoldEnt{ENT_REPLAY, 0u, 0u, (uint32_t)we};
          }
          last = ENT_REPLAY;
          continue;
        }
        for (int i = 0; i < n; ++i) {
          const FoldEnt e = sh.u.c.went[q][i];
          if (e.lo != fold::SPECIAL && e.lo == last) {
            const Tr t = tr_compose(Tr{sh.list[nl - 1].a0, sh.list[nl - 1].a1}, Tr{e.a0, e.a1});
            sh.list[nl - 1] = FoldEnt{e.lo, t.a0, t.a1, e.end};
          } else {
            if (nl >= CL_LIST) return false;
            sh.list[nl++] = e;
          }
          last = e.lo;
        }
      }
      return true;
    };
    // too many entries: the warps with the most entries are replayed in the
    // walk instead, one at a time, until the list fits
    uint32_t repl = 0u;
    while (!merge(repl)) {
      int best = -1, bn = 0;
      for (int q = 0; q < CL_WARPS; ++q)
        if (!((repl >> q) & 1u) && sh.wn[q] > bn) {
          bn = sh.wn[q];
          best = q;
        }
      if (best < 0) {  // cannot happen (CL_WARPS markers fit): the whole range
        sh.list[0] = FoldEnt{ENT_REPLAY, 0u, 0u, (uint32_t)a.wstart[(cr + 1) * CL_WARPS]};
        nl = 1;
        break;
      }
      repl |= 1u << best;
    }
    sh.nlist = nl;
  }
  cl.sync();

  // ---------------- the leader gathers the row's entries and candidates ----------------
  if (cr == 0 && decided < 0) {
    // the CTAs' counts, their offsets in the row (warp 0, one lane per CTA)
    if (w == 0) {
      int ne_c = 0, nc_c = 0;
      if (lane < C) {
        ne_c = *cl.map_shared_rank(&sh.nlist, lane);
        nc_c = *cl.map_shared_rank(&sh.ncand, lane);
      }
      const bool bad = __any_sync(PESTI_FULL_MASK, nc_c > CL_CCAP);
      const int ein = warp_incl_scan_add(ne_c);
      const int cin = warp_incl_scan_add(nc_c);
      if (lane < C) {
        sh.u.f.ccnt[lane] = ein - ne_c;
        sh.u.f.coff[lane] = cin - nc_c;
      }
      const int ne = __shfl_sync(PESTI_FULL_MASK, ein, 31);
      const int ncd = __shfl_sync(PESTI_FULL_MASK, cin, 31);
      if (lane == 0) {
        sh.u.f.ccnt[C] = ne;
        sh.u.f.coff[C] = ncd;
        sh.u.f.nent = ne;
        sh.u.f.ncand = ncd;
        sh.status = (bad || ne > CL_LOCAL || (!nuc && (ncd > FAST_CAND || ncd < keff))) ? 1 : 0;
      }
    }
    __syncthreads();
    if (sh.status == 0) {
      const int ne = sh.u.f.nent, ncd = sh.u.f.ncand;
      for (int i = tid; i < ne; i += CL_NT) {
        int c = 0;
        while (i >= sh.u.f.ccnt[c + 1]) ++c;
        sh.u.f.ent[i] = *cl.map_shared_rank(&sh.list[i - sh.u.f.ccnt[c]], c);
      }
      for (int i = tid; i < ncd; i += CL_NT) {
        int c = 0;
        while (i >= sh.u.f.coff[c + 1]) ++c;
        const int j = i - sh.u.f.coff[c];
        const float e = *cl.map_shared_rank(&sh.cand_e[j], c);
        const uint32_t ix = *cl.map_shared_rank(&sh.cand_i[j], c);
        sh.u.f.key[i] = ((unsigned long long)fbits(e) << 32) | (unsigned long long)(~ix);
      }
    }
  }
  cl.sync();  // after this the other CTAs' shared memory is no longer read
  if (cr != 0) return;

  // ---------------- leader: walk, top-k, draw ----------------
  int status = decided < 0 ? sh.status : decided;
  if (decided == 0 && greedy) {  // generate(): temperature == 0 -> argmax (model.rs:517-521)
    if (w == 0) {
      const uint32_t tok = (prm.flags & PESTI_FLAG_ARGMAX_FIRST) ? (first_max >= 0 ? (uint32_t)first_max : 0u)
                                                                 : (last_max >= 0 ? (uint32_t)last_max : 0u);
      if (lane == 0) {
        a.out[b] = tok;
        if (a.kept_count) a.kept_count[b] = 0;
        a.fb[b] = 0;
      }
      cl_write_pad(a, b, 0);
    }
    return;
  }
  const int ncd = decided < 0 ? sh.u.f.ncand : 0;
  if (status == 0) {
    if (w == 1) {  // candidates by (e desc, index asc) while warp 0 walks
      unsigned long long* key = sh.u.f.key;
      if (ncd <= 32) warp_sort_keys<1>(key, ncd);
      else if (ncd <= 64) warp_sort_keys<2>(key, ncd);
      else if (ncd <= 128) warp_sort_keys<4>(key, ncd);
      else {
        int mm2 = 1;
        while (mm2 < ncd) mm2 <<= 1;
        for (int j = ncd + lane; j < mm2; j += 32) key[j] = 0ull;
        __syncwarp();
        warp_bitonic_desc(key, mm2);
      }
    }
    if (w != 1) {
      // softmax denominator (sampling.rs:128): warp 0 walks the entries with the
      // exact state; an entry the state does not fit (or a replay marker) is
      // folded from the raw logits of its range, from the state before it, by
      // the replay group (warps 0, 2..7)
      const FoldEnt* fent = sh.u.f.ent;
      const int nm = sh.u.f.nent;
      uint32_t s = 0u;
      constexpr int WB = 8;
      int i = 0;
      for (int it = 0;; ++it) {
        int fi = -1;
        if (w == 0 && i < nm) {
          FoldEnt nx[WB];
#pragma unroll
          for (int uu = 0; uu < WB; ++uu) nx[uu] = fent[i + uu < nm ? i + uu : nm - 1];
          for (; i < nm; i += WB) {
            FoldEnt en[WB];
#pragma unroll
            for (int uu = 0; uu < WB; ++uu) {
              en[uu] = nx[uu];
              const int kk = i + WB + uu;
              nx[uu] = fent[kk < nm ? kk : nm - 1];
            }
#pragma unroll
            for (int uu = 0; uu < WB; ++uu) {
              const bool live = fi < 0 && i + uu < nm;
              const bool sp = en[uu].lo == fold::SPECIAL;
              const uint32_t s_sp = fbits(fadd(bitsf(s), bitsf(en[uu].a0)));
              const uint32_t ns = s + ((s & 1u) ? en[uu].a1 : en[uu].a0);
              const bool fits = fold::binade_lo_bits(s) == en[uu].lo && ns < fold::binade_hi_bits(en[uu].lo);
              fi = live && !sp && !fits ? i + uu : fi;
              s = live && (sp || fits) ? (sp ? s_sp : ns) : s;
            }
            if (fi >= 0) break;
          }
        }
        // the entry to replay, double-buffered by parity: a group warp reads
        // slot it&1 before the barrier that lets warp 0 write it again
        if (tid == 0) sh.u.f.rep_fi[it & 1] = fi;
        cl_rbar();
        fi = sh.u.f.rep_fi[it & 1];
        if (fi < 0) break;
        const uint32_t from = fi > 0 ? fent[fi - 1].end : 0u;
        const uint32_t to = fent[fi].end;
        s = cl_replay(row, a.dtype, from, to, s, scale, T, m, sh);
        i = fi + 1;
      }
      if (tid == 0) sh.uscr[0] = s;
    }
    __syncthreads();
    if (nuc) {  // S for the row kernel's sorted folds by distinct values
      if (tid == 0) sh.status = 2;
    } else if (w == 0) {
      const float S = bitsf(sh.uscr[0]);
      unsigned long long* key = sh.u.f.key;
      // p = e/S (sampling.rs:130); the list stays sorted by p except inside
      // groups of equal p, which the stable sort (sampling.rs:60) orders by index
      for (int j = lane; j < ncd; j += 32) {
        const unsigned long long kv = key[j];
        key[j] = ((unsigned long long)fbits(fdiv(bitsf((uint32_t)(kv >> 32)), S)) << 32) | (kv & 0xffffffffull);
      }
      __syncwarp();
      bool viol = false;
      for (int j = lane; j + 1 < ncd; j += 32) viol |= key[j] < key[j + 1];
      if (__any_sync(PESTI_FULL_MASK, viol)) {
        if (lane == 0) {  // insertion sort: only equal-p groups are out of order
          for (int j = 1; j < ncd; ++j) {
            const unsigned long long kv = key[j];
            int t = j - 1;
            while (t >= 0 && key[t] < kv) {
              key[t + 1] = key[t];
              --t;
            }
            key[t + 1] = kv;
          }
        }
        __syncwarp();
      }
      // every element below the candidates (raw < tau) must rank below the keff-th
      const float pk = bitsf((uint32_t)(key[keff - 1] >> 32));
      const bool ok = !(S > 0.0f) ? false : fdiv(sh.e_tau, S) < pk;
      if (ok) {
        const uint32_t r_tau = fold::tau_bits_of(a.u ? a.u[b] : 0.0f);
        float* q = sh.u.f.q;
        for (long long j = lane; j < keff; j += 32) q[j] = bitsf((uint32_t)(key[j] >> 32));
        __syncwarp();
        uint32_t tb = 0u;
        if (lane == 0) tb = serial_fold8(q, keff, 0u, fold::NO_QUERY, false).s_bits;  // sampling.rs:81
        const float total = bitsf(__shfl_sync(PESTI_FULL_MASK, tb, 0));
        for (long long j = lane; j < keff; j += 32) q[j] = fdiv(q[j], total);  // sampling.rs:94
        __syncwarp();
        if (lane == 0) {
          const fold::Result dr = serial_fold8(q, keff, 0u, r_tau, true);  // sampling.rs:99-105
          const long long at = dr.hit >= 0 ? dr.hit : keff - 1;           // sampling.rs:108-111
          a.out[b] = ~(uint32_t)(key[at] & 0xffffffffull);
          if (a.kept_count) a.kept_count[b] = keff;
        }
        for (long long j = lane; j < a.kept_width; j += 32) {
          const bool in = j < keff;
          const unsigned long long kv = in ? key[j] : 0ull;
          if (a.kept_p) a.kept_p[b * a.kept_width + j] = in ? bitsf((uint32_t)(kv >> 32)) : 0.0f;
          if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = in ? ~(uint32_t)(kv & 0xffffffffull) : 0xffffffffu;
        }
      }
      if (lane == 0) sh.status = ok ? 0 : 1;
    }
    __syncthreads();
    status = sh.status;
  }
  if (tid == 0) {
    a.fb[b] = status;
    if (status) {  // the row kernel's generic path takes the row: its prologue
      RowInfo ri;
      ri.max_raw = sh.max_raw;
      ri.m = sh.m;
      ri.tau = INF;
      ri.flags = sh.flags;
      ri.last_max = sh.last_max;
      ri.first_max = sh.first_max;
      ri.last_nan = sh.last_nan;
      ri.uniform = ((sh.flags & MF_NAN) || (scale && T == INF && (sh.flags & (MF_POSINF | MF_NEGINF))) ||
                    !(fabsf(sh.m) < INF)) ? 1 : 0;
      ri.e_tau = 0.0f;
      ri.s_start = 0.0f;
      ri.S = status == 2 ? bitsf(sh.uscr[0]) : 0.0f;
      ri.min_raw = sh.min_raw;
      a.info[b] = ri;
    }
  }
}

}  // namespace pesti
