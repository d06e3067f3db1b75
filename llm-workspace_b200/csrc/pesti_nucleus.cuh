// Top-p rows of bf16 logits, by distinct values instead of a sort
// (sampling.rs:56-111 for rows with top_k == 0 and top_p > 0).
//
// Every copy of one logit value has the same probability, and the stable sort
// by probability (sampling.rs:67) puts the copies of equal probability next
// to each other in index order.  The folds over the sorted list (the top-p
// cumulative sum, total, the draw's cumulative sum, sampling.rs:68-105) only
// see the sequence of values, so they are folds over (probability, count)
// runs in descending order, which fold::block_fold_runs does exactly.  A bf16
// row has a few thousand distinct values: the row becomes a histogram over a
// table of its 16 highest binades (both signs, 128 mantissa steps each), plus
// a short list of the few elements of smaller magnitude.  Only the token and
// the first kept_width entries of the kept list need element indices; they
// come from ordered scans of the row.
//
// One block (K2_NT threads) per row, in the row kernel, once the cluster pass
// has folded the softmax denominator S exactly.  Rows this cannot finish
// (too many small-magnitude elements, too long a kept-list prefix) return
// false and take the generic sorted path.
#pragma once

namespace pesti {

constexpr int NUC_BINADES = 16;                    // binades of the table, per sign
constexpr int NUC_HALF = NUC_BINADES * 128;        // slots per sign
constexpr int NUC_SLOTS = 2 * NUC_HALF;            // positive slots, then negative slots
constexpr int NUC_TINY = 512;                      // elements below the table's magnitude range
constexpr int NUC_ENT = 3072;                      // distinct values of a row this path takes
constexpr int NUC_KEPT = 1024;                     // kept-list prefix taken from the entries above its last group

struct NucSmem {
  union {
    struct {                    // the histogram (until the value sequence is built)
      uint32_t tab[NUC_SLOTS];  // counts per value
      uint32_t tiny_v[NUC_TINY];  // small-magnitude elements: f32 bits and index
      uint32_t tiny_i[NUC_TINY];
      unsigned long long tkey[NUC_TINY];
    } h;
    fold::RunSmem rs;           // the folds
    unsigned long long kkey[NUC_KEPT];  // kept-list prefix: (group, index)
  } u;
  float val[NUC_ENT];           // the distinct values in descending order, their counts
  uint32_t cnt[NUC_ENT];
  float gp[NUC_ENT];            // groups of equal probability: probability, count, lowest value
  uint32_t gc[NUC_ENT];
  float gmin[NUC_ENT];
  float gq[NUC_ENT];            // per entry p, then the normalised probability of each kept group
  uint32_t zero;                // count of +0 and -0
  int ntiny, nent, ngrp, nkey;
};

// Slot of a bf16 value (f32 bits u) in the table whose binades are [E_lo,
// E_lo + NUC_BINADES): -1 outside it (zero has its own count).
__device__ __forceinline__ int nuc_slot(uint32_t u, uint32_t E_lo) {
  const uint32_t E = (u >> 23) & 0xffu;
  if (E < E_lo || E >= E_lo + NUC_BINADES) return -1;
  const int s = (int)((E - E_lo) * 128u + ((u >> 16) & 0x7fu));
  return (u & 0x80000000u) ? NUC_HALF + s : s;
}

// The value of slot s (inverse of nuc_slot).
__device__ __forceinline__ float nuc_value(int s, uint32_t E_lo) {
  const bool neg = s >= NUC_HALF;
  const int t = neg ? s - NUC_HALF : s;
  const uint32_t u = ((E_lo + (uint32_t)(t >> 7)) << 23) | ((uint32_t)(t & 127) << 16) | (neg ? 0x80000000u : 0u);
  return bitsf(u);
}

// Position p (in the descending value order) of the virtual sequence:
// positive slots from the top, small positives, zero, small negatives,
// negative slots by growing magnitude.  tiny[] is sorted by value, largest
// first, with ntp positive ones.
struct NucOrder {
  int ntp, ntn;
  __device__ __forceinline__ int length() const { return NUC_HALF + ntp + 1 + ntn + NUC_HALF; }
};

// Eight consecutive bf16 logits from j (one 16-byte load when the row is
// aligned and whole there), widened; u16[e] = 0 past V with nv the valid count.
__device__ __forceinline__ void nuc_load8(const uint16_t* row, long long j, long long V, bool vec, uint16_t (&h)[8],
                                          int& nv) {
  if (vec && j + 8 <= V) {
    const uint4 w4 = __ldg(reinterpret_cast<const uint4*>(row + j));
    const uint32_t wd[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      h[2 * q] = (uint16_t)(wd[q] & 0xffffu);
      h[2 * q + 1] = (uint16_t)(wd[q] >> 16);
    }
    nv = 8;
    return;
  }
  nv = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const bool in = j + e < V;
    h[e] = in ? row[j + e] : (uint16_t)0;
    nv = in ? e + 1 : nv;
  }
}

// The elements of the row that satisfy pred, in index order: those whose
// ranks among them lie in [first, first + count) are passed to emit(rank, j).
// Each warp owns a contiguous chunk of the row and reads it 32 elements at a
// time (coalesced); the chunks' counts give each warp its first rank.  The
// whole block calls it.
template <typename Pred, typename Emit>
__device__ void nuc_ordered(const uint16_t* row, long long V, bool vec, Pred pred, long long first, long long count,
                            Emit emit, RowShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  constexpr int NW = K2_NT / 32;
  const long long chunk = ((V + NW - 1) / NW + 255) / 256 * 256;  // whole 256-element steps of the warp
  const long long c0 = (long long)wid * chunk, c1 = c0 + chunk < V ? c0 + chunk : V;
  // the warp's count of each 256-element step, kept in the row kernel's
  // shared scratch (free while this path runs), so that the scan for the
  // wanted positions starts at the step that holds the first of them
  uint32_t* scnt = &sh.u.s.hist[wid][0];
  const int nstep = (int)((c1 - c0 + 255) / 256);
  int n = 0;
  {
    int st = 0;
    for (long long j = c0 + lane * 8; st < nstep; j += 256, ++st) {
      uint16_t h[8];
      int nv = 0;
      if (j < c1) nuc_load8(row, j, c1, vec, h, nv);
      int c = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) c += (e < nv && pred(bf16_bits_to_f32(h[e]))) ? 1 : 0;
      c = (int)__reduce_add_sync(PESTI_FULL_MASK, (unsigned)c);
      if (lane == 0 && st < 256) scnt[st] = (uint32_t)c;
      n += c;
    }
  }
  __syncthreads();
  if (lane == 0) sh.iscr[wid] = n;
  __syncthreads();
  long long k = 0;
  for (int q = 0; q < wid; ++q) k += sh.iscr[q];
  if (k + n > first && k < first + count) {
    // skip the whole steps that end before position `first`
    long long j0 = c0;
    if (nstep <= 256) {  // (rows of at most 16 * 256 * 256 elements; longer ones scan from the start)
      long long base = k;
      for (int t0 = 0; t0 < nstep; t0 += 32) {
        const int t = t0 + lane;
        const int c = t < nstep ? (int)scnt[t] : 0;
        const int inc = warp_incl_scan_add(c);
        // the first step of this batch whose running count passes `first`
        const uint32_t past = __ballot_sync(PESTI_FULL_MASK, t < nstep && base + inc > first);
        if (past) {
          const int f = __ffs(past) - 1;
          const int before = __shfl_sync(PESTI_FULL_MASK, inc - c, f);
          j0 = c0 + (long long)(t0 + f) * 256;
          k = base + before;
          break;
        }
        base += __shfl_sync(PESTI_FULL_MASK, inc, 31);
        j0 = c0 + (long long)(t0 + 32) * 256;
        k = base;
      }
    }
    for (; j0 < c1 && k < first + count; j0 += 256) {
      const long long j = j0 + lane * 8;
      uint16_t h[8];
      int nv = 0;
      if (j < c1) nuc_load8(row, j, c1, vec, h, nv);
      uint32_t hm = 0u;
#pragma unroll
      for (int e = 0; e < 8; ++e) hm |= (e < nv && pred(bf16_bits_to_f32(h[e]))) ? (1u << e) : 0u;
      const int c = __popc(hm);
      const int inc = warp_incl_scan_add(c);
      long long r = k + inc - c;
      for (uint32_t mm = hm; mm != 0u; mm &= mm - 1u, ++r)
        if (r >= first && r < first + count) emit(r, j + __ffs(mm) - 1);
      k += __shfl_sync(PESTI_FULL_MASK, inc, 31);
    }
  }
  __syncthreads();
}

__device__ bool nucleus_rows(const RowArgs& a, long long b, const RowInfo& ri, const pesti_sampling_params& prm,
                             const uint16_t* row, RowShared& sh, NucSmem& ns) {
  const int tid = threadIdx.x;
  const long long V = a.V;
  const float T = prm.temperature;
  const bool scale = T > 0.0f;
  const float m = ri.m;
  const float S = ri.S;
  // the table's binades: the 16 highest of the row's magnitudes
  const uint32_t e_hi = (uint32_t)max((int)((fbits(fabsf(ri.max_raw)) >> 23) & 0xff),
                                      (int)((fbits(fabsf(ri.min_raw)) >> 23) & 0xff));
  const uint32_t E_lo = e_hi >= (uint32_t)NUC_BINADES ? e_hi - (NUC_BINADES - 1) : 1u;
  for (int i = tid; i < NUC_SLOTS; i += K2_NT) ns.u.h.tab[i] = 0u;
  if (tid == 0) {
    ns.zero = 0u;
    ns.ntiny = 0;
  }
  __syncthreads();
  // ---- histogram of the row: eight elements per thread and step ----
  const bool vec = ((uintptr_t)row % 16) == 0;
  for (long long j = (long long)tid * 8; j < V; j += (long long)K2_NT * 8) {
    uint16_t h[8];
    int nv;
    nuc_load8(row, j, V, vec, h, nv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (e >= nv) continue;
      const uint32_t u = ((uint32_t)h[e]) << 16;
      if ((u & 0x7fffffffu) == 0u) {
        atomicAdd(&ns.zero, 1u);
        continue;
      }
      const int s = nuc_slot(u, E_lo);
      if (s >= 0) {
        atomicAdd(&ns.u.h.tab[s], 1u);
      } else {
        const int t = atomicAdd(&ns.ntiny, 1);
        if (t < NUC_TINY) {
          ns.u.h.tiny_v[t] = u;
          ns.u.h.tiny_i[t] = (uint32_t)(j + e);
        }
      }
    }
  }
  __syncthreads();
  const int ntiny = ns.ntiny;
  if (ntiny > NUC_TINY) return false;
  // small-magnitude elements by value, largest first (keys: value, then index)
  if (ntiny > 0) {
    int mm2 = 1;
    while (mm2 < ntiny) mm2 <<= 1;
    unsigned long long* key = ns.u.h.tkey;
    for (int i = tid; i < mm2; i += K2_NT)
      key[i] = i < ntiny ? ((unsigned long long)fkey(bitsf(ns.u.h.tiny_v[i])) << 32) | (unsigned long long)(~ns.u.h.tiny_i[i]) : 0ull;
    __syncthreads();
    bitonic_desc(key, mm2);
    for (int i = tid; i < ntiny; i += K2_NT) {
      ns.u.h.tiny_v[i] = fbits(fkey_inv((uint32_t)(key[i] >> 32)));
      ns.u.h.tiny_i[i] = ~(uint32_t)(key[i] & 0xffffffffull);
    }
    __syncthreads();
  }
  int ntp = 0;
  for (int i = tid; i < ntiny; i += K2_NT) ntp += (ns.u.h.tiny_v[i] & 0x80000000u) ? 0 : 1;
  ntp = (int)block_reduce_add((long long)ntp, sh.lscr);
  const NucOrder ord{ntp, ntiny - ntp};
  const int L = ord.length();
  // ---- the distinct values, descending, compacted ----
  auto at = [&](int p, float& v, uint32_t& c) {
    if (p < NUC_HALF) {  // positive slots from the top
      const int s = NUC_HALF - 1 - p;
      c = ns.u.h.tab[s];
      v = nuc_value(s, E_lo);
      return;
    }
    p -= NUC_HALF;
    if (p < ord.ntp) {
      c = 1u;
      v = bitsf(ns.u.h.tiny_v[p]);
      return;
    }
    p -= ord.ntp;
    if (p == 0) {
      c = ns.zero;
      v = 0.0f;
      return;
    }
    p -= 1;
    if (p < ord.ntn) {
      c = 1u;
      v = bitsf(ns.u.h.tiny_v[ord.ntp + p]);
      return;
    }
    p -= ord.ntn;  // negative slots by growing magnitude
    c = ns.u.h.tab[NUC_HALF + p];
    v = nuc_value(NUC_HALF + p, E_lo);
  };
  {
    long long base = 0;
    for (int p0 = 0; p0 < L; p0 += K2_NT) {
      const int p = p0 + tid;
      float v = 0.0f;
      uint32_t c = 0u;
      if (p < L) at(p, v, c);
      long long tot;
      const long long ex = base + block_excl_scan_add((long long)(c > 0u ? 1 : 0), sh.lscr, tot);
      if (c > 0u && ex < NUC_ENT) {
        ns.val[ex] = v;
        ns.cnt[ex] = c;
      }
      base += tot;
    }
    if (tid == 0) ns.nent = (int)base;
    __syncthreads();
  }
  const int ne = ns.nent;
  if (ne > NUC_ENT) return false;
  // probabilities (sampling.rs:46,127,130); equal neighbours form one group
  // (the stable sort orders their elements by index)
  for (int i = tid; i < ne; i += K2_NT) {
    const float v = ns.val[i];
    ns.gq[i] = fdiv(pesti_expf(fsub(scale ? fdiv(v, T) : v, m)), S);  // gq: scratch for p
  }
  __syncthreads();
  {
    long long base = 0;
    for (int i0 = 0; i0 < ne; i0 += K2_NT) {
      const int i = i0 + tid;
      const bool head = i < ne && (i == 0 || ns.gq[i] != ns.gq[i - 1]);
      long long tot;
      const long long g = base + block_excl_scan_add((long long)(head ? 1 : 0), sh.lscr, tot);
      if (head) ns.gp[g] = ns.gq[i];
      base += tot;
    }
    if (tid == 0) ns.ngrp = (int)base;
    __syncthreads();
  }
  const int ng = ns.ngrp;
  // group counts and lowest values (each thread its own entries, in order)
  for (int g = tid; g < ng; g += K2_NT) ns.gc[g] = 0u;
  __syncthreads();
  {
    // entry i belongs to group (number of heads at or before i) - 1
    long long base = 0;
    for (int i0 = 0; i0 < ne; i0 += K2_NT) {
      const int i = i0 + tid;
      const bool head = i < ne && (i == 0 || ns.gq[i] != ns.gq[i - 1]);
      long long tot;
      const long long g = base + block_excl_scan_add((long long)(head ? 1 : 0), sh.lscr, tot) + (head ? 1 : 0) - 1;
      if (i < ne) {
        atomicAdd(&ns.gc[g], ns.cnt[i]);
        const bool last = i + 1 == ne || ns.gq[i + 1] != ns.gq[i];
        if (last) ns.gmin[g] = ns.val[i];
      }
      base += tot;
    }
    __syncthreads();
  }
  // ---- top-p cut: the first position whose cumulative sum reaches top_p (sampling.rs:65-78) ----
  fold::RunResult cut = fold::block_fold_runs(ns.gp, ns.gc, ng, 0u, fold::tau_bits_of(prm.top_p), true, ns.u.rs);
  long long hg, hc;
  float total;
  if (cut.hit >= 0) {
    hg = cut.hit;
    hc = cut.hit_copy;
    total = bitsf(cut.hit_s_bits);  // total_prob (sampling.rs:81) is this same fold
  } else {
    hg = ng - 1;
    hc = (long long)ns.gc[ng - 1] - 1;
    total = bitsf(cut.s_bits);
  }
  if (!(total > 0.0f)) return false;
  // kept count: the groups before hg, and hc + 1 copies of it
  long long before_h = 0;
  for (int g = tid; g < hg; g += K2_NT) before_h += ns.gc[g];
  before_h = block_reduce_add(before_h, sh.lscr);
  const long long K = before_h + hc + 1;
  // ---- draw over the normalised kept list (sampling.rs:94-111) ----
  for (int g = tid; g <= hg; g += K2_NT) ns.gq[g] = fdiv(ns.gp[g], total);
  const uint32_t keep_last = ns.gc[hg];
  __syncthreads();
  if (tid == 0) ns.gc[hg] = (uint32_t)(hc + 1);
  __syncthreads();
  const float r = a.u ? a.u[b] : 0.0f;
  fold::RunResult dr = fold::block_fold_runs(ns.gq, ns.gc, hg + 1, 0u, fold::tau_bits_of(r), true, ns.u.rs);
  long long dg, dc;
  if (dr.hit >= 0) {
    dg = dr.hit;
    dc = dr.hit_copy;
  } else {  // the last kept element (sampling.rs:108-111)
    dg = hg;
    dc = hc;
  }
  __syncthreads();
  if (tid == 0) ns.gc[hg] = keep_last;
  __syncthreads();
  // group g holds the values in [gmin[g], gmin[g-1]) (descending, contiguous)
  auto in_group = [&](float x, long long g) { return x >= ns.gmin[g] && (g == 0 || x < ns.gmin[g - 1]); };
  // the dc-th element (index order) of group dg
  if (tid == 0) sh.n = -1;
  nuc_ordered(row, V, vec, [&](float x) { return in_group(x, dg); }, dc, 1,
              [&](long long, long long j) { sh.n = j; }, sh);
  const long long tok = sh.n;
  __syncthreads();
  if (tok < 0) return false;
  // ---- the kept list's first kept_width entries ----
  const long long kw = a.kept_width < K ? a.kept_width : K;
  if (kw > 0) {
    // the group holding position kw - 1, and the positions before it
    if (tid == 0) {
      long long p = 0;
      int g = 0;
      while (p + (long long)ns.gc[g] < kw) {
        p += ns.gc[g];
        ++g;
      }
      sh.n = g;
      sh.u.c.sel_k = p;  // positions before group g
    }
    __syncthreads();
    const long long gl = sh.n;
    const long long pl = sh.u.c.sel_k;
    __syncthreads();
    if (pl > NUC_KEPT) return false;
    // every element of the groups before gl, sorted by (group, index)
    if (tid == 0) ns.nkey = 0;
    __syncthreads();
    const float lim = gl > 0 ? ns.gmin[gl - 1] : __int_as_float(0x7f800000);
    for (long long j0 = (long long)tid * 8; j0 < V && pl > 0; j0 += (long long)K2_NT * 8) {
      uint16_t h[8];
      int nv;
      nuc_load8(row, j0, V, vec, h, nv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float x = bf16_bits_to_f32(h[e]);
        if (e < nv && x >= lim) {
          int lo2 = 0, hi2 = (int)gl - 1;  // its group: the first g with x >= gmin[g]
          while (lo2 < hi2) {
            const int mid = (lo2 + hi2) >> 1;
            if (x >= ns.gmin[mid]) hi2 = mid;
            else lo2 = mid + 1;
          }
          const int slot = atomicAdd(&ns.nkey, 1);
          if (slot < NUC_KEPT)
            ns.u.kkey[slot] = ((unsigned long long)(0xffffffffu - (uint32_t)lo2) << 32) | (uint32_t)~(uint32_t)(j0 + e);
        }
      }
    }
    __syncthreads();
    const int nk = ns.nkey;
    if (nk != (int)pl) return false;
    if (nk > 0) {
      int mm2 = 1;
      while (mm2 < nk) mm2 <<= 1;
      for (int i = nk + tid; i < mm2; i += K2_NT) ns.u.kkey[i] = 0ull;
      __syncthreads();
      bitonic_desc(ns.u.kkey, mm2);  // (group asc, index asc)
    }
    for (long long j = tid; j < pl; j += K2_NT) {
      const unsigned long long kv = ns.u.kkey[j];
      const uint32_t g = 0xffffffffu - (uint32_t)(kv >> 32);
      if (a.kept_p) a.kept_p[b * a.kept_width + j] = ns.gp[g];
      if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = ~(uint32_t)(kv & 0xffffffffull);
    }
    // then the first kw - pl elements of group gl, in index order
    const float pgl = ns.gp[gl];
    nuc_ordered(row, V, vec, [&](float x) { return in_group(x, gl); }, 0, kw - pl,
                [&](long long r, long long j) {
                  if (a.kept_p) a.kept_p[b * a.kept_width + pl + r] = pgl;
                  if (a.kept_idx) a.kept_idx[b * a.kept_width + pl + r] = (uint32_t)j;
                }, sh);
  }
  for (long long j = kw + tid; j < a.kept_width; j += K2_NT) {
    if (a.kept_p) a.kept_p[b * a.kept_width + j] = 0.0f;
    if (a.kept_idx) a.kept_idx[b * a.kept_width + j] = 0xffffffffu;
  }
  if (tid == 0) {
    a.out[b] = (uint32_t)tok;
    if (a.kept_count) a.kept_count[b] = K;
  }
  return true;
}

}  // namespace pesti
