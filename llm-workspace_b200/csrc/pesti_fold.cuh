// Exact, block-parallel emulation of a sequential f32 fold
//     s = s0;  for j in 0..n: s = fl(s + v[j])          (v[j] >= 0)
// as the reference computes every sum of the sampling step: the softmax
// denominator (sampling.rs:128), the top-p cumulative sum (sampling.rs:68-76),
// the kept-list total (sampling.rs:81) and the draw's cumulative sum
// (sampling.rs:99-105).  A parallel sum in any other order differs from these
// folds by up to 4e-4 relative (small terms are absorbed by a large running
// sum), so the folds are reproduced bit for bit instead.
//
// Why it can be parallel: while the running sum s stays in one binade
// [lo, 2lo) with ulp w, fl(s + v) = s + w*k(v), where k(v) is v rounded to an
// integer multiple of w.  k(v) does not depend on s except through the parity
// of s/w when v/w is exactly half an odd integer (a tie).  With s kept as its
// IEEE bit pattern, "s + w*k" is "bits(s) + k", so a run of such elements is a
// plain integer sum.  k(v) itself is computed exactly as
//     bits(fl(lo + v)) - bits(lo)   (even parity)  and
//     bits(fl(lo + w + v)) - bits(lo + w)   (odd parity),
// and an element is a tie exactly when the two differ.
//
// Each tile of TS elements is classified from an approximate running sum (the
// exact real prefix, in double).  Elements that may leave the binade, that are
// large next to s, that are ties or that may reach the query threshold are
// "special" and are added one at a time with a real f32 add; maximal runs of
// the rest become integer sums.  One thread then walks the segments with the
// exact state and VERIFIES each run: the state must be in the run's binade at
// the start and still below the binade's top at the end.  A failed check
// restarts the tile at that run with the exact state as the new anchor, so
// the result never depends on the approximation being right.
#pragma once
#include "pesti_common.cuh"

namespace pesti {
namespace fold {

constexpr int NT = 512;   // threads of the calling block
constexpr int EPT = 4;    // elements per thread per tile
constexpr int TS = NT * EPT;
constexpr uint32_t SPECIAL = 0xffffffffu;
constexpr uint32_t NO_QUERY = 0xffffffffu;
constexpr double MU = 0x1p-10;  // relative guard band around binade edges and the query
constexpr int SEQ_STEP = 64;    // direct adds taken when a tile makes no progress

struct Smem {
  float v[TS];
  long long pinc[TS];
  uint32_t cls[TS];
  uint32_t seg_lo[TS];
  unsigned short seg_start[TS];
  double dscr[34];
  long long lscr[34];
  int iscr[34];
  uint32_t s_bits;
  uint32_t hit_s_bits;
  long long pos;
  long long hit;
  int done;
  int seq_left;
};

struct Result {
  uint32_t s_bits;      // final state (or the state at the hit when stopping there)
  long long hit;        // first j with fold_j >= tau, -1 if none
  uint32_t hit_s_bits;  // fold value at the hit
};

// Query threshold encoding: the fold "reaches" tau when bits(s) >= tau_bits.
__device__ __forceinline__ uint32_t tau_bits_of(float tau) {
  if (is_nan(tau)) return NO_QUERY;
  if (tau <= 0.0f) return 0u;  // fold_0 >= 0 >= tau: reached at the first element
  return fbits(tau);
}

// Binade of a non-negative finite f32 given by its bits: lo_bits = bits of
// the binade's lowest value (0 for the subnormal range [0, 2^-126)).
__device__ __forceinline__ uint32_t binade_lo_bits(uint32_t s) {
  return s < 0x00800000u ? 0u : (s & 0x7f800000u);
}
__device__ __forceinline__ uint32_t binade_hi_bits(uint32_t lo) {
  return lo == 0u ? 0x00800000u : lo + 0x00800000u;
}

// The block computes the fold of seq[0..n) from s0 (bits; a non-negative
// float).  With a query (tau_bits != NO_QUERY) it records the first position
// whose running sum reaches tau; with stop_at_hit it returns right there.
// All threads of the block must call it; the result is block-uniform.
__device__ __noinline__ Result block_fold(const float* __restrict__ seq, long long n,
                                          uint32_t s0_bits, uint32_t tau_bits, bool stop_at_hit,
                                          Smem& sm) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    sm.s_bits = s0_bits & 0x7fffffffu;  // -0.0 -> +0.0: fl(-0 + v) == fl(+0 + v) for v >= 0
    sm.pos = 0;
    sm.hit = -1;
    sm.hit_s_bits = 0;
    sm.done = 0;
    sm.seq_left = 0;
  }
  __syncthreads();
  const float tauf = bitsf(tau_bits == NO_QUERY ? 0x7f800000u : tau_bits);
  while (true) {
    const long long pos = sm.pos;
    const uint32_t s_bits = sm.s_bits;
    const int done = sm.done;
    const int seq_left = sm.seq_left;
    __syncthreads();
    if (done || pos >= n) break;
    if (seq_left > 0) {
      // Progress guarantee: a few elements added one by one.
      if (tid == 0) {
        uint32_t s = s_bits;
        long long p = pos;
        const long long lim = pos + seq_left < n ? pos + seq_left : n;
        for (; p < lim; ++p) {
          s = fbits(fadd(bitsf(s), seq[p]));
          if (sm.hit < 0 && s >= tau_bits) {
            sm.hit = p;
            sm.hit_s_bits = s;
            if (stop_at_hit) {
              sm.done = 1;
              ++p;
              break;
            }
          }
        }
        sm.s_bits = s;
        sm.pos = p;
        sm.seq_left = 0;
      }
      __syncthreads();
      continue;
    }
    const int len = (int)((n - pos) < (long long)TS ? (n - pos) : (long long)TS);
    // ---- load the tile and form the approximate running sum ----
    float v[EPT];
    double lsum = 0.0;
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int j = tid * EPT + e;
      v[e] = j < len ? seq[pos + j] : 0.0f;
      if (j < len) sm.v[j] = v[e];
      lsum += (double)v[e];
    }
    double dtot;
    double a = (double)bitsf(s_bits) + block_excl_scan_add(lsum, sm.dscr, dtot);
    // ---- classify ----
    long long kk[EPT];
    long long lk = 0;
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int j = tid * EPT + e;
      kk[e] = 0;
      if (j >= len) continue;
      const double b = a + (double)v[e];
      uint32_t lo_bits;
      bool big, near;
      if (a < 0x1p-126) {
        lo_bits = 0u;
        big = v[e] >= 0x1p-127f;
        near = b > 0x1p-126 * (1.0 - MU);
      } else {
        const uint32_t ab = fbits(__double2float_rz(a));
        lo_bits = ab & 0x7f800000u;
        big = fbits(v[e]) >= lo_bits - 0x00800000u;
        const double lo = (double)bitsf(lo_bits);
        near = a < lo * (1.0 + MU) || b > 2.0 * lo * (1.0 - MU);
      }
      const bool q = tau_bits != NO_QUERY && (double)tauf <= b * (1.0 + MU) + 0x1p-149 &&
                     (double)tauf >= a * (1.0 - MU);
      bool sp = big || near || q;
      if (!sp) {
        const uint32_t k0 = fbits(fadd(bitsf(lo_bits), v[e])) - lo_bits;
        const uint32_t k1 = fbits(fadd(bitsf(lo_bits + 1u), v[e])) - (lo_bits + 1u);
        if (k0 != k1) sp = true;
        else kk[e] = (long long)k0;
      }
      sm.cls[j] = sp ? SPECIAL : lo_bits;
      lk += kk[e];
      a = b;
    }
    long long ktot;
    long long kex = block_excl_scan_add(lk, sm.lscr, ktot);  // also orders cls[] writes
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int j = tid * EPT + e;
      kex += kk[e];
      if (j < len) sm.pinc[j] = kex;
    }
    // ---- segment heads ----
    int hc = 0;
    bool head[EPT];
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int j = tid * EPT + e;
      head[e] = false;
      if (j >= len) continue;
      const uint32_t cur = sm.cls[j];
      const uint32_t prev = j > 0 ? sm.cls[j - 1] : SPECIAL;
      head[e] = j == 0 || cur == SPECIAL || prev == SPECIAL || cur != prev;
      hc += head[e] ? 1 : 0;
    }
    int htot;
    int hex = block_excl_scan_add(hc, sm.iscr, htot);
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int j = tid * EPT + e;
      if (head[e]) {
        sm.seg_start[hex] = (unsigned short)j;
        sm.seg_lo[hex] = sm.cls[j];
        ++hex;
      }
    }
    __syncthreads();
    // ---- walk the segments with the exact state ----
    if (tid == 0) {
      uint32_t s = s_bits;
      long long newpos = pos + len;
      for (int g = 0; g < htot; ++g) {
        const int st = sm.seg_start[g];
        const int en = (g + 1 < htot ? (int)sm.seg_start[g + 1] : len) - 1;
        const uint32_t c = sm.seg_lo[g];
        if (c == SPECIAL) {
          s = fbits(fadd(bitsf(s), sm.v[st]));
          if (sm.hit < 0 && s >= tau_bits) {
            sm.hit = pos + st;
            sm.hit_s_bits = s;
            if (stop_at_hit) {
              sm.done = 1;
              newpos = pos + st + 1;
              break;
            }
          }
          continue;
        }
        if (binade_lo_bits(s) != c) {  // predicted binade wrong: restart here
          newpos = pos + st;
          break;
        }
        const long long base = st > 0 ? sm.pinc[st - 1] : 0ll;
        const long long nb = (long long)s + (sm.pinc[en] - base);
        if (nb >= (long long)binade_hi_bits(c)) {  // left the binade inside the run
          newpos = pos + st;
          break;
        }
        if (sm.hit < 0 && nb >= (long long)tau_bits) {
          int l = st, h = en;  // first jj with s + pinc[jj] - base >= tau
          while (l < h) {
            const int mid = (l + h) >> 1;
            if ((long long)s + (sm.pinc[mid] - base) >= (long long)tau_bits) h = mid;
            else l = mid + 1;
          }
          sm.hit = pos + l;
          sm.hit_s_bits = (uint32_t)((long long)s + (sm.pinc[l] - base));
          if (stop_at_hit) {
            sm.done = 1;
            s = sm.hit_s_bits;
            newpos = pos + l + 1;
            break;
          }
        }
        s = (uint32_t)nb;
      }
      if (newpos == pos) sm.seq_left = SEQ_STEP;  // no progress: go element by element
      sm.s_bits = s;
      sm.pos = newpos;
    }
    __syncthreads();
  }
  Result r;
  r.s_bits = sm.s_bits;
  r.hit = sm.hit;
  r.hit_s_bits = sm.hit_s_bits;
  __syncthreads();
  return r;
}

// Sequential fold by the calling thread alone (short lists).
__device__ __forceinline__ Result thread_fold(const float* seq, long long n, uint32_t s0_bits,
                                              uint32_t tau_bits, bool stop_at_hit) {
  Result r;
  uint32_t s = s0_bits & 0x7fffffffu;
  r.hit = -1;
  r.hit_s_bits = 0;
  for (long long j = 0; j < n; ++j) {
    s = fbits(fadd(bitsf(s), seq[j]));
    if (r.hit < 0 && s >= tau_bits) {
      r.hit = j;
      r.hit_s_bits = s;
      if (stop_at_hit) break;
    }
  }
  r.s_bits = s;
  return r;
}

// Fold of `count` copies of the same value v from s0 (the uniform-probability
// case, sampling.rs:132), in O(number of binades) steps: inside a binade each
// copy adds the same integer k to bits(s) (after at most one tie step, which
// always lands on an even multiple of the ulp).
__device__ inline Result repeat_fold(float v, long long count, uint32_t s0_bits,
                                     uint32_t tau_bits, bool stop_at_hit) {
  Result r;
  r.hit = -1;
  r.hit_s_bits = 0;
  uint32_t s = s0_bits & 0x7fffffffu;
  long long i = 0;
  while (i < count) {
    const uint32_t lo = binade_lo_bits(s);
    const uint32_t hi = binade_hi_bits(lo);
    const bool big = lo == 0u ? v >= 0x1p-127f : fbits(v) >= lo - 0x00800000u;
    uint32_t k0 = 0, k1 = 0;
    if (!big) {
      k0 = fbits(fadd(bitsf(lo), v)) - lo;
      k1 = fbits(fadd(bitsf(lo + 1u), v)) - (lo + 1u);
    }
    if (big || (k0 != k1 && (s & 1u))) {  // one direct add
      s = fbits(fadd(bitsf(s), v));
      if (r.hit < 0 && s >= tau_bits) {
        r.hit = i;
        r.hit_s_bits = s;
        if (stop_at_hit) {
          r.s_bits = s;
          return r;
        }
      }
      ++i;
      continue;
    }
    const uint32_t k = k0;  // even parity (or no tie): every step adds k0
    if (k == 0) break;      // absorbed from here on
    // steps that keep s below the top of the binade
    long long room = ((long long)hi - 1 - (long long)s) / (long long)k;
    long long steps = count - i < room ? count - i : room;
    if (steps <= 0) {  // the next add leaves the binade: take it directly
      s = fbits(fadd(bitsf(s), v));
      if (r.hit < 0 && s >= tau_bits) {
        r.hit = i;
        r.hit_s_bits = s;
        if (stop_at_hit) {
          r.s_bits = s;
          return r;
        }
      }
      ++i;
      continue;
    }
    if (r.hit < 0 && tau_bits != NO_QUERY && (long long)s + steps * (long long)k >= (long long)tau_bits) {
      const long long need = tau_bits <= s ? 1 : ((long long)tau_bits - (long long)s + k - 1) / k;
      const long long at = need < 1 ? 1 : need;
      r.hit = i + at - 1;
      r.hit_s_bits = (uint32_t)((long long)s + at * (long long)k);
      if (stop_at_hit) {
        r.s_bits = r.hit_s_bits;
        return r;
      }
    }
    s = (uint32_t)((long long)s + steps * (long long)k);
    i += steps;
  }
  r.s_bits = s;
  return r;
}

// ---------------------------------------------------------------------------
// The same fold over a sequence given as runs of equal values: entry j stands
// for cnt[j] >= 1 consecutive copies of val[j] (the sorted probabilities of a
// row whose logits take few distinct values: every copy of a value has the
// same probability).  Inside a binade each copy of a value adds the same
// integer to bits(s) (after at most one tie step), so a run of cnt copies is
// cnt times that increment; entries that may leave the binade, are large next
// to the state, are ties or may reach the query are folded exactly copy by
// copy (repeat_fold, O(binades) per entry).  Result::hit is the first entry
// whose running sum reaches tau, hit_copy the copy (0-based) inside it.
// ---------------------------------------------------------------------------
struct RunResult {
  uint32_t s_bits;
  long long hit;        // entry of the first copy with fold >= tau, -1 if none
  long long hit_copy;   // that copy's place inside its entry
  uint32_t hit_s_bits;  // fold value at the hit
};

struct RunSmem {
  float v[TS];
  uint32_t c[TS];
  long long pinc[TS];
  uint32_t cls[TS];
  uint32_t seg_lo[TS];
  unsigned short seg_start[TS];
  double dscr[34];
  long long lscr[34];
  int iscr[34];
  uint32_t s_bits;
  uint32_t hit_s_bits;
  long long pos;
  long long hit;
  long long hit_copy;
  int done;
  int seq_left;
};

__device__ __noinline__ RunResult block_fold_runs(const float* __restrict__ val, const uint32_t* __restrict__ cnt,
                                                  long long n, uint32_t s0_bits, uint32_t tau_bits, bool stop_at_hit,
                                                  RunSmem& sm) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    sm.s_bits = s0_bits & 0x7fffffffu;
    sm.pos = 0;
    sm.hit = -1;
    sm.hit_copy = -1;
    sm.hit_s_bits = 0;
    sm.done = 0;
    sm.seq_left = 0;
  }
  __syncthreads();
  const float tauf = bitsf(tau_bits == NO_QUERY ? 0x7f800000u : tau_bits);
  // one entry folded exactly by the calling thread (with the query)
  auto exact_entry = [&](long long at, float v, uint32_t c, uint32_t s) -> uint32_t {
    const Result r = repeat_fold(v, (long long)c, s, sm.hit < 0 ? tau_bits : NO_QUERY, stop_at_hit);
    if (sm.hit < 0 && r.hit >= 0) {
      sm.hit = at;
      sm.hit_copy = r.hit;
      sm.hit_s_bits = r.hit_s_bits;
      if (stop_at_hit) sm.done = 1;
    }
    return r.s_bits;
  };
  while (true) {
    const long long pos = sm.pos;
    const uint32_t s_bits = sm.s_bits;
    const int done = sm.done;
    const int seq_left = sm.seq_left;
    __syncthreads();
    if (done || pos >= n) break;
    if (seq_left > 0) {
      // progress guarantee: a few entries folded one by one
      if (tid == 0) {
        uint32_t s = s_bits;
        long long p = pos;
        const long long lim = pos + seq_left < n ? pos + seq_left : n;
        for (; p < lim && !sm.done; ++p) s = exact_entry(p, val[p], cnt[p], s);
        sm.s_bits = s;
        sm.pos = p;
        sm.seq_left = 0;
      }
      __syncthreads();
      continue;
    }
    const int len = (int)((n - pos) < (long long)TS ? (n - pos) : (long long)TS);
    // ---- load the tile and form the approximate running sum ----
    float v[EPT];
    uint32_t c[EPT];
    double lsum = 0.0;
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int j = tid * EPT + e;
      v[e] = j < len ? val[pos + j] : 0.0f;
      c[e] = j < len ? cnt[pos + j] : 0u;
      if (j < len) {
        sm.v[j] = v[e];
        sm.c[j] = c[e];
      }
      lsum += (double)v[e] * (double)c[e];
    }
    double dtot;
    double a = (double)bitsf(s_bits) + block_excl_scan_add(lsum, sm.dscr, dtot);
    // ---- classify ----
    long long kk[EPT];
    long long lk = 0;
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int j = tid * EPT + e;
      kk[e] = 0;
      if (j >= len) continue;
      const double b = a + (double)v[e] * (double)c[e];
      uint32_t lo_bits;
      bool big, near;
      if (a < 0x1p-126) {
        lo_bits = 0u;
        big = v[e] >= 0x1p-127f;
        near = b > 0x1p-126 * (1.0 - MU);
      } else {
        const uint32_t ab = fbits(__double2float_rz(a));
        lo_bits = ab & 0x7f800000u;
        big = fbits(v[e]) >= lo_bits - 0x00800000u;
        const double lo = (double)bitsf(lo_bits);
        near = a < lo * (1.0 + MU) || b > 2.0 * lo * (1.0 - MU);
      }
      const bool q = tau_bits != NO_QUERY && (double)tauf <= b * (1.0 + MU) + 0x1p-149 &&
                     (double)tauf >= a * (1.0 - MU);
      bool sp = big || near || q;
      if (!sp) {
        const uint32_t k0 = fbits(fadd(bitsf(lo_bits), v[e])) - lo_bits;
        const uint32_t k1 = fbits(fadd(bitsf(lo_bits + 1u), v[e])) - (lo_bits + 1u);
        if (k0 != k1) sp = true;
        else kk[e] = (long long)k0 * (long long)c[e];
      }
      sm.cls[j] = sp ? SPECIAL : lo_bits;
      lk += kk[e];
      a = b;
    }
    long long ktot;
    long long kex = block_excl_scan_add(lk, sm.lscr, ktot);  // also orders cls[] writes
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int j = tid * EPT + e;
      kex += kk[e];
      if (j < len) sm.pinc[j] = kex;
    }
    // ---- segment heads ----
    int hc = 0;
    bool head[EPT];
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int j = tid * EPT + e;
      head[e] = false;
      if (j >= len) continue;
      const uint32_t cur = sm.cls[j];
      const uint32_t prev = j > 0 ? sm.cls[j - 1] : SPECIAL;
      head[e] = j == 0 || cur == SPECIAL || prev == SPECIAL || cur != prev;
      hc += head[e] ? 1 : 0;
    }
    int htot;
    int hex = block_excl_scan_add(hc, sm.iscr, htot);
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int j = tid * EPT + e;
      if (head[e]) {
        sm.seg_start[hex] = (unsigned short)j;
        sm.seg_lo[hex] = sm.cls[j];
        ++hex;
      }
    }
    __syncthreads();
    // ---- walk the segments with the exact state ----
    if (tid == 0) {
      uint32_t s = s_bits;
      long long newpos = pos + len;
      for (int g = 0; g < htot; ++g) {
        const int st = sm.seg_start[g];
        const int en = (g + 1 < htot ? (int)sm.seg_start[g + 1] : len) - 1;
        const uint32_t cl = sm.seg_lo[g];
        if (cl == SPECIAL) {
          s = exact_entry(pos + st, sm.v[st], sm.c[st], s);
          if (sm.done) {
            newpos = pos + st + 1;
            break;
          }
          continue;
        }
        if (binade_lo_bits(s) != cl) {  // predicted binade wrong: restart here
          newpos = pos + st;
          break;
        }
        const long long base = st > 0 ? sm.pinc[st - 1] : 0ll;
        const long long nb = (long long)s + (sm.pinc[en] - base);
        if (nb >= (long long)binade_hi_bits(cl)) {  // left the binade inside the run
          newpos = pos + st;
          break;
        }
        if (sm.hit < 0 && nb >= (long long)tau_bits) {
          int l = st, h = en;  // first entry jj whose last copy reaches tau
          while (l < h) {
            const int mid = (l + h) >> 1;
            if ((long long)s + (sm.pinc[mid] - base) >= (long long)tau_bits) h = mid;
            else l = mid + 1;
          }
          const long long before = (long long)s + ((l > st ? sm.pinc[l - 1] : base) - base);
          const long long k = (sm.pinc[l] - (l > st ? sm.pinc[l - 1] : base)) / (long long)sm.c[l];
          long long need = 1;  // copies of entry l until the fold reaches tau
          if ((long long)tau_bits > before && k > 0) need = ((long long)tau_bits - before + k - 1) / k;
          sm.hit = pos + l;
          sm.hit_copy = need - 1;
          sm.hit_s_bits = (uint32_t)(before + need * k);
          if (stop_at_hit) {
            sm.done = 1;
            s = sm.hit_s_bits;
            newpos = pos + l + 1;
            break;
          }
        }
        s = (uint32_t)nb;
      }
      if (newpos == pos) sm.seq_left = SEQ_STEP;  // no progress: entry by entry
      sm.s_bits = s;
      sm.pos = newpos;
    }
    __syncthreads();
  }
  RunResult r;
  r.s_bits = sm.s_bits;
  r.hit = sm.hit;
  r.hit_copy = sm.hit_copy;
  r.hit_s_bits = sm.hit_s_bits;
  __syncthreads();
  return r;
}

}  // namespace fold

namespace sort {

constexpr int NT = 512;
constexpr int NW = NT / 32;

struct Smem {
  uint32_t hist[NW][256];
  uint32_t iscr[34];
};

// Stable ascending LSD radix sort (8-bit digits) of n (key, value) pairs held
// in global memory, by one block.  Ping-pongs between (k0, v0) and (k1, v1);
// returns 0 if the result is in (k0, v0), 1 if in (k1, v1).  Passes whose
// digit is the same for every key are skipped.
// The lanes of the warp holding the same 9-bit value d as this lane (d <
// 512), as a mask: one ballot per bit, the lanes agreeing on every bit
// (the warp-level multisplit of the radix sort; all 32 lanes call it).
__device__ __forceinline__ uint32_t match_digit9(uint32_t d) {
  uint32_t m = 0xffffffffu;
#pragma unroll
  for (int bit = 0; bit < 9; ++bit) {
    const uint32_t bb = __ballot_sync(0xffffffffu, (d >> bit) & 1u);
    m &= ((d >> bit) & 1u) ? bb : ~bb;
  }
  return m;
}

__device__ __noinline__ int block_radix_sort(uint32_t* k0, uint32_t* v0, uint32_t* k1, uint32_t* v1,
                                             long long n, Smem& sm) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const long long chunk = ((n + NW - 1) / NW + 31) / 32 * 32;
  const long long beg = (long long)w * chunk;
  const long long end = beg + chunk < n ? beg + chunk : n;
  int cur = 0;
  for (int shift = 0; shift < 32; shift += 8) {
    const uint32_t* kin = cur ? k1 : k0;
    const uint32_t* vin = cur ? v1 : v0;
    uint32_t* kout = cur ? k0 : k1;
    uint32_t* vout = cur ? v0 : v1;
    for (int i = tid; i < NW * 256; i += NT) (&sm.hist[0][0])[i] = 0u;
    __syncthreads();
    // RB steps of 32 keys at a time: their loads are issued together, then
    // counted in order (the counters chain through shared memory)
    constexpr int RB = 16;
    for (long long j0 = beg; j0 < end; j0 += 32 * RB) {
      uint32_t kb[RB];
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        const long long j = j0 + r * 32 + lane;
        kb[r] = j < end ? kin[j] : 0u;
      }
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        const long long j = j0 + r * 32 + lane;
        if (j < end) atomicAdd(&sm.hist[w][(kb[r] >> shift) & 255u], 1u);  // the counts only: no order
      }
    }
    __syncthreads();
    // a pass whose digit is the same for every key moves nothing; the
    // decision is taken by the barrier itself, so every warp sees the same
    // value and no shared flag outlives the pass
    bool one_digit = false;
    if (tid < 256) {
      uint32_t t = 0;
      for (int ww = 0; ww < NW; ++ww) t += sm.hist[ww][tid];
      one_digit = (long long)t == n;
    }
    if (__syncthreads_or(one_digit)) continue;
    // exclusive scan in (digit, warp) order: CPT counters per thread
    constexpr int CPT = NW * 256 / NT;
    static_assert(CPT * NT == NW * 256, "counter split");
    uint32_t loc[CPT];
    uint32_t s = 0;
#pragma unroll
    for (int r = 0; r < CPT; ++r) {
      const int i = tid * CPT + r;  // i = digit*NW + warp
      loc[r] = sm.hist[i % NW][i / NW];
      s += loc[r];
    }
    uint32_t tot;
    uint32_t ex = block_excl_scan_add(s, sm.iscr, tot);
#pragma unroll
    for (int r = 0; r < CPT; ++r) {
      const int i = tid * CPT + r;
      sm.hist[i % NW][i / NW] = ex;
      ex += loc[r];
    }
    __syncthreads();
    for (long long j00 = beg; j00 < end; j00 += 32 * RB) {
      uint32_t kb[RB], vb[RB];
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        const long long j = j00 + r * 32 + lane;
        kb[r] = j < end ? kin[j] : 0u;
        vb[r] = j < end ? vin[j] : 0u;
      }
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        const long long j = j00 + r * 32 + lane;
        const bool valid = j < end;
        const uint32_t key = kb[r];
        const uint32_t val = vb[r];
        const uint32_t d = valid ? ((key >> shift) & 255u) : 256u + (uint32_t)lane;
        const uint32_t peers = match_digit9(d);
        const uint32_t lower = peers & ((1u << lane) - 1u);
        uint32_t dst = 0;
        if (valid) dst = sm.hist[w][d] + (uint32_t)__popc(lower);
        __syncwarp();
        if (valid) {
          kout[dst] = key;
          vout[dst] = val;
          if (lower == 0u) sm.hist[w][d] += (uint32_t)__popc(peers);
        }
        __syncwarp();
      }
    }
    __syncthreads();
    cur ^= 1;
  }
  return cur;
}

}  // namespace sort
}  // namespace pesti
