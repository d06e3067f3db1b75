/*
 * CPU oracle for the PESTI token sampler -- TEST INFRASTRUCTURE ONLY.
 * Restates llm-runner/src/transformer/sampling.rs:39-134; see sampler_ref.h.
 *
 * Build flags matter: -O2 -fno-fast-math -ffp-contract=off, so that every f32
 * operation is a single IEEE operation in program order, like the Rust code
 * (Rust never contracts a*b+c into an FMA and never reassociates float sums).
 */
#include "sampler_ref.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <thread>
#include <utility>
#include <vector>

namespace {

struct Pair {
  float p;
  int64_t i;
};

inline float exp_mode_apply(float x, int mode) {
  if (mode == ORACLE_EXP_CORRECTLY_ROUNDED) return oracle_exp_cr(x);
  return expf(x);  // f32::exp -> libm expf (glibc on Linux)
}

// sampling.rs:125-134
std::vector<float> softmax(const std::vector<float>& logits, int exp_mode) {
  // logits.iter().cloned().fold(f32::NEG_INFINITY, f32::max); f32::max returns
  // the non-NaN operand, as fmaxf does.
  float max_val = -std::numeric_limits<float>::infinity();
  for (float v : logits) max_val = fmaxf(max_val, v);
  std::vector<float> exps(logits.size());
  for (size_t i = 0; i < logits.size(); ++i) exps[i] = exp_mode_apply(logits[i] - max_val, exp_mode);
  // exps.iter().sum(): a sequential f32 fold in index order (neutral -0.0).
  float sum = -0.0f;
  for (float e : exps) sum = sum + e;
  std::vector<float> out(logits.size());
  if (sum > 0.0f) {
    for (size_t i = 0; i < exps.size(); ++i) out[i] = exps[i] / sum;
  } else {
    const float u = 1.0f / static_cast<float>(logits.size());
    for (size_t i = 0; i < out.size(); ++i) out[i] = u;
  }
  return out;
}

// Stable sort by probability, descending: slice::sort_by with
// b.0.partial_cmp(&a.0).unwrap_or(Equal) (sampling.rs:60,67).  Probabilities
// are never NaN here (softmax yields finite values or the uniform fallback),
// so `a.p > b.p` is the same strict weak order.
void sort_desc_stable(std::vector<Pair>& v) {
  std::stable_sort(v.begin(), v.end(), [](const Pair& a, const Pair& b) { return a.p > b.p; });
}

}  // namespace

extern "C" {

float oracle_exp_cr(float x) {
  // Correctly rounded exp: the 64-bit-mantissa expl result is rounded once to
  // float.  Over the domain the sampler reaches (x <= 0) this agrees with the
  // CUDA path's exp on every input (checked exhaustively by
  // tests/test_exp_exhaustive.py).
  return static_cast<float>(expl(static_cast<long double>(x)));
}

// sampling.rs:115-122.  Iterator::max_by keeps the running best only when
// compare(best, next) == Greater; Equal (including any NaN comparison) moves
// to `next`, so the last of equal maxima wins and a NaN restarts the scan.
uint32_t oracle_argmax(const float* logits, int64_t V) {
  if (V <= 0) return 0;  // .unwrap_or(0)
  int64_t best = 0;
  for (int64_t i = 1; i < V; ++i) {
    if (!(logits[best] > logits[i])) best = i;
  }
  return static_cast<uint32_t>(best);
}

uint32_t oracle_argmax_first(const float* logits, int64_t V) {
  int64_t best = -1;
  for (int64_t i = 0; i < V; ++i) {
    if (std::isnan(logits[i])) continue;
    if (best < 0 || logits[i] > logits[best]) best = i;
  }
  return best < 0 ? 0u : static_cast<uint32_t>(best);
}

uint32_t oracle_sample(const float* logits, int64_t V, float temperature, float top_p,
                       int64_t top_k, float r, int exp_mode, float* kept_p,
                       uint32_t* kept_idx, int64_t kept_width, int64_t* kept_count,
                       float* boundary_dist) {
  if (boundary_dist) *boundary_dist = std::numeric_limits<float>::infinity();
  // sampling.rs:43-50: temperature scaling (IEEE division, no reciprocal).
  std::vector<float> scaled(static_cast<size_t>(V));
  if (temperature > 0.0f) {
    for (int64_t i = 0; i < V; ++i) scaled[i] = logits[i] / temperature;
  } else {
    for (int64_t i = 0; i < V; ++i) scaled[i] = logits[i];
  }
  // sampling.rs:53
  std::vector<float> probs = softmax(scaled, exp_mode);
  // sampling.rs:56-57
  std::vector<Pair> ip(static_cast<size_t>(V));
  for (int64_t i = 0; i < V; ++i) ip[i] = Pair{probs[i], i};
  // sampling.rs:59-63: top-k
  if (top_k > 0) {
    sort_desc_stable(ip);
    const int64_t k = std::min<int64_t>(top_k, static_cast<int64_t>(ip.size()));
    ip.resize(static_cast<size_t>(k));
  }
  // sampling.rs:65-78: top-p, only when top_k == 0
  if (top_p > 0.0f && top_k == 0) {
    sort_desc_stable(ip);
    float cumsum = 0.0f;
    size_t cutoff = ip.size();
    for (size_t i = 0; i < ip.size(); ++i) {
      cumsum += ip[i].p;
      if (cumsum >= top_p) {
        cutoff = i + 1;
        break;
      }
    }
    ip.resize(cutoff);
  }
  if (kept_count) *kept_count = static_cast<int64_t>(ip.size());
  if (kept_p || kept_idx) {
    for (int64_t j = 0; j < kept_width; ++j) {
      const bool in = j < static_cast<int64_t>(ip.size());
      if (kept_p) kept_p[j] = in ? ip[j].p : 0.0f;
      if (kept_idx) kept_idx[j] = in ? static_cast<uint32_t>(ip[j].i) : 0xffffffffu;
    }
  }
  // sampling.rs:81-90: total and the argmax fallback on the raw logits
  float total = -0.0f;
  for (const Pair& q : ip) total = total + q.p;
  if (total <= 0.0f) return oracle_argmax(logits, V);
  // sampling.rs:92-95
  std::vector<Pair> norm(ip.size());
  for (size_t i = 0; i < ip.size(); ++i) norm[i] = Pair{ip[i].p / total, ip[i].i};
  // sampling.rs:97-105: inverse-CDF walk
  float cumsum = 0.0f;
  float dist = std::numeric_limits<float>::infinity();
  int64_t found = -1;
  for (size_t j = 0; j < norm.size(); ++j) {
    cumsum += norm[j].p;
    if (boundary_dist) dist = std::min(dist, std::fabs(r - cumsum));
    if (found < 0 && r <= cumsum) {
      found = norm[j].i;
      if (!boundary_dist) break;
      // keep scanning the next cumulative sum only, for the distance report
      if (j + 1 < norm.size()) {
        float c2 = cumsum + norm[j + 1].p;
        dist = std::min(dist, std::fabs(r - c2));
      }
      break;
    }
  }
  if (boundary_dist) *boundary_dist = dist;
  if (found >= 0) return static_cast<uint32_t>(found);
  // sampling.rs:107-111: fall back to the last kept token
  return norm.empty() ? 0u : static_cast<uint32_t>(norm.back().i);
}

void oracle_sample_batch(const float* logits, int64_t B, int64_t V, int64_t ld,
                         const oracle_params* params, int params_per_row, const float* u,
                         int exp_mode, uint32_t* out, float* kept_p, uint32_t* kept_idx,
                         int64_t kept_width, int64_t* kept_count, float* boundary_dist,
                         int nthreads) {
  if (nthreads <= 0) nthreads = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
  nthreads = static_cast<int>(std::min<int64_t>(nthreads, std::max<int64_t>(B, 1)));
  auto work = [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) {
      const oracle_params& p = params[params_per_row ? b : 0];
      const float* row = logits + b * ld;
      float* kp = kept_p ? kept_p + b * kept_width : nullptr;
      uint32_t* ki = kept_idx ? kept_idx + b * kept_width : nullptr;
      int64_t* kc = kept_count ? kept_count + b : nullptr;
      float* bd = boundary_dist ? boundary_dist + b : nullptr;
      // model.rs:517-521 / model.rs:823-828
      if ((p.flags & ORACLE_FLAG_GREEDY_IF_ZERO_T) && p.temperature == 0.0f) {
        out[b] = (p.flags & ORACLE_FLAG_ARGMAX_FIRST) ? oracle_argmax_first(row, V)
                                                       : oracle_argmax(row, V);
        if (kc) *kc = 0;
        if (bd) *bd = std::numeric_limits<float>::infinity();
        if (kp || ki) {
          for (int64_t j = 0; j < kept_width; ++j) {
            if (kp) kp[j] = 0.0f;
            if (ki) ki[j] = 0xffffffffu;
          }
        }
        continue;
      }
      out[b] = oracle_sample(row, V, p.temperature, p.top_p, static_cast<int64_t>(p.top_k),
                             u[b], exp_mode, kp, ki, kept_width, kc, bd);
    }
  };
  if (nthreads == 1) {
    work(0, B);
    return;
  }
  std::vector<std::thread> ts;
  const int64_t chunk = (B + nthreads - 1) / nthreads;
  for (int t = 0; t < nthreads; ++t) {
    const int64_t b0 = t * chunk, b1 = std::min(B, b0 + chunk);
    if (b0 >= b1) break;
    ts.emplace_back(work, b0, b1);
  }
  for (auto& t : ts) t.join();
}

// sampling.rs:43-50 (scaling) and :127 (exp of the difference to the max)
void oracle_softmax_terms(const float* logits, int64_t n, float temperature, float m, int exp_mode,
                          float* out) {
  for (int64_t i = 0; i < n; ++i) {
    const float x = temperature > 0.0f ? logits[i] / temperature : logits[i];
    out[i] = exp_mode_apply(x - m, exp_mode);
  }
}

// sampling.rs:128 (exps.iter().sum()) from an arbitrary start
float oracle_fold(const float* v, int64_t n, float s0) {
  float s = s0;
  for (int64_t i = 0; i < n; ++i) s = s + v[i];
  return s;
}

void oracle_bf16_to_f32(const uint16_t* in, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    uint32_t bits = static_cast<uint32_t>(in[i]) << 16;
    std::memcpy(&out[i], &bits, 4);
  }
}

}  // extern "C"
