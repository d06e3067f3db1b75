/*
 * CPU oracle for the PESTI token sampler -- TEST INFRASTRUCTURE ONLY.
 *
 * This is a line-by-line restatement, in C++17, of the reference Rust sampler
 *   llm-runner/src/transformer/sampling.rs:39-134  (sample, argmax, softmax)
 * and of the caller branch in
 *   llm-runner/src/transformer/model.rs:517-521    (temperature == 0 -> argmax)
 *   llm-runner/src/model.rs:823-828                (same branch in CpuModel::run)
 *
 * It exists only to check the CUDA path (tests/, __graft_entry__.smoke()) and
 * to time the reference algorithm on host cores (bench.py's cpu_baseline leg
 * and `--impl reference`).  Nothing in the product library links or calls it.
 *
 * The Rust toolchain is absent from this image, so the reference itself cannot
 * be built; parity of this restatement is pinned only by the reference's own
 * unit tests (sampling.rs:142-207, restated in tests/test_oracle.py), which
 * check properties, not golden token ids.
 *
 * Differences from the Rust function, all forced by the boundary:
 *  - `rng.random::<f32>()` (sampling.rs:98) is replaced by an explicit draw
 *    `r` in [0,1) supplied by the caller (rand 0.10.1 StdRng is not vendored).
 *  - exp: mode 0 calls the platform expf, which is what Rust's f32::exp lowers
 *    to on Linux (glibc).  Mode 1 uses the correctly rounded exp (long double
 *    expl rounded to float); the CUDA path computes the correctly rounded value,
 *    so mode 1 lets the tests check the rest of the arithmetic bit for bit.
 */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
  float temperature; /* SamplingConfig::temperature (sampling.rs:14) */
  float top_p;       /* SamplingConfig::top_p       (sampling.rs:16) */
  uint32_t top_k;    /* SamplingConfig::top_k       (sampling.rs:18) */
  uint32_t flags;    /* ORACLE_FLAG_* below */
} oracle_params;

/* Apply the generate() branch: temperature == 0.0 -> argmax (model.rs:517-521). */
#define ORACLE_FLAG_GREEDY_IF_ZERO_T 1u
/* argmax ties go to the lowest index instead of the last one (sampling.rs:115-122). */
#define ORACLE_FLAG_ARGMAX_FIRST 2u

#define ORACLE_EXP_PLATFORM 0
#define ORACLE_EXP_CORRECTLY_ROUNDED 1

/* sampling.rs:115-122: Iterator::max_by with partial_cmp -> last of equal maxima. */
uint32_t oracle_argmax(const float* logits, int64_t V);
/* Lowest-index variant (NaN entries are skipped). */
uint32_t oracle_argmax_first(const float* logits, int64_t V);

/*
 * sampling.rs:39-112 for one row.
 *  r            : the uniform draw that replaces rng.random::<f32>()
 *  kept_p/idx   : optional; the first kept_width entries of the final kept list
 *                 (after top-k / top-p truncation, in the list's order)
 *  kept_count   : optional; length of the kept list
 *  boundary_dist: optional; min |r - cumsum_j| over the draw's cumulative sums
 *                 (the distance of r from the nearest sampling boundary); set to
 *                 +inf when the draw is not reached (argmax fallback)
 */
uint32_t oracle_sample(const float* logits, int64_t V, float temperature, float top_p,
                       int64_t top_k, float r, int exp_mode, float* kept_p,
                       uint32_t* kept_idx, int64_t kept_width, int64_t* kept_count,
                       float* boundary_dist);

/*
 * Batched driver over rows of a [B, ld] row-major f32 array (first V columns
 * used).  params has B entries when params_per_row != 0, else one entry.
 * Rows are spread over nthreads host threads (<= 0: all hardware threads).
 * Per-row outputs (kept_* have kept_width entries per row) may be NULL.
 */
void oracle_sample_batch(const float* logits, int64_t B, int64_t V, int64_t ld,
                         const oracle_params* params, int params_per_row, const float* u,
                         int exp_mode, uint32_t* out, float* kept_p, uint32_t* kept_idx,
                         int64_t kept_width, int64_t* kept_count, float* boundary_dist,
                         int nthreads);

/* bf16 -> f32 widening of a [n] array (exact). */
void oracle_bf16_to_f32(const uint16_t* in, float* out, int64_t n);

/* The exp used by mode 1, exposed for the exhaustive exp check. */
float oracle_exp_cr(float x);

/*
 * Pieces of sampling.rs:43-50 and :125-128 for checking a vocabulary-sharded
 * evaluation: the softmax terms e_i = exp(scaled_i - m) of n logits
 * (scaled_i = logits_i / temperature when temperature > 0, else logits_i),
 * with m the max of the scaled WHOLE row given by the caller, and the
 * sequential f32 fold s = s0; s = s + v[i] of n terms from any start s0.
 */
void oracle_softmax_terms(const float* logits, int64_t n, float temperature, float m, int exp_mode,
                          float* out);
float oracle_fold(const float* v, int64_t n, float s0);

#ifdef __cplusplus
}
#endif
