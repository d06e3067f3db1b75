/*
 * pesti_testing.h -- test entry points of the sampler library (no
 * counterpart in the reference).
 */
#ifndef PESTI_TESTING_H
#define PESTI_TESTING_H
#include "pesti_sampler.h"
#ifdef __cplusplus
extern "C" {
#endif
/*
 * The sharded call of pesti_sample_batch_sharded, with `shards` equally wide
 * vocabulary shards of the whole matrix d_logits [B, ld] (V a multiple of
 * `shards`) run one after another in this process on the handle's device,
 * the exchanges being plain device memory instead of NCCL: the sharded
 * algorithm on one GPU, for tests.  Results are those of pesti_sample_batch.
 */
int pesti_sample_batch_sharded_emulated(pesti_sampler* s, int shards, const void* d_logits, pesti_dtype dtype,
                                        int64_t B, int64_t V, int64_t ld, const pesti_sampling_params* params,
                                        int params_per_row, int params_on_device, const float* d_u,
                                        uint32_t* d_out_tokens, float* d_kept_p, uint32_t* d_kept_idx,
                                        int64_t kept_width, int64_t* d_kept_count, void* stream);
/* Rows of the handle's last sharded call that took the gathered path. */
int64_t pesti_last_gathered_rows(pesti_sampler* s);
/* The same rows by reason, counts[6]: [1] not a top-k row (top-p, no filter,
 * top_k > 256, NaN, or every probability equal), [2] a shard's fold entries
 * exceeded the row kernel's staging, [3] a shard's candidates exceeded its
 * sort, [4] the chained fold state left a shard's table, [5] the merged
 * candidates could not prove the top-k. */
int pesti_last_gathered_reasons(pesti_sampler* s, int64_t* counts);

/* The cluster pass (one thread-block cluster per row) takes batches of at
 * most 32 greedy and top-k (<= 256) rows, and every batch with bf16 top-p
 * rows (rows of at most 131072 f32 or 262144 16-bit columns).  mode -1 sends
 * every batch through the four-kernel pipeline instead, 1..16 sends every
 * batch the cluster pass can take through it with that many CTAs per row's
 * cluster, 0 restores the default.  Process-wide; for tests and
 * measurements. */
int pesti_testing_set_cluster(int mode);

/* The largest relative error of the hardware 2^y approximation
 * (ex2.approx.ftz.f32) over every float y in [-200, 0] and -inf, against
 * exp2 in double, on the current device (below y = -126 a flushed 0 counts
 * as exact): the classification's cheap exp assumes it is below
 * PESTI_EX2_APPROX_RELERR. */
int pesti_test_ex2_approx_max_relerr(double* out);
#ifdef __cplusplus
}
#endif
#endif
