/*
 * pesti_profile.h -- instrumentation of the sampler library (no counterpart in
 * the reference).  When enabled on a handle, every batch call records CUDA
 * events around each of its three kernels (slice max, survivors, row
 * sampler) on the launching stream; the read call waits for them and returns
 * the summed device times, so a benchmark can report each kernel's own
 * duration.  Recording costs four event records per call.
 */
#ifndef PESTI_PROFILE_H
#define PESTI_PROFILE_H
#include "pesti_sampler.h"
#ifdef __cplusplus
extern "C" {
#endif
/* enable != 0 starts recording (clears earlier records); 0 stops. */
int pesti_profile_enable(pesti_sampler* s, int enable);
/* Sums of the recorded slice-max, survivor and row-kernel times (ms) and the
 * number of calls recorded (at most 4096 are kept).  For a sharded call the
 * three intervals are instead: the HBM pass over the shard, everything from
 * there to the end of the last exchange, and the finish. */
int pesti_profile_read(pesti_sampler* s, double* max_ms, double* surv_ms, double* row_ms, int* calls);
#ifdef __cplusplus
}
#endif
#endif
