/*
 * pesti_sampler.h -- C ABI of the B200 (sm_100a) token sampler.
 *
 * Drop-in boundary for the PESTI sampling step
 *   temperature -> softmax -> top-k -> top-p -> inverse-CDF draw
 * that the reference implements in Rust as
 *   pub fn sample(logits: &[f32], config: &SamplingConfig, rng: &mut StdRng) -> u32
 *                                       (llm-runner/src/transformer/sampling.rs:39)
 *   pub fn argmax(logits: &[f32]) -> u32 (llm-runner/src/transformer/sampling.rs:115)
 * called from LlamaModel::generate (llm-runner/src/transformer/model.rs:517-521) and
 * CpuModel::run (llm-runner/src/model.rs:823-828).  The reference has no GPU
 * sampler; this library takes the place of the stubbed GPU crate
 * (cuda-oxide/src/main.rs:1-3) and is the sampling entry the kernel layer
 * (llm-runner/src/kernel/mod.rs) lacks.
 *
 * Results are those of the reference algorithm, bit for bit, given the same
 * per-row uniform draw u (the value `rng.random::<f32>()` returns at
 * sampling.rs:98) and given exp correctly rounded (the reference calls the
 * platform expf, which differs from the correctly rounded value by one ulp on
 * about 6e-4 of its inputs).
 *
 * Conventions (mirroring the reference kernel layer):
 *  - every call returns 0 on success or a negative PESTI_E_* code; the message
 *    of the last failure on the calling thread is pesti_last_error();
 *  - device pointers are plain addresses (RawHandle(u64) in
 *    llm-runner/src/kernel/memory.rs:22); the caller owns every buffer;
 *  - batch calls are stream-ordered and never synchronize the host;
 *  - there is no CPU fallback: without a usable sm_100 device the calls fail.
 */
#ifndef PESTI_SAMPLER_H
#define PESTI_SAMPLER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PESTI_OK 0
#define PESTI_E_INVALID_ARG (-1)
#define PESTI_E_CUDA (-2)
#define PESTI_E_NCCL (-3)
#define PESTI_E_TIMEOUT (-4)
#define PESTI_E_UNSUPPORTED (-5)
#define PESTI_E_NO_DEVICE (-6)

/* Logit element types.  BF16 and F16 logits are widened to f32 exactly, so
 * results are those of the reference on the widened values (a caller of the
 * reference's &[f32] API would widen them the same way).
 *
 * FP8_E4M3 (OCP E4M3FN: no infinities, S.1111.111 is NaN) and FP8_E5M2 (IEEE
 * layout with infinities and NaNs), the float8 crate's F8E4M3 and F8E5M2,
 * are taken by pesti_sample_batch and pesti_argmax_batch only.  Every value
 * of both formats is an f16 value: the call first widens the [B, V] logits
 * exactly into f16 in the handle's workspace (2 bytes per logit, on the
 * call's stream), then samples those.  The other entry points refuse them
 * with PESTI_E_INVALID_ARG. */
typedef enum { PESTI_F32 = 0, PESTI_BF16 = 1, PESTI_F16 = 2, PESTI_FP8_E4M3 = 3, PESTI_FP8_E5M2 = 4 } pesti_dtype;

/* Per-row sampling parameters: SamplingConfig (sampling.rs:12-21) without the
 * seed, which sample() never reads. */
typedef struct {
  float temperature; /* sampling.rs:14; > 0 scales the logits, otherwise none */
  float top_p;       /* sampling.rs:16; used only when top_k == 0 (sampling.rs:66) */
  uint32_t top_k;    /* sampling.rs:18; 0 = disabled */
  uint32_t flags;    /* PESTI_FLAG_* */
} pesti_sampling_params;

/* Apply the caller branch of generate()/run(): temperature == 0.0 -> argmax
 * (transformer/model.rs:517-521, model.rs:823-828).  Without it a zero
 * temperature means "no scaling", as in sample() itself (sampling.rs:43). */
#define PESTI_FLAG_GREEDY_IF_ZERO_T 1u
/* argmax ties go to the lowest index.  Default: the last index, as
 * Iterator::max_by returns (sampling.rs:115-122). */
#define PESTI_FLAG_ARGMAX_FIRST 2u

typedef struct pesti_sampler pesti_sampler;

/* Creates a sampler bound to CUDA device `device`: events, a workspace that
 * grows on demand, and a private stream for pesti_sample_row_host.  Replaces
 * the context set-up of CudaRuntime::new (llm-runner/src/cuda_runtime.rs:92-176)
 * for this path.  A handle may be used from one thread at a time. */
int pesti_sampler_create(int device, pesti_sampler** out);
void pesti_sampler_destroy(pesti_sampler* s);

/*
 * Batched sample over row-major logits [B, ld] (first V columns of each row),
 * dtype F32, BF16 or F16, on device memory.  Replaces, per row, the call
 *   generate():  if T == 0 { argmax(row) } else { sample(row, cfg, rng) }
 * (model.rs:517-521) when params carry PESTI_FLAG_GREEDY_IF_ZERO_T, and
 * sample(row, cfg, rng) (sampling.rs:39) otherwise.
 *
 *  params          host pointer: B entries if params_per_row, else 1 entry.
 *                  When params_on_device != 0 it is a device pointer instead.
 *  d_u             device [B] f32: the draw r of each row (sampling.rs:98).
 *  d_out_tokens    device [B] u32.
 *  d_kept_p/idx    optional device [B, kept_width]: the first kept_width
 *                  entries of each row's kept list (the (probability, index)
 *                  pairs left after top-k / top-p, sampling.rs:56-78), padded
 *                  with 0 / 0xffffffff.  Either may be NULL.
 *  d_kept_count    optional device [B] i64: length of each kept list (0 for
 *                  greedy rows).
 *  stream          cudaStream_t; NULL is the legacy default stream, as for
 *                  CUDA's own calls (PyTorch's default stream is that stream).
 */
int pesti_sample_batch(pesti_sampler* s, const void* d_logits, pesti_dtype dtype, int64_t B,
                       int64_t V, int64_t ld, const pesti_sampling_params* params,
                       int params_per_row, int params_on_device, const float* d_u,
                       uint32_t* d_out_tokens, float* d_kept_p, uint32_t* d_kept_idx,
                       int64_t kept_width, int64_t* d_kept_count, void* stream);

/* Batched argmax (sampling.rs:115-122, last of equal maxima; NaN handled as
 * Iterator::max_by does) over device logits.  flags: PESTI_FLAG_ARGMAX_FIRST. */
int pesti_argmax_batch(pesti_sampler* s, const void* d_logits, pesti_dtype dtype, int64_t B,
                       int64_t V, int64_t ld, uint32_t flags, uint32_t* d_out_tokens,
                       void* stream);

/* One row from HOST memory, synchronous: the drop-in for
 * sample(&logits, &cfg, &mut rng) (sampling.rs:39) with r drawn by the caller;
 * honours PESTI_FLAG_GREEDY_IF_ZERO_T like the batch call. */
int pesti_sample_row_host(pesti_sampler* s, const float* h_logits, int64_t V,
                          const pesti_sampling_params* params, float u, uint32_t* out_token);

/*
 * No counterpart in the reference.
 *
 * pesti_sample_batch without a handle and without any device allocation, for
 * callers that cannot allocate device memory while they sample: a decode loop
 * that has handed the rest of HBM to its KV-cache page pool, where a
 * cudaMalloc would fail, or one that must not stall its other streams, which
 * cudaMalloc and cudaFree do (pesti_sample_batch grows its workspace with them
 * whenever it meets a larger batch).
 *
 * Arguments and results are those of pesti_sample_batch.  It runs on the
 * calling thread's current device; stream NULL is the legacy default stream.
 * Its only device memory besides the caller's buffers is one static array of
 * PESTI_NOALLOC_SCRATCH_BYTES on each device, shared by every call:
 *  - a call that needs more scratch than the array holds fails with
 *    PESTI_E_INVALID_ARG and launches nothing.  A call needs about 16 bytes
 *    per logit (B*V) when every row is greedy or uses top_k <= 1024, 36 bytes
 *    per logit otherwise (top-p, no filter, larger top_k, or params on the
 *    device), plus host per-row params and at most about 0.3 MB per row:
 *    8 rows of V = 128256 with top-p need about 37 MB;
 *  - calls whose GPU work overlaps (on streams with no order between them)
 *    race on the array: order them on one stream;
 *  - host per-row params are copied into the array on the stream.  From
 *    ordinary (pageable) host memory the copy has taken the values when the
 *    call returns, so the caller may reuse them at once.  From page-locked
 *    host memory (cudaMallocHost, cudaHostRegister, torch's pin_memory) the
 *    copy runs later, when the stream reaches it: the caller must leave those
 *    params unchanged until then (synchronize the stream, or wait on an event
 *    recorded after the call, before rewriting them);
 *  - a single params entry on the device is read back with a stream
 *    synchronization, as in pesti_sample_batch.
 * The first call on a device does the set-up: it looks the array up with
 * cudaGetSymbolAddress, which loads it onto that device.  Make that first call
 * before any stream capture.  No call allocates: none calls cudaMalloc,
 * cudaFree or an allocating library routine.
 */
#define PESTI_NOALLOC_SCRATCH_BYTES (64ull << 20)
int pesti_sample_batch_noalloc(const void* d_logits, pesti_dtype dtype, int64_t B, int64_t V,
                               int64_t ld, const pesti_sampling_params* params,
                               int params_per_row, int params_on_device, const float* d_u,
                               uint32_t* d_out_tokens, float* d_kept_p, uint32_t* d_kept_idx,
                               int64_t kept_width, int64_t* d_kept_count, void* stream);

/*
 * No counterpart in the reference (it has no multi-GPU path).
 *
 * Vocabulary-sharded sampling: each of the communicator's ranks holds one
 * contiguous column range of every row, all ranges V_shard wide and in rank
 * order (rank r holds columns [r*V_shard, (r+1)*V_shard) of rows that are
 * world*V_shard long).  Every rank calls pesti_sample_batch_sharded with the
 * same B, V_shard, params and u (the draws of all B rows), its own shard as
 * d_logits [B, ld], and receives the tokens and kept lists of ALL B rows.
 * Results are those of pesti_sample_batch on the whole rows, bit for bit.
 *
 * Top-k rows (1 <= top_k <= 256) and greedy rows are sampled without moving
 * logits: three NCCL all-gathers of per-row summaries (a few hundred bytes
 * per row and shard).  Other rows (top-p, no filter, larger top_k, NaN, and
 * the rare row the sharded algorithm cannot settle) take a gathered path:
 * their shards are all-gathered into whole rows on every rank and sampled
 * there.  The call synchronizes the stream once, to learn which rows those
 * are.
 *
 * A communicator is made once per rank: one rank calls pesti_comm_id, the
 * caller broadcasts its PESTI_COMM_ID_BYTES bytes to the others, and every
 * rank calls pesti_comm_create with them (ncclGetUniqueId /
 * ncclCommInitRank; NCCL is loaded from libnccl.so.2 on first use).  The
 * sampler and the communicator must be on the same device.
 */
typedef struct pesti_comm pesti_comm;
#define PESTI_COMM_ID_BYTES 128
int pesti_comm_id(void* id);
int pesti_comm_create(int world_size, int rank, const void* id, int device, pesti_comm** out);
/*
 * No counterpart in the reference, whose only failure detection is the HTTP
 * health check of a remote runner with a 3 s limit
 * (llm-runner/src/remote_discovery.rs:36-70).
 *
 * pesti_comm_create with a deadline (pesti_comm_create uses 120000 ms).  The
 * communicator is made non-blocking (ncclCommInitRankConfig with blocking = 0)
 * and its set-up is polled with ncclCommGetAsyncError: if every rank has not
 * joined after timeout_ms, the set-up is aborted (ncclCommAbort) and the call
 * returns PESTI_E_TIMEOUT, so a rank that exits or never starts does not hang
 * the others.  The same deadline bounds, on the host, each
 * pesti_sample_batch_sharded call's exchanges: a call whose all-gathers do not
 * complete within timeout_ms of its start, or that reports an NCCL error,
 * aborts the communicator and returns PESTI_E_TIMEOUT (or PESTI_E_NCCL);
 * every later call on that communicator fails with PESTI_E_NCCL, and
 * pesti_comm_destroy releases it.
 */
int pesti_comm_create_timed(int world_size, int rank, const void* id, int device, int timeout_ms, pesti_comm** out);
void pesti_comm_destroy(pesti_comm* c);
int pesti_sample_batch_sharded(pesti_sampler* s, pesti_comm* c, const void* d_logits, pesti_dtype dtype,
                               int64_t B, int64_t V_shard, int64_t ld, const pesti_sampling_params* params,
                               int params_per_row, int params_on_device, const float* d_u,
                               uint32_t* d_out_tokens, float* d_kept_p, uint32_t* d_kept_idx,
                               int64_t kept_width, int64_t* d_kept_count, void* stream);

/*
 * No counterpart in the reference, whose draw comes from StdRng on the host
 * (sampling.rs:98) once per sample() call.
 *
 * Per-row draws on the device, for a decode loop that keeps its generators
 * on the GPU: no draw crosses from the host each step, and the draws feed
 * d_u of the batch calls directly.  Each row has its own PCG32 generator
 * (O'Neill 2014, XSH-RR 64->32) in d_state: [B][2] u64, state then
 * increment, owned by the caller.
 *  - pesti_pcg32_seed: row b's generator is the one seeded with `seed` on
 *    stream first_stream + b;
 *  - pesti_pcg32_draw: d_u[b] = (next_u32 >> 8) * 2^-24 (the [0, 1) 24-bit
 *    grid of the reference's f32 draw), and row b's generator advances.
 * Both are stream-ordered (NULL: the legacy default stream) and allocate
 * nothing.
 */
int pesti_pcg32_seed(uint64_t* d_state, int64_t B, uint64_t seed, uint64_t first_stream, void* stream);
int pesti_pcg32_draw(uint64_t* d_state, int64_t B, float* d_u, void* stream);

/*
 * The loop control of generate() (transformer/model.rs:508-531: stop tokens,
 * the max_tokens bound, pos >= max_seq_len) on the device, for B sequences
 * decoded together.  Called after each step's sample, it keeps each
 * sequence's tokens on the GPU and feeds the next step's input, so a decode
 * loop reads nothing back per step.  For every row b with d_done[b] == 0,
 * t = d_next[b] (the step's sampled token):
 *  - t in d_stop[0..n_stop): the row finishes (d_done[b] = 1) and t is not
 *    kept (the reference breaks before pushing it);
 *  - otherwise d_generated[b*cap + d_count[b]] = t, d_count[b] += 1 and
 *    d_last[b] = t (the next forward's input token); the row finishes when
 *    d_count[b] reaches max_seq_len (d_done[b] = 3) or max_tokens (2).
 * A row whose d_count[b] is already max_tokens finishes without taking t.
 * Finished rows are left as they are, whatever d_next holds for them.
 * d_active (optional; mapped host memory works) receives the number of rows
 * still running, for a host that checks it now and then instead of
 * synchronising every step.  The caller zeroes d_count and d_done before the
 * first step; cap >= min(max_tokens, max_seq_len).  Stream-ordered (NULL: the
 * legacy default stream); allocates nothing.
 */
int pesti_generate_advance(const uint32_t* d_next, int64_t B, const uint32_t* d_stop, int64_t n_stop,
                           int64_t max_tokens, int64_t max_seq_len, uint32_t* d_generated, int64_t cap,
                           int32_t* d_count, uint8_t* d_done, uint32_t* d_last, int32_t* d_active, void* stream);

/*
 * The sampler chain of PESTI's llama.cpp backend: `build_sampler`
 * (llm-runner/src/llama.rs:465-508) over the fields of its SamplingConfig
 * (llm-runner/src/llama/sampler.rs:19-79), for B rows with one parameter set.
 * The stages run in build_sampler's order and under its gates:
 *   temperature         temperature > 0
 *   top-k               top_k > 0
 *   top-p (min_keep 0)  top_p > 0 (1 or more keeps every candidate)
 *   min-p (min_keep 256) min_p > 0: p >= min_p * p_max, at least 256 kept
 *   top-n-sigma         0 < tfs < 1, n = tfs: logit >= max - n * sigma
 *   typical (min_keep 0) 0 < typical_p < 1
 *   penalties           repetition_penalty != 1, over the last repeat_last_n
 *                       tokens of the row's history (all of it when
 *                       repeat_last_n < 0, none when 0), with
 *                       frequency_penalty and presence_penalty (0.0 in the
 *                       reference)
 * and end with an inverse-CDF draw on d_u[b] over the candidates sorted by
 * logit (the chain as built has no selecting stage; the draw is the Rust
 * sampler's, sampling.rs:97-111).  The stages restate the published filters
 * of llama.cpp, whose sources are not in the reference tree; probabilities
 * are computed in f64.  NaN logits count as -inf.
 *
 * d_history: [B, history_ld] int32 token ids (the row's recent tokens, oldest
 * first), d_history_len (optional): [B] counts of valid leading entries
 * (history_ld for every row when NULL); ids outside [0, V) are ignored.  The
 * window (min(repeat_last_n, history_ld), or history_ld) is at most 8192.
 * d_out_kept (optional): [B] candidates left before the draw.
 * Logits: PESTI_F32, PESTI_BF16, PESTI_F16, and the fp8 types (widened to f16
 * in the handle's workspace first).  Scratch: 16 bytes per logit in the
 * handle's workspace.  Stream-ordered; one 1024-thread block per row.
 */
typedef struct {
  float temperature;        /* llama/sampler.rs:33 */
  int32_t top_k;            /* :36 */
  float top_p;              /* :40 */
  float min_p;              /* :44 */
  float tfs;                /* :47, passed to top-n-sigma (llama.rs:488-491) */
  float typical_p;          /* :50 */
  float repetition_penalty; /* :62 */
  int32_t repeat_last_n;    /* :65 */
  float frequency_penalty;  /* 0.0 in build_sampler (llama.rs:502-503) */
  float presence_penalty;   /* 0.0 in build_sampler */
} pesti_llama_chain_params;

int pesti_llama_chain_batch(pesti_sampler* s, const void* d_logits, pesti_dtype dtype, int64_t B, int64_t V,
                            int64_t ld, const pesti_llama_chain_params* params, const int32_t* d_history,
                            const int32_t* d_history_len, int64_t history_ld, const float* d_u,
                            int32_t* d_out_tokens, int32_t* d_out_kept, void* stream);

/* Message of the last failure on the calling thread ("" if none). */
const char* pesti_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* PESTI_SAMPLER_H */
