// Host side of the sampler library: the C ABI of include/pesti_sampler.h.
// Launch geometry, workspace and error reporting live here; the arithmetic is
// in pesti_kernels.cuh.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <thread>
#include <climits>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/pesti_sampler.h"
#include "../../include/pesti_profile.h"
#include "../../include/pesti_testing.h"
#include "pesti_kernels.cuh"
#include "pesti_cluster.cuh"
#include "pesti_noalloc.h"
#include "pesti_shard.cuh"
#include "pesti_rng.cuh"
#include "pesti_generate.cuh"
#include "pesti_chain.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PESTI_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define PESTI_CUDA_TRY(expr, what)          \
  do {                                      \
    cudaError_t _e = (expr);                \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

}  // namespace

constexpr size_t kRowSmemLimit = 220 * 1024;
static_assert(sizeof(pesti::RowShared) + sizeof(pesti::NucSmem) <= kRowSmemLimit, "nucleus rows' shared memory");

struct pesti_sampler {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // rows whose completion counters (at the start of the workspace) are known
  // to be zero: the kernels leave the counters of their own call zero, and
  // the rest of the workspace may hold anything
  long long ctr_zero_rows = 0;
  pesti_sampling_params* d_params = nullptr;
  size_t d_params_cap = 0;
  pesti_sampling_params* h_params = nullptr;  // pinned staging
  size_t h_params_cap = 0;
  cudaEvent_t params_ev = nullptr;
  bool params_ev_used = false;
  // fp8 logits widened to f16 (grown on demand)
  void* d_wide = nullptr;
  size_t d_wide_cap = 0;
  // llama.cpp chain scratch: per logit an f32 logit, an int32 index and an
  // f64 weight (grown on demand)
  void* d_chain = nullptr;
  size_t d_chain_cap = 0;
  bool chain_smem_set = false;
  // single-row host API buffers
  float* d_row = nullptr;
  size_t d_row_cap = 0;
  float* d_u1 = nullptr;
  uint32_t* d_tok1 = nullptr;
  // instrumentation (pesti_profile.h)
  static constexpr int kProfMax = 4096;
  bool prof = false;
  int prof_n = 0;
  cudaEvent_t prof_ev[kProfMax][4] = {};
  // rows of the last sharded call that took the gathered path, by reason (GR_*)
  long long last_gathered_rows = 0;
  long long last_gathered_why[pesti::GR_KINDS] = {};
};

namespace {

struct Geometry {
  int P;
  long long SL;
};

Geometry pick_geometry(int num_sms, long long B, long long V, int ve) {
  const long long target = 4LL * num_sms;
  long long P = (target + B - 1) / std::max(1LL, B);
  // at most one 1024-element chunk per warp and sub-slice: a short batch of
  // short rows gets as many warps as its rows have chunks
  const long long pmax_v = std::max(1LL, (V + pesti::K1_WARPS * 1024LL - 1) / (pesti::K1_WARPS * 1024LL));
  P = std::max(1LL, std::min({P, pmax_v, (long long)(pesti::MAX_SUBS / pesti::K1_WARPS)}));
  // whole 16-byte-vector chunks per sub-slice (32 lanes x 16 bytes x 8 or 4
  // loads in flight = 1024 elements): only the row's last sub-slice has a tail
  const long long unit = 1024;
  long long SL = (V + P * pesti::K1_WARPS - 1) / (P * pesti::K1_WARPS);
  SL = std::max(unit, (SL + unit - 1) / unit * unit);
  P = std::max(1LL, (V + SL * pesti::K1_WARPS - 1) / (SL * pesti::K1_WARPS));
  return Geometry{(int)P, SL};
}

int ensure_ws(pesti_sampler* s, size_t bytes) {
  if (bytes <= s->ws_bytes) return PESTI_OK;
  if (s->ws) {
    cudaError_t e = cudaStreamSynchronize(s->stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    cudaDeviceSynchronize();
    cudaFree(s->ws);
    s->ws = nullptr;
    s->ws_bytes = 0;
  }
  const size_t want = bytes + bytes / 8;
  cudaError_t e = cudaMalloc(&s->ws, want);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(workspace)");
  // the per-row completion counters must start at zero (the kernels reset them)
  e = cudaMemset(s->ws, 0, want);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(workspace)");
  s->ws_bytes = want;
  s->ctr_zero_rows = LLONG_MAX;
  return PESTI_OK;
}

// The completion counters of B rows at the start of the workspace are zero
// on the stream before the first kernel of the call.
int zero_counters(pesti_sampler* s, long long B, cudaStream_t st) {
  if (B > s->ctr_zero_rows)
    PESTI_CUDA_TRY(cudaMemsetAsync(s->ws, 0, (size_t)B * sizeof(int), st), "cudaMemsetAsync(counters)");
  return PESTI_OK;
}

size_t align_up(size_t x) { return (x + 255) & ~(size_t)255; }

// Some row is neither greedy nor on the fast top-k path, so it needs the
// survivor pass (for the row kernel's generic path).
bool needs_survivor_pass(const pesti_sampling_params* p, long long n, long long V) {
  for (long long i = 0; i < n; ++i) {
    const bool greedy = (p[i].flags & PESTI_FLAG_GREEDY_IF_ZERO_T) && p[i].temperature == 0.0f;
    const long long k = std::min<long long>(p[i].top_k, V);
    if (!greedy && !(k >= 1 && k <= pesti::FAST_K)) return true;
  }
  return false;
}

// What the cluster pass can take of a batch whose host params are p[0..n):
// 0 not every row (some row is neither greedy nor top-k <= 256, nor a bf16
// top-p row), 1 every row greedy or top-k <= 256, 2 also bf16 top-p rows
// (finished by the row kernel from the cluster's exact softmax sum).
int cluster_kind(const pesti_sampling_params* p, long long n, long long V, pesti_dtype dtype) {
  int kind = 1;
  for (long long i = 0; i < n; ++i) {
    const bool greedy = (p[i].flags & PESTI_FLAG_GREEDY_IF_ZERO_T) && p[i].temperature == 0.0f;
    const long long k = std::min<long long>(p[i].top_k, V);
    if (greedy || (k >= 1 && k <= pesti::FAST_K)) continue;
    if (dtype == PESTI_BF16 && p[i].top_k == 0 && p[i].top_p > 0.0f) {
      kind = 2;
      continue;
    }
    return 0;
  }
  return kind;
}

bool needs_sorted_buffers(const pesti_sampling_params* p, long long n) {
  for (long long i = 0; i < n; ++i) {
    const bool greedy = (p[i].flags & PESTI_FLAG_GREEDY_IF_ZERO_T) && p[i].temperature == 0.0f;
    if (greedy) continue;
    if (p[i].top_k == 0) return true;  // top-p or no filter
    if (p[i].top_k > (uint32_t)pesti::TOPK_SMALL) return true;
  }
  return false;
}

// The row kernel's dynamic shared memory limit is a property of the function
// on each device, shared by every caller in the process: it is raised once,
// to the largest size any launch asks for, so that no caller lowers it under
// another.
constexpr int kMaxDevices = 64;
std::atomic<bool> g_row_limit_set[kMaxDevices];

int ensure_row_smem_limit(int device) {
  const bool cached = device >= 0 && device < kMaxDevices;
  if (cached && g_row_limit_set[device].load(std::memory_order_acquire)) return PESTI_OK;
  PESTI_CUDA_TRY(cudaFuncSetAttribute(pesti::row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kRowSmemLimit),
                 "cudaFuncSetAttribute(row_kernel)");
  PESTI_CUDA_TRY(cudaFuncSetAttribute(pesti::shard_table_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)pesti::TAB_SMEM),
                 "cudaFuncSetAttribute(shard_table_kernel)");
  const int fused = (int)sizeof(pesti::FusedShared);
  PESTI_CUDA_TRY(cudaFuncSetAttribute(pesti::fused_classify_kernel<float, 4, true>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, fused), "cudaFuncSetAttribute(fused)");
  PESTI_CUDA_TRY(cudaFuncSetAttribute(pesti::fused_classify_kernel<float, 4, false>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, fused), "cudaFuncSetAttribute(fused)");
  PESTI_CUDA_TRY(cudaFuncSetAttribute(pesti::fused_classify_kernel<uint16_t, 8, true>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, fused), "cudaFuncSetAttribute(fused)");
  PESTI_CUDA_TRY(cudaFuncSetAttribute(pesti::fused_classify_kernel<uint16_t, 8, false>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, fused), "cudaFuncSetAttribute(fused)");
  PESTI_CUDA_TRY(cudaFuncSetAttribute(pesti::fused_classify_kernel<__half, 8, true>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, fused), "cudaFuncSetAttribute(fused)");
  PESTI_CUDA_TRY(cudaFuncSetAttribute(pesti::fused_classify_kernel<__half, 8, false>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, fused), "cudaFuncSetAttribute(fused)");
  if (cached) g_row_limit_set[device].store(true, std::memory_order_release);
  return PESTI_OK;
}

// Launch of a kernel that may start while the previous kernel of the stream
// is finishing (programmatic dependent launch): it waits on the device for
// that kernel's results (griddepcontrol.wait) before reading them.
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Launch geometry and workspace layout of one batch call: byte offsets into
// one workspace, each region 256-byte aligned.
struct Plan {
  Geometry g;
  int num_sms;
  long long nsub, nseg, jmax;
  bool sorted_bufs;
  bool survivors = true;  // some row may need the survivor pass (not on the fast path)
  size_t o_ctr, o_stats, o_pre, o_info, o_surv, o_segmax, o_upre, o_se, o_si, o_cc, o_ce, o_ci;
  size_t o_gsurv, o_inext, o_tasks, o_tctr, o_pctr, o_pool;
  size_t o_E, o_I, o_status, o_fb;
  size_t o_sk0 = 0, o_sv0 = 0, o_sk1 = 0, o_sv1 = 0, o_q = 0;
  size_t bytes;  // workspace the call needs
};

Plan make_plan(int num_sms, pesti_dtype dtype, long long B, long long V, bool sorted_bufs) {
  const int esize = dtype == PESTI_F32 ? 4 : 2;
  const int ve = 16 / esize;
  Plan p;
  p.g = pick_geometry(num_sms, B, V > 0 ? V : 1, ve);
  p.num_sms = num_sms;
  p.nsub = (long long)p.g.P * pesti::K1_WARPS;
  p.nseg = (std::max(1LL, V) + 32LL * ve - 1) / (32LL * ve);
  p.jmax = (p.g.SL + pesti::UNIT - 1) / pesti::UNIT;
  const size_t ngrp = (size_t)B * p.nsub * p.jmax;
  p.sorted_bufs = sorted_bufs;
  const size_t bv = (size_t)B * (size_t)std::max(1LL, V);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes);
    return o;
  };
  p.o_ctr = take((size_t)B * 4);  // must be zero at the start of a call; the kernels leave it zero
  p.o_stats = take((size_t)B * p.nsub * sizeof(pesti::SubStat));
  p.o_pre = take((size_t)B * p.nsub * sizeof(pesti::SubPre));
  p.o_info = take((size_t)B * sizeof(pesti::RowInfo));
  p.o_surv = take((size_t)B * p.nsub * sizeof(pesti::SubSurv));
  p.o_segmax = take((size_t)B * p.nseg * 4);
  p.o_upre = take((size_t)B * ((std::max(1LL, V) + pesti::UNIT - 1) / pesti::UNIT) * sizeof(pesti::UnitPre));
  p.o_se = take(bv * 4);
  p.o_si = take(bv * 4);
  p.o_cc = take((size_t)B * 4);
  p.o_ce = take((size_t)B * pesti::CAND_CAP * 4);
  p.o_ci = take((size_t)B * pesti::CAND_CAP * 4);
  p.o_E = take(bv * 4);
  p.o_I = take(bv * 4);
  p.o_status = take(16);
  p.o_fb = take((size_t)B * sizeof(int));
  p.o_gsurv = take(ngrp * sizeof(pesti::GroupEnt));
  p.o_inext = take(sizeof(int));
  p.o_tasks = take(ngrp * sizeof(pesti::ClassTask));
  p.o_tctr = take(3 * sizeof(int));
  p.o_pctr = take((size_t)B * sizeof(int));
  p.o_pool = take((size_t)B * pesti::POOL_CAP * sizeof(pesti::FoldEnt));
  if (sorted_bufs) {
    p.o_sk0 = take(bv * 4);
    p.o_sv0 = take(bv * 4);
    p.o_sk1 = take(bv * 4);
    p.o_sv1 = take(bv * 4);
    p.o_q = take(bv * 4);
  }
  p.bytes = off;
  return p;
}

// Arguments of the slice kernels over workspace `ws` laid out by `p`.
pesti::SliceArgs make_slice_args(const Plan& p, char* ws, const void* d_logits, pesti_dtype dtype, long long B,
                                 long long V, long long ld, const pesti_sampling_params& uni,
                                 const pesti_sampling_params* d_per_row) {
  pesti::SliceArgs sa{};
  sa.logits = d_logits;
  sa.dtype = (int)dtype;
  sa.B = B;
  sa.V = V;
  sa.ld = ld;
  sa.uni = uni;
  sa.per_row = d_per_row;
  sa.P = p.g.P;
  sa.SL = p.g.SL;
  sa.nseg = p.nseg;
  sa.stats = (pesti::SubStat*)(ws + p.o_stats);
  sa.pre = (pesti::SubPre*)(ws + p.o_pre);
  sa.info = (pesti::RowInfo*)(ws + p.o_info);
  sa.row_ctr = (int*)(ws + p.o_ctr);
  sa.surv = (pesti::SubSurv*)(ws + p.o_surv);
  sa.seg_max = (float*)(ws + p.o_segmax);
  sa.unit_pre = (pesti::UnitPre*)(ws + p.o_upre);
  sa.surv_raw = (float*)(ws + p.o_se);
  sa.surv_idx = (uint32_t*)(ws + p.o_si);
  sa.jmax = (int)p.jmax;
  sa.item_next = (int*)(ws + p.o_inext);
  sa.tasks = (pesti::ClassTask*)(ws + p.o_tasks);
  sa.task_count = (int*)(ws + p.o_tctr);
  sa.task_next = sa.task_count + 1;
  sa.task_count_h = sa.task_count + 2;
  // the fused pass (vocabulary shards: set by their caller) or the survivor
  // pass and the task queue, as measured on B200: the fused pass is faster on
  // rows beyond 128k columns and on short rows (at most 64k) when every row is
  // on the top-k fast path (it needs no survivor pass then) in batches of 32
  // rows or more: 3.07 M against 2.20 M rows/s on 1000 rows of 32000; the
  // task queue on rows of 128k (913 k against 798 k rows/s, 64 rows), on
  // mixed batches and on single rows (B=1 p50 62.2 against 64.7 us)
  sa.fused = (V > 131072 || (V <= 65536 && !p.survivors && B >= 32)) ? 1 : 0;
  sa.gsurv = (pesti::GroupEnt*)(ws + p.o_gsurv);
  sa.pool = (pesti::FoldEnt*)(ws + p.o_pool);
  sa.pool_ctr = (int*)(ws + p.o_pctr);
  sa.cand_count = (int*)(ws + p.o_cc);
  sa.cand_e = (float*)(ws + p.o_ce);
  sa.cand_idx = (uint32_t*)(ws + p.o_ci);
  sa.V_total = V;
  // guard band of the fold classification: the speculation runs ahead of the
  // fold by the mass the fold absorbs, which grows along the row (up to about
  // 6e-4 of it on rows of 256k)
  sa.band = V > 131072 ? 0x1p-10f : 0x1p-12f;
  // the fast path stages the row's fold entries in shared memory; with very
  // many sub-slices it does not fit and all rows take the generic path
  const size_t fast_bytes = pesti::fast_smem_bytes((int)p.nsub, pesti::FAST_ENTS);
  sa.fast_enabled = sizeof(pesti::RowShared) + fast_bytes <= kRowSmemLimit ? 1 : 0;
  return sa;
}

bool rows_aligned(const void* d_logits, pesti_dtype dtype, long long ld) {
  const int esize = dtype == PESTI_F32 ? 4 : 2;
  return ((uintptr_t)d_logits % 16 == 0) && ((ld * esize) % 16 == 0);
}

// The HBM pass (slice_stats_kernel): row prologues, or shard summaries when
// sa.shard_out is set.
int launch_slice_stats(const Plan& p, const pesti::SliceArgs& sa, cudaStream_t st) {
  const bool aligned = rows_aligned(sa.logits, (pesti_dtype)sa.dtype, sa.ld);
  const dim3 g1((unsigned)(p.g.P * sa.B));
  if (sa.dtype == PESTI_F16) {
    if (aligned) pesti::slice_stats_kernel<__half, 8, 4, true><<<g1, pesti::K1_NT, 0, st>>>(sa);
    else pesti::slice_stats_kernel<__half, 8, 4, false><<<g1, pesti::K1_NT, 0, st>>>(sa);
  } else if (sa.dtype == PESTI_BF16) {
    if (aligned) pesti::slice_stats_kernel<uint16_t, 8, 4, true><<<g1, pesti::K1_NT, 0, st>>>(sa);
    else pesti::slice_stats_kernel<uint16_t, 8, 4, false><<<g1, pesti::K1_NT, 0, st>>>(sa);
  } else {
    if (aligned) pesti::slice_stats_kernel<float, 4, 8, true><<<g1, pesti::K1_NT, 0, st>>>(sa);
    else pesti::slice_stats_kernel<float, 4, 8, false><<<g1, pesti::K1_NT, 0, st>>>(sa);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "slice_stats_kernel launch");
  return PESTI_OK;
}

// The survivor pass and the classification of the fast path's rows: either
// the task queue over the survivors, or (sa.fused) the fused pass, with the
// survivor pass only for the rows off the fast path (skipped when the call
// has none).
int launch_survivors(const Plan& p, const pesti::SliceArgs& sa, int device, cudaStream_t st) {
  const bool aligned = rows_aligned(sa.logits, (pesti_dtype)sa.dtype, sa.ld);
  const dim3 b1(pesti::K1_NT);
  cudaError_t e;
  if (!sa.fused || p.survivors || !sa.fast_enabled) {
    // the survivor pass reads from L2: fewer loads in flight, smaller code
    const dim3 g1((unsigned)(p.g.P * sa.B));
    if (sa.dtype == PESTI_F16) {
      if (aligned) e = launch_dependent(pesti::survivor_kernel<__half, 8, true>, g1, b1, 0, st, sa);
      else e = launch_dependent(pesti::survivor_kernel<__half, 8, false>, g1, b1, 0, st, sa);
    } else if (sa.dtype == PESTI_BF16) {
      if (aligned) e = launch_dependent(pesti::survivor_kernel<uint16_t, 8, true>, g1, b1, 0, st, sa);
      else e = launch_dependent(pesti::survivor_kernel<uint16_t, 8, false>, g1, b1, 0, st, sa);
    } else {
      if (aligned) e = launch_dependent(pesti::survivor_kernel<float, 4, true>, g1, b1, 0, st, sa);
      else e = launch_dependent(pesti::survivor_kernel<float, 4, false>, g1, b1, 0, st, sa);
    }
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "survivor_kernel launch");
  }
  if (!sa.fused) {
    // classification tasks: a persistent grid takes them from a counter
    const long long most = (long long)sa.B * p.nsub * p.jmax;
    const long long blocks = std::min<long long>(4LL * p.num_sms, (most + pesti::K1_WARPS - 1) / pesti::K1_WARPS);
    e = launch_dependent(pesti::classify_kernel, dim3((unsigned)std::max(1LL, blocks)), b1, 0, st, sa);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "classify_kernel launch");
    return PESTI_OK;
  }
  if (!sa.fast_enabled) return PESTI_OK;
  int rc = ensure_row_smem_limit(device);
  if (rc) return rc;
  // a persistent grid over the rows' UNIT-element units: as many blocks as
  // fit on the device at once
  const size_t smem = sizeof(pesti::FusedShared);
  void (*kern)(pesti::SliceArgs) =
      sa.dtype == PESTI_F16    ? (aligned ? pesti::fused_classify_kernel<__half, 8, true>
                                          : pesti::fused_classify_kernel<__half, 8, false>)
      : sa.dtype == PESTI_BF16 ? (aligned ? pesti::fused_classify_kernel<uint16_t, 8, true>
                                          : pesti::fused_classify_kernel<uint16_t, 8, false>)
                             : (aligned ? pesti::fused_classify_kernel<float, 4, true>
                                        : pesti::fused_classify_kernel<float, 4, false>);
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, pesti::K1_NT, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  const long long units = sa.B * ((sa.V + pesti::UNIT - 1) / pesti::UNIT);
  const long long blocks =
      std::min<long long>((long long)std::max(1, per_sm) * p.num_sms, (units + pesti::K1_WARPS - 1) / pesti::K1_WARPS);
  e = launch_dependent(kern, dim3((unsigned)std::max(1LL, blocks)), b1, smem, st, sa);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fused_classify_kernel launch");
  return PESTI_OK;
}

// Arguments of the row kernel for the slice arguments `sa`.
pesti::RowArgs make_row_args(const Plan& p, char* ws, const pesti::SliceArgs& sa, const float* d_u, uint32_t* d_out,
                             float* d_kept_p, uint32_t* d_kept_idx, long long kept_width, int64_t* d_kept_count) {
  const bool sorted_bufs = p.sorted_bufs;
  const void* d_logits = sa.logits;
  const pesti_dtype dtype = (pesti_dtype)sa.dtype;
  const long long B = sa.B, V = sa.V, ld = sa.ld;
  const pesti_sampling_params uni = sa.uni;
  const pesti_sampling_params* d_per_row = sa.per_row;
  pesti::RowArgs ra{};
  ra.logits = d_logits;
  ra.dtype = (int)dtype;
  ra.B = B;
  ra.V = V;
  ra.ld = ld;
  ra.uni = uni;
  ra.per_row = d_per_row;
  ra.P = p.g.P;
  ra.SL = p.g.SL;
  ra.info = sa.info;
  ra.surv = sa.surv;
  ra.jmax = sa.jmax;
  ra.gsurv = sa.gsurv;
  ra.pool = sa.pool;
  ra.surv_raw = sa.surv_raw;
  ra.surv_idx = sa.surv_idx;
  ra.cand_count = sa.cand_count;
  ra.cand_e = sa.cand_e;
  ra.cand_idx = sa.cand_idx;
  ra.E = (float*)(ws + p.o_E);
  ra.I = (uint32_t*)(ws + p.o_I);
  ra.SK0 = sorted_bufs ? (uint32_t*)(ws + p.o_sk0) : nullptr;
  ra.SV0 = sorted_bufs ? (uint32_t*)(ws + p.o_sv0) : nullptr;
  ra.SK1 = sorted_bufs ? (uint32_t*)(ws + p.o_sk1) : nullptr;
  ra.SV1 = sorted_bufs ? (uint32_t*)(ws + p.o_sv1) : nullptr;
  ra.Q = sorted_bufs ? (float*)(ws + p.o_q) : nullptr;
  ra.u = d_u;
  ra.out = d_out;
  ra.kept_p = d_kept_p;
  ra.kept_idx = d_kept_idx;
  ra.kept_width = (d_kept_p || d_kept_idx) ? kept_width : 0;
  ra.kept_count = d_kept_count;
  ra.status = (int*)(ws + p.o_status);
  ra.fast_enabled = sa.fast_enabled;
  ra.V_total = sa.V_total;
  // fold entries the row kernel stages per row: rows up to 128k columns make
  // a few hundred (about one per 256 survivors, plus the single elements)
  ra.fast_ents = sa.V_total > 131072 || sa.fused ? pesti::FAST_ENTS : pesti::FAST_ENTS_SHORT;
  return ra;
}

int launch_row(const Plan& p, int device, const pesti::RowArgs& ra, cudaStream_t st) {
  size_t smem2 =
      sizeof(pesti::RowShared) + (ra.fast_enabled ? pesti::fast_smem_bytes((int)p.nsub, ra.fast_ents) : 0);
  if (ra.nucleus) smem2 = std::max(smem2, sizeof(pesti::RowShared) + sizeof(pesti::NucSmem));
  if (smem2 > 48 * 1024) {
    int rc = ensure_row_smem_limit(device);
    if (rc) return rc;
  }
  cudaError_t e = launch_dependent(pesti::row_kernel, dim3((unsigned)ra.B), dim3(pesti::K2_NT), smem2, st, ra);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "row_kernel launch");
  return PESTI_OK;
}

// Enqueues the four passes of one batch call on `st` over workspace `ws`
// (laid out by `p`).  pev: four events bracketing the passes, or null.
int run_plan(const Plan& p, char* ws, int device, cudaEvent_t* pev, const void* d_logits,
             pesti_dtype dtype, long long B, long long V, long long ld,
             const pesti_sampling_params& uni, const pesti_sampling_params* d_per_row,
             const float* d_u, uint32_t* d_out, float* d_kept_p, uint32_t* d_kept_idx,
             long long kept_width, int64_t* d_kept_count, cudaStream_t st) {
  const pesti::SliceArgs sa = make_slice_args(p, ws, d_logits, dtype, B, V, ld, uni, d_per_row);
  if (pev) PESTI_CUDA_TRY(cudaEventRecord(pev[0], st), "cudaEventRecord(profile)");
  int rc = launch_slice_stats(p, sa, st);
  if (rc) return rc;
  if (pev) PESTI_CUDA_TRY(cudaEventRecord(pev[1], st), "cudaEventRecord(profile)");
  rc = launch_survivors(p, sa, device, st);
  if (rc) return rc;
  if (pev) PESTI_CUDA_TRY(cudaEventRecord(pev[2], st), "cudaEventRecord(profile)");
  const pesti::RowArgs ra = make_row_args(p, ws, sa, d_u, d_out, d_kept_p, d_kept_idx, kept_width, d_kept_count);
  rc = launch_row(p, device, ra, st);
  if (rc) return rc;
  if (pev) PESTI_CUDA_TRY(cudaEventRecord(pev[3], st), "cudaEventRecord(profile)");
  return PESTI_OK;
}

// ---------------------------------------------------------------------------
// The cluster pass: one thread-block cluster per row (pesti_cluster.cuh), then
// the row kernel for the rows it leaves (usually none: its blocks return at
// once).  Used when every row is greedy or on the top-k fast path and rows are
// at most CL_MAX_V long.
// ---------------------------------------------------------------------------
std::atomic<int> g_cluster_override{0};  // pesti_testing_set_cluster

using ClusterKernel = void (*)(pesti::ClusterArgs);

ClusterKernel cluster_kernel_for(pesti_dtype dtype, bool aligned) {
  if (dtype == PESTI_F16) return aligned ? pesti::row_cluster_kernel<__half, 8, true> : pesti::row_cluster_kernel<__half, 8, false>;
  if (dtype == PESTI_BF16)
    return aligned ? pesti::row_cluster_kernel<uint16_t, 8, true> : pesti::row_cluster_kernel<uint16_t, 8, false>;
  return aligned ? pesti::row_cluster_kernel<float, 4, true> : pesti::row_cluster_kernel<float, 4, false>;
}

// Largest cluster (16 or 8 CTAs) the device runs this kernel with; 16 needs
// the non-portable size, allowed once per device and kernel.
constexpr int kClusterKinds = 6;
std::atomic<int> g_cluster_max[kMaxDevices][kClusterKinds];

int cluster_max_for(int device, ClusterKernel kern, int kind) {
  const bool cached = device >= 0 && device < kMaxDevices;
  if (cached) {
    const int v = g_cluster_max[device][kind].load(std::memory_order_acquire);
    if (v) return v;
  }
  int best = 8;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(16);
    cfg.blockDim = dim3(pesti::CL_NT);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 16;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) best = 16;
  }
  cudaGetLastError();  // a refused query leaves no error behind
  if (cached) g_cluster_max[device][kind].store(best, std::memory_order_release);
  return best;
}

struct ClusterGeom {
  int C;  // CTAs per row
  int wstart[pesti::CL_MAXC * pesti::CL_WARPS + 1];  // warp ranges (ClusterArgs::wstart)
};

// Relative lengths of the first warp ranges of a row: there the running sum
// is small, most elements survive the pruning and the state crosses binades
// often, so those warps have more to do per element.
constexpr double kHeadWeight[4] = {0.25, 0.25, 0.5, 0.5};

// Cluster size and warp ranges for rows of V elements: 16 CTAs for short
// batches (latency), 8 otherwise; every range a multiple of 32*VE elements and
// at most CL_SEGS of them.
bool cluster_geometry(long long B, long long V, int esize, int cmax, ClusterGeom& g) {
  const long long seg = 32LL * (16 / esize);
  const int forced = g_cluster_override.load(std::memory_order_relaxed);
  auto standard = [&](int c) {  // the length of an ordinary warp range
    const int n = c * pesti::CL_WARPS;
    double w = 0.0;
    for (int q = 0; q < n; ++q) w += q < 4 ? kHeadWeight[q] : 1.0;
    const long long per = (long long)std::ceil((double)V / w);
    return std::max(seg, (per + seg - 1) / seg * seg);
  };
  int C = forced > 0 ? forced : (B <= 16 ? 16 : 8);
  if (C > cmax) C = cmax;
  if (forced <= 0 && standard(C) > pesti::CL_SEGS * seg && cmax >= 16) C = 16;
  // no more CTAs than the row has warp ranges for
  const long long need = (V + pesti::CL_WARPS * seg - 1) / (pesti::CL_WARPS * seg);
  if ((long long)C > need && forced <= 0) C = (int)std::max(1LL, need);
  const long long L = standard(C);
  if (L > pesti::CL_SEGS * seg) return false;
  const int n = C * pesti::CL_WARPS;
  long long pos = 0;
  for (int q = 0; q < n; ++q) {
    const double wq = q < 4 ? kHeadWeight[q] : 1.0;
    long long len = (long long)std::ceil(wq * (double)L / (double)seg) * seg;
    g.wstart[q] = (int)std::min(pos, V);
    pos += len;
  }
  g.wstart[n] = (int)V;
  if (pos < V) return false;  // (cannot happen: the lengths sum to at least V)
  g.C = C;
  return true;
}

// Batches of at most this many rows take the cluster pass when they can (its
// one launch per call is what a short batch's latency needs); longer batches
// of top-k rows keep the four-kernel pipeline, which was faster on B200 at 64
// rows of 128k (72.6 against 110 us per step) and at 1000 rows of 32k.
constexpr long long kClusterMaxRows = 32;

bool use_cluster_path(long long B, long long V, int esize, int ckind) {
  const long long vmax = esize == 4 ? pesti::CL_MAX_V : pesti::CL_MAX_V16;
  const int ov = g_cluster_override.load(std::memory_order_relaxed);
  if (ov < 0 || ckind <= 0 || V < 1 || V > vmax) return false;
  // bf16 top-p rows always (their sorted folds by distinct values need the
  // cluster's exact softmax sum); others for short batches, or when a test forces it
  return ckind == 2 || B <= kClusterMaxRows || ov > 0;
}

int run_cluster(const Plan& p, const ClusterGeom& cgm, char* ws, int device, cudaEvent_t* pev,
                const void* d_logits, pesti_dtype dtype, long long B, long long V, long long ld,
                const pesti_sampling_params& uni, const pesti_sampling_params* d_per_row, const float* d_u,
                uint32_t* d_out, float* d_kept_p, uint32_t* d_kept_idx, long long kept_width,
                int64_t* d_kept_count, bool nucleus, cudaStream_t st) {
  const bool aligned = rows_aligned(d_logits, dtype, ld);
  pesti::ClusterArgs ca{};
  ca.logits = d_logits;
  ca.dtype = (int)dtype;
  ca.B = B;
  ca.V = V;
  ca.ld = ld;
  ca.uni = uni;
  ca.per_row = d_per_row;
  std::memcpy(ca.wstart, cgm.wstart, sizeof(int) * (cgm.C * pesti::CL_WARPS + 1));
  ca.u = d_u;
  ca.out = d_out;
  ca.kept_p = d_kept_p;
  ca.kept_idx = d_kept_idx;
  ca.kept_width = (d_kept_p || d_kept_idx) ? kept_width : 0;
  ca.kept_count = d_kept_count;
  ca.fb = (int*)(ws + p.o_fb);
  ca.info = (pesti::RowInfo*)(ws + p.o_info);
  // guard band: the speculation runs ahead of the fold by the mass the fold
  // absorbs, which grows along the row (about 1.2e-4 of it at 128k columns,
  // up to 6e-4 at 256k).  A run predicted in the wrong binade is replayed, so
  // the band trades replays against general segments: on rows of 128k columns
  // 2^-13 gave the fewest of both (against 2^-11, 2^-12 and 2^-14); on bf16
  // rows of 152064 columns 2^-12 was 6 % faster than 2^-10 and 2^-11
  ca.band = V > 196608 ? 0x1p-10f : (V > 131072 ? 0x1p-12f : 0x1p-13f);
  ca.nucleus = nucleus ? 1 : 0;
  // a short batch lets the row kernel's few blocks be scheduled while the
  // cluster pass runs (they wait for it on the device), hiding that launch
  ca.early_dependents = B <= 16 ? 1 : 0;
  if (pev) PESTI_CUDA_TRY(cudaEventRecord(pev[0], st), "cudaEventRecord(profile)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(B * cgm.C));
  cfg.blockDim = dim3(pesti::CL_NT);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cgm.C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, cluster_kernel_for(dtype, aligned), ca);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "row_cluster_kernel launch");
  if (pev) {
    PESTI_CUDA_TRY(cudaEventRecord(pev[1], st), "cudaEventRecord(profile)");
    PESTI_CUDA_TRY(cudaEventRecord(pev[2], st), "cudaEventRecord(profile)");
  }
  // the rows the cluster pass left: the row kernel's generic path over whole rows
  pesti::SliceArgs sa = make_slice_args(p, ws, d_logits, dtype, B, V, ld, uni, d_per_row);
  sa.fast_enabled = 0;
  pesti::RowArgs ra = make_row_args(p, ws, sa, d_u, d_out, d_kept_p, d_kept_idx, kept_width, d_kept_count);
  ra.only = ca.fb;
  ra.fast_enabled = 0;
  ra.nucleus = nucleus ? 1 : 0;
  int rc = launch_row(p, device, ra, st);
  if (rc) return rc;
  if (pev) PESTI_CUDA_TRY(cudaEventRecord(pev[3], st), "cudaEventRecord(profile)");
  return PESTI_OK;
}

int launch(pesti_sampler* s, const void* d_logits, pesti_dtype dtype, long long B, long long V,
           long long ld, const pesti_sampling_params& uni, const pesti_sampling_params* d_per_row,
           bool sorted_bufs, bool survivors, int ckind, const float* d_u, uint32_t* d_out, float* d_kept_p,
           uint32_t* d_kept_idx, long long kept_width, int64_t* d_kept_count, cudaStream_t st) {
  const int esize = dtype == PESTI_F32 ? 4 : 2;
  ClusterGeom cgm{};
  if (use_cluster_path(B, V, esize, ckind)) {
    const int kind = (int)dtype * 2 + (rows_aligned(d_logits, dtype, ld) ? 1 : 0);
    const int cmax = cluster_max_for(s->device, cluster_kernel_for(dtype, kind & 1), kind);
    if (cluster_geometry(B, V, esize, cmax, cgm)) {
      // the row kernel's generic path may take any row: whole-row buffers
      Plan p = make_plan(s->num_sms, dtype, B, V, true);
      int rc = ensure_ws(s, p.bytes);
      if (rc) return rc;
      cudaEvent_t* pev = nullptr;
      if (s->prof && s->prof_n < pesti_sampler::kProfMax) {
        pev = s->prof_ev[s->prof_n++];
        for (int q = 0; q < 4; ++q)
          if (!pev[q]) PESTI_CUDA_TRY(cudaEventCreate(&pev[q]), "cudaEventCreate(profile)");
      }
      return run_cluster(p, cgm, (char*)s->ws, s->device, pev, d_logits, dtype, B, V, ld, uni, d_per_row, d_u,
                         d_out, d_kept_p, d_kept_idx, kept_width, d_kept_count, ckind == 2, st);
    }
  }
  Plan p = make_plan(s->num_sms, dtype, B, V, sorted_bufs);
  p.survivors = survivors;
  int rc = ensure_ws(s, p.bytes);
  if (rc) return rc;
  rc = zero_counters(s, B, st);
  if (rc) return rc;
  cudaEvent_t* pev = nullptr;
  if (s->prof && s->prof_n < pesti_sampler::kProfMax) {
    pev = s->prof_ev[s->prof_n++];
    for (int q = 0; q < 4; ++q)
      if (!pev[q]) PESTI_CUDA_TRY(cudaEventCreate(&pev[q]), "cudaEventCreate(profile)");
  }
  rc = run_plan(p, (char*)s->ws, s->device, pev, d_logits, dtype, B, V, ld, uni, d_per_row, d_u,
                d_out, d_kept_p, d_kept_idx, kept_width, d_kept_count, st);
  s->ctr_zero_rows = rc ? 0 : B;
  return rc;
}

// Per-row parameters as the kernels read them: one uniform entry, or a
// device array (the caller's, or the host entries copied to the handle's).
int stage_params(pesti_sampler* s, const pesti_sampling_params* params, int params_per_row, int params_on_device,
                 long long B, long long V, cudaStream_t st, pesti_sampling_params& uni,
                 const pesti_sampling_params*& d_per_row, bool& sorted_bufs, bool& survivors,
                 pesti_dtype dtype = PESTI_F32, int* ckind = nullptr) {
  uni = pesti_sampling_params{};
  d_per_row = nullptr;
  sorted_bufs = true;
  survivors = true;
  if (ckind) *ckind = 0;  // params on the device: not known here
  if (params_on_device) {
    if (params_per_row) d_per_row = params;
    else {
      // single device entry: read it back once (rare API use)
      PESTI_CUDA_TRY(cudaMemcpyAsync(&uni, params, sizeof(uni), cudaMemcpyDeviceToHost, st), "params copy");
      PESTI_CUDA_TRY(cudaStreamSynchronize(st), "params sync");
      sorted_bufs = needs_sorted_buffers(&uni, 1);
      survivors = needs_survivor_pass(&uni, 1, V);
      if (ckind) *ckind = cluster_kind(&uni, 1, V, dtype);
    }
  } else if (params_per_row) {
    sorted_bufs = needs_sorted_buffers(params, B);
    survivors = needs_survivor_pass(params, B, V);
    if (ckind) *ckind = cluster_kind(params, B, V, dtype);
    if ((size_t)B > s->h_params_cap) {
      if (s->params_ev_used) cudaEventSynchronize(s->params_ev);
      if (s->h_params) cudaFreeHost(s->h_params);
      if (s->d_params) cudaFree(s->d_params);
      s->h_params = nullptr;
      s->d_params = nullptr;
      PESTI_CUDA_TRY(cudaMallocHost(&s->h_params, (size_t)B * sizeof(pesti_sampling_params)), "cudaMallocHost(params)");
      PESTI_CUDA_TRY(cudaMalloc(&s->d_params, (size_t)B * sizeof(pesti_sampling_params)), "cudaMalloc(params)");
      s->h_params_cap = s->d_params_cap = (size_t)B;
    } else if (s->params_ev_used) {
      PESTI_CUDA_TRY(cudaEventSynchronize(s->params_ev), "cudaEventSynchronize(params)");
    }
    std::memcpy(s->h_params, params, (size_t)B * sizeof(pesti_sampling_params));
    PESTI_CUDA_TRY(cudaMemcpyAsync(s->d_params, s->h_params, (size_t)B * sizeof(pesti_sampling_params),
                                   cudaMemcpyHostToDevice, st), "params copy");
    PESTI_CUDA_TRY(cudaEventRecord(s->params_ev, st), "cudaEventRecord(params)");
    s->params_ev_used = true;
    d_per_row = s->d_params;
  } else {
    uni = params[0];
    sorted_bufs = needs_sorted_buffers(&uni, 1);
    survivors = needs_survivor_pass(&uni, 1, V);
    if (ckind) *ckind = cluster_kind(&uni, 1, V, dtype);
  }
  return PESTI_OK;
}

// ---------------------------------------------------------------------------
// Vocabulary shards: every rank holds one contiguous, equally wide column
// range of each row (pesti_shard.cuh describes the algorithm).
// ---------------------------------------------------------------------------

// NCCL is loaded when the first communicator is made, so that the library
// itself has no link-time dependency on it (libnccl.so.2: the copy the
// process already holds, if any, else the system's).
struct NcclApi {
  bool loaded = false;
  std::string err;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
};

const NcclApi& nccl_api() {
  static const NcclApi api = [] {
    NcclApi a;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* why = dlerror();
      a.err = std::string("cannot load libnccl.so.2: ") + (why ? why : "unknown");
      return a;
    }
    a.get_unique_id = (decltype(a.get_unique_id))dlsym(h, "ncclGetUniqueId");
    a.comm_init_rank = (decltype(a.comm_init_rank))dlsym(h, "ncclCommInitRank");
    a.comm_destroy = (decltype(a.comm_destroy))dlsym(h, "ncclCommDestroy");
    a.all_gather = (decltype(a.all_gather))dlsym(h, "ncclAllGather");
    a.error_string = (decltype(a.error_string))dlsym(h, "ncclGetErrorString");
    a.comm_init_rank_config = (decltype(a.comm_init_rank_config))dlsym(h, "ncclCommInitRankConfig");
    a.get_async_error = (decltype(a.get_async_error))dlsym(h, "ncclCommGetAsyncError");
    a.comm_abort = (decltype(a.comm_abort))dlsym(h, "ncclCommAbort");
    a.loaded = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.all_gather && a.error_string &&
               a.comm_init_rank_config && a.get_async_error && a.comm_abort;
    if (!a.loaded) a.err = "libnccl.so.2 lacks an entry point";
    return a;
  }();
  return api;
}

int nccl_fail(ncclResult_t r, const char* what) {
  const NcclApi& n = nccl_api();
  return fail(PESTI_E_NCCL, std::string(what) + ": " + (n.error_string ? n.error_string(r) : "error"));
}

}  // namespace

struct pesti_comm {
  int world = 1;
  int rank = 0;
  int device = 0;
  ncclComm_t comm = nullptr;
  int timeout_ms = 120000;  // deadline of the set-up and of each sharded call's exchanges
  bool aborted = false;     // a deadline passed or an exchange failed: the communicator is gone
};

namespace {

using Clock = std::chrono::steady_clock;

Clock::time_point deadline_of(const pesti_comm* c) { return Clock::now() + std::chrono::milliseconds(c->timeout_ms); }

void comm_abort(pesti_comm* c) {
  if (c->comm && !c->aborted) nccl_api().comm_abort(c->comm);
  c->aborted = true;
}

// Waits, on the host, until the communicator's pending operation (its
// set-up, or the enqueueing of a collective) has completed: polls
// ncclCommGetAsyncError until it no longer reports ncclInProgress.  An error,
// or the deadline passing first, aborts the communicator.
int comm_settle(pesti_comm* c, ncclResult_t issued, Clock::time_point deadline, const char* what) {
  const NcclApi& n = nccl_api();
  if (issued != ncclSuccess && issued != ncclInProgress) {
    comm_abort(c);
    return nccl_fail(issued, what);
  }
  for (;;) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t r = n.get_async_error(c->comm, &st);
    if (r != ncclSuccess) {
      comm_abort(c);
      return nccl_fail(r, "ncclCommGetAsyncError");
    }
    if (st == ncclSuccess) return PESTI_OK;
    if (st != ncclInProgress) {
      comm_abort(c);
      return nccl_fail(st, what);
    }
    if (Clock::now() >= deadline) {
      comm_abort(c);
      return fail(PESTI_E_TIMEOUT, std::string(what) + ": not complete after " + std::to_string(c->timeout_ms) +
                                       " ms (a rank did not join or stopped); the communicator was aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// Waits for stream st with the communicator's deadline: the stream's work
// includes the communicator's collectives, which wait for every rank.
int stream_settle(pesti_comm* c, cudaStream_t st, Clock::time_point deadline, const char* what) {
  const NcclApi& n = nccl_api();
  for (;;) {
    const cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return PESTI_OK;
    if (e != cudaErrorNotReady) return cuda_fail(e, what);
    ncclResult_t as = ncclSuccess;
    if (n.get_async_error(c->comm, &as) == ncclSuccess && as != ncclSuccess && as != ncclInProgress) {
      comm_abort(c);
      return nccl_fail(as, what);
    }
    if (Clock::now() >= deadline) {
      comm_abort(c);
      return fail(PESTI_E_TIMEOUT, std::string(what) + ": the exchanges did not finish within " +
                                       std::to_string(c->timeout_ms) + " ms; the communicator was aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

}  // namespace

namespace {

// Relative guard band of the fold classification for shards: the
// approximate start of a shard (the true mass of the earlier shards) runs
// ahead of the fold by the mass the fold absorbs, up to about 6e-4 of it on
// rows of 256k; the band keeps the fold entries valid at the exact start.
constexpr float kShardBand = 0x1p-10f;

// Workspace of one sharded call: one set of single-shard passes per shard the
// process holds (one with NCCL, all of them when emulated), then the
// exchange buffers.  Each shard's region starts with its completion counters.
struct ShardPlan {
  Plan local;            // one shard's passes over [B, Vs]
  int G = 1, nlocal = 1;
  long long B = 0, Vs = 0, VT = 0;
  int ksh = 0;
  long long rec_stride = 0;
  size_t local_stride = 0;
  size_t o_ment = 0, o_nment = 0;  // within a shard's region
  size_t o_sum_recv = 0, o_sum_send = 0, o_rec_recv = 0, o_rec_send = 0, o_tab_recv = 0, o_tab_send = 0;
  size_t o_nflag = 0, o_flags = 0;
  size_t bytes = 0;
};

ShardPlan make_shard_plan(int num_sms, pesti_dtype dtype, long long B, long long Vs, int G, int nlocal, int ksh) {
  ShardPlan sp;
  sp.local = make_plan(num_sms, dtype, B, Vs, false);
  sp.local.survivors = false;  // rows off the fast path take the gathered path
  sp.G = G;
  sp.nlocal = nlocal;
  sp.B = B;
  sp.Vs = Vs;
  sp.VT = Vs * G;
  sp.ksh = ksh;
  sp.rec_stride = (long long)((sizeof(pesti::ShardRec) + (size_t)ksh * sizeof(pesti::ShardCand) + 15) / 16 * 16);
  sp.o_ment = align_up(sp.local.bytes);
  sp.o_nment = sp.o_ment + align_up((size_t)B * pesti::FAST_ENTS * sizeof(pesti::FoldEnt));
  sp.local_stride = sp.o_nment + align_up((size_t)B * sizeof(int));
  size_t off = sp.local_stride * (size_t)nlocal;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes);
    return o;
  };
  const size_t nsum = (size_t)B * sizeof(pesti::ShardSum);
  const size_t nrec = (size_t)B * (size_t)sp.rec_stride;
  const size_t ntab = (size_t)B * sizeof(pesti::ShardTab);
  sp.o_sum_recv = take(nsum * G);
  sp.o_sum_send = take(nsum);
  sp.o_rec_recv = take(nrec * G);
  sp.o_rec_send = take(nrec);
  sp.o_tab_recv = take(ntab * G);
  sp.o_tab_send = take(ntab);
  sp.o_nflag = take(16);
  sp.o_flags = take((size_t)B * sizeof(int));
  sp.bytes = off;
  return sp;
}

struct ShardCall {
  pesti_dtype dtype;
  long long B, Vs, ld;
  pesti_sampling_params uni;
  const pesti_sampling_params* d_per_row;
  const float* d_u;
  uint32_t* d_out;
  float* d_kept_p;
  uint32_t* d_kept_idx;
  long long kept_width;
  int64_t* d_kept_count;
  cudaStream_t st;
};

// First phase of shard r held in region li: its summary (max, flags, mass,
// candidate threshold, argmax columns) to `sum_out`.
int shard_phase1(const ShardPlan& sp, char* ws, int li, const ShardCall& c, const void* lg,
                 pesti::ShardSum* sum_out) {
  char* lws = ws + (size_t)li * sp.local_stride;
  PESTI_CUDA_TRY(cudaMemsetAsync(lws + sp.local.o_ctr, 0, (size_t)c.B * sizeof(int), c.st), "cudaMemsetAsync(counters)");
  pesti::SliceArgs sa = make_slice_args(sp.local, lws, lg, c.dtype, c.B, c.Vs, c.ld, c.uni, c.d_per_row);
  sa.V_total = sp.VT;
  sa.band = kShardBand;
  sa.shard_out = sum_out;
  sa.fused = 1;  // the second phase's fused pass reads this pass's per-unit states
  return launch_slice_stats(sp.local, sa, c.st);
}

// Second phase of shard r (region li), once every summary is in `sums`:
// the shard's prologue, survivor and classification passes, and its
// exchange record (fold increment and candidates) to `rec_out`.
int shard_phase2(const ShardPlan& sp, char* ws, int li, int r, int device, const ShardCall& c, const void* lg,
                 const pesti::ShardSum* sums, unsigned char* rec_out) {
  char* lws = ws + (size_t)li * sp.local_stride;
  pesti::SliceArgs sa = make_slice_args(sp.local, lws, lg, c.dtype, c.B, c.Vs, c.ld, c.uni, c.d_per_row);
  sa.V_total = sp.VT;
  sa.band = kShardBand;
  sa.shard_all = sums;
  sa.shard_G = sp.G;
  sa.shard_rank = r;
  sa.fused = 1;
  if (c.dtype == PESTI_F16) pesti::shard_prologue_kernel<__half, 8><<<(unsigned)c.B, pesti::K1_NT, 0, c.st>>>(sa);
  else if (c.dtype == PESTI_BF16) pesti::shard_prologue_kernel<uint16_t, 8><<<(unsigned)c.B, pesti::K1_NT, 0, c.st>>>(sa);
  else pesti::shard_prologue_kernel<float, 4><<<(unsigned)c.B, pesti::K1_NT, 0, c.st>>>(sa);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "shard_prologue_kernel launch");
  int rc = launch_survivors(sp.local, sa, device, c.st);
  if (rc) return rc;
  pesti::RowArgs ra = make_row_args(sp.local, lws, sa, c.d_u, c.d_out, nullptr, nullptr, 0, nullptr);
  ra.shard = 1;
  ra.fast_ents = pesti::FAST_ENTS;
  ra.col0 = (long long)r * c.Vs;
  ra.rec = rec_out;
  ra.rec_stride = sp.rec_stride;
  ra.ksh = sp.ksh;
  ra.ment_g = (pesti::FoldEnt*)(lws + sp.o_ment);
  ra.nment_g = (int*)(lws + sp.o_nment);
  return launch_row(sp.local, device, ra, c.st);
}

// Third phase of shard r (region li), once every record is in `recs`: its
// table of exact folds around the chained estimate of its start, to `tab_out`.
int shard_phase3(const ShardPlan& sp, char* ws, int li, int r, int device, const ShardCall& c, const void* lg,
                 const unsigned char* recs, pesti::ShardTab* tab_out) {
  char* lws = ws + (size_t)li * sp.local_stride;
  pesti::TabArgs ta{};
  ta.logits = lg;
  ta.dtype = (int)c.dtype;
  ta.B = c.B;
  ta.ld = c.ld;
  ta.uni = c.uni;
  ta.per_row = c.d_per_row;
  ta.info = (const pesti::RowInfo*)(lws + sp.local.o_info);
  ta.recs = recs;
  ta.rec_stride = sp.rec_stride;
  ta.rank = r;
  ta.ment_g = (const pesti::FoldEnt*)(lws + sp.o_ment);
  ta.nment_g = (const int*)(lws + sp.o_nment);
  ta.tab_out = tab_out;
  int rc = ensure_row_smem_limit(device);
  if (rc) return rc;
  pesti::shard_table_kernel<<<(unsigned)c.B, 32, pesti::TAB_SMEM, c.st>>>(ta);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "shard_table_kernel launch");
  return PESTI_OK;
}

// Every row on every rank: chain, merge, draw; rows it cannot settle are listed.
int shard_finish(const ShardPlan& sp, char* ws, const ShardCall& c) {
  int* nflag = (int*)(ws + sp.o_nflag);
  PESTI_CUDA_TRY(cudaMemsetAsync(nflag, 0, sizeof(int), c.st), "cudaMemsetAsync(flags)");
  pesti::FinishArgs fa{};
  fa.B = c.B;
  fa.V_total = sp.VT;
  fa.G = sp.G;
  fa.uni = c.uni;
  fa.per_row = c.d_per_row;
  fa.info = (const pesti::RowInfo*)(ws + sp.local.o_info);  // region 0
  fa.recs = (const unsigned char*)(ws + sp.o_rec_recv);
  fa.rec_stride = sp.rec_stride;
  fa.ksh = sp.ksh;
  fa.tabs = (const pesti::ShardTab*)(ws + sp.o_tab_recv);
  fa.u = c.d_u;
  fa.out = c.d_out;
  fa.kept_p = c.d_kept_p;
  fa.kept_idx = c.d_kept_idx;
  fa.kept_width = (c.d_kept_p || c.d_kept_idx) ? c.kept_width : 0;
  fa.kept_count = c.d_kept_count;
  fa.nflag = nflag;
  fa.flag_rows = (int*)(ws + sp.o_flags);
  pesti::shard_finish_kernel<<<(unsigned)c.B, pesti::K2_NT, 0, c.st>>>(fa);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "shard_finish_kernel launch");
  return PESTI_OK;
}

// The rows listed by the finish (a host copy, sorted: every rank sees the
// same list), and how many for each reason.  Synchronizes the stream.
int read_flagged(const ShardPlan& sp, char* ws, cudaStream_t st, std::vector<int>& rows, long long* why,
                 pesti_comm* comm, Clock::time_point deadline) {
  int n = 0;
  PESTI_CUDA_TRY(cudaMemcpyAsync(&n, ws + sp.o_nflag, sizeof(int), cudaMemcpyDeviceToHost, st), "flag count copy");
  if (comm) {
    const int rc = stream_settle(comm, st, deadline, "sharded exchanges");
    if (rc) return rc;
  } else {
    PESTI_CUDA_TRY(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  }
  rows.assign((size_t)n, 0);
  for (int q = 0; q < pesti::GR_KINDS; ++q) why[q] = 0;
  if (n > 0) {
    PESTI_CUDA_TRY(cudaMemcpy(rows.data(), ws + sp.o_flags, (size_t)n * sizeof(int), cudaMemcpyDeviceToHost),
                   "flag list copy");
    for (int& r : rows) {
      const uint32_t q = (uint32_t)r >> 28;
      ++why[q < pesti::GR_KINDS ? q : 0];
      r = (int)((uint32_t)r & 0x0fffffffu);
    }
    std::sort(rows.begin(), rows.end());
  }
  return PESTI_OK;
}

// Gathered path for the listed rows: whole rows are assembled (from the
// shards by an NCCL all-gather, or from the whole matrix when emulated) and
// sampled by the single-device passes; the results go to their rows.
int shard_gathered(pesti_sampler* s, pesti_comm* comm, const ShardPlan& sp, const ShardCall& c,
                   const void* local_logits, const void* whole_logits, const std::vector<int>& rows) {
  const long long nf = (long long)rows.size();
  if (nf == 0) return PESTI_OK;
  const int esize = c.dtype == PESTI_F32 ? 4 : 2;
  const long long VT = sp.VT;
  const long long W = (c.d_kept_p || c.d_kept_idx) ? c.kept_width : 0;
  const Plan pf = make_plan(s->num_sms, c.dtype, nf, VT, true);
  size_t off = align_up(pf.bytes);
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes);
    return o;
  };
  const size_t o_rows = take((size_t)nf * sizeof(int));
  const size_t o_full = take((size_t)nf * VT * esize);
  const size_t o_u = take((size_t)nf * sizeof(float));
  const size_t o_prm = take((size_t)nf * sizeof(pesti_sampling_params));
  const size_t o_tok = take((size_t)nf * sizeof(uint32_t));
  const size_t o_kp = take((size_t)nf * std::max<long long>(W, 1) * sizeof(float));
  const size_t o_ki = take((size_t)nf * std::max<long long>(W, 1) * sizeof(uint32_t));
  const size_t o_kc = take((size_t)nf * sizeof(int64_t));
  const size_t o_send = take(comm ? (size_t)nf * c.Vs * esize : 0);
  const size_t o_recv = take(comm ? (size_t)nf * VT * esize : 0);
  // the sharded passes are done with the workspace (the stream was synchronized)
  int rc = ensure_ws(s, off);
  if (rc) return rc;
  char* ws = (char*)s->ws;
  // the gathered plan's counters: zero on the first sp.B rows after the sharded passes
  if (nf > sp.B) PESTI_CUDA_TRY(cudaMemsetAsync(ws, 0, (size_t)nf * sizeof(int), c.st), "cudaMemsetAsync(counters)");
  int* d_rows = (int*)(ws + o_rows);
  PESTI_CUDA_TRY(cudaMemcpyAsync(d_rows, rows.data(), (size_t)nf * sizeof(int), cudaMemcpyHostToDevice, c.st),
                 "row list copy");
  unsigned char* full = (unsigned char*)(ws + o_full);
  const long long row_bytes = VT * esize;
  if (comm) {
    const long long sh_bytes = c.Vs * esize;
    unsigned char* send = (unsigned char*)(ws + o_send);
    unsigned char* recv = (unsigned char*)(ws + o_recv);
    pesti::gather_rows_kernel<<<dim3(16, (unsigned)nf), 256, 0, c.st>>>(
        (const unsigned char*)local_logits, c.ld * esize, d_rows, (int)nf, sh_bytes, send, sh_bytes);
    PESTI_CUDA_TRY(cudaGetLastError(), "gather_rows_kernel launch");
    const ncclResult_t nr = nccl_api().all_gather(send, recv, (size_t)(nf * sh_bytes), ncclUint8, comm->comm, c.st);
    const int src = comm_settle(comm, nr, deadline_of(comm), "ncclAllGather(rows)");
    if (src) return src;
    for (int g = 0; g < sp.G; ++g)
      PESTI_CUDA_TRY(cudaMemcpy2DAsync(full + (size_t)g * sh_bytes, (size_t)row_bytes, recv + (size_t)g * nf * sh_bytes,
                                       (size_t)sh_bytes, (size_t)sh_bytes, (size_t)nf, cudaMemcpyDeviceToDevice, c.st),
                     "row assembly copy");
  } else {
    pesti::gather_rows_kernel<<<dim3(16, (unsigned)nf), 256, 0, c.st>>>(
        (const unsigned char*)whole_logits, c.ld * esize, d_rows, (int)nf, row_bytes, full, row_bytes);
    PESTI_CUDA_TRY(cudaGetLastError(), "gather_rows_kernel launch");
  }
  float* u_f = (float*)(ws + o_u);
  pesti_sampling_params* prm_f = (pesti_sampling_params*)(ws + o_prm);
  pesti::gather_row_values_kernel<<<(unsigned)((nf + 255) / 256), 256, 0, c.st>>>(d_rows, (int)nf, c.d_u, u_f,
                                                                                    c.d_per_row, prm_f);
  PESTI_CUDA_TRY(cudaGetLastError(), "gather_row_values_kernel launch");
  uint32_t* tok = (uint32_t*)(ws + o_tok);
  float* kp = (float*)(ws + o_kp);
  uint32_t* ki = (uint32_t*)(ws + o_ki);
  int64_t* kc = (int64_t*)(ws + o_kc);
  rc = run_plan(pf, ws, s->device, nullptr, full, c.dtype, nf, VT, VT, c.uni, c.d_per_row ? prm_f : nullptr, u_f,
                tok, W ? kp : nullptr, W ? ki : nullptr, W, kc, c.st);
  s->ctr_zero_rows = rc ? 0 : nf;
  if (rc) return rc;
  pesti::scatter_results_kernel<<<(unsigned)nf, 256, 0, c.st>>>(d_rows, (int)nf, tok, kp, ki, kc, W, c.d_out,
                                                                 c.d_kept_p, c.d_kept_idx, c.d_kept_count);
  PESTI_CUDA_TRY(cudaGetLastError(), "scatter_results_kernel launch");
  return PESTI_OK;
}

// Candidates each shard lists per row: the largest top-k of the call's
// top-k rows plus 8 (so that the bound on the unlisted ones lies well below
// the k-th), at most FIN_KEYS over all shards.
int shard_list_size(const pesti_sampling_params* params, int per_row, int on_device, long long B, long long VT, int G) {
  long long kmax = pesti::FAST_K;
  if (!on_device) {
    kmax = 1;
    const long long n = per_row ? B : 1;
    for (long long i = 0; i < n; ++i) {
      const long long k = std::min<long long>(params[i].top_k, VT);
      if (k >= 1 && k <= pesti::FAST_K) kmax = std::max(kmax, k);
    }
  }
  return (int)std::min<long long>(kmax + 8, pesti::FIN_KEYS / std::max(1, G));
}

// The sharded call.  comm == nullptr emulates `G` shards of the whole matrix
// `d_logits` in one process; otherwise d_logits is this rank's shard.
int sample_sharded(pesti_sampler* s, pesti_comm* comm, int G, const void* d_logits, pesti_dtype dtype,
                   long long B, long long Vs, long long ld, const pesti_sampling_params* params, int params_per_row,
                   int params_on_device, const float* d_u, uint32_t* d_out, float* d_kept_p, uint32_t* d_kept_idx,
                   long long kept_width, int64_t* d_kept_count, void* stream) {
  PESTI_CUDA_TRY(cudaSetDevice(s->device), "cudaSetDevice");
  cudaStream_t st = (cudaStream_t)stream;  // NULL: the legacy default stream
  if (comm && comm->aborted) return fail(PESTI_E_NCCL, "the communicator was aborted by an earlier failure");
  const Clock::time_point deadline = comm ? deadline_of(comm) : Clock::time_point{};
  ShardCall c{};
  c.dtype = dtype;
  c.B = B;
  c.Vs = Vs;
  c.ld = ld;
  c.d_u = d_u;
  c.d_out = d_out;
  c.d_kept_p = d_kept_p;
  c.d_kept_idx = d_kept_idx;
  c.kept_width = kept_width;
  c.d_kept_count = d_kept_count;
  c.st = st;
  bool sorted_bufs = false, survivors = false;
  int rc = stage_params(s, params, params_per_row, params_on_device, B, Vs * G, st, c.uni, c.d_per_row, sorted_bufs,
                        survivors);
  if (rc) return rc;
  const int esize = dtype == PESTI_F32 ? 4 : 2;
  const int nlocal = comm ? 1 : G;
  const int ksh = shard_list_size(params, params_per_row, params_on_device, B, Vs * G, G);
  const ShardPlan sp = make_shard_plan(s->num_sms, dtype, B, Vs, G, nlocal, ksh);
  rc = ensure_ws(s, sp.bytes);
  if (rc) return rc;
  char* ws = (char*)s->ws;
  auto lg = [&](int g) {  // shard g's columns
    return comm ? d_logits : (const void*)((const char*)d_logits + (size_t)g * Vs * esize);
  };
  pesti::ShardSum* sum_recv = (pesti::ShardSum*)(ws + sp.o_sum_recv);
  unsigned char* rec_recv = (unsigned char*)(ws + sp.o_rec_recv);
  pesti::ShardTab* tab_recv = (pesti::ShardTab*)(ws + sp.o_tab_recv);
  s->ctr_zero_rows = 0;
  // instrumentation (pesti_profile.h): the HBM pass, everything up to the
  // last exchange, the finish
  cudaEvent_t* pev = nullptr;
  if (s->prof && s->prof_n < pesti_sampler::kProfMax) {
    pev = s->prof_ev[s->prof_n++];
    for (int q = 0; q < 4; ++q)
      if (!pev[q]) PESTI_CUDA_TRY(cudaEventCreate(&pev[q]), "cudaEventCreate(profile)");
  }
  auto mark = [&](int q) { return pev ? cudaEventRecord(pev[q], st) : cudaSuccess; };
  PESTI_CUDA_TRY(mark(0), "cudaEventRecord(profile)");
  if (comm) {
    const NcclApi& n = nccl_api();
    pesti::ShardSum* sum_send = (pesti::ShardSum*)(ws + sp.o_sum_send);
    unsigned char* rec_send = (unsigned char*)(ws + sp.o_rec_send);
    pesti::ShardTab* tab_send = (pesti::ShardTab*)(ws + sp.o_tab_send);
    rc = shard_phase1(sp, ws, 0, c, d_logits, sum_send);
    if (rc) return rc;
    PESTI_CUDA_TRY(mark(1), "cudaEventRecord(profile)");
    ncclResult_t nr = n.all_gather(sum_send, sum_recv, (size_t)B * sizeof(pesti::ShardSum), ncclUint8, comm->comm, st);
    if ((rc = comm_settle(comm, nr, deadline, "ncclAllGather(summaries)"))) return rc;
    rc = shard_phase2(sp, ws, 0, comm->rank, s->device, c, d_logits, sum_recv, rec_send);
    if (rc) return rc;
    nr = n.all_gather(rec_send, rec_recv, (size_t)(B * sp.rec_stride), ncclUint8, comm->comm, st);
    if ((rc = comm_settle(comm, nr, deadline, "ncclAllGather(records)"))) return rc;
    rc = shard_phase3(sp, ws, 0, comm->rank, s->device, c, d_logits, rec_recv, tab_send);
    if (rc) return rc;
    nr = n.all_gather(tab_send, tab_recv, (size_t)B * sizeof(pesti::ShardTab), ncclUint8, comm->comm, st);
    if ((rc = comm_settle(comm, nr, deadline, "ncclAllGather(tables)"))) return rc;
  } else {
    for (int g = 0; g < G; ++g)
      if ((rc = shard_phase1(sp, ws, g, c, lg(g), sum_recv + (size_t)g * B))) return rc;
    PESTI_CUDA_TRY(mark(1), "cudaEventRecord(profile)");
    for (int g = 0; g < G; ++g)
      if ((rc = shard_phase2(sp, ws, g, g, s->device, c, lg(g), sum_recv, rec_recv + (size_t)g * B * sp.rec_stride)))
        return rc;
    for (int g = 0; g < G; ++g)
      if ((rc = shard_phase3(sp, ws, g, g, s->device, c, lg(g), rec_recv, tab_recv + (size_t)g * B))) return rc;
  }
  PESTI_CUDA_TRY(mark(2), "cudaEventRecord(profile)");
  rc = shard_finish(sp, ws, c);
  if (rc) return rc;
  PESTI_CUDA_TRY(mark(3), "cudaEventRecord(profile)");
  s->ctr_zero_rows = B;
  std::vector<int> rows;
  rc = read_flagged(sp, ws, st, rows, s->last_gathered_why, comm, deadline);
  if (rc) return rc;
  s->last_gathered_rows = (long long)rows.size();
  return shard_gathered(s, comm, sp, c, d_logits, d_logits, rows);
}

// fp8 logits -> f16, exactly (every E4M3 and E5M2 value, NaN and the E5M2
// infinities included, is an f16 value).  Row b's V bytes at src + b*ld go to
// dst + b*V; each thread widens 8 consecutive bytes, with an 8-byte load and a
// 16-byte store where both are aligned.
template <bool E4M3>
__global__ void __launch_bounds__(256) widen_fp8_kernel(const uint8_t* __restrict__ src, long long ld,
                                                        __half* __restrict__ dst, long long B, long long V) {
  constexpr __nv_fp8_interpretation_t kind = E4M3 ? __NV_E4M3 : __NV_E5M2;
  const long long c0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= V) return;
  for (long long b = blockIdx.y; b < B; b += gridDim.y) {  // gridDim.y is at most 65535
    const uint8_t* s = src + b * ld + c0;
    __half* d = dst + b * V + c0;
    if (c0 + 8 <= V && ((uintptr_t)s % 8 == 0) && ((uintptr_t)d % 16 == 0)) {
      const uint2 w = *reinterpret_cast<const uint2*>(s);
      uint4 o;
      const uint32_t in[2] = {w.x, w.y};
      uint32_t out[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const __nv_fp8x2_storage_t pair = (__nv_fp8x2_storage_t)((in[h >> 1] >> (16 * (h & 1))) & 0xffffu);
        const __half2_raw r = __nv_cvt_fp8x2_to_halfraw2(pair, kind);
        out[h] = (uint32_t)r.x | ((uint32_t)r.y << 16);
      }
      o.x = out[0]; o.y = out[1]; o.z = out[2]; o.w = out[3];
      *reinterpret_cast<uint4*>(d) = o;
      continue;
    }
    for (int e = 0; e < 8 && c0 + e < V; ++e) {
      const __half_raw r = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)s[e], kind);
      d[e] = __half(r);
    }
  }
}

bool is_fp8(pesti_dtype dtype) { return dtype == PESTI_FP8_E4M3 || dtype == PESTI_FP8_E5M2; }

// Widens fp8 logits into the handle's f16 buffer on stream st; the call then
// samples (*out, PESTI_F16, ld = V).
int widen_fp8(pesti_sampler* s, const void* d_logits, pesti_dtype dtype, long long B, long long V, long long ld,
              cudaStream_t st, const void** out) {
  const size_t need = (size_t)B * (size_t)V * 2;
  if (need > s->d_wide_cap) {
    if (s->d_wide) {
      PESTI_CUDA_TRY(cudaStreamSynchronize(st), "cudaStreamSynchronize");
      cudaFree(s->d_wide);
      s->d_wide = nullptr;
      s->d_wide_cap = 0;
    }
    PESTI_CUDA_TRY(cudaMalloc(&s->d_wide, need), "cudaMalloc(fp8 widening buffer)");
    s->d_wide_cap = need;
  }
  const dim3 grid((unsigned)((V + 256 * 8 - 1) / (256 * 8)), (unsigned)(B < 65535 ? B : 65535));
  if (dtype == PESTI_FP8_E4M3)
    widen_fp8_kernel<true><<<grid, 256, 0, st>>>((const uint8_t*)d_logits, ld, (__half*)s->d_wide, B, V);
  else
    widen_fp8_kernel<false><<<grid, 256, 0, st>>>((const uint8_t*)d_logits, ld, (__half*)s->d_wide, B, V);
  PESTI_CUDA_TRY(cudaGetLastError(), "widen_fp8_kernel launch");
  *out = s->d_wide;
  return PESTI_OK;
}

int check_shapes(const void* d_logits, pesti_dtype dtype, int64_t B, int64_t V, int64_t ld) {
  if (dtype != PESTI_F32 && dtype != PESTI_BF16 && dtype != PESTI_F16) return fail(PESTI_E_INVALID_ARG, "unsupported dtype");
  if (B < 0 || V < 0) return fail(PESTI_E_INVALID_ARG, "negative B or V");
  if (V > 0x7fffffffLL) return fail(PESTI_E_INVALID_ARG, "V exceeds 2^31-1");
  if (B > 0x7fffffffLL) return fail(PESTI_E_INVALID_ARG, "B exceeds 2^31-1");
  if (B > 0 && V > 0 && !d_logits) return fail(PESTI_E_INVALID_ARG, "null logits");
  if (B > 0 && ld < V) return fail(PESTI_E_INVALID_ARG, "leading dimension smaller than V");
  return PESTI_OK;
}

int check_common(pesti_sampler* s, const void* d_logits, pesti_dtype dtype, int64_t B, int64_t V,
                 int64_t ld) {
  if (!s) return fail(PESTI_E_INVALID_ARG, "null sampler handle");
  return check_shapes(d_logits, dtype, B, V, ld);
}

}  // namespace

extern "C" {

const char* pesti_last_error(void) { return g_last_error.c_str(); }

int pesti_sampler_create(int device, pesti_sampler** out) {
  if (!out) return fail(PESTI_E_INVALID_ARG, "null output pointer");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess || n == 0) return fail(PESTI_E_NO_DEVICE, "no CUDA device available");
  if (device < 0 || device >= n) return fail(PESTI_E_INVALID_ARG, "device index out of range");
  cudaDeviceProp prop;
  PESTI_CUDA_TRY(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major < 10) return fail(PESTI_E_UNSUPPORTED, "the sampler is built for sm_100a (B200)");
  PESTI_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
  pesti_sampler* s = new pesti_sampler();
  s->device = device;
  s->num_sms = prop.multiProcessorCount;
  e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) { delete s; return cuda_fail(e, "cudaStreamCreate"); }
  e = cudaEventCreateWithFlags(&s->params_ev, cudaEventDisableTiming);
  if (e != cudaSuccess) { cudaStreamDestroy(s->stream); delete s; return cuda_fail(e, "cudaEventCreate"); }
  *out = s;
  return PESTI_OK;
}

void pesti_sampler_destroy(pesti_sampler* s) {
  if (!s) return;
  cudaSetDevice(s->device);
  if (s->stream) cudaStreamSynchronize(s->stream);
  cudaDeviceSynchronize();
  if (s->ws) cudaFree(s->ws);
  if (s->d_params) cudaFree(s->d_params);
  if (s->h_params) cudaFreeHost(s->h_params);
  if (s->d_row) cudaFree(s->d_row);
  if (s->d_wide) cudaFree(s->d_wide);
  if (s->d_chain) cudaFree(s->d_chain);
  if (s->d_u1) cudaFree(s->d_u1);
  if (s->d_tok1) cudaFree(s->d_tok1);
  if (s->params_ev) cudaEventDestroy(s->params_ev);
  for (int i = 0; i < pesti_sampler::kProfMax; ++i)
    for (int q = 0; q < 4; ++q)
      if (s->prof_ev[i][q]) cudaEventDestroy(s->prof_ev[i][q]);
  if (s->stream) cudaStreamDestroy(s->stream);
  delete s;
}

int pesti_sample_batch(pesti_sampler* s, const void* d_logits, pesti_dtype dtype, int64_t B,
                       int64_t V, int64_t ld, const pesti_sampling_params* params,
                       int params_per_row, int params_on_device, const float* d_u,
                       uint32_t* d_out_tokens, float* d_kept_p, uint32_t* d_kept_idx,
                       int64_t kept_width, int64_t* d_kept_count, void* stream) {
  const bool fp8 = is_fp8(dtype);
  int rc = check_common(s, d_logits, fp8 ? PESTI_F16 : dtype, B, V, ld);
  if (rc) return rc;
  if (!params) return fail(PESTI_E_INVALID_ARG, "null params");
  if (B > 0 && (!d_u || !d_out_tokens)) return fail(PESTI_E_INVALID_ARG, "null u or output tokens");
  if ((d_kept_p || d_kept_idx) && kept_width <= 0) return fail(PESTI_E_INVALID_ARG, "kept_width must be > 0");
  if (B == 0) return PESTI_OK;
  PESTI_CUDA_TRY(cudaSetDevice(s->device), "cudaSetDevice");
  cudaStream_t st = (cudaStream_t)stream;  // NULL: the legacy default stream
  if (fp8 && V > 0) {  // widened exactly to f16 first
    rc = widen_fp8(s, d_logits, dtype, B, V, ld, st, &d_logits);
    if (rc) return rc;
    dtype = PESTI_F16;
    ld = V;
  } else if (fp8) {
    dtype = PESTI_F16;
  }
  pesti_sampling_params uni{};
  const pesti_sampling_params* d_per_row = nullptr;
  bool sorted_bufs = true, survivors = true;
  int ckind = 0;
  rc = stage_params(s, params, params_per_row, params_on_device, B, V, st, uni, d_per_row, sorted_bufs, survivors,
                    dtype, &ckind);
  if (rc) return rc;
  return launch(s, d_logits, dtype, B, V, ld, uni, d_per_row, sorted_bufs, survivors, ckind, d_u, d_out_tokens,
                d_kept_p, d_kept_idx, kept_width, d_kept_count, st);
}

int pesti_argmax_batch(pesti_sampler* s, const void* d_logits, pesti_dtype dtype, int64_t B,
                       int64_t V, int64_t ld, uint32_t flags, uint32_t* d_out_tokens, void* stream) {
  const bool fp8 = is_fp8(dtype);
  int rc = check_common(s, d_logits, fp8 ? PESTI_F16 : dtype, B, V, ld);
  if (rc) return rc;
  if (B > 0 && !d_out_tokens) return fail(PESTI_E_INVALID_ARG, "null output tokens");
  if (B == 0) return PESTI_OK;
  PESTI_CUDA_TRY(cudaSetDevice(s->device), "cudaSetDevice");
  cudaStream_t st = (cudaStream_t)stream;  // NULL: the legacy default stream
  if (fp8 && V > 0) {  // widened exactly to f16 first
    rc = widen_fp8(s, d_logits, dtype, B, V, ld, st, &d_logits);
    if (rc) return rc;
    dtype = PESTI_F16;
    ld = V;
  } else if (fp8) {
    dtype = PESTI_F16;
  }
  pesti_sampling_params uni{};
  uni.temperature = 0.0f;
  uni.flags = PESTI_FLAG_GREEDY_IF_ZERO_T | (flags & PESTI_FLAG_ARGMAX_FIRST);
  return launch(s, d_logits, dtype, B, V, ld, uni, nullptr, false, false, 1, nullptr, d_out_tokens, nullptr,
                nullptr, 0, nullptr, st);
}

int pesti_sample_row_host(pesti_sampler* s, const float* h_logits, int64_t V,
                          const pesti_sampling_params* params, float u, uint32_t* out_token) {
  if (!s || !params || !out_token) return fail(PESTI_E_INVALID_ARG, "null argument");
  if (V < 0 || V > 0x7fffffffLL) return fail(PESTI_E_INVALID_ARG, "bad V");
  if (V > 0 && !h_logits) return fail(PESTI_E_INVALID_ARG, "null logits");
  PESTI_CUDA_TRY(cudaSetDevice(s->device), "cudaSetDevice");
  const size_t need = (size_t)std::max<int64_t>(V, 4);
  if (need > s->d_row_cap) {
    if (s->d_row) cudaFree(s->d_row);
    s->d_row = nullptr;
    PESTI_CUDA_TRY(cudaMalloc(&s->d_row, need * sizeof(float)), "cudaMalloc(row)");
    s->d_row_cap = need;
  }
  if (!s->d_u1) PESTI_CUDA_TRY(cudaMalloc(&s->d_u1, 16), "cudaMalloc(u)");
  if (!s->d_tok1) PESTI_CUDA_TRY(cudaMalloc(&s->d_tok1, 16), "cudaMalloc(token)");
  cudaStream_t st = s->stream;
  if (V > 0)
    PESTI_CUDA_TRY(cudaMemcpyAsync(s->d_row, h_logits, (size_t)V * sizeof(float), cudaMemcpyHostToDevice, st), "logits copy");
  PESTI_CUDA_TRY(cudaMemcpyAsync(s->d_u1, &u, sizeof(float), cudaMemcpyHostToDevice, st), "u copy");
  int rc = launch(s, s->d_row, PESTI_F32, 1, V, std::max<int64_t>(V, 1), *params, nullptr,
                  needs_sorted_buffers(params, 1), needs_survivor_pass(params, 1, V),
                  cluster_kind(params, 1, V, PESTI_F32), s->d_u1, s->d_tok1, nullptr, nullptr, 0, nullptr, st);
  if (rc) return rc;
  uint32_t tok = 0;
  PESTI_CUDA_TRY(cudaMemcpyAsync(&tok, s->d_tok1, sizeof(uint32_t), cudaMemcpyDeviceToHost, st), "token copy");
  PESTI_CUDA_TRY(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  *out_token = tok;
  return PESTI_OK;
}

int pesti_sample_batch_noalloc(const void* d_logits, pesti_dtype dtype, int64_t B, int64_t V,
                               int64_t ld, const pesti_sampling_params* params,
                               int params_per_row, int params_on_device, const float* d_u,
                               uint32_t* d_out_tokens, float* d_kept_p, uint32_t* d_kept_idx,
                               int64_t kept_width, int64_t* d_kept_count, void* stream) {
  int rc = check_shapes(d_logits, dtype, B, V, ld);
  if (rc) return rc;
  if (!params) return fail(PESTI_E_INVALID_ARG, "null params");
  if (B > 0 && (!d_u || !d_out_tokens)) return fail(PESTI_E_INVALID_ARG, "null u or output tokens");
  if ((d_kept_p || d_kept_idx) && kept_width <= 0) return fail(PESTI_E_INVALID_ARG, "kept_width must be > 0");
  if (B == 0) return PESTI_OK;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
    return fail(PESTI_E_NO_DEVICE, "no CUDA device available");
  int device = 0;
  PESTI_CUDA_TRY(cudaGetDevice(&device), "cudaGetDevice");
  pesti_noalloc_device dev{};
  PESTI_CUDA_TRY(pesti_noalloc_setup(device, &dev), "no-allocation scratch set-up");
  if (dev.cc_major < 10) return fail(PESTI_E_UNSUPPORTED, "the sampler is built for sm_100a (B200)");
  cudaStream_t st = (cudaStream_t)stream;

  pesti_sampling_params uni{};
  const pesti_sampling_params* d_per_row = nullptr;
  bool sorted_bufs = true, survivors = true;
  size_t params_bytes = 0;  // host per-row params go to the front of the scratch
  if (params_on_device) {
    if (params_per_row) d_per_row = params;
    else {
      PESTI_CUDA_TRY(cudaMemcpyAsync(&uni, params, sizeof(uni), cudaMemcpyDeviceToHost, st), "params copy");
      PESTI_CUDA_TRY(cudaStreamSynchronize(st), "params sync");
      sorted_bufs = needs_sorted_buffers(&uni, 1);
      survivors = needs_survivor_pass(&uni, 1, V);
    }
  } else if (params_per_row) {
    sorted_bufs = needs_sorted_buffers(params, B);
    survivors = needs_survivor_pass(params, B, V);
    params_bytes = align_up((size_t)B * sizeof(pesti_sampling_params));
  } else {
    uni = params[0];
    sorted_bufs = needs_sorted_buffers(&uni, 1);
    survivors = needs_survivor_pass(&uni, 1, V);
  }
  Plan p = make_plan(dev.num_sms, dtype, B, V, sorted_bufs);
  p.survivors = survivors;
  const size_t need = params_bytes + p.bytes;
  if (need > (size_t)PESTI_NOALLOC_SCRATCH_BYTES)
    return fail(PESTI_E_INVALID_ARG,
                "batch too large for pesti_sample_batch_noalloc: it needs " + std::to_string(need) +
                    " bytes of scratch, the static array holds " +
                    std::to_string((size_t)PESTI_NOALLOC_SCRATCH_BYTES) +
                    " (PESTI_NOALLOC_SCRATCH_BYTES); split the batch or use pesti_sample_batch");
  if (params_bytes) {
    PESTI_CUDA_TRY(cudaMemcpyAsync(dev.scratch, params, (size_t)B * sizeof(pesti_sampling_params),
                                   cudaMemcpyHostToDevice, st), "params copy");
    d_per_row = (const pesti_sampling_params*)dev.scratch;
  }
  char* ws = dev.scratch + params_bytes;
  // the per-row completion counters must start at zero, and the array holds
  // whatever the previous call (or an aborted one) left there
  PESTI_CUDA_TRY(cudaMemsetAsync(ws + p.o_ctr, 0, (size_t)B * sizeof(int), st), "cudaMemsetAsync(counters)");
  return run_plan(p, ws, device, nullptr, d_logits, dtype, B, V, ld, uni, d_per_row, d_u, d_out_tokens,
                  d_kept_p, d_kept_idx, kept_width, d_kept_count, st);
}

int pesti_comm_id(void* id) {
  if (!id) return fail(PESTI_E_INVALID_ARG, "null id buffer");
  const NcclApi& n = nccl_api();
  if (!n.loaded) return fail(PESTI_E_NCCL, n.err);
  ncclUniqueId u;
  const ncclResult_t r = n.get_unique_id(&u);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  static_assert(sizeof(ncclUniqueId) == PESTI_COMM_ID_BYTES, "NCCL unique id size");
  std::memcpy(id, &u, sizeof(u));
  return PESTI_OK;
}

int pesti_comm_create(int world_size, int rank, const void* id, int device, pesti_comm** out) {
  return pesti_comm_create_timed(world_size, rank, id, device, 120000, out);
}

int pesti_comm_create_timed(int world_size, int rank, const void* id, int device, int timeout_ms, pesti_comm** out) {
  if (!out || !id) return fail(PESTI_E_INVALID_ARG, "null argument");
  *out = nullptr;
  if (world_size < 1 || world_size > pesti::FIN_MAXG || rank < 0 || rank >= world_size)
    return fail(PESTI_E_INVALID_ARG, "bad world size or rank (1..64 ranks)");
  if (timeout_ms < 1) return fail(PESTI_E_INVALID_ARG, "timeout_ms must be >= 1");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(PESTI_E_NO_DEVICE, "no CUDA device available");
  if (device < 0 || device >= ndev) return fail(PESTI_E_INVALID_ARG, "device index out of range");
  const NcclApi& n = nccl_api();
  if (!n.loaded) return fail(PESTI_E_NCCL, n.err);
  PESTI_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  pesti_comm* c = new pesti_comm();
  c->world = world_size;
  c->rank = rank;
  c->device = device;
  c->timeout_ms = timeout_ms;
  // non-blocking: the set-up runs in the background and is polled with a
  // deadline, so a rank that never joins cannot hang the others
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  const Clock::time_point deadline = deadline_of(c);
  const ncclResult_t r = n.comm_init_rank_config(&c->comm, world_size, u, rank, &cfg);
  if (!c->comm) {
    delete c;
    return nccl_fail(r == ncclSuccess ? ncclInternalError : r, "ncclCommInitRankConfig");
  }
  const int rc = comm_settle(c, r, deadline, "ncclCommInitRankConfig");
  if (rc) {  // the communicator was aborted (ncclCommAbort frees it)
    delete c;
    return rc;
  }
  *out = c;
  return PESTI_OK;
}

void pesti_comm_destroy(pesti_comm* c) {
  if (!c) return;
  if (c->comm && !c->aborted) {
    cudaSetDevice(c->device);
    nccl_api().comm_destroy(c->comm);
  }
  delete c;
}

int pesti_sample_batch_sharded(pesti_sampler* s, pesti_comm* c, const void* d_logits, pesti_dtype dtype,
                               int64_t B, int64_t V_shard, int64_t ld, const pesti_sampling_params* params,
                               int params_per_row, int params_on_device, const float* d_u,
                               uint32_t* d_out_tokens, float* d_kept_p, uint32_t* d_kept_idx,
                               int64_t kept_width, int64_t* d_kept_count, void* stream) {
  int rc = check_common(s, d_logits, dtype, B, V_shard, ld);
  if (rc) return rc;
  if (!c) return fail(PESTI_E_INVALID_ARG, "null communicator");
  if (c->device != s->device) return fail(PESTI_E_INVALID_ARG, "sampler and communicator on different devices");
  if (!params) return fail(PESTI_E_INVALID_ARG, "null params");
  if (V_shard < 1) return fail(PESTI_E_INVALID_ARG, "every shard needs at least one column");
  if ((long long)V_shard * c->world > 0x7fffffffLL) return fail(PESTI_E_INVALID_ARG, "whole rows exceed 2^31-1");
  if (B > 0 && (!d_u || !d_out_tokens)) return fail(PESTI_E_INVALID_ARG, "null u or output tokens");
  if ((d_kept_p || d_kept_idx) && kept_width <= 0) return fail(PESTI_E_INVALID_ARG, "kept_width must be > 0");
  if (B == 0) return PESTI_OK;
  return sample_sharded(s, c, c->world, d_logits, dtype, B, V_shard, ld, params, params_per_row, params_on_device,
                        d_u, d_out_tokens, d_kept_p, d_kept_idx, kept_width, d_kept_count, stream);
}

int pesti_sample_batch_sharded_emulated(pesti_sampler* s, int shards, const void* d_logits, pesti_dtype dtype,
                                        int64_t B, int64_t V, int64_t ld, const pesti_sampling_params* params,
                                        int params_per_row, int params_on_device, const float* d_u,
                                        uint32_t* d_out_tokens, float* d_kept_p, uint32_t* d_kept_idx,
                                        int64_t kept_width, int64_t* d_kept_count, void* stream) {
  int rc = check_common(s, d_logits, dtype, B, V, ld);
  if (rc) return rc;
  if (shards < 1 || shards > pesti::FIN_MAXG) return fail(PESTI_E_INVALID_ARG, "shards must be 1..64");
  if (V < shards || V % shards != 0) return fail(PESTI_E_INVALID_ARG, "V must be a multiple of the shard count");
  if (!params) return fail(PESTI_E_INVALID_ARG, "null params");
  if (B > 0 && (!d_u || !d_out_tokens)) return fail(PESTI_E_INVALID_ARG, "null u or output tokens");
  if ((d_kept_p || d_kept_idx) && kept_width <= 0) return fail(PESTI_E_INVALID_ARG, "kept_width must be > 0");
  if (B == 0) return PESTI_OK;
  return sample_sharded(s, nullptr, shards, d_logits, dtype, B, V / shards, ld, params, params_per_row,
                        params_on_device, d_u, d_out_tokens, d_kept_p, d_kept_idx, kept_width, d_kept_count, stream);
}

int64_t pesti_last_gathered_rows(pesti_sampler* s) { return s ? s->last_gathered_rows : -1; }

int pesti_testing_set_cluster(int mode) {
  if (mode != -1 && mode != 0 && !(mode >= 1 && mode <= pesti::CL_MAXC))
    return fail(PESTI_E_INVALID_ARG, "cluster mode must be -1, 0 or 1..16");
  g_cluster_override.store(mode, std::memory_order_relaxed);
  return PESTI_OK;
}

int pesti_pcg32_seed(uint64_t* d_state, int64_t B, uint64_t seed, uint64_t first_stream, void* stream) {
  if (B < 0) return fail(PESTI_E_INVALID_ARG, "B < 0");
  if (B == 0) return PESTI_OK;
  if (!d_state) return fail(PESTI_E_INVALID_ARG, "null state");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(PESTI_E_NO_DEVICE, "no CUDA device available");
  const long long blocks = (B + 255) / 256;
  pesti::pcg32_seed_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(d_state, B, seed, first_stream);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PESTI_OK : cuda_fail(e, "pcg32_seed_kernel launch");
}

int pesti_pcg32_draw(uint64_t* d_state, int64_t B, float* d_u, void* stream) {
  if (B < 0) return fail(PESTI_E_INVALID_ARG, "B < 0");
  if (B == 0) return PESTI_OK;
  if (!d_state || !d_u) return fail(PESTI_E_INVALID_ARG, "null state or draws");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(PESTI_E_NO_DEVICE, "no CUDA device available");
  const long long blocks = (B + 255) / 256;
  pesti::pcg32_draw_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(d_state, B, d_u);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PESTI_OK : cuda_fail(e, "pcg32_draw_kernel launch");
}

int pesti_generate_advance(const uint32_t* d_next, int64_t B, const uint32_t* d_stop, int64_t n_stop,
                           int64_t max_tokens, int64_t max_seq_len, uint32_t* d_generated, int64_t cap,
                           int32_t* d_count, uint8_t* d_done, uint32_t* d_last, int32_t* d_active, void* stream) {
  if (B < 0 || n_stop < 0) return fail(PESTI_E_INVALID_ARG, "B or n_stop < 0");
  if (max_tokens < 0 || max_seq_len < 0) return fail(PESTI_E_INVALID_ARG, "max_tokens or max_seq_len < 0");
  if (max_tokens > 0x7fffffffLL || max_seq_len > 0x7fffffffLL) return fail(PESTI_E_INVALID_ARG, "limits exceed 2^31-1");
  if (cap < std::min(max_tokens, max_seq_len)) return fail(PESTI_E_INVALID_ARG, "cap is below min(max_tokens, max_seq_len)");
  if (B == 0) return PESTI_OK;
  if (!d_next || !d_generated || !d_count || !d_done || !d_last) return fail(PESTI_E_INVALID_ARG, "null argument");
  if (n_stop > 0 && !d_stop) return fail(PESTI_E_INVALID_ARG, "null stop list");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(PESTI_E_NO_DEVICE, "no CUDA device available");
  pesti::generate_advance_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(d_next, B, d_stop, n_stop, max_tokens,
                                                                      max_seq_len, d_generated, cap, d_count,
                                                                      d_done, d_last, d_active);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PESTI_OK : cuda_fail(e, "generate_advance_kernel launch");
}

int pesti_llama_chain_batch(pesti_sampler* s, const void* d_logits, pesti_dtype dtype, int64_t B, int64_t V,
                            int64_t ld, const pesti_llama_chain_params* params, const int32_t* d_history,
                            const int32_t* d_history_len, int64_t history_ld, const float* d_u,
                            int32_t* d_out_tokens, int32_t* d_out_kept, void* stream) {
  const bool fp8 = is_fp8(dtype);
  int rc = check_common(s, d_logits, fp8 ? PESTI_F16 : dtype, B, V, ld);
  if (rc) return rc;
  if (!params) return fail(PESTI_E_INVALID_ARG, "null params");
  if (B == 0) return PESTI_OK;
  if (V < 1) return fail(PESTI_E_INVALID_ARG, "V must be at least 1");
  if (!d_u || !d_out_tokens) return fail(PESTI_E_INVALID_ARG, "null u or output tokens");
  if (history_ld < 0) return fail(PESTI_E_INVALID_ARG, "history_ld < 0");
  const pesti_llama_chain_params& p = *params;
  const bool penalties = p.repetition_penalty != 1.0f && p.repeat_last_n != 0 && history_ld > 0;
  if (penalties) {
    if (!d_history) return fail(PESTI_E_INVALID_ARG, "null history");
    const int64_t win = p.repeat_last_n < 0 ? history_ld : std::min<int64_t>(p.repeat_last_n, history_ld);
    if (win > pesti::CH_WINDOW) return fail(PESTI_E_INVALID_ARG, "repetition window above 8192 tokens");
  }
  PESTI_CUDA_TRY(cudaSetDevice(s->device), "cudaSetDevice");
  cudaStream_t st = (cudaStream_t)stream;
  if (fp8) {
    rc = widen_fp8(s, d_logits, dtype, B, V, ld, st, &d_logits);
    if (rc) return rc;
    dtype = PESTI_F16;
    ld = V;
  }
  // scratch of 16 bytes per logit; refuse sizes whose byte count overflows
  if ((size_t)B > (SIZE_MAX / 16) / (size_t)V) return fail(PESTI_E_INVALID_ARG, "B * V too large");
  const size_t per = (size_t)B * (size_t)V;
  const size_t need = per * (sizeof(float) + sizeof(int) + sizeof(double));
  if (need > s->d_chain_cap) {
    if (s->d_chain) {
      PESTI_CUDA_TRY(cudaStreamSynchronize(st), "cudaStreamSynchronize");
      cudaFree(s->d_chain);
      s->d_chain = nullptr;
      s->d_chain_cap = 0;
    }
    PESTI_CUDA_TRY(cudaMalloc(&s->d_chain, need), "cudaMalloc(chain scratch)");
    s->d_chain_cap = need;
  }
  double* sw = (double*)s->d_chain;
  float* sl = (float*)(sw + per);
  int* si = (int*)(sl + per);
  pesti::ChainArgs a{p.temperature,        p.top_k,         p.top_p,
                     p.min_p,              p.tfs,           p.typical_p,
                     p.repetition_penalty, p.repeat_last_n, p.frequency_penalty,
                     p.presence_penalty};
  if (!penalties) a.repetition_penalty = 1.0f;
  const size_t smem = sizeof(pesti::ChainShared);
  if (!s->chain_smem_set) {
    PESTI_CUDA_TRY(cudaFuncSetAttribute(pesti::llama_chain_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)smem),
                   "cudaFuncSetAttribute(chain)");
    PESTI_CUDA_TRY(cudaFuncSetAttribute(pesti::llama_chain_kernel<uint16_t>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                   "cudaFuncSetAttribute(chain)");
    PESTI_CUDA_TRY(cudaFuncSetAttribute(pesti::llama_chain_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)smem),
                   "cudaFuncSetAttribute(chain)");
    s->chain_smem_set = true;
  }
  const int32_t* hp = penalties ? d_history : nullptr;
  const dim3 grid((unsigned)B), block(pesti::CH_THREADS);
  if (dtype == PESTI_BF16)
    pesti::llama_chain_kernel<uint16_t><<<grid, block, smem, st>>>((const uint16_t*)d_logits, (int)V, ld, a, hp,
                                                                   d_history_len, history_ld, d_u, d_out_tokens,
                                                                   d_out_kept, sl, si, sw);
  else if (dtype == PESTI_F16)
    pesti::llama_chain_kernel<__half><<<grid, block, smem, st>>>((const __half*)d_logits, (int)V, ld, a, hp,
                                                                 d_history_len, history_ld, d_u, d_out_tokens,
                                                                 d_out_kept, sl, si, sw);
  else
    pesti::llama_chain_kernel<float><<<grid, block, smem, st>>>((const float*)d_logits, (int)V, ld, a, hp,
                                                                d_history_len, history_ld, d_u, d_out_tokens,
                                                                d_out_kept, sl, si, sw);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PESTI_OK : cuda_fail(e, "llama_chain_kernel launch");
}

int pesti_test_ex2_approx_max_relerr(double* out) {
  if (!out) return fail(PESTI_E_INVALID_ARG, "null output");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(PESTI_E_NO_DEVICE, "no CUDA device available");
  unsigned long long* d = nullptr;
  PESTI_CUDA_TRY(cudaMalloc(&d, sizeof(unsigned long long)), "cudaMalloc");
  cudaError_t e = cudaMemset(d, 0, sizeof(unsigned long long));
  if (e == cudaSuccess) {
    pesti::ex2_approx_error_kernel<<<1184, 256>>>(d);
    e = cudaGetLastError();
  }
  unsigned long long bits = 0ull;
  if (e == cudaSuccess) e = cudaMemcpy(&bits, d, sizeof(bits), cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (e != cudaSuccess) return cuda_fail(e, "ex2_approx_error_kernel");
  std::memcpy(out, &bits, sizeof(double));
  return PESTI_OK;
}

int pesti_last_gathered_reasons(pesti_sampler* s, int64_t* counts) {
  if (!s || !counts) return fail(PESTI_E_INVALID_ARG, "null argument");
  for (int q = 0; q < pesti::GR_KINDS; ++q) counts[q] = s->last_gathered_why[q];
  return PESTI_OK;
}

int pesti_profile_enable(pesti_sampler* s, int enable) {
  if (!s) return fail(PESTI_E_INVALID_ARG, "null sampler handle");
  s->prof = enable != 0;
  s->prof_n = 0;
  return PESTI_OK;
}

int pesti_profile_read(pesti_sampler* s, double* max_ms, double* surv_ms, double* row_ms, int* calls) {
  if (!s || !max_ms || !surv_ms || !row_ms || !calls) return fail(PESTI_E_INVALID_ARG, "null argument");
  double t[3] = {0.0, 0.0, 0.0};
  for (int i = 0; i < s->prof_n; ++i) {
    PESTI_CUDA_TRY(cudaEventSynchronize(s->prof_ev[i][3]), "cudaEventSynchronize(profile)");
    for (int q = 0; q < 3; ++q) {
      float ms = 0.f;
      PESTI_CUDA_TRY(cudaEventElapsedTime(&ms, s->prof_ev[i][q], s->prof_ev[i][q + 1]), "cudaEventElapsedTime");
      t[q] += ms;
    }
  }
  *max_ms = t[0];
  *surv_ms = t[1];
  *row_ms = t[2];
  *calls = s->prof_n;
  return PESTI_OK;
}

}  // extern "C"
