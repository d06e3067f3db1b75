// Host side of the sampler library: the C ABI of include/pesti_sampler.h.
// Launch geometry, workspace and error reporting live here; the arithmetic is
// in pesti_kernels.cuh.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/pesti_sampler.h"
#include "../../include/pesti_profile.h"
#include "pesti_kernels.cuh"
#include "pesti_noalloc.h"

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

struct pesti_sampler {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  pesti_sampling_params* d_params = nullptr;
  size_t d_params_cap = 0;
  pesti_sampling_params* h_params = nullptr;  // pinned staging
  size_t h_params_cap = 0;
  cudaEvent_t params_ev = nullptr;
  bool params_ev_used = false;
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
};

namespace {

struct Geometry {
  int P;
  long long SL;
};

Geometry pick_geometry(int num_sms, long long B, long long V, int ve) {
  const long long target = 4LL * num_sms;
  long long P = (target + B - 1) / std::max(1LL, B);
  const long long pmax_v = std::max(1LL, V / (pesti::K1_WARPS * 1024LL));
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
  return PESTI_OK;
}

size_t align_up(size_t x) { return (x + 255) & ~(size_t)255; }

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
  size_t o_ctr, o_stats, o_pre, o_info, o_surv, o_segmax, o_se, o_si, o_cc, o_ce, o_ci;
  size_t o_gsurv, o_tasks, o_tctr, o_pctr, o_pool;
  size_t o_E, o_I, o_status;
  size_t o_sk0 = 0, o_sv0 = 0, o_sk1 = 0, o_sv1 = 0, o_q = 0;
  size_t bytes;  // workspace the call needs
};

Plan make_plan(int num_sms, pesti_dtype dtype, long long B, long long V, bool sorted_bufs) {
  const int esize = dtype == PESTI_BF16 ? 2 : 4;
  const int ve = 16 / esize;
  Plan p;
  p.g = pick_geometry(num_sms, B, V > 0 ? V : 1, ve);
  p.num_sms = num_sms;
  p.nsub = (long long)p.g.P * pesti::K1_WARPS;
  p.nseg = (std::max(1LL, V) + 32LL * ve - 1) / (32LL * ve);
  p.jmax = (p.g.SL + pesti::GROUP - 1) / pesti::GROUP;
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
  p.o_se = take(bv * 4);
  p.o_si = take(bv * 4);
  p.o_cc = take((size_t)B * 4);
  p.o_ce = take((size_t)B * pesti::CAND_CAP * 4);
  p.o_ci = take((size_t)B * pesti::CAND_CAP * 4);
  p.o_E = take(bv * 4);
  p.o_I = take(bv * 4);
  p.o_status = take(16);
  p.o_gsurv = take(ngrp * sizeof(pesti::GroupEnt));
  p.o_tasks = take(ngrp * sizeof(pesti::ClassTask));
  p.o_tctr = take(2 * sizeof(int));
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

// Enqueues the three passes of one batch call on `st` over workspace `ws`
// (laid out by `p`).  pev: four events bracketing the passes, or null.
int run_plan(const Plan& p, char* ws, int device, cudaEvent_t* pev, const void* d_logits,
             pesti_dtype dtype, long long B, long long V, long long ld,
             const pesti_sampling_params& uni, const pesti_sampling_params* d_per_row,
             const float* d_u, uint32_t* d_out, float* d_kept_p, uint32_t* d_kept_idx,
             long long kept_width, int64_t* d_kept_count, cudaStream_t st) {
  const int esize = dtype == PESTI_BF16 ? 2 : 4;
  const bool sorted_bufs = p.sorted_bufs;

  pesti::SliceArgs sa;
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
  sa.surv_raw = (float*)(ws + p.o_se);
  sa.surv_idx = (uint32_t*)(ws + p.o_si);
  sa.jmax = (int)p.jmax;
  sa.tasks = (pesti::ClassTask*)(ws + p.o_tasks);
  sa.task_count = (int*)(ws + p.o_tctr);
  sa.task_next = sa.task_count + 1;
  sa.gsurv = (pesti::GroupEnt*)(ws + p.o_gsurv);
  sa.pool = (pesti::FoldEnt*)(ws + p.o_pool);
  sa.pool_ctr = (int*)(ws + p.o_pctr);
  sa.cand_count = (int*)(ws + p.o_cc);
  sa.cand_e = (float*)(ws + p.o_ce);
  sa.cand_idx = (uint32_t*)(ws + p.o_ci);

  // the fast path stages the row's fold entries in shared memory; with very
  // many sub-slices it does not fit and all rows take the generic path
  const size_t fast_bytes = pesti::fast_smem_bytes((int)p.nsub);
  sa.fast_enabled = sizeof(pesti::RowShared) + fast_bytes <= kRowSmemLimit ? 1 : 0;

  if (pev) PESTI_CUDA_TRY(cudaEventRecord(pev[0], st), "cudaEventRecord(profile)");
  const bool aligned = ((uintptr_t)d_logits % 16 == 0) && ((ld * esize) % 16 == 0);
  const dim3 g1((unsigned)(p.g.P * B));
  if (dtype == PESTI_BF16) {
    if (aligned) pesti::slice_stats_kernel<uint16_t, 8, 4, true><<<g1, pesti::K1_NT, 0, st>>>(sa);
    else pesti::slice_stats_kernel<uint16_t, 8, 4, false><<<g1, pesti::K1_NT, 0, st>>>(sa);
  } else {
    if (aligned) pesti::slice_stats_kernel<float, 4, 8, true><<<g1, pesti::K1_NT, 0, st>>>(sa);
    else pesti::slice_stats_kernel<float, 4, 8, false><<<g1, pesti::K1_NT, 0, st>>>(sa);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "slice_stats_kernel launch");
  if (pev) PESTI_CUDA_TRY(cudaEventRecord(pev[1], st), "cudaEventRecord(profile)");
  // the survivor pass reads from L2: fewer loads in flight, smaller code
  const dim3 b1(pesti::K1_NT);
  if (dtype == PESTI_BF16) {
    if (aligned) e = launch_dependent(pesti::survivor_kernel<uint16_t, 8, true>, g1, b1, 0, st, sa);
    else e = launch_dependent(pesti::survivor_kernel<uint16_t, 8, false>, g1, b1, 0, st, sa);
  } else {
    if (aligned) e = launch_dependent(pesti::survivor_kernel<float, 4, true>, g1, b1, 0, st, sa);
    else e = launch_dependent(pesti::survivor_kernel<float, 4, false>, g1, b1, 0, st, sa);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "survivor_kernel launch");
  // classification tasks: a persistent grid takes them from a counter
  {
    const long long most = (long long)B * p.nsub * p.jmax;
    const long long blocks = std::min<long long>(4LL * p.num_sms, (most + pesti::K1_WARPS - 1) / pesti::K1_WARPS);
    e = launch_dependent(pesti::classify_kernel, dim3((unsigned)std::max(1LL, blocks)), b1, 0, st, sa);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "classify_kernel launch");
  }
  if (pev) PESTI_CUDA_TRY(cudaEventRecord(pev[2], st), "cudaEventRecord(profile)");

  pesti::RowArgs ra;
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
  const size_t smem2 = sizeof(pesti::RowShared) + (ra.fast_enabled ? fast_bytes : 0);
  if (smem2 > 48 * 1024) {
    int rc = ensure_row_smem_limit(device);
    if (rc) return rc;
  }
  e = launch_dependent(pesti::row_kernel, dim3((unsigned)B), dim3(pesti::K2_NT), smem2, st, ra);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "row_kernel launch");
  if (pev) PESTI_CUDA_TRY(cudaEventRecord(pev[3], st), "cudaEventRecord(profile)");
  return PESTI_OK;
}

int launch(pesti_sampler* s, const void* d_logits, pesti_dtype dtype, long long B, long long V,
           long long ld, const pesti_sampling_params& uni, const pesti_sampling_params* d_per_row,
           bool sorted_bufs, const float* d_u, uint32_t* d_out, float* d_kept_p,
           uint32_t* d_kept_idx, long long kept_width, int64_t* d_kept_count, cudaStream_t st) {
  const Plan p = make_plan(s->num_sms, dtype, B, V, sorted_bufs);
  int rc = ensure_ws(s, p.bytes);
  if (rc) return rc;
  cudaEvent_t* pev = nullptr;
  if (s->prof && s->prof_n < pesti_sampler::kProfMax) {
    pev = s->prof_ev[s->prof_n++];
    for (int q = 0; q < 4; ++q)
      if (!pev[q]) PESTI_CUDA_TRY(cudaEventCreate(&pev[q]), "cudaEventCreate(profile)");
  }
  return run_plan(p, (char*)s->ws, s->device, pev, d_logits, dtype, B, V, ld, uni, d_per_row, d_u,
                  d_out, d_kept_p, d_kept_idx, kept_width, d_kept_count, st);
}

int check_shapes(const void* d_logits, pesti_dtype dtype, int64_t B, int64_t V, int64_t ld) {
  if (dtype != PESTI_F32 && dtype != PESTI_BF16) return fail(PESTI_E_INVALID_ARG, "unsupported dtype");
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
  int rc = check_common(s, d_logits, dtype, B, V, ld);
  if (rc) return rc;
  if (!params) return fail(PESTI_E_INVALID_ARG, "null params");
  if (B > 0 && (!d_u || !d_out_tokens)) return fail(PESTI_E_INVALID_ARG, "null u or output tokens");
  if ((d_kept_p || d_kept_idx) && kept_width <= 0) return fail(PESTI_E_INVALID_ARG, "kept_width must be > 0");
  if (B == 0) return PESTI_OK;
  PESTI_CUDA_TRY(cudaSetDevice(s->device), "cudaSetDevice");
  cudaStream_t st = stream ? (cudaStream_t)stream : s->stream;
  pesti_sampling_params uni{};
  const pesti_sampling_params* d_per_row = nullptr;
  bool sorted_bufs = true;
  if (params_on_device) {
    if (params_per_row) d_per_row = params;
    else {
      // single device entry: read it back once (rare API use)
      PESTI_CUDA_TRY(cudaMemcpyAsync(&uni, params, sizeof(uni), cudaMemcpyDeviceToHost, st), "params copy");
      PESTI_CUDA_TRY(cudaStreamSynchronize(st), "params sync");
      sorted_bufs = needs_sorted_buffers(&uni, 1);
    }
  } else if (params_per_row) {
    sorted_bufs = needs_sorted_buffers(params, B);
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
  }
  return launch(s, d_logits, dtype, B, V, ld, uni, d_per_row, sorted_bufs, d_u, d_out_tokens,
                d_kept_p, d_kept_idx, kept_width, d_kept_count, st);
}

int pesti_argmax_batch(pesti_sampler* s, const void* d_logits, pesti_dtype dtype, int64_t B,
                       int64_t V, int64_t ld, uint32_t flags, uint32_t* d_out_tokens, void* stream) {
  int rc = check_common(s, d_logits, dtype, B, V, ld);
  if (rc) return rc;
  if (B > 0 && !d_out_tokens) return fail(PESTI_E_INVALID_ARG, "null output tokens");
  if (B == 0) return PESTI_OK;
  PESTI_CUDA_TRY(cudaSetDevice(s->device), "cudaSetDevice");
  cudaStream_t st = stream ? (cudaStream_t)stream : s->stream;
  pesti_sampling_params uni{};
  uni.temperature = 0.0f;
  uni.flags = PESTI_FLAG_GREEDY_IF_ZERO_T | (flags & PESTI_FLAG_ARGMAX_FIRST);
  return launch(s, d_logits, dtype, B, V, ld, uni, nullptr, false, nullptr, d_out_tokens, nullptr,
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
                  needs_sorted_buffers(params, 1), s->d_u1, s->d_tok1, nullptr, nullptr, 0, nullptr, st);
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
  bool sorted_bufs = true;
  size_t params_bytes = 0;  // host per-row params go to the front of the scratch
  if (params_on_device) {
    if (params_per_row) d_per_row = params;
    else {
      PESTI_CUDA_TRY(cudaMemcpyAsync(&uni, params, sizeof(uni), cudaMemcpyDeviceToHost, st), "params copy");
      PESTI_CUDA_TRY(cudaStreamSynchronize(st), "params sync");
      sorted_bufs = needs_sorted_buffers(&uni, 1);
    }
  } else if (params_per_row) {
    sorted_bufs = needs_sorted_buffers(params, B);
    params_bytes = align_up((size_t)B * sizeof(pesti_sampling_params));
  } else {
    uni = params[0];
    sorted_bufs = needs_sorted_buffers(&uni, 1);
  }
  const Plan p = make_plan(dev.num_sms, dtype, B, V, sorted_bufs);
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
