"""Benchmark of the B200 token sampler (one JSON line on stdout, rank 0).

Workload (default): the batched Llama-3-vocab case -- logits [64, 128256] f32,
N(0,1)*3 plus a Zipf(1.1) rank bias, temperature 0.7, top-k 50, top-p 0.9,
per-row draws from PCG32 seed 1.  A step samples one token for every row of
one batch already resident in HBM.  Under torchrun (N > 1) the configured
batch is split into N contiguous row blocks, one per rank, with no collective
on the data path (strong scaling: the total work is fixed).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload 1..5]

--workload 5 under torchrun (N > 1) runs the vocabulary-sharded path instead:
the [1024, 256000] f32 batch is split into N contiguous column ranges, one
per rank (strong scaling), and every rank receives all 1024 tokens
(pesti_sample_batch_sharded; three NCCL all-gathers of per-row records, no
logits moved).

Keys beyond the base contract:
  roofline      the whole step: logit bytes per step / step time against the
                measured HBM copy bandwidth; `kernels` gives each timed
                interval's own figure (profiled pass, CUDA events on the
                launching stream); `traffic` is the step's DRAM bytes from an
                ncu capture of the same loop (warm L2, see TRAFFIC_PER_STEP)
  parity        the batch's results against the oracle: rows bit-exact with
                exp correctly rounded, and against the platform-expf oracle
                the token mismatch rate outside the 1e-6 boundary band, the
                largest relative probability error and the share of top-k
                rows whose index sets are identical
  b1_latency_us p50/p99 wall time of one B=1 row (workload 1 shape, [1,32000]
                f32, device-resident), launch and sync included
  cpu_baseline  the reference algorithm (C++ restatement of sampling.rs) on the
                host cores, on a bounded sample of the same workload
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (os.path.join(ROOT, "llm-workspace_b200"), os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

METRIC = "sampled rows/s (B=64, V=128256 f32, T0.7 k50 p0.9)"


def metric_for(w: int) -> str:
    """The metric line of workload w (workload 2 is the headline)."""
    import synth
    if w == 2:
        return METRIC
    spec = synth.WORKLOADS[w]
    return f"sampled rows/s ({spec['name']})"


def params_text(w: int) -> str:
    import synth
    spec = synth.WORKLOADS[w]
    ps_ = synth.params_for(w, spec["B"], spec["V"])
    if len(set(ps_)) == 1:
        t, p, k = ps_[0]
        note = " (top-p unused since top_k > 0, sampling.rs:66)" if k > 0 and p > 0 else ""
        return f"T{t} top_k{k} top_p{p}{note}"
    return "per-row mix (synth.ROW_CLASSES_4)"
UNIT = "rows/s"
L2_BYTES = 126 * 1024 * 1024

# DRAM bytes (read + write) of one step, summed over its kernels, from one
# ncu capture per workload of this loop with the caches left warm: one-pass
# metrics (dram__bytes_read.sum, dram__bytes_write.sum, gpu__time_duration.sum,
# --cache-control none) over `bench.py --workload N --kernels-only --steps 3 --warmup 3`.
TRAFFIC_PER_STEP = {
    1: 246_770_000,  # [1000 x 32000] f32: K0 142.4 MB, K1f 102.1 MB, K2 2.2 MB
    2: 40_580_000,   # [64 x 128256] f32: K0 37.6 MB, K1a 2.0 MB, K1b 0.7 MB, K2 0.3 MB
    3: 98_740_000,   # [256 x 152064] bf16: cluster pass 88.0 MB, nucleus rows 10.8 MB
}


def cluster_pass(V, params, bf16=False, mode=0):
    """The batch takes the cluster pass: every row greedy (T == 0), top-k
    <= 256 or (bf16) top-p, rows of at most 131072 columns (262144 for bf16),
    and either some bf16 top-p row, at most 32 rows, or the pass forced
    (mode > 0); mode -1 sends every batch through the pipeline."""
    if mode < 0 or not 1 <= V <= (262144 if bf16 else 131072):
        return False
    nuc = [bf16 and k == 0 and p > 0 for (t, p, k) in params]
    if not all(t == 0.0 or 1 <= k <= 256 or n for (t, p, k), n in zip(params, nuc)):
        return False
    return any(nuc) or len(params) <= 32 or mode > 0


def kernels_per_step(V, params, bf16=False, mode=0):
    """This library's launches in one step.  The cluster pass: the cluster
    kernel and the row kernel (whose blocks return at once unless the cluster
    left their row).  Otherwise: the HBM pass; the fused pass (rows beyond 128k
    columns, or of at most 64k in batches of 32 rows or more when every row is
    on the top-k fast path), plus the survivor pass when some row is off that
    path, else the survivor pass and the task-queue classification; the row
    kernel."""
    if cluster_pass(V, params, bf16, mode):
        return 2
    off_fast = any(not (1 <= k <= 256) or t <= 0 for (t, _, k) in params)
    fused = V > 131072 or (V <= 65536 and not off_fast and len(params) >= 32)
    if not fused:
        return 4
    return 4 if off_fast else 3


def b1_latency(s, ps, synth, dev, rows=1000, warm=64):
    """p50/p99 host wall time (us) of one B=1 pesti_sample_batch call on a
    device-resident [1, 32000] f32 row (T 0.8, top-k 40) followed by
    cudaStreamSynchronize, with the call's arguments prepared beforehand as a
    decode loop would hold them."""
    import ctypes
    import glob

    import torch
    x1 = torch.from_numpy(synth.make_logits(1, B=64)).to(dev)
    u1 = torch.from_numpy(synth.make_u(1, 64)).to(dev)
    o1 = torch.empty(1, dtype=torch.int32, device=dev)
    lib = ps.load_library()
    prm = (ps._Params * 1)(ps.SamplingConfig(0.8, 0.95, 40).to_params(True))
    st = torch.cuda.current_stream(dev).cuda_stream
    V = x1.shape[1]
    rowp = [x1[r:r + 1].data_ptr() for r in range(64)]
    up = [u1[r:r + 1].data_ptr() for r in range(64)]
    outp = o1.data_ptr()
    sync = None
    for path in glob.glob(os.path.join(os.path.dirname(torch.__file__), "..", "nvidia", "cuda_runtime", "lib",
                                       "libcudart.so*")):
        try:
            cudart = ctypes.CDLL(path)
            cudart.cudaStreamSynchronize.argtypes = [ctypes.c_void_p]
            sync = lambda: cudart.cudaStreamSynchronize(st)  # noqa: E731
            break
        except OSError:
            continue
    if sync is None:
        sync = torch.cuda.synchronize
    call = lib.pesti_sample_batch
    h = s._h
    ts = []
    for i in range(rows + warm):
        r = i % 64
        t0 = time.perf_counter()
        rc = call(h, rowp[r], ps.PESTI_F32, 1, V, V, prm, 0, 0, up[r], outp, None, None, 0, None, st)
        sync()
        t1 = time.perf_counter()
        if rc != 0:
            raise RuntimeError(lib.pesti_last_error().decode())
        if i >= warm:
            ts.append((t1 - t0) * 1e6)
    return {"p50": float(np.percentile(ts, 50)), "p99": float(np.percentile(ts, 99)), "rows": len(ts),
            "how": "pesti_sample_batch through ctypes on a device-resident [1, 32000] f32 row, then "
                   "cudaStreamSynchronize; host wall clock"}


def merge_parity(reps):
    """The parity figures of every rank's rows, as one batch."""
    reps = [r for r in reps if r]
    if not reps:
        return None
    rows = sum(r["rows"] for r in reps)
    topk_rows = sum(r["topk_rows"] for r in reps)
    topk_ok = sum((r["topk_sets_exact"] or 0.0) * r["topk_rows"] for r in reps)
    outside = sum(r["token_mismatches_outside_band"] for r in reps)
    return {
        "rows": rows,
        "rows_exact_cr_exp": sum(r["rows_exact"] for r in reps),
        "token_mismatch_rate": outside / max(rows, 1),
        "token_mismatches": sum(r["token_mismatches"] for r in reps),
        "rows_near_boundary": sum(r["rows_near_boundary"] for r in reps),
        "max_prob_rel_err": max(r["max_prob_rel_err"] for r in reps),
        "topk_sets_exact": (topk_ok / topk_rows) if topk_rows else None,
        "against": "oracle (C++ restatement of sampling.rs:39-134): bit-exact rows with exp correctly "
                   "rounded; the other figures against glibc expf, 1e-6 boundary band",
    }


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_baseline(x, params, u, budget_s=10.0, threads=0):
    """Reference algorithm (oracle, platform expf) on the host cores."""
    import oracle as O
    nthreads = threads or os.cpu_count() or 1
    B = x.shape[0]
    rows, t0 = 0, time.perf_counter()
    while True:
        O.sample_batch(x, params, u, O.EXP_PLATFORM, nthreads=nthreads)
        rows += B
        dt = time.perf_counter() - t0
        if dt >= budget_s:
            break
    return rows / dt, nthreads, rows


def run_reference(args):
    """`--impl reference`: the reference algorithm on the host cores (rank 0)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    import oracle as O
    import synth
    w = args.workload
    spec = synth.WORKLOADS[w]
    B, V = spec["B"], spec["V"]
    x = synth.make_logits(w)
    params = synth.params_for(w, B, V)
    u = synth.make_u(w)
    nthreads = os.cpu_count() or 1
    # calibrate: rows per step so that warmup + steps fit in ~90 s
    t0 = time.perf_counter()
    O.sample_batch(x[: min(B, nthreads)], params[: min(B, nthreads)], u[: min(B, nthreads)], O.EXP_PLATFORM,
                   nthreads=nthreads)
    per_row = (time.perf_counter() - t0) / min(B, nthreads) * nthreads  # one row on one core
    per_row_par = per_row / nthreads
    rows_per_step = max(1, min(B, int(90.0 / max(1, args.steps + args.warmup) / max(per_row_par, 1e-9))))
    for i in range(args.warmup):
        O.sample_batch(x[:rows_per_step], params[:rows_per_step], u[:rows_per_step], O.EXP_PLATFORM,
                       nthreads=nthreads)
    t0 = time.perf_counter()
    for i in range(args.steps):
        O.sample_batch(x[:rows_per_step], params[:rows_per_step], u[:rows_per_step], O.EXP_PLATFORM,
                       nthreads=nthreads)
    dt = time.perf_counter() - t0
    value = rows_per_step * args.steps / dt
    line = {
        "metric": metric_for(w), "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": spec["dtype"],
        "data": "synthetic",
        "config": {"workload": spec["name"], "B": B, "B_per_gpu": B, "V": V, "input_dtype": spec["dtype"],
                   "params": params_text(w), "l2": "not applicable (host memory)",
                   "parallelism": f"{nthreads} host threads, rows in parallel; {rows_per_step} of the {B} rows "
                                  "per step"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": nthreads, "kind": "port",
                         "sample": f"{rows_per_step} of the {B} rows per step, {args.steps} steps; "
                                   "C++ restatement of sampling.rs:39-134 with glibc expf (the Rust "
                                   "reference cannot be built here)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def run_vocab_sharded(args, rank, world, local, dev):
    """Workload 5 over `world` ranks, each holding one column range of every row."""
    import ctypes

    import torch
    import torch.distributed as dist

    import pesti_sampler as ps
    import synth
    from rows import max_over_ranks
    w = 5
    spec = synth.WORKLOADS[w]
    B, V = spec["B"], spec["V"]
    if V % world:
        raise SystemExit(f"V={V} is not a multiple of {world} ranks")
    Vs = V // world
    cols = range(rank * Vs, (rank + 1) * Vs)
    x = synth.make_logits(w, cols=cols)
    u = synth.make_u(w, B)
    T, P, K = synth.params_for(w, 1, V)[0]
    cfg = ps.SamplingConfig(T, P, K)
    host = torch.from_numpy(x)
    step_bytes = B * Vs * 4  # this rank's logits
    nbuf = max(2, math.ceil(2 * L2_BYTES / step_bytes))
    bufs = [host.to(dev) for _ in range(nbuf)]
    ud = torch.from_numpy(u).to(dev)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    s = ps.Sampler(local)
    comm = ps.Comm(local)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        s.sample_batch_sharded(comm, bufs[i % nbuf], cfg, ud, out=out)

    # correctness guard: every rank's tokens against the whole rows sampled on
    # rank 0's GPU, and rank 0's results (tokens and kept lists of all rows)
    # against the oracle
    KW = 64
    tok, kp, ki, kc = s.sample_batch_sharded(comm, bufs[0], cfg, ud, kept_width=KW)
    torch.cuda.synchronize()
    gathered_first = s.last_gathered_rows()
    gathered_why = s.last_gathered_reasons()
    mine = tok.cpu().numpy().view(np.uint32).copy()
    check = None
    parity = None
    if rank == 0:
        import oracle as O
        full = synth.make_logits(w)
        whole = torch.from_numpy(full).to(dev)
        ref = s.sample_batch(whole, cfg, ud)
        torch.cuda.synchronize()
        check = ref.cpu().numpy().view(np.uint32)
        del whole
        torch.cuda.empty_cache()
        parity = merge_parity([O.parity_report(full, (T, P, K), u, mine, kp.cpu().numpy(), ki.cpu().numpy(),
                                               kc.cpu().numpy(), KW)])
        del full
    all_tok = [None] * world
    dist.all_gather_object(all_tok, mine)
    exact = int(sum(int((t == check).sum()) for t in all_tok)) if rank == 0 else None

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        step(i)
    t_end.record(stream)
    torch.cuda.synchronize()
    elapsed_ms = t_start.elapsed_time(t_end)
    clk = clocks.stop()
    dist.barrier()
    elapsed_ms = max_over_ranks(elapsed_ms, dev)
    ms_per_step = elapsed_ms / args.steps
    value = B * args.steps / (elapsed_ms / 1e3)

    # the HBM pass over the shard, timed alone (profiled steps)
    lib = ps.load_library()
    lib.pesti_profile_enable.argtypes = [ctypes.c_void_p, ctypes.c_int]
    lib.pesti_profile_read.argtypes = [ctypes.c_void_p] + [ctypes.POINTER(ctypes.c_double)] * 3 + \
        [ctypes.POINTER(ctypes.c_int)]
    lib.pesti_profile_enable(s._h, 1)
    prof_steps = min(args.steps, 50)
    for i in range(prof_steps):
        step(i)
    torch.cuda.synchronize()
    t_max, t_mid, t_fin, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
    lib.pesti_profile_read(s._h, ctypes.byref(t_max), ctypes.byref(t_mid), ctypes.byref(t_fin), ctypes.byref(n))
    lib.pesti_profile_enable(s._h, 0)
    scan_ms = max_over_ranks(t_max.value / max(1, n.value), dev)
    mid_ms = max_over_ranks(t_mid.value / max(1, n.value), dev)
    fin_ms = max_over_ranks(t_fin.value / max(1, n.value), dev)
    peak, peak_kind = measured_peaks()
    achieved = step_bytes / (scan_ms / 1e3) / 1e9

    # end to end: each rank's shard from pinned host memory, all tokens back
    pinned = host.pin_memory()
    u_pinned = torch.from_numpy(u).pin_memory()
    dbuf = torch.empty_like(bufs[0])
    ubuf = torch.empty_like(ud)
    tok_host = torch.empty(B, dtype=torch.int32).pin_memory()
    e2e_steps = max(5, min(args.steps, 50))

    def e2e_step():
        dbuf.copy_(pinned, non_blocking=True)
        ubuf.copy_(u_pinned, non_blocking=True)
        s.sample_batch_sharded(comm, dbuf, cfg, ubuf, out=out)
        tok_host.copy_(out, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), dev)
    e2e_value = B * e2e_steps / (e2e_ms / 1e3)
    if rank == 0:
        line = {
            "metric": "sampled rows/s, vocabulary-sharded (B=1024, V=256000 f32, T0.9 k64 p0.92)",
            "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": spec["name"], "B": B, "V": V, "V_per_gpu": Vs,
                       "l2": f"rotating {nbuf} input buffers per rank ({nbuf * step_bytes / 2**20:.0f} MiB > 126 MiB L2)",
                       "parallelism": f"vocab shards, {world} GPU(s), 3 NCCL all-gathers of per-row records"},
            "roofline": {"bound": "hbm", "kernel": "slice_stats_kernel", "achieved": achieved, "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak, "traffic": None,
                         "bytes_per_launch": step_bytes},
            "phase_us": {"slice_stats": scan_ms * 1e3, "to_last_exchange": mid_ms * 1e3, "finish": fin_ms * 1e3},
            "step_hbm_gbs_per_gpu": step_bytes / (ms_per_step / 1e3) / 1e9,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": step_bytes + B * 4,
                    "d2h_bytes_per_step": B * 4},
            # shard_stats, shard_prologue, survivor, classify, row (record), table, finish
            "gpu_launches": 7 * args.steps,
            "clocks": clk,
            "cpu_baseline": None,
            "rows_equal_whole_row_sampler": exact, "rows_checked": B * world, "parity": parity,
            "gathered_rows_first_step": gathered_first, "gathered_reasons": gathered_why,
        }
        print(json.dumps(line))
    comm.close()
    s.close()
    dist.destroy_process_group()
    return 0


def run_chain(args, dev):
    """The llama.cpp backend's sampler chain (llm-runner/src/llama.rs:465-508)
    with one SamplingConfig preset over the workload's [B, V] logits and a
    256-token history per row; every row checked against the chain's CPU
    restatement before timing."""
    import torch

    import llama_chain as LC
    import pesti_sampler as ps
    import synth

    w = args.workload
    spec = synth.WORKLOADS[w]
    B, V = (args.rows or spec["B"]), spec["V"]
    bf16 = spec["dtype"] == "bf16"
    x = synth.make_logits(w, rows=range(B))
    u = synth.make_u(w, B)
    rng = np.random.default_rng(20240)
    hist = rng.integers(0, V, size=(B, 256)).astype(np.int32)
    p = ps.LlamaChainParams() if args.chain == "default" else getattr(ps.LlamaChainParams, args.chain)()
    if bf16:
        host = torch.from_numpy(synth.f32_to_bf16_bits(x).view(np.int16)).view(torch.bfloat16)
    else:
        host = torch.from_numpy(x)
    step_bytes = B * V * (2 if bf16 else 4)
    nbuf = max(2, math.ceil(2 * L2_BYTES / step_bytes))
    bufs = [host.to(dev) for _ in range(nbuf)]
    ud = torch.from_numpy(u).to(dev)
    hd = torch.from_numpy(hist).to(dev)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    kept = torch.empty(B, dtype=torch.int32, device=dev)
    s = ps.Sampler(dev.index or 0)
    stream = torch.cuda.current_stream(dev)

    parity = None
    if not args.kernels_only:
        s.llama_chain_batch(bufs[0], p, ud, history=hd, out=out, kept=kept)
        torch.cuda.synchronize()
        xw = bufs[0].float().cpu().numpy()
        ot, ok, om = LC.chain_batch(xw, p.as_dict(), hist, u)
        near = om < 1e-9
        tok, kp = out.cpu().numpy(), kept.cpu().numpy()
        agree = (ot == tok) & (ok == kp)
        parity = {"rows": B, "rows_agree": int(agree.sum()), "rows_near_boundary": int(near.sum()),
                  "rows_disagree_off_boundary": int((~agree & ~near).sum())}

    for i in range(args.warmup):
        s.llama_chain_batch(bufs[i % nbuf], p, ud, history=hd, out=out, kept=kept)
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index or 0)
    clocks.start()
    time.sleep(0.3)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        s.llama_chain_batch(bufs[i % nbuf], p, ud, history=hd, out=out, kept=kept)
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    # the logits are the algorithmic bytes of a step (read once); the
    # history and draws are a few KB
    peak, peak_kind = measured_peaks()
    gbs = step_bytes / (ms / 1e3) / 1e9
    line = {
        "metric": f"rows/s, llama.cpp sampler chain ({args.chain} preset)", "value": round(B / (ms / 1e3), 1),
        "unit": "rows/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "vs_baseline": None, "dtype": spec["dtype"], "data": "synthetic",
        "config": {"workload": f"[{B} x {V}] {spec['dtype']}", "chain": p.as_dict(), "history": 256,
                   "l2": f"{nbuf} rotating input buffers, {nbuf * step_bytes / 1e6:.0f} MB > L2"},
        "gpu_launches": args.steps, "parity": parity, "clocks": clk,
        "roofline": {"bound": "hbm", "kernel": "llama_chain_kernel", "achieved": round(gbs, 1), "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": round(gbs / peak, 4), "traffic": None},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", type=int, default=2)
    ap.add_argument("--rows", type=int, default=0,
                    help="rows per GPU instead of the workload's batch (small cases for profiler captures)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernels-only", action="store_true",
                    help="only the warm-up and timed steps (for profiler captures); prints ms_per_step")
    ap.add_argument("--chain", default="",
                    choices=["", "default", "greedy", "creative", "balanced", "precise"],
                    help="time the llama.cpp backend's sampler chain (pesti_llama_chain_batch) with that "
                         "SamplingConfig preset on the workload's shape, on one GPU")
    ap.add_argument("--cluster", type=int, default=0,
                    help="path of the batch: 0 the library's routing, -1 the four-kernel pipeline, "
                         "1..16 the cluster pass with that many CTAs per row (profiles of either path)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist

    import pesti_sampler as ps
    import synth
    from rows import max_over_ranks, rank_rows

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.chain:
        if world > 1:
            raise SystemExit("--chain runs on one GPU")
        return run_chain(args, dev)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        if args.workload == 5:
            return run_vocab_sharded(args, rank, world, local, dev)

    w = args.workload
    spec = synth.WORKLOADS[w]
    B_total, V = (args.rows or spec["B"]), spec["V"]
    if B_total % world:
        raise SystemExit(f"the batch of {B_total} rows does not split over {world} ranks")
    B = B_total // world  # this rank's contiguous row block of the configured batch
    rows = rank_rows(rank, world, B)
    x = synth.make_logits(w, rows=rows)
    params = synth.params_for(w, B_total, V)[rows.start:rows.stop]
    u = synth.make_u(w, B_total)[rows.start:rows.stop]
    bf16 = spec["dtype"] == "bf16"
    if bf16:
        host = torch.from_numpy(synth.f32_to_bf16_bits(x).view(np.int16)).view(torch.bfloat16)
    else:
        host = torch.from_numpy(x)
    esize = 2 if bf16 else 4
    step_bytes = B * V * esize
    nbuf = max(2, math.ceil(2 * L2_BYTES / step_bytes))
    bufs = [host.to(dev) for _ in range(nbuf)]
    ud = torch.from_numpy(u).to(dev)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    # one SamplingConfig when every row shares it (as the reference's API
    # takes it), else the per-row list converted once
    cfgs = (ps.SamplingConfig(*params[0]) if len(set(params)) == 1
            else ps.PreparedParams([ps.SamplingConfig(t, p, k) for (t, p, k) in params]))
    s = ps.Sampler(local)
    ps.set_cluster_mode(args.cluster)
    stream = torch.cuda.current_stream(dev)

    # the timed loop calls the C ABI entry point directly with its arguments
    # prepared once, as a decode loop holding its buffers would, so that the
    # host's per-call Python work does not starve the GPU between steps
    _, _, dt_, arr_, per_row_, _, _, _, _, st_ = ps._batch_args(bufs[0], cfgs, out, True, False, 0, None)
    ptrs_ = [bf.data_ptr() for bf in bufs]
    ld_ = bufs[0].stride(0)
    u_ptr_, out_ptr_ = ud.data_ptr(), out.data_ptr()
    call_ = s._lib.pesti_sample_batch
    h_ = s._h

    def step(i):
        rc = call_(h_, ptrs_[i % nbuf], dt_, B, V, ld_, arr_, per_row_, 0, u_ptr_, out_ptr_, None, None, 0, None, st_)
        if rc:
            ps._check(rc)

    def barrier():
        if world > 1:
            dist.barrier()

    # correctness guard on the benchmark's own input: every rank's rows
    # against the oracle (the parity figures of the drop-in contract)
    parity = None
    if not args.kernels_only:
        import oracle as O
        KW = 64
        tok, kp, ki, kc = s.sample_batch(bufs[0], cfgs, ud, kept_width=KW)
        torch.cuda.synchronize()
        rep = O.parity_report(x, params, u, tok.cpu().numpy(), kp.cpu().numpy(), ki.cpu().numpy(),
                              kc.cpu().numpy(), KW)
        reps = [rep]
        if world > 1:
            reps = [None] * world
            dist.all_gather_object(reps, rep)
        parity = merge_parity(reps)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if args.kernels_only:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for i in range(args.steps):
            step(i)
        t_end.record(stream)
        torch.cuda.synchronize()
        if rank == 0:
            print(json.dumps({"kernels_only": True, "workload": spec["name"], "steps": args.steps,
                              "ms_per_step": t_start.elapsed_time(t_end) / args.steps}))
        return 0
    clocks = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        step(i)
    t_end.record(stream)
    torch.cuda.synchronize()
    elapsed_ms = t_start.elapsed_time(t_end)
    # keep the clock sampler running across a longer loop if the timed region was short
    extra_until = time.perf_counter() + 0.6
    j = 0
    while time.perf_counter() < extra_until:
        step(j)
        j += 1
        if j % 64 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier()
    elapsed_ms = max_over_ranks(elapsed_ms, dev)
    ms_per_step = elapsed_ms / args.steps
    value = B_total * args.steps / (elapsed_ms / 1e3)

    # per-kernel device times (profiled pass, separate from the timed loop)
    lib = ps.load_library()
    import ctypes
    lib.pesti_profile_enable.argtypes = [ctypes.c_void_p, ctypes.c_int]
    lib.pesti_profile_read.argtypes = [ctypes.c_void_p] + [ctypes.POINTER(ctypes.c_double)] * 3 + \
        [ctypes.POINTER(ctypes.c_int)]
    lib.pesti_profile_enable(s._h, 1)
    prof_steps = min(args.steps, 1000)
    for i in range(prof_steps):
        step(i)
    torch.cuda.synchronize()
    t_max, t_surv, t_row, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
    lib.pesti_profile_read(s._h, ctypes.byref(t_max), ctypes.byref(t_surv), ctypes.byref(t_row), ctypes.byref(n))
    lib.pesti_profile_enable(s._h, 0)
    scan_ms = max_over_ranks(t_max.value / max(1, n.value), dev)
    surv_ms = max_over_ranks(t_surv.value / max(1, n.value), dev)
    row_ms = max_over_ranks(t_row.value / max(1, n.value), dev)
    peak, peak_kind = measured_peaks()
    achieved = step_bytes / (ms_per_step / 1e3) / 1e9

    def kern(ms):
        gbs = step_bytes / (ms / 1e3) / 1e9 if ms > 0 else None
        return {"us": ms * 1e3, "logit_gbs": gbs, "frac": gbs / peak if gbs else None}

    # end to end through the public API with host buffers
    pinned = host.pin_memory()
    u_pinned = torch.from_numpy(u).pin_memory()
    dbuf = torch.empty_like(bufs[0])
    ubuf = torch.empty_like(ud)
    tok_host = torch.empty(B, dtype=torch.int32).pin_memory()
    e2e_steps = max(10, min(args.steps, 200))

    def e2e_step():
        dbuf.copy_(pinned, non_blocking=True)
        ubuf.copy_(u_pinned, non_blocking=True)
        s.sample_batch(dbuf, cfgs, ubuf, out=out)
        tok_host.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    e2e_ms = max_over_ranks(e2e_ms, dev)
    e2e_value = B_total * e2e_steps / (e2e_ms / 1e3)

    # B = 1 latency (workload 1 shape, [1, 32000] f32 rows already on the
    # device): host wall clock of one pesti_sample_batch call through the C ABI
    # plus the stream synchronisation that waits for its token
    lat = None
    if rank == 0:
        lat = b1_latency(s, ps, synth, dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, nrows = cpu_baseline(x, params, u, budget_s=10.0)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{nrows} rows of this workload (the {B}-row batch repeated for ~10 s), all host "
                         "threads; C++ restatement of sampling.rs:39-134 with glibc expf"}

    if rank == 0:
        nk = kernels_per_step(V, params, bf16, args.cluster)
        line = {
            "metric": metric_for(w), "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": spec["dtype"], "data": "synthetic",
            "config": {"workload": spec["name"], "B": B_total, "B_per_gpu": B, "V": V, "input_dtype": spec["dtype"],
                       "params": params_text(w),
                       "l2": f"rotating {nbuf} input buffers ({nbuf * step_bytes / 2**20:.0f} MiB > 126 MiB L2)",
                       "parallelism": f"row blocks of {B} rows on each of {world} GPU(s), no collective",
                       "path": ("cluster pass" if cluster_pass(V, params, bf16, args.cluster) else "four-kernel pipeline")
                       + (f" (forced, --cluster {args.cluster})" if args.cluster else "")},
            "roofline": {"bound": "hbm", "kernel": f"whole step ({nk} launches)", "achieved": achieved,
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": (TRAFFIC_PER_STEP.get(w) if world == 1 and not args.rows and not args.cluster
                                     else None),
                         "bytes_per_launch": step_bytes,
                         "kernels": ({"row_cluster": kern(scan_ms), "row (rows the cluster pass left)": kern(row_ms)}
                                     if cluster_pass(V, params, bf16, args.cluster) else
                                     {"slice_stats": kern(scan_ms), "survivor+classify": kern(surv_ms),
                                      "row": kern(row_ms)})},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": step_bytes + B * 4,
                    "d2h_bytes_per_step": B * 4},
            "gpu_launches": nk * args.steps,
            "clocks": clk,
            "b1_latency_us": lat,
            "cpu_baseline": cpu,
            "parity": parity,
        }
        print(json.dumps(line))
    s.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
