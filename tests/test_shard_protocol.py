"""Vocabulary-sharded sampling (workload 5's path), its protocol on CPU ranks.

Two and four gloo ranks each hold one contiguous column range of the same
rows and run the protocol of the sharded path (oracle/sharded.py, the CPU
restatement of what the kernels compute) with torch.distributed all-gathers
between its phases.  Every rank must end with the softmax sum, token and kept
list of the whole-row oracle (sampling.rs:39-134, exp correctly rounded),
bit for bit: the chained shard tables reproduce the sequential fold exactly.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
W5 = 5
ROWS = 4
K, T, TOP_P = 64, 0.9, 0.92


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import sys
    for p in (os.path.join(ROOT, "llm-workspace_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    import torch.distributed as dist
    import sharded as P
    import synth
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        x = synth.make_logits(W5, B=ROWS)
        u = synth.make_u(W5, ROWS)
        V = x.shape[1]
        Vs = V // world
        cols = slice(rank * Vs, (rank + 1) * Vs)
        results = []
        for b in range(ROWS):
            xs = np.ascontiguousarray(x[b, cols])
            sums = [None] * world
            dist.all_gather_object(sums, P.summary(xs, T))
            recs = [None] * world
            dist.all_gather_object(recs, P.record(xs, rank * Vs, T, sums, rank, K + 8))
            gmx = max(mr for mr, _ in sums)
            tabs = [None] * world
            dist.all_gather_object(tabs, P.table(xs, T, gmx, [r[0] for r in recs], rank))
            res = P.finish(tabs, recs, K, float(u[b]))
            results.append(None if res is None else (P.f32_bits(res[0]), res[1],
                                                     [(P.f32_bits(p), c) for p, c in res[2]]))
        out.put((rank, results))
    finally:
        dist.destroy_process_group()


def _whole_rows():
    import oracle as O
    import synth
    x = synth.make_logits(W5, B=ROWS)
    u = synth.make_u(W5, ROWS)
    want = []
    for b in range(ROWS):
        m = np.float32(np.float32(x[b].max()) / np.float32(T))
        S = O.fold(O.softmax_terms(x[b], T, m))
        tok, kp, ki, kc, _ = O.sample(x[b], T, TOP_P, K, float(u[b]), O.EXP_CR, kept_width=K)
        want.append((int(np.float32(S).view(np.uint32)), tok, list(zip(kp.view(np.uint32).tolist(), ki.tolist()))))
    return want


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_protocol_on_gloo_ranks_matches_whole_rows(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = _whole_rows()
    for rank in range(world):
        for b in range(ROWS):
            res = got[rank][b]
            assert res is not None, f"rank {rank} row {b}: protocol could not settle the row"
            S_bits, tok, kept = res
            assert S_bits == want[b][0], f"rank {rank} row {b}: softmax sum differs"
            assert tok == want[b][1], f"rank {rank} row {b}: token {tok} != {want[b][1]}"
            assert kept == want[b][2], f"rank {rank} row {b}: kept list differs"
