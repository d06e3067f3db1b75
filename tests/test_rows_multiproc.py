"""Row split over ranks (bench.py --gpus N): two gloo ranks on CPU.

Each rank generates and samples its own contiguous row block with the oracle;
together the blocks must give exactly what one process gives for the whole
batch, and the timing reduction must return the maximum over ranks.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

W, ROWS_PER_RANK, WORLD = 1, 4, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, out):
    import sys
    for p in (os.path.join(ROOT, "llm-workspace_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    import torch.distributed as dist
    import oracle as O
    import synth
    from rows import max_over_ranks, rank_rows
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD)
    try:
        rows = rank_rows(rank, WORLD, ROWS_PER_RANK)
        x = synth.make_logits(W, rows=rows)
        u = synth.make_u(W, WORLD * ROWS_PER_RANK)[rows.start:rows.stop]
        params = synth.params_for(W, WORLD * ROWS_PER_RANK, x.shape[1])[rows.start:rows.stop]
        tok = O.sample_batch(x, params, u, O.EXP_CR)["tokens"]
        gathered = [None] * WORLD
        dist.all_gather_object(gathered, (rows.start, tok.tolist()))
        mx = max_over_ranks(rank + 1.5)
        if rank == 0:
            out.put((gathered, mx))
    finally:
        dist.destroy_process_group()


def test_row_blocks_over_two_gloo_ranks_match_one_process():
    import oracle as O
    import synth
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    gathered, mx = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert mx == WORLD + 0.5
    B = WORLD * ROWS_PER_RANK
    x = synth.make_logits(W, B=B)
    want = O.sample_batch(x, synth.params_for(W, B, x.shape[1]), synth.make_u(W, B), O.EXP_CR)["tokens"]
    got = np.zeros(B, np.uint32)
    for start, toks in gathered:
        got[start:start + ROWS_PER_RANK] = toks
    assert np.array_equal(got, want)


def test_rank_rows_partition():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "llm-workspace_b200"))
    from rows import rank_rows
    blocks = [rank_rows(r, 4, 64) for r in range(4)]
    assert [b.start for b in blocks] == [0, 64, 128, 192] and all(len(b) == 64 for b in blocks)
    with pytest.raises(ValueError):
        rank_rows(4, 4, 64)
