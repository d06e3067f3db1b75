"""Vocabulary-sharded sampling on the GPU, through the C ABI.

The sharded call splits every row into equal contiguous column ranges and
samples without moving logits (pesti_shard.cuh).  Its results must be those of
pesti_sample_batch on the whole rows, bit for bit: tokens, kept lists and kept
probabilities.  On one GPU the shards run one after another
(pesti_sample_batch_sharded_emulated); on two or more GPUs one process per GPU
runs pesti_sample_batch_sharded over NCCL.
"""
import os
import socket

import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KW = 64


def _dev(x, bf16=False):
    import torch
    if bf16:
        return torch.from_numpy(synth.f32_to_bf16_bits(x).view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _same(a, b, what):
    a = [t.cpu().numpy() for t in a]
    b = [t.cpu().numpy() for t in b]
    assert np.array_equal(a[0], b[0]), f"{what}: tokens differ at rows {np.nonzero(a[0] != b[0])[0][:8]}"
    assert np.array_equal(a[3], b[3]), f"{what}: kept counts differ"
    assert np.array_equal(a[2], b[2]), f"{what}: kept indices differ"
    assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32)), f"{what}: kept probabilities differ"


def test_emulated_shards_of_workload5_rows_match_whole_rows(sampler):
    import torch
    import oracle as O
    import pesti_sampler as ps
    B = 32
    x = synth.make_logits(5, B=B)  # [32, 256000] f32, T0.9 k64 p0.92
    u = synth.make_u(5, B)
    cfg = ps.SamplingConfig(0.9, 0.92, 64)
    d, du = _dev(x), torch.from_numpy(u).cuda()
    whole = sampler.sample_batch(d, cfg, du, kept_width=KW)
    want = O.sample_batch(x, (0.9, 0.92, 64), u, O.EXP_CR, kept_width=KW)
    assert np.array_equal(whole[0].cpu().numpy().view(np.uint32), want["tokens"])
    for G in (2, 4, 8):
        got = sampler.sample_batch_sharded_emulated(d, cfg, du, G, kept_width=KW)
        torch.cuda.synchronize()
        _same(got, whole, f"{G} shards")
        # the rows settled without gathering (the gathered path is for rare rows)
        assert sampler.last_gathered_rows() <= B // 8, sampler.last_gathered_rows()


def test_emulated_shards_of_mixed_rows_match_whole_rows(sampler):
    """Greedy rows (both tie rules, duplicate maxima), top-k 1 and 64, and
    rows the sharded path hands to the gathered path: top-p, no filter,
    top_k = V and a NaN row; f32 and bf16."""
    import torch
    import pesti_sampler as ps
    B, V = 12, 3 * 4096
    x = synth.make_logits(4, B=B, V=V) * np.float32(2.0)
    x[1, [7, 9000]] = x[1].max() + 1.0          # duplicate maxima across two shards
    x[8, 5000] = np.nan
    cfgs = [ps.SamplingConfig(0.0, 0.0, 0), ps.SamplingConfig(0.0, 0.0, 0), ps.SamplingConfig(0.8, 0.0, 1),
            ps.SamplingConfig(0.9, 0.0, 64), ps.SamplingConfig(1.0, 0.9, 0), ps.SamplingConfig(0.7, 0.0, 0),
            ps.SamplingConfig(1.0, 0.0, V), ps.SamplingConfig(1.3, 0.0, 40), ps.SamplingConfig(0.9, 0.0, 50),
            ps.SamplingConfig(0.9, 0.0, 256), ps.SamplingConfig(0.5, 0.0, 2), ps.SamplingConfig(2.0, 0.0, 64)]
    u = np.random.default_rng(5).random(B).astype(np.float32)
    du = torch.from_numpy(u).cuda()
    for bf16 in (False, True):
        d = _dev(x, bf16)
        for first in (False, True):
            whole = sampler.sample_batch(d, cfgs, du, kept_width=KW, argmax_first=first)
            got = sampler.sample_batch_sharded_emulated(d, cfgs, du, 3, kept_width=KW, argmax_first=first)
            torch.cuda.synchronize()
            _same(got, whole, f"bf16={bf16} argmax_first={first}")
            assert sampler.last_gathered_rows() >= 4  # top-p, no filter, top_k = V, NaN


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, out):
    import sys
    for p in (os.path.join(ROOT, "llm-workspace_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist
    import pesti_sampler as ps
    import synth as S
    torch.cuda.set_device(rank)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        B = 64
        x = S.make_logits(5, B=B)
        u = S.make_u(5, B)
        Vs = x.shape[1] // world
        s = ps.Sampler(rank)
        comm = ps.Comm(rank)
        shard = torch.from_numpy(np.ascontiguousarray(x[:, rank * Vs:(rank + 1) * Vs])).cuda()
        du = torch.from_numpy(u).cuda()
        cfg = ps.SamplingConfig(0.9, 0.92, 64)
        got = s.sample_batch_sharded(comm, shard, cfg, du, kept_width=KW)
        torch.cuda.synchronize()
        res = [t.cpu().numpy() for t in got]
        whole = None
        if rank == 0:
            w = s.sample_batch(torch.from_numpy(x).cuda(), cfg, du, kept_width=KW)
            whole = [t.cpu().numpy() for t in w]
        out.put((rank, res, whole, s.last_gathered_rows()))
        dist.barrier()
        comm.close()
        s.close()
    finally:
        dist.destroy_process_group()


def test_nccl_shards_match_whole_rows():
    import torch
    import torch.multiprocessing as mp
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        rank, res, whole, ng = q.get(timeout=300)
        got[rank] = (res, whole, ng)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    whole = got[0][1]
    for rank in range(world):
        res = got[rank][0]
        assert np.array_equal(res[0], whole[0]), f"rank {rank}: tokens differ"
        assert np.array_equal(res[2], whole[2]) and np.array_equal(res[3], whole[3])
        assert np.array_equal(res[1].view(np.uint32), whole[1].view(np.uint32))
        assert got[rank][2] <= 8
