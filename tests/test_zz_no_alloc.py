"""pesti_sample_batch_noalloc against pesti_sample_batch, through the C ABI.

The no-allocation entry point runs the same kernels in one static scratch array
that every call shares.  Consecutive calls with different batches (sizes,
dtypes, parameter forms) must each give exactly what the allocating entry point
gives -- tokens, kept lists and kept probabilities bit for bit -- so nothing a
call leaves in the array changes the next call's result.  A batch larger than
the array is refused with an error and leaves the outputs untouched.
"""
import ctypes

import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu

KW = 64


def _device_batch(x_f32, bf16):
    import torch
    if bf16:
        bits = synth.f32_to_bf16_bits(x_f32)
        return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(np.ascontiguousarray(x_f32)).cuda()


def _batches():
    """Three consecutive calls: per-row host params over every filter kind,
    one uniform top-k config, and bf16 rows with top-p."""
    import pesti_sampler as ps
    x1 = synth.make_logits(2, B=8)  # [8, 128256] f32
    c1 = [ps.SamplingConfig(0.7, 0.9, 50), ps.SamplingConfig(1.0, 0.95, 0), ps.SamplingConfig(0.0, 0.0, 0),
          ps.SamplingConfig(1.0, 0.0, 0), ps.SamplingConfig(0.8, 0.0, 2000), ps.SamplingConfig(0.7, 0.5, 0),
          ps.SamplingConfig(1.3, 0.0, 1), ps.SamplingConfig(0.9, 0.0, 64)]
    x2 = synth.make_logits(1, B=5)  # [5, 32000] f32
    c2 = ps.SamplingConfig(0.8, 0.0, 40)
    x3 = synth.make_logits(3, B=6)  # [6, 152064] as bf16
    c3 = [ps.SamplingConfig(1.0, 0.95, 0)] * 3 + [ps.SamplingConfig(0.7, 0.0, 50)] * 3
    rng = np.random.default_rng(17)
    return [(x1, c1, False, rng.random(8).astype(np.float32)),
            (x2, c2, False, rng.random(5).astype(np.float32)),
            (x3, c3, True, rng.random(6).astype(np.float32))]


def _outputs(B):
    import torch
    return (torch.full((B,), -7, dtype=torch.int32, device="cuda"),
            torch.empty(B, KW, dtype=torch.float32, device="cuda"),
            torch.empty(B, KW, dtype=torch.int32, device="cuda"),
            torch.empty(B, dtype=torch.int64, device="cuda"))


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls(sampler):
    import torch
    import pesti_sampler as ps
    batches = _batches()
    dev = [(_device_batch(x, bf16), cfg, torch.from_numpy(u).cuda()) for (x, cfg, bf16, u) in batches]
    # the no-allocation calls back to back on one stream, then the allocating ones
    got = []
    for logits, cfg, u in dev:
        out, kp, ki, kc = _outputs(logits.shape[0])
        ps.sample_batch_noalloc(logits, cfg, u, out, kept=(kp, ki, kc))
        got.append((out, kp, ki, kc))
    want = [sampler.sample_batch(logits, cfg, u, kept_width=KW) for logits, cfg, u in dev]
    torch.cuda.synchronize()
    for n, (g, w) in enumerate(zip(got, want)):
        g = [t.cpu().numpy() for t in g]
        w = [t.cpu().numpy() for t in w]
        assert np.array_equal(g[0], w[0]), f"call {n}: tokens {g[0]} != {w[0]}"
        assert np.array_equal(g[3], w[3]), f"call {n}: kept counts differ"
        assert np.array_equal(g[2], w[2]), f"call {n}: kept indices differ"
        assert np.array_equal(g[1].view(np.uint32), w[1].view(np.uint32)), f"call {n}: kept probabilities differ"
    # the greedy row of the first batch is the argmax of its row
    assert int(got[0][0][2]) == int(np.argmax(batches[0][0][2]))


def test_noalloc_refuses_a_batch_larger_than_its_scratch():
    import torch
    import pesti_sampler as ps
    lib = ps.load_library()
    B, V = 64, 128256  # top-p rows need about 36 bytes per logit: ~296 MB > 64 MiB
    logits = torch.zeros(B, V, dtype=torch.float32, device="cuda")
    u = torch.full((B,), 0.5, dtype=torch.float32, device="cuda")
    out = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    p = ps.SamplingConfig(1.0, 0.9, 0).to_params(True)
    rc = lib.pesti_sample_batch_noalloc(logits.data_ptr(), ps.PESTI_F32, B, V, V, ctypes.byref(p), 0, 0,
                                        u.data_ptr(), out.data_ptr(), None, None, 0, None,
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == ps.PESTI_E_INVALID_ARG
    msg = lib.pesti_last_error().decode()
    assert "PESTI_NOALLOC_SCRATCH_BYTES" in msg and str(ps.NOALLOC_SCRATCH_BYTES) in msg, msg
    torch.cuda.synchronize()
    assert bool((out == -7).all())


def test_noalloc_page_locked_params(sampler):
    """Per-row params in page-locked host memory: the copy into the scratch
    array runs when the stream reaches it, so the caller rewrites the params
    for the next call only after synchronizing.  Two calls from the same
    page-locked array, each with its own configs, give the allocating entry
    point's results bit for bit."""
    import torch
    import pesti_sampler as ps
    lib = ps.load_library()
    B = 8
    x = torch.from_numpy(synth.make_logits(2, B=B)).cuda()
    u = torch.from_numpy(synth.make_u(2, B)).cuda()
    sets = [[ps.SamplingConfig(0.7, 0.9, 50)] * 4 + [ps.SamplingConfig(1.0, 0.0, 5)] * 4,
            [ps.SamplingConfig(0.0, 0.0, 0), ps.SamplingConfig(0.9, 0.0, 64)] * 4]
    page_locked = torch.empty(B * ctypes.sizeof(ps._Params), dtype=torch.uint8).pin_memory()
    arr = (ps._Params * B).from_address(page_locked.data_ptr())
    st = torch.cuda.current_stream().cuda_stream
    for cfgs in sets:
        for i, c in enumerate(cfgs):
            arr[i] = c.to_params(True)
        out, kp, ki, kc = _outputs(B)
        rc = lib.pesti_sample_batch_noalloc(x.data_ptr(), ps.PESTI_F32, B, x.shape[1], x.shape[1], arr, 1, 0,
                                            u.data_ptr(), out.data_ptr(), kp.data_ptr(), ki.data_ptr(), KW,
                                            kc.data_ptr(), st)
        assert rc == ps.PESTI_OK, lib.pesti_last_error().decode()
        torch.cuda.synchronize()  # the stream has passed the call: the params may change now
        want = [t.cpu().numpy() for t in sampler.sample_batch(x, cfgs, u, kept_width=KW)]
        got = [t.cpu().numpy() for t in (out, kp, ki, kc)]
        for g, w_ in zip(got, want):
            assert np.array_equal(g.view(np.uint8), w_.view(np.uint8))
