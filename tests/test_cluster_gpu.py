"""The cluster pass (one thread-block cluster per row) against the oracle and
against the four-kernel pipeline, through the C ABI.

Batches of at most 32 rows that are all greedy or top-k <= 256, and batches
with bf16 top-p rows, take the cluster pass by default;
pesti_testing_set_cluster(-1) sends every batch through the four-kernel
pipeline instead, and 1..16 sends every batch the cluster pass can take
through it with that cluster size.  Every result must be bit-identical to the oracle with exp correctly
rounded (tokens, kept lists, kept probabilities), whatever the cluster size,
including the rows the cluster pass hands to the row kernel (NaN and infinite
rows, too many tied candidates).
"""
import numpy as np
import pytest

import oracle as O
import synth
from test_gpu_parity import KW, check_exact, run_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture
def cluster_mode():
    import pesti_sampler as ps
    yield ps.set_cluster_mode
    ps.set_cluster_mode(0)


@pytest.mark.parametrize("w,B", [(1, 64), (2, 16), (2, 64), (5, 4)])
@pytest.mark.parametrize("mode", [0, 1, 2, 4, 8, 16])
def test_cluster_sizes_match_the_oracle(sampler, cluster_mode, w, B, mode):
    """Workload rows (workload 5's rows cut to 131072 columns) under every
    cluster size: bit for bit against the oracle."""
    spec = synth.WORKLOADS[w]
    x = synth.make_logits(w, B=B)
    if x.shape[1] > 131072:
        x = np.ascontiguousarray(x[:, :131072])
    params = synth.params_for(w, B, x.shape[1])
    u = synth.make_u(w, B)
    cluster_mode(mode)
    got = run_gpu(sampler, x, params, u, bf16=spec["dtype"] == "bf16")
    check_exact(x, params, u, got, f"workload{w} cluster mode {mode}")


def test_cluster_pass_equals_the_pipeline(sampler, cluster_mode):
    """The same batches through both paths: identical bits."""
    for w, B in ((1, 100), (2, 32)):
        x = synth.make_logits(w, B=B)
        params = synth.params_for(w, B, x.shape[1])
        u = synth.make_u(w, B)
        cluster_mode(-1)
        want = run_gpu(sampler, x, params, u)
        cluster_mode(8)  # the cluster pass whatever the batch size
        got = run_gpu(sampler, x, params, u)
        for g, w_ in zip(got, want):
            assert np.array_equal(np.asarray(g).view(np.uint8), np.asarray(w_).view(np.uint8))


def _single_config_cases():
    """Rows that all share one fast-path config, so that the batch takes the
    cluster pass; the rows cover what the pass hands on to the row kernel."""
    rng = np.random.default_rng(21)
    cases = []
    cases.append(("tiny-V", np.array([[0.1, 0.9, 0.3, 0.7]], np.float32), (1.0, 0.0, 2)))
    cases.append(("V1", np.array([[3.0]], np.float32), (1.0, 0.9, 5)))
    x = (rng.standard_normal((4, 997)) * 3).astype(np.float32)
    x[0, 5] = np.nan
    x[1, 7] = np.inf
    x[2, :] = -np.inf
    cases.append(("nan-inf-rows", x, (0.9, 0.0, 10)))
    x = np.zeros((3, 3000), np.float32)
    x[1, 17] = 1.0
    cases.append(("constant", x, (1.0, 0.0, 7)))
    x = np.round(rng.standard_normal((6, 4096)) * 2).astype(np.float32)
    cases.append(("ties", x, (1.0, 0.0, 10)))
    x = (rng.standard_normal((6, 20001)) * 40).astype(np.float32)
    cases.append(("wide", x, (0.1, 0.0, 50)))
    x = (rng.standard_normal((5, 50001)) * 3).astype(np.float32)
    cases.append(("odd-V", x, (0.9, 0.0, 256)))
    x = (rng.standard_normal((3, 131072)) * 2).astype(np.float32)
    cases.append(("max-V", x, (0.8, 0.0, 64)))
    x = (rng.standard_normal((4, 3000)) * 2).astype(np.float32)
    cases.append(("T<0 and k=1", x, (-1.0, 0.0, 1)))
    return cases


@pytest.mark.parametrize("case", _single_config_cases(), ids=lambda c: c[0])
@pytest.mark.parametrize("mode", [0, 2, 16])
def test_cluster_edge_rows(sampler, cluster_mode, case, mode):
    name, x, cfg = case
    B = x.shape[0]
    params = [cfg] * B
    cluster_mode(mode)
    for u in (np.zeros(B, np.float32), np.full(B, 0.5, np.float32), np.full(B, np.float32(0.99999994))):
        check_exact(x, params, u, run_gpu(sampler, x, params, u), f"{name} mode {mode}")


@pytest.mark.parametrize("mode", [0, 4])
def test_cluster_greedy_rows(sampler, cluster_mode, mode):
    """Greedy rows (argmax, both tie rules) with duplicate maxima, -inf rows
    and NaN rows (handed to the row kernel for the last-index rule)."""
    import torch
    rng = np.random.default_rng(3)
    x = rng.standard_normal((8, 32768)).astype(np.float32)
    x[1, [100, 30000]] = 50.0
    x[2, :] = -np.inf
    x[3, 9] = np.nan
    x[4, [5, 20000, 32767]] = 9.0
    x[5, :] = 1.5
    d = torch.from_numpy(x).cuda()
    cluster_mode(mode)
    last = sampler.argmax_batch(d).cpu().numpy()
    first = sampler.argmax_batch(d, first=True).cpu().numpy()
    assert list(last) == [O.argmax(r) for r in x]
    assert list(first) == [O.argmax_first(r) for r in x]
    params = [(0.0, 0.0, 0)] * 8
    u = np.full(8, 0.5, np.float32)
    check_exact(x, params, u, run_gpu(sampler, x, params, u), f"greedy mode {mode}")


@pytest.mark.parametrize("ld_extra", [0, 1])
def test_cluster_half_precision_and_unaligned(sampler, cluster_mode, ld_extra):
    """bf16 and f16 rows, and rows whose leading dimension breaks the 16-byte
    alignment (scalar loads)."""
    import torch
    import pesti_sampler as ps
    cluster_mode(0)
    x = synth.make_logits(2, B=8)[:, :60000]
    xb = synth.bf16_bits_to_f32(synth.f32_to_bf16_bits(x))
    params = [(0.7, 0.0, 50)] * 8
    u = synth.make_u(2, 8)
    ld = 60000 + ld_extra if ld_extra else None
    check_exact(xb, params, u, run_gpu(sampler, xb, params, u, bf16=True, ld=ld), "bf16")
    check_exact(x, params, u, run_gpu(sampler, x, params, u, ld=ld), "f32")
    x16 = x.astype(np.float16)
    host = torch.from_numpy(x16)
    if ld_extra:
        big = torch.zeros((8, 60000 + ld_extra), dtype=torch.float16)
        big[:, :60000] = host
        dev = big.cuda()[:, :60000]
    else:
        dev = host.cuda()
    cfgs = [ps.SamplingConfig(*p) for p in params]
    tok, kp, ki, kc = sampler.sample_batch(dev, cfgs, torch.from_numpy(u).cuda(), kept_width=KW)
    got = (tok.cpu().numpy().view(np.uint32), kp.cpu().numpy(), ki.cpu().numpy().view(np.uint32), kc.cpu().numpy())
    check_exact(x16.astype(np.float32), params, u, got, "f16")


def test_cluster_single_rows_from_the_host(sampler, cluster_mode):
    """The B=1 host API (the latency path) on workload 1 rows."""
    import pesti_sampler as ps
    cluster_mode(0)
    x = synth.make_logits(1, B=32)
    u = synth.make_u(1, 32)
    for b in range(32):
        t = sampler.sample_with_u(x[b], ps.SamplingConfig(0.8, 0.95, 40), float(u[b]))
        assert t == O.sample(x[b], 0.8, 0.95, 40, float(u[b]), O.EXP_CR)


def _nucleus_cases():
    """bf16 rows with top-p (the cluster pass folds S, the row kernel takes the
    sorted folds by distinct values), including what that path hands on to
    the generic sorted path."""
    rng = np.random.default_rng(33)
    bf = lambda a: synth.bf16_bits_to_f32(synth.f32_to_bf16_bits(np.asarray(a, np.float32)))
    cases = []
    x = synth.make_logits(3, B=6)
    cases.append(("workload3", x, [(1.0, 0.95, 0)] * 6))
    x = bf(rng.standard_normal((4, 20000)) * 2)
    cases.append(("top-p 1.0 and 1e-6", x, [(0.9, 1.0, 0), (1.1, 1e-6, 0), (0.7, 0.5, 0), (1.0, 0.999, 0)]))
    x = bf(np.zeros((2, 5000)))
    x[1, ::7] = 1.0
    cases.append(("constant and two-valued", x, [(1.0, 0.9, 0), (1.0, 0.3, 0)]))
    x = bf(rng.standard_normal((3, 9000)) * 1e-6)  # magnitudes far below the top binade
    x[0, 5] = 3.0
    cases.append(("tiny magnitudes", x, [(1.0, 0.9, 0), (0.5, 0.99, 0), (2.0, 0.2, 0)]))
    x = bf(-np.abs(rng.standard_normal((2, 7000))) * 3 - 1)  # only negative logits
    cases.append(("negative", x, [(1.0, 0.9, 0), (0.8, 0.7, 0)]))
    x = bf(np.round(rng.standard_normal((3, 30000)) * 4) / 4)  # few distinct values, big groups
    cases.append(("few values", x, [(1.0, 0.95, 0), (0.6, 0.8, 0), (1.3, 0.1, 0)]))
    x = bf(rng.standard_normal((4, 40000)) * 2)
    cases.append(("mixed kinds", x, [(1.0, 0.9, 0), (0.7, 0.0, 50), (0.0, 0.0, 0), (1.0, 0.95, 0)]))
    return cases


@pytest.mark.parametrize("case", _nucleus_cases(), ids=lambda c: c[0])
@pytest.mark.parametrize("kw", [KW, 2000])
def test_cluster_nucleus_rows(sampler, cluster_mode, case, kw):
    """bf16 top-p rows: tokens, kept lists (their first kw entries) and kept
    counts bit for bit against the oracle, and equal to the four-kernel
    pipeline's."""
    name, x, params = case
    B = x.shape[0]
    cluster_mode(0)
    for u in (np.zeros(B, np.float32), np.full(B, 0.5, np.float32), np.full(B, np.float32(0.99999994)),
              synth.make_u(3, B)):
        got = run_gpu(sampler, x, params, u, bf16=True, kept_width=kw)
        want = O.sample_batch(x, params, u, O.EXP_CR, kept_width=kw)
        tok, kp, ki, kc = got
        assert np.array_equal(tok, want["tokens"]), (name, tok, want["tokens"])
        assert np.array_equal(kc, want["kept_count"]), name
        assert np.array_equal(ki, want["kept_idx"]), name
        assert np.array_equal(kp.view(np.uint32), want["kept_p"].view(np.uint32)), name
    cluster_mode(-1)
    pipe = run_gpu(sampler, x, params, u, bf16=True, kept_width=kw)
    for g, w_ in zip(got, pipe):
        assert np.array_equal(np.asarray(g).view(np.uint8), np.asarray(w_).view(np.uint8))
