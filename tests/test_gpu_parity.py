"""GPU parity: the CUDA sampler against the CPU oracle, through the C ABI.

Bar (from the drop-in contract):
  * with exp correctly rounded in the oracle, every output is bit-identical:
    token, kept-list length, kept indices and kept probabilities (bits);
  * against the oracle with the platform expf (what the Rust reference calls),
    top-k index sets are identical, probabilities agree within 1e-5 relative,
    and tokens differ on at most 1e-4 of the rows whose draw is not within
    1e-6 of a cumulative-probability boundary.
"""
import numpy as np
import pytest

import oracle as O
import synth

pytestmark = pytest.mark.gpu

KW = 64  # kept-list entries compared per row
PROB_RTOL = 1e-5
BAND = 1e-6


def run_gpu(sampler, x_f32, params, u, bf16=False, ld=None, kept_width=KW):
    import torch
    import pesti_sampler as ps
    B, V = x_f32.shape
    if bf16:
        bits = synth.f32_to_bf16_bits(x_f32)
        host = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)
    else:
        host = torch.from_numpy(np.ascontiguousarray(x_f32))
    if ld is not None and ld != V:
        big = torch.zeros((B, ld), dtype=host.dtype)
        big[:, :V] = host
        dev = big.cuda()[:, :V]
    else:
        dev = host.cuda()
    cfgs = [ps.SamplingConfig(temperature=t, top_p=p, top_k=k) for (t, p, k) in params]
    ud = torch.from_numpy(np.ascontiguousarray(u, dtype=np.float32)).cuda()
    tok, kp, ki, kc = sampler.sample_batch(dev, cfgs, ud, kept_width=kept_width)
    torch.cuda.synchronize()
    return (tok.cpu().numpy().view(np.uint32), kp.cpu().numpy(), ki.cpu().numpy().view(np.uint32),
            kc.cpu().numpy())


def check_exact(x, params, u, got, label):
    want = O.sample_batch(x, params, u, O.EXP_CR, kept_width=KW)
    tok, kp, ki, kc = got
    bad = np.nonzero(tok != want["tokens"])[0]
    assert bad.size == 0, f"{label}: token mismatch rows {bad[:10]} got {tok[bad[:5]]} want {want['tokens'][bad[:5]]}"
    assert np.array_equal(kc, want["kept_count"]), f"{label}: kept counts differ"
    assert np.array_equal(ki, want["kept_idx"]), f"{label}: kept indices differ"
    assert np.array_equal(kp.view(np.uint32), want["kept_p"].view(np.uint32)), f"{label}: kept probabilities differ"


def check_reference_tolerances(x, params, u, got, label):
    ref = O.sample_batch(x, params, u, O.EXP_PLATFORM, kept_width=KW)
    tok, kp, ki, kc = got
    B = len(tok)
    mism = tok != ref["tokens"]
    near = ref["boundary_dist"] <= BAND
    outside = int((mism & ~near).sum())
    # top-k sets (top_k > 0 rows that are not greedy)
    for b in range(B):
        t, p, k = params[b]
        if t != 0.0 and k > 0 and k <= KW:
            assert set(ki[b, :k].tolist()) == set(ref["kept_idx"][b, :k].tolist()), f"{label}: top-k set row {b}"
    valid = ref["kept_idx"] != 0xFFFFFFFF
    rp, gp = ref["kept_p"][valid].astype(np.float64), kp[valid].astype(np.float64)
    same_idx = ki[valid] == ref["kept_idx"][valid]
    rel = np.abs(gp[same_idx] - rp[same_idx]) / np.maximum(np.abs(rp[same_idx]), 1e-38)
    print(f"[{label}] rows={B} token mismatches={int(mism.sum())} (outside 1e-6 band: {outside}, "
          f"rows near a boundary: {int(near.sum())}) max rel prob err={rel.max() if rel.size else 0:.3g}")
    assert rel.size == 0 or rel.max() <= PROB_RTOL
    assert outside <= max(1e-4 * B, 0), f"{label}: {outside} token mismatches outside the boundary band"


@pytest.mark.parametrize("w,B", [(1, 64), (2, 16), (3, 8), (4, 200), (5, 8)])
def test_workloads_reduced_batch(sampler, w, B):
    spec = synth.WORKLOADS[w]
    V = spec["V"]
    x = synth.make_logits(w, B=B)
    params = synth.params_for(w, B, V)
    u = synth.make_u(w, B)
    got = run_gpu(sampler, x, params, u, bf16=spec["dtype"] == "bf16")
    check_exact(x, params, u, got, f"workload{w}")
    check_reference_tolerances(x, params, u, got, f"workload{w}")


_FULL = {}


def full_workload(w):
    """The whole configured batch of workload w (logits, params, draws),
    generated once per test session."""
    if w not in _FULL:
        spec = synth.WORKLOADS[w]
        x = synth.make_logits(w)
        _FULL[w] = (x, synth.params_for(w, spec["B"], spec["V"]), synth.make_u(w))
    return _FULL[w]


@pytest.mark.parametrize("w", [1, 2, 3, 4, 5])
def test_workloads_full_size(sampler, w):
    """Every row of every configured batch: bit for bit against the oracle
    with exp correctly rounded, and within the drop-in tolerances against the
    oracle with the platform expf (top-k sets identical, probabilities within
    1e-5 relative, at most 1e-4 token mismatches outside the 1e-6 band)."""
    spec = synth.WORKLOADS[w]
    x, params, u = full_workload(w)
    tok, kp, ki, kc = run_gpu(sampler, x, params, u, bf16=spec["dtype"] == "bf16")
    rep = O.parity_report(x, params, u, tok, kp, ki, kc, KW)
    print(f"[workload{w}-full] {rep}")
    assert rep["rows_exact"] == rep["rows"], f"workload {w}: {rep['rows'] - rep['rows_exact']} rows differ"
    assert rep["token_mismatch_rate"] <= 1e-4
    assert rep["max_prob_rel_err"] <= PROB_RTOL
    assert rep["topk_sets_exact"] in (None, 1.0)


@pytest.mark.parametrize("shards", [2, 4, 8])
def test_workload5_full_size_emulated_shards(sampler, shards):
    """All 1024 rows of workload 5 as 2, 4 and 8 vocabulary shards (one GPU
    emulating the ranks): tokens, kept lists and kept probabilities equal the
    whole-row sampler's bit for bit (which the full-size test above holds to
    the oracle)."""
    import torch
    import pesti_sampler as ps
    x, params, u = full_workload(5)
    d = torch.from_numpy(x).cuda()
    ud = torch.from_numpy(u).cuda()
    cfg = ps.SamplingConfig(*params[0])
    whole = [t.cpu().numpy() for t in sampler.sample_batch(d, cfg, ud, kept_width=KW)]
    got = [t.cpu().numpy() for t in sampler.sample_batch_sharded_emulated(d, cfg, ud, shards, kept_width=KW)]
    for g, w_ in zip(got, whole):
        assert np.array_equal(g.view(np.uint8), w_.view(np.uint8))
    print(f"[workload5 {shards} shards] rows taking the gathered path: {sampler.last_gathered_rows()}")


def _edge_cases():
    rng = np.random.default_rng(5)
    cases = []
    cases.append(("tiny-V", np.array([[0.1, 0.9, 0.3, 0.7]], np.float32), [(1.0, 0.0, 2)]))
    cases.append(("V1", np.array([[3.0]], np.float32), [(1.0, 0.9, 0)]))
    cases.append(("all-neg-inf", np.full((1, 37), -np.inf, np.float32), [(1.0, 0.9, 0)]))
    x = rng.standard_normal((3, 97)).astype(np.float32)
    x[0, 5] = np.nan
    x[1, 7] = np.inf
    cases.append(("nan-inf", x, [(1.0, 0.0, 5), (0.8, 0.95, 0), (1.0, 0.0, 0)]))
    x = rng.standard_normal((4, 1000)).astype(np.float32)
    cases.append(("temperatures", x, [(-1.0, 0.9, 0), (float("nan"), 0.0, 3), (1e-30, 0.0, 0), (1e30, 0.5, 0)]))
    x = (rng.standard_normal((6, 5000)) * 40).astype(np.float32)  # large dynamic range: pruning
    cases.append(("wide", x, [(0.1, 0.9, 0), (0.1, 0.0, 50), (1.0, 0.0, 0), (3.0, 0.95, 0), (0.5, 0.0, 3000), (0.5, 0.0, 5000)]))
    x = np.round(rng.standard_normal((6, 4096)) * 2).astype(np.float32)  # many equal logits
    cases.append(("ties", x, [(1.0, 0.0, 10), (1.0, 0.9, 0), (0.7, 0.0, 0), (1.0, 0.0, 4096), (1.0, 0.0, 1), (1.0, 1.0, 0)]))
    x = np.zeros((2, 3000), np.float32)
    cases.append(("constant", x, [(1.0, 0.9, 0), (1.0, 0.0, 7)]))
    # near-equal probabilities: the sort keys share their upper digits, so the
    # block radix sort skips passes (every pass on the constant row)
    x = (np.arange(6000) % 3).astype(np.float32)[None, :] * np.float32(1e-6) * np.ones((3, 1), np.float32)
    x[2] = 0.0
    cases.append(("near-equal", x, [(1.0, 0.5, 0), (1.0, 0.999, 0), (1.0, 0.3, 0)]))
    x = (rng.standard_normal((3, 20001)) * 3).astype(np.float32)  # odd V, vector tails
    cases.append(("odd-V", x, [(0.9, 0.0, 64), (1.0, 0.95, 0), (0.8, 0.0, 1500)]))
    return cases


@pytest.mark.parametrize("case", _edge_cases(), ids=lambda c: c[0])
def test_edge_cases(sampler, case):
    name, x, params = case
    B = x.shape[0]
    for u in (np.zeros(B, np.float32), np.full(B, 0.5, np.float32), np.full(B, np.float32(0.99999994))):
        got = run_gpu(sampler, x, params, u)
        check_exact(x, params, u, got, name)


def test_unaligned_rows_and_bf16(sampler):
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((5, 3001)) * 2).astype(np.float32)
    params = [(0.8, 0.0, 40)] * 5
    u = rng.random(5).astype(np.float32)
    check_exact(x, params, u, run_gpu(sampler, x, params, u, ld=3003), "unaligned")
    xb = synth.bf16_bits_to_f32(synth.f32_to_bf16_bits(x))
    params = [(1.0, 0.95, 0), (0.7, 0.0, 50), (0.0, 0.0, 0), (1.0, 0.0, 0), (1.2, 0.5, 0)]
    check_exact(xb, params, u, run_gpu(sampler, xb, params, u, bf16=True), "bf16")
    check_exact(xb, params, u, run_gpu(sampler, xb, params, u, bf16=True, ld=3005), "bf16-unaligned")


def test_reference_unit_tests_on_gpu(sampler):
    import pesti_sampler as ps
    assert sampler.argmax([0.1, 0.9, 0.3, 0.7]) == 1
    cfg = ps.SamplingConfig(temperature=1.0, top_p=0.0, top_k=2)
    seen = {sampler.sample_with_u([0.1, 0.9, 0.3, 0.7], cfg, float(r)) for r in np.linspace(0, 0.9999, 65)}
    assert seen == {1, 3}
    x = [i * 0.01 for i in range(100)]
    rng = ps.Pcg32(42)
    assert sampler.sample(x, ps.SamplingConfig(), rng) < 100
    assert sampler.sample_with_u([], ps.SamplingConfig(), 0.5) == 0


def test_argmax_batch_semantics(sampler):
    import torch
    x = np.array([[1.0, 3.0, 3.0, 2.0], [5.0, np.nan, 1.0, 2.0], [5.0, 1.0, np.nan, np.nan],
                  [-np.inf, -np.inf, -np.inf, -np.inf]], np.float32)
    d = torch.from_numpy(x).cuda()
    last = sampler.argmax_batch(d).cpu().numpy()
    first = sampler.argmax_batch(d, first=True).cpu().numpy()
    assert list(last) == [O.argmax(r) for r in x]
    assert list(first) == [O.argmax_first(r) for r in x]


def test_host_row_api_matches_oracle(sampler):
    import pesti_sampler as ps
    x = synth.make_logits(1, B=20)
    u = synth.make_u(1, 20)
    for b in range(20):
        t = sampler.sample_with_u(x[b], ps.SamplingConfig(0.8, 0.95, 40), float(u[b]))
        assert t == O.sample(x[b], 0.8, 0.95, 40, float(u[b]), O.EXP_CR)


def test_prepared_params_and_single_config_match_the_list(sampler):
    """The three ways of passing the rows' configs (one SamplingConfig, a list,
    PreparedParams made once and reused) give the same tokens and kept lists,
    and PreparedParams refuses a batch of another size."""
    import torch
    import pesti_sampler as ps
    B = 16
    x = synth.make_logits(2, B=B)
    u = synth.make_u(2, B)
    d = torch.from_numpy(x).cuda()
    ud = torch.from_numpy(u).cuda()
    cfg = ps.SamplingConfig(0.7, 0.9, 50)
    prep = ps.PreparedParams([cfg] * B)
    want = [t.cpu().numpy() for t in sampler.sample_batch(d, [cfg] * B, ud, kept_width=KW)]
    for how in (cfg, prep, prep):  # the prepared params are reused
        got = [t.cpu().numpy() for t in sampler.sample_batch(d, how, ud, kept_width=KW)]
        for g, w_ in zip(got, want):
            assert np.array_equal(g.view(np.uint8), w_.view(np.uint8))
    with pytest.raises(ValueError):
        sampler.sample_batch(d[:8], prep, ud[:8])


def test_device_draws_equal_the_host_generator(sampler):
    """Per-row PCG32 draws on the device (pesti_pcg32_seed/draw) are those of
    the host Pcg32 on the same seed and stream, bit for bit, draw after draw;
    a batch sampled with them equals one sampled with the host draws."""
    import torch
    import pesti_sampler as ps
    B, seed, first = 100, 7, 11
    rng = ps.DeviceRng(B, seed, first_stream=first)
    host = [ps.Pcg32(seed, stream=first + b) for b in range(B)]
    for _ in range(3):
        got = rng.draw().cpu().numpy()
        want = np.array([h.next_f32() for h in host], dtype=np.float32)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    x = synth.make_logits(2, B=16)
    d = torch.from_numpy(x).cuda()
    cfg = ps.SamplingConfig(0.7, 0.9, 50)
    rng16 = ps.DeviceRng(16, 3, first_stream=0)
    ud = rng16.draw()
    hu = np.array([ps.Pcg32(3, stream=b).next_f32() for b in range(16)], dtype=np.float32)
    a = sampler.sample_batch(d, cfg, ud).cpu().numpy()
    b_ = sampler.sample_batch(d, cfg, torch.from_numpy(hu).cuda()).cpu().numpy()
    assert np.array_equal(a, b_)


def _run_f16(sampler, x16, params, u, ld=None, kept_width=KW):
    import torch
    import pesti_sampler as ps
    B, V = x16.shape
    host = torch.from_numpy(np.ascontiguousarray(x16))
    if ld is not None and ld != V:
        big = torch.zeros((B, ld), dtype=torch.float16)
        big[:, :V] = host
        dev = big.cuda()[:, :V]
    else:
        dev = host.cuda()
    cfgs = [ps.SamplingConfig(temperature=t, top_p=p, top_k=k) for (t, p, k) in params]
    ud = torch.from_numpy(np.ascontiguousarray(u, dtype=np.float32)).cuda()
    tok, kp, ki, kc = sampler.sample_batch(dev, cfgs, ud, kept_width=kept_width)
    torch.cuda.synchronize()
    return (tok.cpu().numpy().view(np.uint32), kp.cpu().numpy(), ki.cpu().numpy().view(np.uint32),
            kc.cpu().numpy())


@pytest.mark.parametrize("w,B,ld_extra", [(2, 16, 0), (2, 8, 1), (3, 4, 0), (4, 60, 0), (5, 8, 0)])
def test_f16_logits(sampler, w, B, ld_extra):
    """f16 logits: the results of the oracle on the same values widened to f32
    (what a caller of the reference's &[f32] API would pass), bit for bit;
    the rounding to f16 also makes many ties.  ld_extra 1 takes the unaligned
    (scalar-load) paths."""
    spec = synth.WORKLOADS[w]
    V = spec["V"]
    x16 = synth.make_logits(w, B=B).astype(np.float16)
    x = x16.astype(np.float32)
    params = synth.params_for(w, B, V)
    u = synth.make_u(w, B)
    got = _run_f16(sampler, x16, params, u, ld=V + ld_extra if ld_extra else None)
    check_exact(x, params, u, got, f"f16 workload{w}")


def test_f16_emulated_shards_match_whole_rows(sampler):
    """Vocabulary shards of f16 logits (one GPU emulating 4 shards) give the
    whole-row results bit for bit."""
    import torch
    import pesti_sampler as ps
    B = 16
    x16 = synth.make_logits(5, B=B).astype(np.float16)
    d = torch.from_numpy(x16).cuda()
    u = torch.from_numpy(synth.make_u(5, B)).cuda()
    cfg = ps.SamplingConfig(0.9, 0.92, 64)
    whole = [t.cpu().numpy() for t in sampler.sample_batch(d, cfg, u, kept_width=KW)]
    got = [t.cpu().numpy() for t in sampler.sample_batch_sharded_emulated(d, cfg, u, 4, kept_width=KW)]
    for g, w_ in zip(got, whole):
        assert np.array_equal(g.view(np.uint8), w_.view(np.uint8))


def _fp8_case(fmt, B, V, seed):
    """fp8 logits of one format ([B, V] uint8 bits) and their exact f32
    values, with the format's specials planted: NaN (both formats), the
    infinities (E5M2), signed zeros and subnormals."""
    import torch
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((B, V)) * 3).astype(np.float32)
    tdt = torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2
    bits = torch.from_numpy(x).to(tdt).view(torch.uint8).numpy().copy()
    bits[0, 3] = 0x01            # the smallest subnormal
    bits[0, 4] = 0x80            # -0
    bits[1, 5] = 0x7f            # NaN (E4M3) / NaN (E5M2)
    if fmt == "e5m2":
        bits[2, 6] = 0x7c        # +inf
        bits[3, 7] = 0xfc        # -inf
    widened = torch.from_numpy(bits).view(tdt).to(torch.float32).numpy()
    return bits, widened, tdt


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("V,ld_extra", [(32000, 0), (5001, 3)])
def test_fp8_logits(sampler, fmt, V, ld_extra):
    """fp8 logits (E4M3FN and E5M2): the oracle's results on the same values
    widened to f32, bit for bit, for sampled rows of every kind and for
    argmax; rows with NaN or infinities included.  ld_extra takes the
    unaligned (byte-wise) widening."""
    import torch
    import pesti_sampler as ps
    B = 12
    bits, x, tdt = _fp8_case(fmt, B, V, 7 if fmt == "e4m3" else 8)
    kinds = [(0.8, 0.0, 40), (1.0, 0.9, 0), (0.7, 0.0, 0), (0.0, 0.0, 0), (1.2, 0.0, 256), (0.9, 0.95, 1000)]
    params = [kinds[r % len(kinds)] for r in range(B)]
    u = synth.make_u(1, B)
    ld = V + ld_extra
    host = np.zeros((B, ld), np.uint8)
    host[:, :V] = bits
    dev = torch.from_numpy(host).cuda().view(tdt)[:, :V]
    cfgs = [ps.SamplingConfig(temperature=t, top_p=p, top_k=k) for (t, p, k) in params]
    ud = torch.from_numpy(u).cuda()
    tok, kp, ki, kc = sampler.sample_batch(dev, cfgs, ud, kept_width=KW)
    got = (tok.cpu().numpy().view(np.uint32), kp.cpu().numpy(), ki.cpu().numpy().view(np.uint32), kc.cpu().numpy())
    check_exact(x, params, u, got, f"fp8 {fmt}")
    last = sampler.argmax_batch(dev).cpu().numpy()
    first = sampler.argmax_batch(dev, first=True).cpu().numpy()
    assert list(last) == [O.argmax(r) for r in x]
    assert list(first) == [O.argmax_first(r) for r in x]
