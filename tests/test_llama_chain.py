"""The llama.cpp backend's sampler chain (llm-runner/src/llama.rs:465-508):
the CPU restatement's own properties, and pesti_llama_chain_batch on the GPU
against it.

Parity bar (the chain's stages are third-party semantics whose sources are not
in the reference tree, so the restatement is unpinned): probabilities are f64
on both sides, summed in different orders, so a decision may differ only
where the restatement reports a boundary closer than 1e-9 relative (`margin`).
Every other row must give the same token and the same number of candidates
before the draw; at most one row in twenty may sit that close."""
import zlib

import numpy as np
import pytest

import llama_chain as LC

MARGIN = 1e-9

# The presets of llm-runner/src/llama/sampler.rs:81-173 and a few that reach
# the whole-row paths (top_k = 0).
PRESETS = {
    "default": dict(temperature=0.7, top_k=40, top_p=0.95),
    "greedy": dict(temperature=0.0, top_k=1, top_p=0.0),
    "creative": dict(temperature=1.0, top_k=50, top_p=0.99, min_p=0.05, tfs=0.5, typical_p=0.5),
    "balanced": dict(temperature=0.7, top_k=40, top_p=0.95),
    "precise": dict(temperature=0.3, top_k=20, top_p=0.9, min_p=0.1, repetition_penalty=1.1,
                    repeat_last_n=128),
    "whole_row_top_p_typical": dict(temperature=0.8, top_k=0, top_p=0.9, typical_p=0.7),
    "whole_row_min_p_sigma": dict(temperature=1.0, top_k=0, top_p=0.0, min_p=0.02, tfs=0.8),
    "whole_row_penalties": dict(temperature=1.0, top_k=0, top_p=0.0, repetition_penalty=1.3,
                                repeat_last_n=-1, frequency_penalty=0.1, presence_penalty=0.2),
    "none": dict(temperature=0.0, top_k=0, top_p=0.0),
}


def _logits(rng, B, V, scale=2.5):
    x = (rng.standard_normal((B, V)) * scale).astype(np.float32)
    # a few peaked rows and a duplicated maximum
    if B > 2:
        x[1, rng.integers(0, V)] += 12.0
        x[2, :] = np.round(x[2, :])
    return x


def _history(rng, x, H):
    """Recent tokens drawn mostly from each row's largest logits, so that the
    penalties land on candidates."""
    B, V = x.shape
    top = np.argsort(-x, axis=1, kind="stable")[:, :64]
    h = np.where(rng.random((B, H)) < 0.8, top[np.arange(B)[:, None], rng.integers(0, 64, (B, H))],
                 rng.integers(0, V, (B, H)))
    return h.astype(np.int32)


def _u(rng, B):
    u = rng.random(B).astype(np.float32)
    u[0] = 0.0
    if B > 3:
        u[3] = np.float32(0.99999994)
    return u


# ---- the restatement's own properties (no GPU) ----

def test_greedy_preset_is_the_first_maximum():
    x = np.array([0.5, 3.0, -1.0, 3.0, 2.0], dtype=np.float32)
    for u in (0.0, 0.5, 0.99):
        tok, kept, _ = LC.chain_row(x, u=u, **PRESETS["greedy"])
        assert (tok, kept) == (1, 1)


def test_unfiltered_draw_is_the_inverse_cdf_by_logit():
    rng = np.random.default_rng(1)
    x = rng.standard_normal(300).astype(np.float32)
    w = np.exp(x.astype(np.float64) - float(x.max()))
    order = np.lexsort((np.arange(300), LC.desc_key(x)))
    cum = np.cumsum(w[order]) / w.sum()
    for u in (0.0, 0.1, 0.5, 0.9, 0.9999):
        tok, kept, _ = LC.chain_row(x, u=u, **PRESETS["none"])
        assert kept == 300
        assert tok == order[int(np.searchsorted(cum, np.float32(u), side="left"))]


def test_min_p_keeps_at_least_256():
    rng = np.random.default_rng(2)
    x = rng.standard_normal(1000).astype(np.float32)
    x[7] = 40.0  # every other token far below min_p * p_max
    _, kept, _ = LC.chain_row(x, temperature=1.0, top_k=0, top_p=0.0, min_p=0.5, u=0.3)
    assert kept == 256
    _, kept, _ = LC.chain_row(x[:100], temperature=1.0, top_k=0, top_p=0.0, min_p=0.5, u=0.3)
    assert kept == 100


def test_top_p_keeps_the_shortest_prefix_reaching_p():
    x = np.log(np.array([0.5, 0.3, 0.15, 0.05], dtype=np.float64)).astype(np.float32)
    for p, want in ((0.5, 1), (0.79, 2), (0.81, 3), (0.96, 4)):
        _, kept, _ = LC.chain_row(x, temperature=1.0, top_k=0, top_p=p, u=0.0)
        assert kept == want, p


def test_penalties_move_the_draw_off_repeated_tokens():
    x = np.array([2.0, 2.0, -1.0, 0.5], dtype=np.float32)
    tok, _, _ = LC.chain_row(x, **PRESETS["none"], u=0.0)
    assert tok == 0
    tok, _, _ = LC.chain_row(x, temperature=0.0, top_k=0, top_p=0.0, repetition_penalty=1.5,
                             repeat_last_n=4, history=[0, 3], u=0.0)
    assert tok == 1
    # a negative logit is multiplied by the penalty: -1 * 1.5 falls below -1.2
    y = np.array([-1.0, -1.2], dtype=np.float32)
    assert LC.chain_row(y, **PRESETS["none"], u=0.0)[0] == 0
    assert LC.chain_row(y, temperature=0.0, top_k=0, top_p=0.0, repetition_penalty=1.5, repeat_last_n=4,
                        history=[0], u=0.0)[0] == 1


def test_typical_keeps_mass_at_least_p():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(2000) * 2).astype(np.float32)
    _, kept_all, _ = LC.chain_row(x, temperature=1.0, top_k=0, top_p=0.0, u=0.5)
    _, kept, _ = LC.chain_row(x, temperature=1.0, top_k=0, top_p=0.0, typical_p=0.5, u=0.5)
    assert 1 <= kept < kept_all


def test_library_presets_are_the_configs_presets():
    import pesti_sampler as ps
    for name in ("greedy", "creative", "balanced", "precise"):
        got = getattr(ps.LlamaChainParams, name)().as_dict()
        want = ps.LlamaChainParams(**PRESETS[name]).as_dict()
        assert got == want, name
    assert ps.LlamaChainParams().as_dict() == ps.LlamaChainParams(**PRESETS["default"]).as_dict()


# ---- GPU parity ----

def _gpu_chain(x, params, u, hist=None, dtype="f32"):
    import torch
    import pesti_sampler as ps
    s = _sampler()
    t = torch.from_numpy(x).cuda()
    if dtype == "bf16":
        t = t.to(torch.bfloat16)
    elif dtype == "f16":
        t = t.half()
    elif dtype == "e4m3":
        t = t.to(torch.float8_e4m3fn)
    ud = torch.from_numpy(u).cuda()
    hd = None if hist is None else torch.from_numpy(hist).cuda()
    kept = torch.empty(x.shape[0], dtype=torch.int32, device="cuda")
    tok = s.llama_chain_batch(t, ps.LlamaChainParams(**params), ud, history=hd, kept=kept)
    torch.cuda.synchronize()
    widened = t.float().cpu().numpy()
    return tok.cpu().numpy(), kept.cpu().numpy(), widened


_S = None


def _sampler():
    global _S
    if _S is None:
        import pesti_sampler as ps
        _S = ps.Sampler(0)
    return _S


def _check(x, params, u, hist, tok, kept, exact=False):
    ot, ok, om = LC.chain_batch(x, params, hist, u)
    near = np.zeros_like(om, dtype=bool) if exact else om < MARGIN
    bad = np.nonzero(~near & ((ot != tok) | (ok != kept)))[0]
    assert bad.size == 0, [(int(b), int(ot[b]), int(tok[b]), int(ok[b]), int(kept[b])) for b in bad[:5]]
    assert near.sum() <= max(1, x.shape[0] // 20), int(near.sum())


@pytest.mark.gpu
@pytest.mark.parametrize("preset", list(PRESETS))
@pytest.mark.parametrize("B,V,dtype", [(32, 32000, "f32"), (8, 128256, "f32"), (16, 5001, "bf16")])
def test_chain_matches_the_restatement(preset, B, V, dtype):
    rng = np.random.default_rng(zlib.crc32(f"{preset}/{V}".encode()))
    x = _logits(rng, B, V)
    u = _u(rng, B)
    hist = _history(rng, x, 200)
    params = PRESETS[preset]
    tok, kept, xw = _gpu_chain(x, params, u, hist, dtype)
    _check(xw, params, u, hist, tok, kept)


@pytest.mark.gpu
def test_chain_edge_rows():
    V = 3000
    x = np.zeros((6, V), dtype=np.float32)
    x[0, :] = -np.inf                 # every logit -inf
    x[1, :] = 1.25                    # all equal
    x[2, :] = np.nan                  # NaN counts as -inf
    x[2, 17] = 0.0
    x[3, :] = np.linspace(-5, 5, V, dtype=np.float32)
    x[3, ::7] = np.nan
    x[4, :] = -np.inf
    x[4, [5, 900]] = np.inf           # two +inf logits
    x[5, :] = np.float32(-0.0)
    x[5, ::2] = 0.0                   # +0 and -0
    u = np.array([0.3, 0.999, 0.5, 0.7, 0.6, 0.5], dtype=np.float32)
    # ties and infinities: both sides compute the same weights exactly, so
    # every row must agree, boundaries included
    for name in ("default", "creative", "whole_row_top_p_typical", "whole_row_min_p_sigma", "none"):
        params = PRESETS[name]
        tok, kept, xw = _gpu_chain(x, params, u)
        _check(xw, params, u, None, tok, kept, exact=True)


@pytest.mark.gpu
def test_chain_small_rows_and_large_k():
    rng = np.random.default_rng(9)
    for V in (1, 2, 33, 1025):
        x = _logits(rng, 4, V)
        u = _u(rng, 4)
        for params in (dict(temperature=0.9, top_k=V + 10, top_p=0.8), PRESETS["creative"], PRESETS["none"]):
            tok, kept, xw = _gpu_chain(x, params, u)
            _check(xw, params, u, None, tok, kept)


@pytest.mark.gpu
def test_chain_fp8_logits():
    rng = np.random.default_rng(11)
    x = _logits(rng, 8, 32000, scale=2.0)
    u = _u(rng, 8)
    tok, kept, xw = _gpu_chain(x, PRESETS["creative"], u, dtype="e4m3")
    _check(xw, PRESETS["creative"], u, None, tok, kept)


@pytest.mark.gpu
@pytest.mark.parametrize("last_n", [0, 1, 37, 500, -1])
def test_chain_penalty_windows_and_history_lengths(last_n):
    """Per-row history lengths (d_history_len) and every window rule:
    repeat_last_n 0 (no penalty), shorter and longer than the history, -1
    (all of it)."""
    import torch
    import pesti_sampler as ps
    rng = np.random.default_rng(100 + last_n)
    B, V, H = 12, 20000, 300
    x = _logits(rng, B, V)
    u = _u(rng, B)
    hist = _history(rng, x, H)
    hl = rng.integers(0, H + 1, size=B).astype(np.int32)
    hl[0], hl[1] = 0, H
    params = dict(temperature=0.9, top_k=0, top_p=0.0, repetition_penalty=1.4, repeat_last_n=last_n,
                  frequency_penalty=0.05, presence_penalty=0.3)
    s = _sampler()
    kept = torch.empty(B, dtype=torch.int32, device="cuda")
    tok = s.llama_chain_batch(torch.from_numpy(x).cuda(), ps.LlamaChainParams(**params), torch.from_numpy(u).cuda(),
                              history=torch.from_numpy(hist).cuda(), history_len=torch.from_numpy(hl).cuda(),
                              kept=kept)
    torch.cuda.synchronize()
    rows_hist = [hist[b, :hl[b]] for b in range(B)]
    _check(x, params, u, rows_hist, tok.cpu().numpy(), kept.cpu().numpy())


@pytest.mark.gpu
def test_chain_f16_logits():
    rng = np.random.default_rng(13)
    x = _logits(rng, 8, 32000, scale=2.0)
    u = _u(rng, 8)
    hist = _history(rng, x, 128)
    tok, kept, xw = _gpu_chain(x, PRESETS["precise"], u, hist, dtype="f16")
    _check(xw, PRESETS["precise"], u, hist, tok, kept)


@pytest.mark.gpu
def test_chain_is_deterministic():
    rng = np.random.default_rng(12)
    x = _logits(rng, 16, 128256)
    u = _u(rng, 16)
    hist = _history(rng, x, 300)
    params = PRESETS["whole_row_top_p_typical"]
    a = _gpu_chain(x, params, u, hist)
    b = _gpu_chain(x, params, u, hist)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


@pytest.mark.gpu
def test_chain_invalid_window():
    import torch
    import pesti_sampler as ps
    s = _sampler()
    x = torch.zeros(2, 100, device="cuda")
    u = torch.zeros(2, device="cuda")
    h = torch.zeros(2, 9000, dtype=torch.int32, device="cuda")
    with pytest.raises(ps.SamplerError) as e:
        s.llama_chain_batch(x, ps.LlamaChainParams(repetition_penalty=1.2, repeat_last_n=-1), u, history=h)
    assert e.value.code == ps.PESTI_E_INVALID_ARG
