"""The CPU oracle against the reference's own tests and a second restatement.

The reference's sampler tests (llm-runner/src/transformer/sampling.rs:142-207)
check properties, not token ids; each is restated here against the C++ oracle
(and, where it applies, the pure-Python restatement).  The two restatements
are then cross-checked bit for bit (exp correctly rounded in both) on seeded
random rows and on the edge cases the reference's code paths distinguish.
"""
import math

import numpy as np
import pytest

import oracle as O


def _kept_probs(logits):
    # top_k = 0 and top_p = 0: no sort, the kept list is the softmax in index order
    tok, kp, ki, kc, _ = O.sample(logits, 1.0, 0.0, 0, 0.5, O.EXP_PLATFORM, kept_width=len(logits))
    assert list(ki) == list(range(len(logits)))
    return kp


def test_softmax_basic():  # sampling.rs:143-151
    p = _kept_probs([1.0, 2.0, 3.0])
    assert len(p) == 3
    assert abs(float(np.float64(p).sum()) - 1.0) < 1e-5
    assert p[2] > p[1] > p[0]


def test_softmax_numerical_stability():  # sampling.rs:154-160
    p = _kept_probs([1000.0, 1001.0, 1002.0])
    assert abs(float(np.float64(p).sum()) - 1.0) < 1e-5
    assert p[2] > p[1] > p[0]


def test_argmax_returns_largest():  # sampling.rs:163-166
    assert O.argmax([0.1, 0.9, 0.3, 0.7]) == 1
    assert O.py_argmax([0.1, 0.9, 0.3, 0.7]) == 1


def test_zero_temperature_is_argmax():  # sampling.rs:169-181 and model.rs:517-521
    x = np.array([[0.1, 0.9, 0.3, 0.7]], np.float32)
    out = O.sample_batch(x, (0.0, 0.0, 0), np.array([0.3], np.float32))
    assert out["tokens"][0] == 1


def test_sample_with_top_k():  # sampling.rs:184-196, over a sweep of draws
    x = [0.1, 0.9, 0.3, 0.7]
    seen = set()
    for r in np.linspace(0.0, 0.999999, 257):
        t = O.sample(x, 1.0, 0.0, 2, float(r))
        assert t in (1, 3)
        seen.add(t)
    assert seen == {1, 3}


def test_sample_returns_valid_token():  # sampling.rs:199-207 (default config)
    x = [i * 0.01 for i in range(100)]
    for r in (0.0, 0.25, 0.5, 0.999):
        assert O.sample(x, 0.7, 0.9, 0, r) < 100


def test_argmax_ties_go_last_and_nan_restarts():
    assert O.argmax([1.0, 3.0, 3.0, 2.0]) == 2
    assert O.argmax_first([1.0, 3.0, 3.0, 2.0]) == 1
    # a NaN is adopted, the next element replaces it, then max_by resumes
    assert O.argmax([5.0, float("nan"), 1.0, 2.0, 0.5]) == 3
    assert O.argmax([5.0, 1.0, float("nan")]) == 2
    assert O.argmax([]) == 0
    for x in ([5.0, float("nan"), 1.0, 2.0, 0.5], [5.0, 1.0, float("nan")], [3.0, 3.0, 1.0]):
        assert O.argmax(x) == O.py_argmax(x)


def _edge_rows(rng):
    rows = []
    rows.append(([0.0] * 7, (1.0, 0.0, 0)))
    rows.append(([float("-inf")] * 5, (1.0, 0.9, 0)))               # all -inf -> uniform
    rows.append(([1.0, float("nan"), 2.0], (1.0, 0.0, 2)))          # NaN -> uniform
    rows.append(([1.0, float("inf"), 2.0], (0.5, 0.95, 0)))         # +inf -> uniform
    rows.append(([1.0, float("-inf"), 2.0, 2.0], (1.0, 0.0, 3)))    # -inf entry, tie
    rows.append(([3.0], (1.0, 0.9, 0)))                             # V = 1
    rows.append(([1.0, 2.0, 3.0], (-1.0, 0.9, 0)))                  # T < 0: no scaling
    rows.append(([1.0, 2.0, 3.0], (float("nan"), 0.0, 5)))          # T NaN: no scaling; k > V
    rows.append(([100.0, 0.0, -100.0], (1e-30, 0.0, 0)))           # x/T overflows -> uniform
    rows.append(([2.0, 2.0, 2.0, 1.0], (1.0, 1.0, 0)))              # top-p 1.0
    rows.append(([2.0, 2.0, 2.0, 1.0], (1.0, 1e-6, 0)))             # top-p tiny
    for _ in range(40):
        V = int(rng.integers(1, 300))
        x = (rng.standard_normal(V) * rng.uniform(0.1, 20)).astype(np.float32)
        if rng.random() < 0.3:
            x[rng.integers(0, V, size=max(1, V // 10))] = x.max()
        if rng.random() < 0.2:
            x = np.round(x)
        t = float(rng.choice([0.0, 0.5, 0.7, 1.0, 1.3, -1.0]))
        k = int(rng.choice([0, 0, 1, 2, 5, 40, V, V + 3]))
        p = float(rng.choice([0.0, 0.5, 0.9, 0.95, 1.0, 1e-6]))
        rows.append((x.tolist(), (t, p, k)))
    return rows


def test_two_restatements_agree_bit_for_bit():
    rng = np.random.default_rng(7)
    for x, (t, p, k) in _edge_rows(rng):
        for r in (0.0, 0.1, 0.5, 0.9, 0.99999994):
            a = O.sample(x, t, p, k, r, O.EXP_CR, kept_width=len(x))
            b_tok, b_kept = O.py_sample(x, t, p, k, r)
            assert a[0] == b_tok, (x, t, p, k, r)
            assert a[3] == len(b_kept)
            kp = a[1][: a[3]].view(np.uint32)
            bk = np.array([q for q, _ in b_kept], np.float32).view(np.uint32)
            assert np.array_equal(kp, bk)
            assert list(a[2][: a[3]]) == [i for _, i in b_kept]


def test_batch_driver_matches_rows():
    rng = np.random.default_rng(3)
    B, V = 24, 500
    x = (rng.standard_normal((B, V)) * 3).astype(np.float32)
    params = [(float(rng.choice([0.0, 0.8, 1.0])), 0.9, int(rng.choice([0, 10]))) for _ in range(B)]
    u = rng.random(B).astype(np.float32)
    out = O.sample_batch(x, params, u, O.EXP_CR, kept_width=8, nthreads=4)
    for b in range(B):
        t, p, k = params[b]
        want = O.argmax(x[b]) if t == 0.0 else O.sample(x[b], t, p, k, u[b], O.EXP_CR)
        assert out["tokens"][b] == want


def test_platform_exp_rarely_differs():
    # glibc's expf is not correctly rounded; on sampler-sized rows the two exp
    # modes still give the same tokens on almost every row.
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((32, 4096)) * 2).astype(np.float32)
    u = rng.random(32).astype(np.float32)
    a = O.sample_batch(x, (0.8, 0.95, 40), u, O.EXP_PLATFORM)["tokens"]
    b = O.sample_batch(x, (0.8, 0.95, 40), u, O.EXP_CR)["tokens"]
    assert (a != b).sum() <= 1


def test_generate_control_exits():
    """The restated loop control of generate() (transformer/model.rs:508-531)
    on its three exits and on a loop still running."""
    assert O.generate_control([1, 2, 3, 4], stop_tokens=[3], max_tokens=10, max_seq_len=10) == ([1, 2], "stop")
    assert O.generate_control([1, 2, 3, 4], stop_tokens=[], max_tokens=2, max_seq_len=10) == ([1, 2], "max_tokens")
    assert O.generate_control([1, 2, 3, 4], stop_tokens=[], max_tokens=10, max_seq_len=3) == ([1, 2, 3], "max_seq_len")
    assert O.generate_control([1, 2], stop_tokens=[], max_tokens=10, max_seq_len=10) == ([1, 2], None)
    assert O.generate_control([5], stop_tokens=[5], max_tokens=0, max_seq_len=10) == ([], "max_tokens")
