"""ctypes binding of the CPU oracle (liboracle.so) -- TEST INFRASTRUCTURE ONLY.

Used by tests/, __graft_entry__.smoke() (as the checker) and bench.py's
cpu_baseline / `--impl reference` leg (as the timed reference algorithm).  The
product library never imports this module.

Also holds `py_sample`, a second, independent restatement of
llm-runner/src/transformer/sampling.rs:39-134 written with numpy float32
scalars in plain Python loops.  It is slow and meant for small rows; the tests
use it to cross-check the C++ oracle (both must agree bit for bit when exp is
correctly rounded).

Parity pin: the Rust reference cannot be built in this image (no cargo or
rustc), and its own tests (sampling.rs:142-207) pin properties only, not token
ids; tests/test_oracle.py restates those six tests against both restatements.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(_HERE, "_build", "liboracle.so")

EXP_PLATFORM = 0
EXP_CR = 1
FLAG_GREEDY_IF_ZERO_T = 1
FLAG_ARGMAX_FIRST = 2


class OracleParams(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_float), ("top_p", ctypes.c_float),
                ("top_k", ctypes.c_uint32), ("flags", ctypes.c_uint32)]


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return LIB


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        fp, i64, vp = ctypes.POINTER(ctypes.c_float), ctypes.c_int64, ctypes.c_void_p
        L.oracle_argmax.argtypes = [fp, i64]
        L.oracle_argmax.restype = ctypes.c_uint32
        L.oracle_argmax_first.argtypes = [fp, i64]
        L.oracle_argmax_first.restype = ctypes.c_uint32
        L.oracle_sample.argtypes = [fp, i64, ctypes.c_float, ctypes.c_float, i64, ctypes.c_float,
                                    ctypes.c_int, vp, vp, i64, vp, vp]
        L.oracle_sample.restype = ctypes.c_uint32
        L.oracle_sample_batch.argtypes = [fp, i64, i64, i64, ctypes.POINTER(OracleParams), ctypes.c_int,
                                          fp, ctypes.c_int, vp, vp, vp, i64, vp, vp, ctypes.c_int]
        L.oracle_sample_batch.restype = None
        L.oracle_exp_cr.argtypes = [ctypes.c_float]
        L.oracle_exp_cr.restype = ctypes.c_float
        L.oracle_softmax_terms.argtypes = [fp, i64, ctypes.c_float, ctypes.c_float, ctypes.c_int, fp]
        L.oracle_softmax_terms.restype = None
        L.oracle_fold.argtypes = [fp, i64, ctypes.c_float]
        L.oracle_fold.restype = ctypes.c_float
        _lib = L
    return _lib


def _fp(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def argmax(logits) -> int:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().oracle_argmax(_fp(x), x.size))


def argmax_first(logits) -> int:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().oracle_argmax_first(_fp(x), x.size))


def sample(logits, temperature, top_p, top_k, r, exp_mode=EXP_PLATFORM, kept_width=0):
    """One row of sampling.rs:39.  Returns token, or (token, kept_p, kept_idx,
    kept_count, boundary_dist) when kept_width > 0."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    kp = np.zeros(max(kept_width, 1), np.float32)
    ki = np.zeros(max(kept_width, 1), np.uint32)
    kc = np.zeros(1, np.int64)
    bd = np.zeros(1, np.float32)
    tok = lib().oracle_sample(_fp(x), x.size, float(temperature), float(top_p), int(top_k), float(r),
                              exp_mode, kp.ctypes.data, ki.ctypes.data, kept_width,
                              kc.ctypes.data, bd.ctypes.data)
    if kept_width > 0:
        return int(tok), kp[:kept_width], ki[:kept_width], int(kc[0]), float(bd[0])
    return int(tok)


def softmax_terms(logits, temperature, m, exp_mode=EXP_CR) -> np.ndarray:
    """exp(scaled_i - m) of each logit (sampling.rs:43-50, :127), m being the
    max of the scaled whole row (the caller's, when `logits` is a shard)."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    out = np.empty_like(x)
    lib().oracle_softmax_terms(_fp(x), x.size, float(temperature), float(m), exp_mode, _fp(out))
    return out


def fold(v, s0=0.0) -> np.float32:
    """The sequential f32 fold s = s0; s = s + v[i] (sampling.rs:128 from any start)."""
    x = np.ascontiguousarray(v, dtype=np.float32)
    return np.float32(lib().oracle_fold(_fp(x), x.size, float(np.float32(s0))))


def sample_batch(logits: np.ndarray, params, u: np.ndarray, exp_mode=EXP_PLATFORM, kept_width=0,
                 nthreads=0, greedy_if_zero_t=True, argmax_first=False):
    """Rows of a [B, V] f32 array.  params: list of (temperature, top_p, top_k)
    per row (or one tuple).  Returns dict(tokens, kept_p, kept_idx, kept_count,
    boundary_dist)."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    B, V = x.shape
    flags = (FLAG_GREEDY_IF_ZERO_T if greedy_if_zero_t else 0) | (FLAG_ARGMAX_FIRST if argmax_first else 0)
    if isinstance(params, tuple):
        arr = (OracleParams * 1)(OracleParams(params[0], params[1], params[2], flags))
        per_row = 0
    else:
        arr = (OracleParams * B)(*[OracleParams(t, p, k, flags) for (t, p, k) in params])
        per_row = 1
    uu = np.ascontiguousarray(u, dtype=np.float32)
    out = np.zeros(B, np.uint32)
    kw = max(kept_width, 0)
    kp = np.zeros((B, max(kw, 1)), np.float32)
    ki = np.zeros((B, max(kw, 1)), np.uint32)
    kc = np.zeros(B, np.int64)
    bd = np.zeros(B, np.float32)
    lib().oracle_sample_batch(_fp(x), B, V, V, arr, per_row, _fp(uu), exp_mode, out.ctypes.data,
                              kp.ctypes.data if kw else None, ki.ctypes.data if kw else None, kw,
                              kc.ctypes.data, bd.ctypes.data, int(nthreads))
    return dict(tokens=out, kept_p=kp[:, :kw], kept_idx=ki[:, :kw], kept_count=kc, boundary_dist=bd)


# ---------------------------------------------------------------------------
# Independent pure-Python restatement (numpy float32 scalars), small rows only.
# ---------------------------------------------------------------------------
def _exp_cr(x: np.float32) -> np.float32:
    if np.isnan(x):
        return np.float32(np.nan)
    if x == -np.inf:
        return np.float32(0.0)
    return np.float32(math.exp(float(x)))


def py_argmax(logits) -> int:
    x = [np.float32(v) for v in logits]
    if not x:
        return 0
    best = 0
    for i in range(1, len(x)):
        if not (x[best] > x[i]):
            best = i
    return best


def py_sample(logits, temperature, top_p, top_k, r):
    """sampling.rs:39-112 with exp correctly rounded; returns (token, kept list)."""
    f32 = np.float32
    lg = [f32(v) for v in logits]
    T = f32(temperature)
    scaled = [v / T for v in lg] if T > f32(0.0) else list(lg)
    m = f32(-np.inf)
    for v in scaled:
        m = v if np.isnan(m) else (m if np.isnan(v) else max(m, v))
    with np.errstate(invalid="ignore", over="ignore"):
        exps = [_exp_cr(f32(v - m)) for v in scaled]
        s = f32(-0.0)
        for e in exps:
            s = f32(s + e)
        if s > f32(0.0):
            probs = [f32(e / s) for e in exps]
        else:
            probs = [f32(1.0) / f32(len(lg))] * len(lg)
    ip = [(p, i) for i, p in enumerate(probs)]
    if top_k > 0:
        ip = sorted(ip, key=lambda t: -float(t[0]))
        ip = ip[:min(top_k, len(ip))]
    if f32(top_p) > f32(0.0) and top_k == 0:
        ip = sorted(ip, key=lambda t: -float(t[0]))
        c = f32(0.0)
        cut = len(ip)
        for i, (p, _) in enumerate(ip):
            c = f32(c + p)
            if c >= f32(top_p):
                cut = i + 1
                break
        ip = ip[:cut]
    total = f32(-0.0)
    for p, _ in ip:
        total = f32(total + p)
    if total <= f32(0.0):
        return py_argmax(logits), ip
    norm = [(f32(p / total), i) for p, i in ip]
    c = f32(0.0)
    rr = f32(r)
    for p, i in norm:
        c = f32(c + p)
        if rr <= c:
            return i, ip
    return (norm[-1][1] if norm else 0), ip


# ---------------------------------------------------------------------------
# Parity figures of a batch against both oracle modes (tests and the bench's
# correctness guard).
# ---------------------------------------------------------------------------
BOUNDARY_BAND = 1e-6


def parity_report(logits: np.ndarray, params, u: np.ndarray, tokens, kept_p, kept_idx, kept_count,
                  kept_width: int, nthreads: int = 0) -> dict:
    """The figures the drop-in contract is stated in, for one batch:

    rows_exact        rows whose token, kept-list length, kept indices and kept
                      probabilities (bits, first kept_width entries) equal the
                      oracle's with exp correctly rounded;
    token_mismatch_rate  against the oracle with the platform expf (what the
                      Rust reference calls): tokens that differ, outside the
                      rows whose draw lies within 1e-6 of a cumulative-
                      probability boundary, over all rows;
    rows_near_boundary   rows inside that band;
    max_prob_rel_err  largest relative difference of a kept probability from
                      the platform-expf oracle's, over entries with the same
                      index at the same position;
    topk_sets_exact   fraction of the top-k rows (T != 0, 0 < top_k <=
                      kept_width) whose top-k index set equals the
                      platform-expf oracle's."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    B = x.shape[0]
    tok = np.asarray(tokens).view(np.uint32).reshape(B)
    kp = np.asarray(kept_p, dtype=np.float32).reshape(B, kept_width)
    ki = np.asarray(kept_idx).view(np.uint32).reshape(B, kept_width)
    kc = np.asarray(kept_count).reshape(B)
    cr = sample_batch(x, params, u, EXP_CR, kept_width=kept_width, nthreads=nthreads)
    exact = ((tok == cr["tokens"]) & (kc == cr["kept_count"]) & (ki == cr["kept_idx"]).all(axis=1)
             & (kp.view(np.uint32) == cr["kept_p"].view(np.uint32)).all(axis=1))
    ref = sample_batch(x, params, u, EXP_PLATFORM, kept_width=kept_width, nthreads=nthreads)
    mism = tok != ref["tokens"]
    near = ref["boundary_dist"] <= BOUNDARY_BAND
    valid = ref["kept_idx"] != 0xFFFFFFFF
    same = valid & (ki == ref["kept_idx"])
    rp = ref["kept_p"][same].astype(np.float64)
    gp = kp[same].astype(np.float64)
    rel = np.abs(gp - rp) / np.maximum(np.abs(rp), 1e-38)
    plist = [params] * B if isinstance(params, tuple) else list(params)
    topk_rows, topk_ok = 0, 0
    for b in range(B):
        t, _, k = plist[b]
        if t != 0.0 and 0 < k <= kept_width:
            topk_rows += 1
            topk_ok += int(set(ki[b, :k].tolist()) == set(ref["kept_idx"][b, :k].tolist()))
    return {
        "rows": B,
        "rows_exact": int(exact.sum()),
        "token_mismatches": int(mism.sum()),
        "token_mismatches_outside_band": int((mism & ~near).sum()),
        "token_mismatch_rate": float((mism & ~near).sum()) / max(B, 1),
        "rows_near_boundary": int(near.sum()),
        "max_prob_rel_err": float(rel.max()) if rel.size else 0.0,
        "topk_rows": topk_rows,
        "topk_sets_exact": (topk_ok / topk_rows) if topk_rows else None,
    }


def generate_control(steps, stop_tokens, max_tokens, max_seq_len):
    """The loop control of generate() (transformer/model.rs:508-531) for one
    sequence, given the token each step would sample (`steps`, in order):
    the generated tokens and why the loop ended ("stop", "max_tokens",
    "max_seq_len", or None while it would still run).  Test infrastructure:
    restates the loop with the sampler replaced by the given tokens."""
    generated = []
    pos = 0
    it = iter(steps)
    for _ in range(max_tokens):  # for _ in 0..max_tokens
        try:
            next_token = next(it)
        except StopIteration:
            return generated, None
        if next_token in stop_tokens:  # stop_tokens.contains(&next_token) -> break
            return generated, "stop"
        generated.append(next_token)  # generated.push; context.push
        pos += 1
        if pos >= max_seq_len:
            return generated, "max_seq_len"
    return generated, "max_tokens"
