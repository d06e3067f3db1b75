"""CPU restatement of the llama.cpp sampler chain that PESTI builds for its
llama.cpp backend -- TEST INFRASTRUCTURE ONLY.

Used by tests/ as the checker of pesti_llama_chain_batch; the product library
never imports this module.

The chain is the one `build_sampler` makes (llm-runner/src/llama.rs:465-508),
stage by stage and with the same gates:

  temperature    if temperature > 0             (llama.rs:468-471)
  top-k          if top_k > 0                   (llama.rs:473-476)
  top-p          if top_p > 0, min_keep 0       (llama.rs:478-481)
  min-p          if min_p > 0, min_keep 256     (llama.rs:483-486)
  top-n-sigma    n = tfs, if 0 < tfs < 1        (llama.rs:488-491)
  typical        if 0 < typical_p < 1, min_keep 0 (llama.rs:493-496)
  penalties      if repetition_penalty != 1, window repeat_last_n,
                 frequency and presence 0 in the reference (llama.rs:498-506)

The stages themselves live in llama.cpp (the llama-cpp-2 crate, version
0.1.146 in the reference's Cargo.toml:29, which wraps it), whose sources are
not in the reference tree.  They are restated here from their published
definitions:
  - temperature: logits divided by T (f32);
  - top-k: the k largest logits;
  - top-p (nucleus, Holtzman et al. 2020): the shortest prefix of the
    candidates sorted by probability whose mass reaches p;
  - min-p (Nguyen et al. 2024): tokens with p >= min_p * p_max, and at least
    min_keep of the largest;
  - top-n-sigma (Tang et al. 2024): tokens with logit >= max - n * sigma,
    sigma the standard deviation of the finite logits;
  - locally typical sampling (Meister et al. 2023): candidates sorted by
    |-log p - H| ascending, H the entropy, the shortest prefix whose mass
    reaches p;
  - repetition penalty (Keskar et al. 2019, CTRL) with frequency and
    presence penalties (OpenAI's published formula): each distinct token of
    the window that is still a candidate has its logit divided by the penalty
    when positive and multiplied by it otherwise, then lowered by
    count * frequency + (count > 0) * presence.
The chain as built ends without a selecting stage; as the Rust sampler does
(llm-runner/src/transformer/sampling.rs:97-111), the last stage here draws by
inverse CDF with the caller's uniform u over the candidates sorted by logit
(descending, ties by index), with the last candidate as the fallback.

Conventions that both this restatement and the CUDA kernel follow (llama.cpp's
own floating-point order is not known here, so parity is unpinned for this
chain): NaN logits count as -inf; probabilities are computed in f64 as
w = exp(l - max) (1 for l == max); sorts are stable, keys compared as the
ordered bit patterns of the f32 logit (+0 before -0) or of the f64 typical
deviation; a mass-based cut keeps the shortest prefix whose running f64 sum
reaches target * S (the whole list when rounding leaves the target unreached).
Every stage reports how close its decision came to a boundary, relative to the
quantities compared, so that a test can set aside rows that rounding could
flip (`margin`).
"""
from __future__ import annotations

import numpy as np

MIN_P_KEEP = 256


def desc_key(l: np.ndarray) -> np.ndarray:
    """uint32 key whose ascending order is descending f32 logit order."""
    u = np.ascontiguousarray(l, dtype=np.float32).view(np.uint32)
    asc = np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000))
    return (~asc).astype(np.uint32)


def _weights(l: np.ndarray):
    mx = np.float32(l.max())
    with np.errstate(invalid="ignore"):  # inf - inf where l == mx, masked
        d = np.where(l == mx, 0.0, l.astype(np.float64) - np.float64(mx))
    w = np.exp(d)
    return mx, d, w


def _mass_cut(order: np.ndarray, w: np.ndarray, target: float):
    """Position in `order` of the last kept element, and the relative margin."""
    cum = np.cumsum(w[order])
    total = cum[-1] if len(cum) else 0.0
    pos = int(np.searchsorted(cum, target, side="left"))
    if pos >= len(order):
        return len(order) - 1, 1.0
    lo = cum[pos - 1] if pos > 0 else 0.0
    scale = max(total, 1e-300)
    margin = min(abs(cum[pos] - target), abs(target - lo)) / scale
    if pos == 0 and target <= 0.0:
        margin = 1.0
    return pos, margin


def chain_row(logits, *, temperature=0.0, top_k=0, top_p=0.0, min_p=0.0, tfs=1.0, typical_p=1.0,
              repetition_penalty=1.0, repeat_last_n=64, frequency_penalty=0.0, presence_penalty=0.0,
              history=(), u=0.5):
    """One row through the chain.  Returns (token, kept_count, margin)."""
    x = np.asarray(logits, dtype=np.float32).copy()
    x[np.isnan(x)] = -np.inf
    if temperature > 0.0:
        x = (x / np.float32(temperature)).astype(np.float32)
    idx = np.arange(len(x), dtype=np.int64)
    l = x
    margin = 1.0

    def by_logit(l, idx):
        return np.lexsort((idx, desc_key(l)))

    if top_k > 0 and top_k < len(l):
        o = by_logit(l, idx)[:top_k]
        o.sort()
        l, idx = l[o], idx[o]
    if top_p > 0.0 and top_p < 1.0:
        _, _, w = _weights(l)
        o = by_logit(l, idx)
        pos, mg = _mass_cut(o, w, float(np.float64(np.float32(top_p)) * w.sum()))
        margin = min(margin, mg)
        o = np.sort(o[:pos + 1])
        l, idx = l[o], idx[o]
    if min_p > 0.0:
        _, d, _ = _weights(l)
        thr = np.log(np.float64(np.float32(min_p)))
        c = int(np.count_nonzero(d >= thr))
        keep = max(c, min(MIN_P_KEEP, len(l)))
        if c > 0 and keep == c:
            gap = np.abs(d[np.isfinite(d)] - thr)
            if gap.size:
                margin = min(margin, float(gap.min()) / max(abs(thr), 1.0))
        o = np.sort(by_logit(l, idx)[:keep])
        l, idx = l[o], idx[o]
    if 0.0 < tfs < 1.0:
        fin = np.isfinite(l)
        if fin.any():
            mx = np.float64(l.max())
            lf = l[fin].astype(np.float64)
            mu = lf.sum() / lf.size
            sigma = np.sqrt(((lf - mu) ** 2).sum() / lf.size)
            thr = mx - np.float64(np.float32(tfs)) * sigma
            keepm = l.astype(np.float64) >= thr
            gap = np.abs(l[fin].astype(np.float64) - thr)
            if np.isfinite(thr) and sigma > 0:
                margin = min(margin, float(gap.min()) / max(abs(thr), sigma, 1.0))
            l, idx = l[keepm], idx[keepm]
    if 0.0 < typical_p < 1.0:
        mx, d, w = _weights(l)
        S = w.sum()
        lnS = np.log(S)
        H = lnS - np.where(w > 0, w * d, 0.0).sum() / S
        dev = np.abs(lnS - d - H)
        key = dev.astype(np.float64).view(np.uint64)
        o = np.lexsort((idx, key))
        pos, mg = _mass_cut(o, w, float(np.float64(np.float32(typical_p)) * S))
        margin = min(margin, mg)
        # the pair at the cut, which rounding of H or log S could reorder
        # (equal logits have equal deviations on both sides)
        if pos + 1 < len(o) and d[o[pos + 1]] != d[o[pos]]:
            gap = float(abs(dev[o[pos + 1]] - dev[o[pos]]))
            margin = min(margin, gap / max(abs(H), 1.0))
        o = np.sort(o[:pos + 1])
        l, idx = l[o], idx[o]
    if repetition_penalty != 1.0 and repeat_last_n != 0:
        hist = list(history)
        win = hist if repeat_last_n < 0 else hist[max(0, len(hist) - repeat_last_n):]
        counts = {}
        for t in win:
            counts[int(t)] = counts.get(int(t), 0) + 1
        pos_of = {int(t): i for i, t in enumerate(idx)}
        l = l.copy()
        rp = np.float32(repetition_penalty)
        fq = np.float32(frequency_penalty)
        pr = np.float32(presence_penalty)
        for t, c in counts.items():
            i = pos_of.get(t)
            if i is None:
                continue
            v = l[i]
            v = np.float32(v * rp) if v <= 0 else np.float32(v / rp)
            sub = np.float32(np.float32(np.float32(c) * fq) + (pr if c > 0 else np.float32(0)))
            l[i] = np.float32(v - sub)
    _, _, w = _weights(l)
    o = np.lexsort((idx, desc_key(l)))
    pos, mg = _mass_cut(o, w, float(np.float64(np.float32(u)) * w.sum()))
    margin = min(margin, mg)
    return int(idx[o[pos]]), int(len(l)), float(margin)


def chain_batch(logits: np.ndarray, params: dict, history=None, u=None):
    """Rows of a [B, V] batch through the chain with one parameter set."""
    B = logits.shape[0]
    toks = np.zeros(B, dtype=np.int64)
    kept = np.zeros(B, dtype=np.int64)
    margins = np.zeros(B, dtype=np.float64)
    for b in range(B):
        h = () if history is None else history[b]
        toks[b], kept[b], margins[b] = chain_row(logits[b], history=h, u=float(u[b]), **params)
    return toks, kept, margins
