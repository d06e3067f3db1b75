"""CPU restatement of the vocabulary-sharded sampling protocol -- TEST INFRASTRUCTURE ONLY.

The sharded path (pesti_sample_batch_sharded) never moves logits between
ranks: each rank holds one contiguous, equally wide column range of every row
and exchanges three small per-row records.  The reference has no such path;
what must hold is that its results are those of sampling.rs:39-134 on the
whole row.  This module restates the protocol's arithmetic with the oracle's
exact exps and sequential folds, so that the protocol itself (the chain of
shard folds and the candidate bound) can be checked on CPU ranks against the
whole-row oracle.  It is not the product: the CUDA kernels implement the same
steps on the device.

The softmax denominator is one f32 fold over the whole row in index order
(sampling.rs:126-128), so shard r's part of it is a function F_r of the fold
state s_r at its first column: s_0 = 0, s_{r+1} = F_r(s_r), S = s_G.
  1. summary: each shard's raw max and approximate mass (relative to it);
  2. record: the exact increment delta_r = F_r(start_r) - start_r from an
     approximate start (the true mass of the earlier shards), plus the
     shard's top candidates by (exp desc, column asc) and a bound on the rest;
  3. table: F_r at TAB_W consecutive floats around the chained increments;
  4. finish: the tables chained from s_0 = 0 give S exactly; the merged
     candidates give the top-k, then total, normalisation and draw
     (sampling.rs:59-111).  None means the row needs the gathered path.
"""
from __future__ import annotations

import numpy as np

import oracle as O

TAB_W, TAB_BELOW = 32, 16


def f32_bits(x) -> int:
    return int(np.array([x], dtype=np.float32).view(np.uint32)[0])


def bits_f32(b: int) -> np.float32:
    return np.array([b], dtype=np.uint32).view(np.float32)[0]


def scaled_max(gmx: float, T: float) -> np.float32:
    """m of sampling.rs:126: the division is monotone, so the max of the
    scaled row is the scaled raw max (sampling.rs:46)."""
    return np.float32(np.float32(gmx) / np.float32(T)) if T > 0 else np.float32(gmx)


def summary(x_shard: np.ndarray, T: float):
    """Phase 1: (raw max, approximate mass relative to it)."""
    mx = float(np.max(x_shard))
    t = T if T > 0 else 1.0
    return mx, float(np.sum(np.exp((x_shard.astype(np.float64) - mx) / t)))


def record(x_shard: np.ndarray, col0: int, T: float, sums, rank: int, ksh: int):
    """Phase 2: (delta, start, candidates [(e, column)], bound)."""
    gmx = max(mr for mr, _ in sums)
    t = T if T > 0 else 1.0
    m = scaled_max(gmx, T)
    start = np.float32(sum(ms * np.exp((mr - gmx) / t) for mr, ms in sums[:rank]))
    e = O.softmax_terms(x_shard, T, m)
    delta = float(O.fold(e, start)) - float(start)
    order = np.lexsort((np.arange(e.size), -e.astype(np.float64)))
    cands = [(np.float32(e[i]), col0 + int(i)) for i in order[:ksh]]
    bound = np.float32(e[order[ksh]]) if e.size > ksh else np.float32(0.0)
    return delta, start, cands, bound


def table(x_shard: np.ndarray, T: float, gmx: float, deltas, rank: int):
    """Phase 3: (base, [F_r(bits base + j) for j < TAB_W]) around the chained estimate."""
    eb = f32_bits(np.float32(sum(deltas[:rank])))
    base = eb - TAB_BELOW if eb >= TAB_BELOW else 0
    e = O.softmax_terms(x_shard, T, scaled_max(gmx, T))
    return base, [f32_bits(O.fold(e, bits_f32(base + j))) for j in range(TAB_W)]


def finish(tables, records, k: int, u: float):
    """Phase 4: (S, token, kept [(p, column)]) or None (gathered path)."""
    s = 0
    for base, tab in tables:
        j = s - base
        if not 0 <= j < TAB_W:
            return None
        s = tab[j]
    S = bits_f32(s)
    merged = [(np.float32(e / S), col) for (_, _, cands, _) in records for (e, col) in cands]
    merged.sort(key=lambda pc: (-float(pc[0]), pc[1]))  # the stable sort of sampling.rs:60
    if len(merged) < k:
        return None
    pk = merged[k - 1][0]
    if not all(np.float32(bound / S) < pk for (_, _, _, bound) in records):
        return None
    kept = merged[:k]
    total = O.fold(np.array([p for p, _ in kept], np.float32))               # sampling.rs:81
    q = np.array([np.float32(p / total) for p, _ in kept], np.float32)       # sampling.rs:94
    cum = np.float32(0.0)
    for j in range(k):                                                       # sampling.rs:99-111
        cum = np.float32(cum + q[j])
        if np.float32(u) <= cum:
            return S, kept[j][1], kept
    return S, kept[-1][1], kept
