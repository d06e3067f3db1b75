"""Seeded synthetic workloads for the sampler (the five benchmark configurations).

The reference publishes no benchmark inputs; these generators produce logits
with the stated shapes, dtypes and distributions.  Everything is a pure
function of (workload, seed), computed with numpy on the host, so the CUDA
path and the CPU oracle see identical bytes.

Normal deviates: a counter-based generator.  Element i of a workload with data
seed D takes two 53-bit uniforms from splitmix64(D*2^40 + 2i) and
splitmix64(D*2^40 + 2i + 1) and maps them with Box-Muller (cosine branch) in
float64, then rounds once to float32 (or to bfloat16, round-to-nearest-even).

Draws u: one PCG32 stream per workload (seed = workload number - 1, PCG
stream 54), u_b = (next_u32() >> 8) * 2^-24 for b = 0..B-1 in row order.

Choices that are this generator's own (the workload text leaves them open):
  * workload 2's Zipf bias: bias[perm[r-1]] = -1.1*ln(r) for rank r = 1..V, with
    perm the argsort of splitmix64 hashes of the column index (per row);
  * workload 1's 32 boosted indices per row: the 32 smallest hashes of the row;
  * workload 5's boosted entries: hash < 0.001 * 2^64;
  * workload 4's row classes: by row index mod 20 (see ROW_CLASSES_4).
"""
from __future__ import annotations

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def splitmix64(x: np.ndarray) -> np.ndarray:
    z = (x + np.uint64(0x9E3779B97F4A7C15)) & _M64
    z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & _M64
    z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & _M64
    return z ^ (z >> np.uint64(31))


def _u53(h: np.ndarray) -> np.ndarray:
    return (h >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def normals(seed: int, start: int, count: int) -> np.ndarray:
    """float64 standard normals for element indices [start, start+count)."""
    with np.errstate(over="ignore"):
        base = np.uint64(seed) << np.uint64(40)
        i = np.arange(start, start + count, dtype=np.uint64)
        h1 = splitmix64(base + np.uint64(2) * i)
        h2 = splitmix64(base + np.uint64(2) * i + np.uint64(1))
    u1 = 1.0 - _u53(h1)  # (0, 1]
    u2 = _u53(h2)
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)


def row_hash(seed: int, row: int, V: int, salt: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        base = (np.uint64(seed) << np.uint64(40)) ^ (np.uint64(salt) << np.uint64(56)) ^ (np.uint64(row) << np.uint64(20))
        return splitmix64(base ^ (np.arange(V, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)))


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    out = ((u + r) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(x)
    out[nan] = np.uint16(0x7FC0)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def pcg32_draws(seed: int, n: int, stream: int = 54) -> np.ndarray:
    mult, mask = 6364136223846793005, (1 << 64) - 1
    inc = ((stream << 1) | 1) & mask
    state = 0

    def step(st):
        return (st * mult + inc) & mask

    state = step(state)
    state = (state + seed) & mask
    state = step(state)
    out = np.empty(n, dtype=np.float32)
    for k in range(n):
        old = state
        state = step(old)
        xs = (((old >> 18) ^ old) >> 27) & 0xFFFFFFFF
        rot = old >> 59
        v = ((xs >> rot) | (xs << ((-rot) & 31))) & 0xFFFFFFFF
        out[k] = np.float32((v >> 8) * (1.0 / (1 << 24)))
    return out


# (temperature, top_p, top_k, duplicate maxima) per class r % 20 of workload 4
ROW_CLASSES_4 = {
    0: (0.0, 0.0, 0, True), 1: (0.0, 0.0, 0, False), 2: (0.0, 0.0, 0, False),
    3: (0.0, 0.0, 0, False), 4: (0.0, 0.0, 0, False), 5: (0.0, 0.0, 0, False),
    6: (0.0, 0.0, 0, False), 7: (0.0, 0.0, 0, False), 8: (0.0, 0.0, 0, False),
    9: (0.0, 0.0, 0, False),
    10: (0.8, 0.0, 1, True), 11: (0.8, 0.0, 1, False),
    12: (1.0, 0.0, -1, False), 13: (1.0, 0.0, -1, False),   # top_k = V
    14: (0.9, 1.0, 0, False), 15: (0.9, 1.0, 0, False),     # top-p 1.0
    16: (1.1, 1e-6, 0, False), 17: (1.1, 1e-6, 0, False),   # top-p 1e-6
    18: (0.7, 0.0, 0, False),                               # no filter (index-order draw)
    19: (1.0, 0.5, 40, False),                              # top-k with top-p ignored
}

WORKLOADS = {
    1: dict(name="single-row [1000 x 32000] f32, T0.8 k40 p0.95", B=1000, V=32000, dtype="f32"),
    2: dict(name="batched [64 x 128256] f32, T0.7 k50 p0.9", B=64, V=128256, dtype="f32"),
    3: dict(name="nucleus [256 x 152064] bf16, T1.0 k0 p0.95", B=256, V=152064, dtype="bf16"),
    4: dict(name="greedy+edge [512 x 32768] f32, mixed", B=512, V=32768, dtype="f32"),
    5: dict(name="vocab-sharded [1024 x 256000] f32, T0.9 k64 p0.92", B=1024, V=256000, dtype="f32"),
}


def params_for(w: int, B: int, V: int):
    """Per-row (temperature, top_p, top_k) lists for workload w."""
    if w == 1:
        return [(0.8, 0.95, 40)] * B
    if w == 2:
        return [(0.7, 0.9, 50)] * B
    if w == 3:
        return [(1.0, 0.95, 0)] * B
    if w == 5:
        return [(0.9, 0.92, 64)] * B
    out = []
    for r in range(B):
        t, p, k, _ = ROW_CLASSES_4[r % 20]
        out.append((t, p, V if k < 0 else k))
    return out


def make_logits(w: int, B: int = None, V: int = None, rows=None, cols=None) -> np.ndarray:
    """float32 logits of workload w ([B, V], or the rows `rows` and columns
    `cols` (a range) of it); for workload 3 the values are already
    bf16-representable (use f32_to_bf16_bits for the device copy)."""
    spec = WORKLOADS[w]
    B = spec["B"] if B is None else B
    V = spec["V"] if V is None else V
    seed = 100 + w
    rows = range(B) if rows is None else rows
    if cols is not None:
        if w == 5:  # element-wise generator: only the columns asked for
            out = np.empty((len(rows), len(cols)), dtype=np.float32)
            for o, r in enumerate(rows):
                z = normals(seed, r * V + cols.start, len(cols))
                boost = row_hash(seed, r, V, 5)[cols.start:cols.stop] < np.uint64(int(0.001 * 2**64))
                out[o] = (z * 2.5 + 6.0 * boost).astype(np.float32)
            return out
        return np.ascontiguousarray(make_logits(w, B, V, rows)[:, cols.start:cols.stop])
    out = np.empty((len(rows), V), dtype=np.float32)
    for o, r in enumerate(rows):
        z = normals(seed, r * V, V)
        if w == 1:
            x = (z * 2.0).astype(np.float32)
            h = row_hash(seed, r, V, 1)
            idx = np.argpartition(h, 32)[:32]
            x[idx] = (x[idx].astype(np.float64) + 8.0).astype(np.float32)
        elif w == 2:
            h = row_hash(seed, r, V, 2)
            perm = np.argsort(h, kind="stable")
            bias = np.empty(V, dtype=np.float64)
            bias[perm] = -1.1 * np.log(np.arange(1, V + 1, dtype=np.float64))
            x = (z * 3.0 + bias).astype(np.float32)
        elif w == 3:
            x = bf16_bits_to_f32(f32_to_bf16_bits((z * 1.5).astype(np.float32)))
        elif w == 4:
            x = z.astype(np.float32)
            if ROW_CLASSES_4[r % 20][3]:
                h = row_hash(seed, r, V, 4)
                mx = x.max()
                dup = np.argpartition(h, 2)[:2]
                x[dup] = mx
        elif w == 5:
            x = z * 2.5
            h = row_hash(seed, r, V, 5)
            boost = h < np.uint64(int(0.001 * 2**64))
            x = (x + 6.0 * boost).astype(np.float32)
        else:
            raise ValueError(w)
        out[o] = x
    return out


def make_u(w: int, B: int = None) -> np.ndarray:
    spec = WORKLOADS[w]
    B = spec["B"] if B is None else B
    return pcg32_draws(w - 1, B)
