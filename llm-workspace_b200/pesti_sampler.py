"""Host-side mirror of the reference sampler API over the sm_100a C ABI.

The reference (Rust) exposes, in llm-runner/src/transformer/sampling.rs:
    pub struct SamplingConfig { temperature: f32, top_p: f32, top_k: usize, seed: Option<u64> }  (:12-21)
    impl Default for SamplingConfig -> T=0.7, top_p=0.9, top_k=0, seed=None                      (:23-32)
    pub fn sample(logits: &[f32], config: &SamplingConfig, rng: &mut StdRng) -> u32              (:39)
    pub fn argmax(logits: &[f32]) -> u32                                                          (:115)
and its callers branch on `temperature == 0.0` (transformer/model.rs:517-521).

This module keeps those names and meanings and adds the batched form the
decode loop needs (`Sampler.sample_batch`, rows of a [B, V] device tensor).
Every call runs the CUDA kernels of libpesti_sampler.so; there is no CPU
path: without the library or a B200 the calls raise.

`rng` stands for the reference's StdRng: any object with `next_f32()`
returning the next uniform draw in [0, 1) (sampling.rs:98 draws exactly one
per `sample` call and none for argmax).  `Pcg32` below is the generator the
benchmarks and tests use.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from typing import Optional, Sequence, Union

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpesti_sampler.so")
CSRC = os.path.join(_HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(_HERE), "include")

PESTI_OK = 0
PESTI_E_INVALID_ARG = -1
PESTI_E_CUDA = -2
PESTI_E_NCCL = -3
PESTI_E_TIMEOUT = -4
PESTI_E_UNSUPPORTED = -5
PESTI_E_NO_DEVICE = -6

PESTI_F32 = 0
PESTI_BF16 = 1
PESTI_F16 = 2
PESTI_FP8_E4M3 = 3  # sample_batch and argmax_batch only (widened exactly to f16 first)
PESTI_FP8_E5M2 = 4

FLAG_GREEDY_IF_ZERO_T = 1
FLAG_ARGMAX_FIRST = 2

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def build(verbose: bool = False) -> str:
    """Compiles csrc/ into libpesti_sampler.so for sm_100a (in-tree)."""
    srcs = [os.path.join(CSRC, "pesti_sampler.cu"), os.path.join(CSRC, "pesti_noalloc.cu")]
    cmd = ["nvcc", *NVCC_FLAGS, "-o", LIB_PATH, *srcs, "-ldl"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    return LIB_PATH


class SamplerError(RuntimeError):
    """A failed library call: `code` is the PESTI_E_* value."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"pesti error {code}: {msg}")
        self.code = code


class _Params(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_float), ("top_p", ctypes.c_float),
                ("top_k", ctypes.c_uint32), ("flags", ctypes.c_uint32)]


_lib = None


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads the sampler library; raises if it is missing (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"{path} is missing: build it with __graft_entry__.build() (there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    vp, i64, c_int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.pesti_sampler_create.argtypes = [c_int, ctypes.POINTER(vp)]
    lib.pesti_sampler_create.restype = c_int
    lib.pesti_sampler_destroy.argtypes = [vp]
    lib.pesti_sampler_destroy.restype = None
    lib.pesti_sample_batch.argtypes = [vp, vp, c_int, i64, i64, i64, ctypes.POINTER(_Params), c_int,
                                       c_int, vp, vp, vp, vp, i64, vp, vp]
    lib.pesti_sample_batch.restype = c_int
    lib.pesti_argmax_batch.argtypes = [vp, vp, c_int, i64, i64, i64, ctypes.c_uint32, vp, vp]
    lib.pesti_argmax_batch.restype = c_int
    lib.pesti_sample_row_host.argtypes = [vp, ctypes.POINTER(ctypes.c_float), i64,
                                          ctypes.POINTER(_Params), ctypes.c_float,
                                          ctypes.POINTER(ctypes.c_uint32)]
    lib.pesti_sample_row_host.restype = c_int
    lib.pesti_sample_batch_noalloc.argtypes = [vp, c_int, i64, i64, i64, ctypes.POINTER(_Params), c_int,
                                               c_int, vp, vp, vp, vp, i64, vp, vp]
    lib.pesti_sample_batch_noalloc.restype = c_int
    lib.pesti_last_error.argtypes = []
    lib.pesti_last_error.restype = ctypes.c_char_p
    lib.pesti_comm_id.argtypes = [vp]
    lib.pesti_comm_id.restype = c_int
    lib.pesti_comm_create.argtypes = [c_int, c_int, vp, c_int, ctypes.POINTER(vp)]
    lib.pesti_comm_create.restype = c_int
    lib.pesti_comm_create_timed.argtypes = [c_int, c_int, vp, c_int, c_int, ctypes.POINTER(vp)]
    lib.pesti_comm_create_timed.restype = c_int
    lib.pesti_comm_destroy.argtypes = [vp]
    lib.pesti_comm_destroy.restype = None
    lib.pesti_sample_batch_sharded.argtypes = [vp, vp, vp, c_int, i64, i64, i64, ctypes.POINTER(_Params), c_int,
                                               c_int, vp, vp, vp, vp, i64, vp, vp]
    lib.pesti_sample_batch_sharded.restype = c_int
    lib.pesti_sample_batch_sharded_emulated.argtypes = [vp, c_int, vp, c_int, i64, i64, i64, ctypes.POINTER(_Params),
                                                        c_int, c_int, vp, vp, vp, vp, i64, vp, vp]
    lib.pesti_sample_batch_sharded_emulated.restype = c_int
    lib.pesti_pcg32_seed.argtypes = [vp, i64, ctypes.c_uint64, ctypes.c_uint64, vp]
    lib.pesti_pcg32_seed.restype = c_int
    lib.pesti_pcg32_draw.argtypes = [vp, i64, vp, vp]
    lib.pesti_pcg32_draw.restype = c_int
    lib.pesti_generate_advance.argtypes = [vp, i64, vp, i64, i64, i64, vp, i64, vp, vp, vp, vp, vp]
    lib.pesti_generate_advance.restype = c_int
    lib.pesti_llama_chain_batch.argtypes = [vp, vp, c_int, i64, i64, i64, ctypes.POINTER(LlamaChainParams), vp, vp,
                                            i64, vp, vp, vp, vp]
    lib.pesti_llama_chain_batch.restype = c_int
    lib.pesti_last_gathered_rows.argtypes = [vp]
    lib.pesti_last_gathered_rows.restype = i64
    lib.pesti_last_gathered_reasons.argtypes = [vp, vp]
    lib.pesti_last_gathered_reasons.restype = c_int
    lib.pesti_testing_set_cluster.argtypes = [c_int]
    lib.pesti_testing_set_cluster.restype = c_int
    _lib = lib
    return lib


def _check(rc: int) -> None:
    if rc != PESTI_OK:
        raise SamplerError(rc, load_library().pesti_last_error().decode())


@dataclass
class SamplingConfig:
    """sampling.rs:12-32 (defaults included)."""
    temperature: float = 0.7
    top_p: float = 0.9
    top_k: int = 0
    seed: Optional[int] = None

    def to_params(self, greedy_if_zero_t: bool = False, argmax_first: bool = False) -> _Params:
        flags = (FLAG_GREEDY_IF_ZERO_T if greedy_if_zero_t else 0) | (FLAG_ARGMAX_FIRST if argmax_first else 0)
        return _Params(float(self.temperature), float(self.top_p), int(self.top_k), flags)


class LlamaChainParams(ctypes.Structure):
    """pesti_llama_chain_params: the fields of the llama.cpp backend's
    SamplingConfig (llm-runner/src/llama/sampler.rs:19-79) that build_sampler
    (llm-runner/src/llama.rs:465-508) reads.  Defaults are that config's."""
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_int32), ("top_p", ctypes.c_float),
                ("min_p", ctypes.c_float), ("tfs", ctypes.c_float), ("typical_p", ctypes.c_float),
                ("repetition_penalty", ctypes.c_float), ("repeat_last_n", ctypes.c_int32),
                ("frequency_penalty", ctypes.c_float), ("presence_penalty", ctypes.c_float)]

    def __init__(self, temperature=0.7, top_k=40, top_p=0.95, min_p=0.0, tfs=1.0, typical_p=1.0,
                 repetition_penalty=1.0, repeat_last_n=64, frequency_penalty=0.0, presence_penalty=0.0):
        super().__init__(temperature, top_k, top_p, min_p, tfs, typical_p, repetition_penalty, repeat_last_n,
                         frequency_penalty, presence_penalty)

    def as_dict(self) -> dict:
        return {f: getattr(self, f) for f, _ in self._fields_}

    # the presets of llm-runner/src/llama/sampler.rs:116-173
    @classmethod
    def greedy(cls) -> "LlamaChainParams":
        return cls(temperature=0.0, top_k=1, top_p=0.0, min_p=0.0, tfs=1.0, typical_p=1.0, repetition_penalty=1.0)

    @classmethod
    def creative(cls) -> "LlamaChainParams":
        return cls(temperature=1.0, top_k=50, top_p=0.99, min_p=0.05, tfs=0.5, typical_p=0.5)

    @classmethod
    def balanced(cls) -> "LlamaChainParams":
        return cls(temperature=0.7, top_k=40, top_p=0.95, min_p=0.0, tfs=1.0, typical_p=1.0)

    @classmethod
    def precise(cls) -> "LlamaChainParams":
        return cls(temperature=0.3, top_k=20, top_p=0.9, min_p=0.1, tfs=1.0, typical_p=1.0,
                   repetition_penalty=1.1, repeat_last_n=128)


class PreparedParams:
    """Per-row sampling parameters converted once into the C layout, for
    callers that sample many batches with the same rows' configs: pass it to
    the batch calls in place of the list (converting a long list on every
    call costs host time comparable to the GPU step)."""

    def __init__(self, configs: Sequence[SamplingConfig], greedy_if_zero_t: bool = True,
                 argmax_first: bool = False):
        self.rows = len(configs)
        self.greedy_if_zero_t = greedy_if_zero_t
        self.argmax_first = argmax_first
        self.arr = (_Params * self.rows)(*[c.to_params(greedy_if_zero_t, argmax_first) for c in configs])


class Pcg32:
    """PCG32 (O'Neill 2014, XSH-RR 64->32) with the reference's f32 draw.

    next_f32() = (next_u32() >> 8) * 2^-24: the [0,1) 24-bit grid that rand's
    `random::<f32>()` produces (sampling.rs:98).
    """

    MULT = 6364136223846793005
    MASK = (1 << 64) - 1

    def __init__(self, seed: int, stream: int = 54):
        self.state = 0
        self.inc = ((stream << 1) | 1) & self.MASK
        self.next_u32()
        self.state = (self.state + seed) & self.MASK
        self.next_u32()

    def next_u32(self) -> int:
        old = self.state
        self.state = (old * self.MULT + self.inc) & self.MASK
        xs = (((old >> 18) ^ old) >> 27) & 0xFFFFFFFF
        rot = old >> 59
        return ((xs >> rot) | (xs << ((-rot) & 31))) & 0xFFFFFFFF

    def next_f32(self) -> float:
        return float(self.next_u32() >> 8) * (1.0 / (1 << 24))

    def draws(self, n: int):
        import numpy as np
        return np.array([self.next_f32() for _ in range(n)], dtype=np.float32)


class DeviceRng:
    """Per-row PCG32 generators on the device (pesti_pcg32_seed /
    pesti_pcg32_draw): row b's draws are those of Pcg32(seed, first_stream + b)
    in sequence, produced where the batch calls read them, with no host copy."""

    def __init__(self, B: int, seed: int, first_stream: int = 0, device: int = 0, stream=None):
        import torch
        self._lib = load_library()
        self.B = int(B)
        self.state = torch.empty((self.B, 2), dtype=torch.int64, device=f"cuda:{device}")
        st = stream if stream is not None else torch.cuda.current_stream(self.state.device).cuda_stream
        _check(self._lib.pesti_pcg32_seed(self.state.data_ptr(), self.B, int(seed) & ((1 << 64) - 1),
                                          int(first_stream) & ((1 << 64) - 1), st))

    def draw(self, out=None, stream=None):
        """The next draw of every row: a [B] float32 CUDA tensor."""
        import torch
        if out is None:
            out = torch.empty(self.B, dtype=torch.float32, device=self.state.device)
        st = stream if stream is not None else torch.cuda.current_stream(self.state.device).cuda_stream
        _check(self._lib.pesti_pcg32_draw(self.state.data_ptr(), self.B, out.data_ptr(), st))
        return out


class DecodeState:
    """The loop control of generate() (transformer/model.rs:508-531) for B
    sequences on the device (pesti_generate_advance): after each step's
    sample, advance(tokens) keeps the tokens on the GPU and finishes rows on
    a stop token, after max_tokens tokens, or at max_seq_len.  `last` is the
    next step's input token per row; `active()` reads the number of rows
    still running (a host read: call it now and then, not every step)."""

    def __init__(self, B: int, max_tokens: int, max_seq_len: int, stop_tokens=(), device=0):
        import torch
        self._lib = load_library()
        self.B, self.max_tokens, self.max_seq_len = int(B), int(max_tokens), int(max_seq_len)
        self.cap = max(1, min(self.max_tokens, self.max_seq_len))
        dev = torch.device("cuda", device)
        self.generated = torch.zeros(self.B, self.cap, dtype=torch.int32, device=dev)
        self.count = torch.zeros(self.B, dtype=torch.int32, device=dev)
        self.done = torch.zeros(self.B, dtype=torch.uint8, device=dev)
        self.last = torch.zeros(self.B, dtype=torch.int32, device=dev)
        self._active = torch.zeros(1, dtype=torch.int32, device=dev)
        self.stop = torch.tensor(list(stop_tokens) or [0], dtype=torch.int64).to(torch.int32).to(dev)
        self.n_stop = len(stop_tokens)

    def advance(self, tokens, stream=None):
        """Takes the step's [B] sampled tokens (int32 u32 bits, on the device)."""
        import torch
        st = stream if stream is not None else torch.cuda.current_stream(tokens.device).cuda_stream
        _check(self._lib.pesti_generate_advance(
            tokens.data_ptr(), self.B, self.stop.data_ptr(), self.n_stop, self.max_tokens, self.max_seq_len,
            self.generated.data_ptr(), self.cap, self.count.data_ptr(), self.done.data_ptr(), self.last.data_ptr(),
            self._active.data_ptr(), st))

    def active(self) -> int:
        return int(self._active.item())

    def sequences(self):
        """The generated tokens of every row (lists of ints, u32)."""
        g = self.generated.cpu().numpy().view("uint32")
        c = self.count.cpu().numpy()
        return [list(map(int, g[b, :c[b]])) for b in range(self.B)]


class Sampler:
    """A device-bound sampler handle (pesti_sampler_create / _destroy)."""

    def __init__(self, device: int = 0):
        lib = load_library()
        h = ctypes.c_void_p()
        _check(lib.pesti_sampler_create(int(device), ctypes.byref(h)))
        self._h = h
        self._lib = lib
        self.device = device

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.pesti_sampler_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- batched API (device tensors) --------------------------------------
    def sample_batch(self, logits, configs: Union[SamplingConfig, Sequence[SamplingConfig]], u,
                     out=None, greedy_if_zero_t: bool = True, argmax_first: bool = False,
                     kept_width: int = 0, stream=None):
        """Samples one token per row of `logits` ([B, V] f32 or bf16 CUDA tensor).

        configs: one SamplingConfig for all rows or one per row.  u: [B] f32
        CUDA tensor of draws.  Returns the [B] int32 token tensor (u32 bits),
        or (tokens, kept_p, kept_idx, kept_count) when kept_width > 0.
        """
        B, V, dtype, arr, per_row, out, kp, ki, kc, st = _batch_args(
            logits, configs, out, greedy_if_zero_t, argmax_first, kept_width, stream)
        _check(self._lib.pesti_sample_batch(
            self._h, logits.data_ptr(), dtype, B, V, logits.stride(0), arr, per_row, 0,
            u.data_ptr(), out.data_ptr(), _ptr(kp), _ptr(ki), kept_width, _ptr(kc), st))
        if kept_width > 0:
            return out, kp, ki, kc
        return out

    def sample_batch_sharded(self, comm: "Comm", logits_shard, configs, u, out=None,
                             greedy_if_zero_t: bool = True, argmax_first: bool = False,
                             kept_width: int = 0, stream=None):
        """pesti_sample_batch_sharded: `logits_shard` is this rank's column range
        [B, V_shard] of rows that are comm.world * V_shard long (rank r holds
        columns [r*V_shard, (r+1)*V_shard)).  Every rank passes the same
        configs and u ([B], all rows) and receives the results of all B rows.
        """
        B, Vs, dtype, arr, per_row, out, kp, ki, kc, st = _batch_args(
            logits_shard, configs, out, greedy_if_zero_t, argmax_first, kept_width, stream)
        _check(self._lib.pesti_sample_batch_sharded(
            self._h, comm._h, logits_shard.data_ptr(), dtype, B, Vs, logits_shard.stride(0), arr, per_row, 0,
            u.data_ptr(), out.data_ptr(), _ptr(kp), _ptr(ki), kept_width, _ptr(kc), st))
        if kept_width > 0:
            return out, kp, ki, kc
        return out

    def sample_batch_sharded_emulated(self, logits, configs, u, shards: int, out=None,
                                      greedy_if_zero_t: bool = True, argmax_first: bool = False,
                                      kept_width: int = 0, stream=None):
        """The sharded algorithm over `shards` equal column ranges of the whole
        matrix `logits`, all on this device (pesti_testing.h)."""
        B, V, dtype, arr, per_row, out, kp, ki, kc, st = _batch_args(
            logits, configs, out, greedy_if_zero_t, argmax_first, kept_width, stream)
        _check(self._lib.pesti_sample_batch_sharded_emulated(
            self._h, int(shards), logits.data_ptr(), dtype, B, V, logits.stride(0), arr, per_row, 0,
            u.data_ptr(), out.data_ptr(), _ptr(kp), _ptr(ki), kept_width, _ptr(kc), st))
        if kept_width > 0:
            return out, kp, ki, kc
        return out

    def last_gathered_rows(self) -> int:
        """Rows of the last sharded call that took the gathered path."""
        return int(self._lib.pesti_last_gathered_rows(self._h))

    GATHER_REASONS = ("", "row kind", "fold entries", "candidates", "chain", "top-k bound")

    def last_gathered_reasons(self) -> dict:
        """Those rows by reason (pesti_testing.h)."""
        c = (ctypes.c_int64 * 6)()
        _check(self._lib.pesti_last_gathered_reasons(self._h, c))
        return {n: int(c[i]) for i, n in enumerate(self.GATHER_REASONS) if i and c[i]}

    def sample_batch_device_params(self, logits, d_params, u, out, stream=None):
        """Per-row parameters already on the device (a [B, 4] int32/f32 view of
        pesti_sampling_params records)."""
        import torch
        B, V = logits.shape
        dtype = _dtype_of(logits)
        st = stream if stream is not None else torch.cuda.current_stream(logits.device).cuda_stream
        _check(self._lib.pesti_sample_batch(
            self._h, logits.data_ptr(), dtype, B, V, logits.stride(0),
            ctypes.cast(ctypes.c_void_p(d_params.data_ptr()), ctypes.POINTER(_Params)), 1, 1,
            u.data_ptr(), out.data_ptr(), None, None, 0, None, st))
        return out

    def argmax_batch(self, logits, first: bool = False, out=None, stream=None):
        """sampling.rs:115-122 over each row (last of equal maxima unless first)."""
        import torch
        B, V = logits.shape
        dtype = _dtype_of(logits)
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=logits.device)
        st = stream if stream is not None else torch.cuda.current_stream(logits.device).cuda_stream
        _check(self._lib.pesti_argmax_batch(self._h, logits.data_ptr(), dtype, B, V, logits.stride(0),
                                            FLAG_ARGMAX_FIRST if first else 0, out.data_ptr(), st))
        return out

    def llama_chain_batch(self, logits, params: LlamaChainParams, u, history=None, history_len=None,
                          out=None, kept=None, stream=None):
        """pesti_llama_chain_batch: the llama.cpp backend's sampler chain
        (llama.rs:465-508) over each row of `logits` ([B, V] CUDA tensor, f32,
        bf16, f16 or fp8).  history: [B, H] int32 CUDA tensor of recent tokens
        (oldest first) for the penalties, history_len: optional [B] int32.
        Returns the [B] int32 tokens, and `kept` ([B] int32, candidates left
        before the draw) filled when given."""
        import torch
        B, V = logits.shape
        dtype = _dtype_of(logits)
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=logits.device)
        st = stream if stream is not None else torch.cuda.current_stream(logits.device).cuda_stream
        hld = 0
        if history is not None:
            if history.dim() != 2 or history.shape[0] != B or not history.is_contiguous():
                raise ValueError("history must be a contiguous [B, H] tensor")
            hld = history.shape[1]
        _check(self._lib.pesti_llama_chain_batch(
            self._h, logits.data_ptr(), dtype, B, V, logits.stride(0), ctypes.byref(params),
            _ptr(history), _ptr(history_len), hld, u.data_ptr(), out.data_ptr(), _ptr(kept), st))
        return out

    # -- single row from host memory (the reference's own signature) -------
    def sample(self, logits, config: SamplingConfig, rng, greedy_if_zero_t: bool = False) -> int:
        """sample(&logits, &config, &mut rng) (sampling.rs:39): one draw from rng."""
        import numpy as np
        x = np.ascontiguousarray(np.asarray(logits, dtype=np.float32))
        r = rng.next_f32()
        tok = ctypes.c_uint32()
        p = config.to_params(greedy_if_zero_t)
        _check(self._lib.pesti_sample_row_host(
            self._h, x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), int(x.size), ctypes.byref(p),
            ctypes.c_float(r), ctypes.byref(tok)))
        return int(tok.value)

    def sample_with_u(self, logits, config: SamplingConfig, u: float, greedy_if_zero_t: bool = False) -> int:
        import numpy as np
        x = np.ascontiguousarray(np.asarray(logits, dtype=np.float32))
        tok = ctypes.c_uint32()
        p = config.to_params(greedy_if_zero_t)
        _check(self._lib.pesti_sample_row_host(
            self._h, x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), int(x.size), ctypes.byref(p),
            ctypes.c_float(u), ctypes.byref(tok)))
        return int(tok.value)

    def argmax(self, logits) -> int:
        """argmax(&logits) (sampling.rs:115): greedy, no draw."""
        import numpy as np
        x = np.ascontiguousarray(np.asarray(logits, dtype=np.float32))
        tok = ctypes.c_uint32()
        p = _Params(0.0, 0.0, 0, FLAG_GREEDY_IF_ZERO_T)
        _check(self._lib.pesti_sample_row_host(
            self._h, x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), int(x.size), ctypes.byref(p),
            ctypes.c_float(0.0), ctypes.byref(tok)))
        return int(tok.value)


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _dtype_of(logits) -> int:
    """pesti_dtype of a logits tensor (float32, bfloat16, float16, or the fp8
    formats float8_e4m3fn and float8_e5m2)."""
    import torch
    dtype = {torch.float32: PESTI_F32, torch.bfloat16: PESTI_BF16, torch.float16: PESTI_F16,
             getattr(torch, "float8_e4m3fn", None): PESTI_FP8_E4M3,
             getattr(torch, "float8_e5m2", None): PESTI_FP8_E5M2}.get(logits.dtype)
    if dtype is None:
        raise ValueError("logits must be float32, bfloat16, float16, float8_e4m3fn or float8_e5m2")
    return dtype


def _batch_args(logits, configs, out, greedy_if_zero_t, argmax_first, kept_width, stream):
    """Shape, dtype, parameter array and output tensors of a batch call."""
    import torch
    if logits.dim() != 2:
        raise ValueError("logits must be [B, V]")
    B, V = logits.shape
    dtype = _dtype_of(logits)
    if logits.stride(1) != 1:
        raise ValueError("logits rows must be contiguous")
    if isinstance(configs, SamplingConfig):
        arr = (_Params * 1)(configs.to_params(greedy_if_zero_t, argmax_first))
        per_row = 0
    elif isinstance(configs, PreparedParams):
        if configs.rows != B:
            raise ValueError("need one config per row")
        if (configs.greedy_if_zero_t, configs.argmax_first) != (greedy_if_zero_t, argmax_first):
            raise ValueError("PreparedParams were made with other flags")
        arr = configs.arr
        per_row = 1
    else:
        if len(configs) != B:
            raise ValueError("need one config per row")
        arr = (_Params * B)(*[c.to_params(greedy_if_zero_t, argmax_first) for c in configs])
        per_row = 1
    if out is None:
        out = torch.empty(B, dtype=torch.int32, device=logits.device)
    kp = ki = kc = None
    if kept_width > 0:
        kp = torch.empty(B, kept_width, dtype=torch.float32, device=logits.device)
        ki = torch.empty(B, kept_width, dtype=torch.int32, device=logits.device)
        kc = torch.empty(B, dtype=torch.int64, device=logits.device)
    st = stream if stream is not None else torch.cuda.current_stream(logits.device).cuda_stream
    return B, V, dtype, arr, per_row, out, kp, ki, kc, st


COMM_ID_BYTES = 128  # PESTI_COMM_ID_BYTES


class Comm:
    """A pesti_comm (an NCCL communicator over this process group's ranks) for
    Sampler.sample_batch_sharded.  Rank 0 makes the id (pesti_comm_id); it is
    broadcast over the default torch.distributed group, then every rank
    calls pesti_comm_create_timed.  Collective: every rank constructs it.
    timeout_ms bounds the set-up and each sharded call's exchanges (a rank
    that does not join or stops makes the others fail with PESTI_E_TIMEOUT
    instead of hanging)."""

    def __init__(self, device: int, timeout_ms: int = 120000):
        import torch
        import torch.distributed as dist
        lib = load_library()
        rank, world = dist.get_rank(), dist.get_world_size()
        buf = (ctypes.c_uint8 * COMM_ID_BYTES)()
        if rank == 0:
            _check(lib.pesti_comm_id(buf))
        t = torch.tensor(list(bytes(buf)), dtype=torch.uint8)
        if dist.get_backend() == "nccl":
            t = t.to(f"cuda:{device}")
        dist.broadcast(t, 0)
        buf = (ctypes.c_uint8 * COMM_ID_BYTES).from_buffer_copy(bytes(t.cpu().tolist()))
        h = ctypes.c_void_p()
        _check(lib.pesti_comm_create_timed(world, rank, buf, int(device), int(timeout_ms), ctypes.byref(h)))
        self._h = h
        self._lib = lib
        self.rank, self.world, self.device = rank, world, device

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.pesti_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def set_cluster_mode(mode: int) -> None:
    """pesti_testing_set_cluster: -1 sends greedy/top-k batches through the
    four-kernel pipeline instead of the cluster pass, 1..16 forces that many
    CTAs per row's cluster, 0 restores the default (process-wide)."""
    _check(load_library().pesti_testing_set_cluster(int(mode)))


NOALLOC_SCRATCH_BYTES = 64 << 20  # PESTI_NOALLOC_SCRATCH_BYTES


def sample_batch_noalloc(logits, configs: Union[SamplingConfig, Sequence[SamplingConfig]], u, out,
                         greedy_if_zero_t: bool = True, argmax_first: bool = False, kept=None,
                         stream=None):
    """Sampler.sample_batch through pesti_sample_batch_noalloc: no handle and no
    device allocation inside the call, for callers that cannot allocate while
    they sample (every output buffer is the caller's).

    out: [B] int32 CUDA tensor for the tokens.  kept: None or a tuple
    (kept_p [B, W] f32, kept_idx [B, W] int32, kept_count [B] int64).  Runs on
    the current CUDA device in a static scratch array of NOALLOC_SCRATCH_BYTES
    shared by every call: larger batches raise SamplerError, and calls on
    unordered streams race.  The first call on a device sets the array up.
    """
    import torch
    lib = load_library()
    B, V = logits.shape
    dtype = _dtype_of(logits)
    if logits.stride(1) != 1:
        raise ValueError("logits rows must be contiguous")
    if isinstance(configs, SamplingConfig):
        arr = (_Params * 1)(configs.to_params(greedy_if_zero_t, argmax_first))
        per_row = 0
    else:
        if len(configs) != B:
            raise ValueError("need one config per row")
        arr = (_Params * B)(*[c.to_params(greedy_if_zero_t, argmax_first) for c in configs])
        per_row = 1
    kp, ki, kc = kept if kept is not None else (None, None, None)
    width = kp.shape[1] if kp is not None else 0
    st = stream if stream is not None else torch.cuda.current_stream(logits.device).cuda_stream
    _check(lib.pesti_sample_batch_noalloc(
        logits.data_ptr(), dtype, B, V, logits.stride(0), arr, per_row, 0, u.data_ptr(), out.data_ptr(),
        kp.data_ptr() if kp is not None else None, ki.data_ptr() if ki is not None else None, width,
        kc.data_ptr() if kc is not None else None, st))
    return out


_default: Optional[Sampler] = None


def _default_sampler() -> Sampler:
    global _default
    if _default is None:
        _default = Sampler(0)
    return _default


def sample(logits, config: SamplingConfig, rng) -> int:
    """Module-level drop-in for sampling.rs:39 on CUDA device 0."""
    return _default_sampler().sample(logits, config, rng)


def argmax(logits) -> int:
    """Module-level drop-in for sampling.rs:115 on CUDA device 0."""
    return _default_sampler().argmax(logits)


def generate_step(logits, config: SamplingConfig, rng) -> int:
    """The branch of LlamaModel::generate (transformer/model.rs:517-521)."""
    if config.temperature == 0.0:
        return argmax(logits)
    return sample(logits, config, rng)
