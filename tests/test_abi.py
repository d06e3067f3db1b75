"""The C-ABI library: builds, loads, exports every declared entry point, and
fails loudly (no CPU fallback) when no GPU is present."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in sorted(os.listdir(os.path.join(ROOT, "include")))
           if h.endswith(".h")]
LIB = os.path.join(ROOT, "llm-workspace_b200", "libpesti_sampler.so")


def declared_functions():
    text = "\n".join(open(h).read() for h in HEADERS)
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pesti_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for want in ("pesti_sampler_create", "pesti_sampler_destroy", "pesti_sample_batch",
                 "pesti_argmax_batch", "pesti_sample_row_host", "pesti_last_error"):
        assert want in names


def test_library_exports_every_declared_symbol():
    assert os.path.exists(LIB), "build the library first (__graft_entry__.build())"
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (pesti_[a-z0-9_]+)$", out, flags=re.M))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    lib = ctypes.CDLL(LIB)
    for n in declared_functions():
        assert hasattr(lib, n)


def test_no_device_is_an_error_not_a_fallback():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import pesti_sampler
    with pytest.raises(pesti_sampler.SamplerError) as e:
        pesti_sampler.Sampler(0)
    assert e.value.code == pesti_sampler.PESTI_E_NO_DEVICE
    lib = pesti_sampler.load_library()
    assert b"device" in lib.pesti_last_error()


def test_invalid_arguments_are_rejected_without_a_device():
    import pesti_sampler
    lib = pesti_sampler.load_library()
    assert lib.pesti_sample_batch(None, None, 0, 1, 1, 1, None, 0, 0, None, None, None, None, 0, None, None) \
        == pesti_sampler.PESTI_E_INVALID_ARG
    assert lib.pesti_argmax_batch(None, None, 0, 1, 1, 1, 0, None, None) == pesti_sampler.PESTI_E_INVALID_ARG
    # the device draws: a negative row count and a null state are refused before any device work
    assert lib.pesti_pcg32_seed(None, -1, 1, 0, None) == pesti_sampler.PESTI_E_INVALID_ARG
    assert lib.pesti_pcg32_draw(None, 4, None, None) == pesti_sampler.PESTI_E_INVALID_ARG
    # a communicator needs a positive deadline; refused before any device or NCCL work
    import ctypes
    h = ctypes.c_void_p()
    buf = (ctypes.c_uint8 * pesti_sampler.COMM_ID_BYTES)()
    assert lib.pesti_comm_create_timed(2, 0, buf, 0, 0, ctypes.byref(h)) == pesti_sampler.PESTI_E_INVALID_ARG
    assert lib.pesti_comm_create_timed(2, 2, buf, 0, 1000, ctypes.byref(h)) == pesti_sampler.PESTI_E_INVALID_ARG
    # the device loop control: bad limits and a too-small output are refused before any device work
    assert lib.pesti_generate_advance(None, 4, None, 0, -1, 8, None, 8, None, None, None, None, None) \
        == pesti_sampler.PESTI_E_INVALID_ARG
    assert lib.pesti_generate_advance(None, 4, None, 0, 10, 8, None, 4, None, None, None, None, None) \
        == pesti_sampler.PESTI_E_INVALID_ARG
    assert lib.pesti_generate_advance(None, 4, None, 0, 10, 8, None, 8, None, None, None, None, None) \
        == pesti_sampler.PESTI_E_INVALID_ARG
    # the llama.cpp chain: a null handle is refused before any device work
    assert lib.pesti_llama_chain_batch(None, None, 0, 1, 1, 1, None, None, None, 0, None, None, None, None) \
        == pesti_sampler.PESTI_E_INVALID_ARG
    # fp8 logits are taken by the batch calls only; the others refuse them
    assert lib.pesti_sample_batch_noalloc(None, pesti_sampler.PESTI_FP8_E4M3, 1, 1, 1, None, 0, 0, None, None,
                                          None, None, 0, None, None) == pesti_sampler.PESTI_E_INVALID_ARG
