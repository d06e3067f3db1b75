"""The hardware 2^y approximation behind the classification's cheap exp
(ex2.approx.ftz.f32), checked exhaustively: over every float y in [-200, 0]
and -inf (below y = -126 a flushed 0 counts as exact) its relative error
against exp2 in double must not exceed
PESTI_EX2_APPROX_RELERR, the bound from which the classification's decision
margins are derived (exp_hw in pesti_kernels.cuh)."""
import ctypes
import math
import os
import re

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_bound():
    text = open(os.path.join(ROOT, "llm-workspace_b200", "csrc", "pesti_exp.cuh")).read()
    m = re.search(r"#define PESTI_EX2_APPROX_RELERR (0x[0-9a-fp.+-]+)f", text)
    assert m, "PESTI_EX2_APPROX_RELERR not found"
    return float.fromhex(m.group(1))


def test_ex2_approx_error_within_the_declared_bound():
    import pesti_sampler as ps
    lib = ps.load_library()
    fn = lib.pesti_test_ex2_approx_max_relerr
    fn.argtypes = [ctypes.POINTER(ctypes.c_double)]
    fn.restype = ctypes.c_int
    out = ctypes.c_double()
    assert fn(ctypes.byref(out)) == 0, lib.pesti_last_error()
    print(f"max relative error of ex2.approx.ftz.f32 on [-200, 0]: {out.value:.6g} (2^{math.log2(out.value):.3f})")
    assert 0.0 < out.value <= _declared_bound()
