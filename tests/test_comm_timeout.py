"""Failure detection of the vocabulary-sharded path's communicator, with the
failure made on the host: a rank that exits before it joins.

Two processes (one GPU is enough: the rank that leaves never touches its
device).  Rank 0 makes the communicator id and hands it to rank 1, which
exits without calling pesti_comm_create.  Rank 0's pesti_comm_create_timed
must give up within its deadline with PESTI_E_TIMEOUT (the set-up is
non-blocking and aborted when the deadline passes) instead of waiting for the
missing rank forever.  NVLS is off, as for every failure test here.
"""
import multiprocessing as mp
import os
import time

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TIMEOUT_MS = 3000


def _leaver(q):
    q.get(timeout=60)  # the id arrives; this rank leaves without joining


def _waiter(q, out):
    import ctypes
    import sys
    sys.path.insert(0, os.path.join(ROOT, "llm-workspace_b200"))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import pesti_sampler as ps
    lib = ps.load_library()
    buf = (ctypes.c_uint8 * ps.COMM_ID_BYTES)()
    rc = lib.pesti_comm_id(buf)
    if rc:
        out.put(("id", rc, lib.pesti_last_error().decode(), 0.0))
        return
    q.put(bytes(buf))
    h = ctypes.c_void_p()
    t0 = time.monotonic()
    rc = lib.pesti_comm_create_timed(2, 0, buf, 0, TIMEOUT_MS, ctypes.byref(h))
    out.put(("create", rc, lib.pesti_last_error().decode(), time.monotonic() - t0))


def test_a_rank_that_never_joins_times_out():
    import pesti_sampler as ps
    ctx = mp.get_context("spawn")
    q, out = ctx.Queue(), ctx.Queue()
    leaver = ctx.Process(target=_leaver, args=(q,))
    waiter = ctx.Process(target=_waiter, args=(q, out))
    leaver.start()
    waiter.start()
    try:
        what, rc, msg, dt = out.get(timeout=120)
    finally:
        for p in (waiter, leaver):
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join()
    assert what == "create", msg
    assert rc == ps.PESTI_E_TIMEOUT, (rc, msg)
    assert "aborted" in msg, msg
    assert TIMEOUT_MS / 1e3 * 0.9 <= dt <= TIMEOUT_MS / 1e3 + 10.0, dt
