"""Failure detection on the host, without a GPU fault: a rank that leaves before
the exchange step makes the others' next collective end with an error within
the process-group timeout instead of hanging."""
import os
import time

import torch

from gqa_kernels import sharded as S
from tests._dist import run_ranks


def _leaver(rank, world):
    packed = torch.ones(S.packed_size((1, 4, 1, 64)))
    if rank == world - 1:
        os._exit(0)  # leaves between steps: no collective of it is in flight
    t0 = time.time()
    try:
        S.gather_partials(packed)
    except Exception as e:
        return ("raised", type(e).__name__, time.time() - t0)
    return ("returned", None, time.time() - t0)


def test_peer_exit_is_reported_not_hung():
    res = run_ranks(_leaver, 2, timeout_s=10, join_s=90)
    assert 0 in res
    status, val = res[0]
    if status == "ok":
        what, name, dt = val
        assert what == "raised", val
        assert dt < 60
    else:  # the error surfaced while tearing down; still not a hang
        assert "Error" in val or "error" in val


def _raiser(rank, world):
    if rank == 0:
        raise RuntimeError("injected host-side failure on rank 0")
    packed = torch.ones(S.packed_size((1, 4, 1, 64)))
    t0 = time.time()
    try:
        S.gather_partials(packed)
    except Exception as e:
        return ("raised", type(e).__name__, time.time() - t0)
    return ("returned", None, time.time() - t0)


def test_peer_exception_is_reported():
    res = run_ranks(_raiser, 2, timeout_s=10, join_s=90)
    assert res[0][0] == "error" and "injected" in res[0][1]
    status, val = res[1]
    assert status == "error" or val[0] == "raised", res[1]


def test_device_error_drops_cached_workspaces(monkeypatch):
    """A nonzero device error word (an aborted launch) makes the split kernels' cached
    workspaces untrusted: reading it drops them, so the next call starts from zeroed
    ticket counters. A fake library stands in for the GPU."""
    import ctypes

    from gqa_kernels import _lib

    class FakeLib:
        def __init__(self, code):
            self.code = code

        def gqa_device_error(self, code_p, site_p, clear):
            ctypes.cast(code_p, ctypes.POINTER(ctypes.c_int))[0] = self.code
            ctypes.cast(site_p, ctypes.POINTER(ctypes.c_int))[0] = 103 if self.code else 0
            return 0

    dropped = []
    monkeypatch.setattr(_lib.WORKSPACES, "drop", lambda device: dropped.append(device))
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    monkeypatch.setattr(_lib, "load", lambda: FakeLib(0))
    assert _lib.device_error() == (0, 0) and dropped == []
    monkeypatch.setattr(_lib, "load", lambda: FakeLib(5))
    assert _lib.device_error() == (5, 103)
    assert dropped == [torch.device("cuda", 0)]
