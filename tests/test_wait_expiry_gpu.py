"""Failure detection on the GPU: a bounded in-kernel wait that runs out.

Every mbarrier wait in the kernels is bounded. When one expires, the kernel records
GQA_ERR_TIMEOUT and a site id in the device error word, raises its CTA's abort flag
(the CTA's other waits end), lets the copies it issued land, frees its TMEM and
returns; the host reads the word with gqa_device_error. Nothing faults and nothing
hangs, so the context stays usable.

The checked build's test hook (gqa_debug_inject) makes the TMA producer of CTA 0
withhold one of its loads and shortens every wait to 20 ms: the consumer's wait on
that load then expires -- a flag nothing sets, the form of fault injection this pool
allows. Each case checks that the launch returns, that the error word names the
timeout, and that a following normal call on the SAME workspace (ticket counters
included) is bit-identical to the release library's output and reports no error.
"""
import ctypes
import os
import time

import pytest
import torch

from gqa_kernels import _lib
from tests._common import make_inputs

pytestmark = pytest.mark.gpu
LOG2E = 1.4426950408889634
GQA_ERR_TIMEOUT = 5
LIMIT_NS = 20_000_000

PREFILL_SITES = set(range(1, 26))     # producer 1-2, MMA issuer 10-19, softmax 20-25
STREAM_SITES = set(range(101, 105))   # producer 101-102, compute 103, combine 104


def _load(path):
    lib = ctypes.CDLL(path)
    for name, (res, args) in _lib.SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


@pytest.fixture(scope="module")
def libs(cuda_lib, lib_path):
    dbg = os.path.join(os.path.dirname(lib_path), "libgqa_sm100_debug.so")
    assert os.path.exists(dbg), "build.py --debug first"
    return _load(lib_path), _load(dbg)


def _fwd(lib, q, k, v, ws):
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    o = torch.full_like(q, float("nan"))
    rc = lib.gqa_fwd(*(ctypes.c_void_p(t.data_ptr()) for t in (q, k, v, o)), *(_lib.strides(t) for t in (q, k, v, o)),
                     B, Hq, Hkv, Sq, Skv, D, ctypes.c_float(D ** -0.5 * LOG2E), 1, _lib.dtype_code(q),
                     ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()),
                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, rc
    torch.cuda.synchronize()  # raises if the launch faulted; a timeout is not a fault
    return o


def _error(lib):
    code, site = ctypes.c_int(0), ctypes.c_int(0)
    assert lib.gqa_device_error(ctypes.byref(code), ctypes.byref(site), 1) == 0
    return code.value, site.value


def _workspace(lib, q, k):
    B, Hq, Sq, D = q.shape
    nb = lib.gqa_fwd_workspace_bytes(B, Hq, k.shape[1], Sq, k.shape[2], D)
    return torch.zeros(max(nb, 256), dtype=torch.uint8, device=q.device)


@pytest.mark.parametrize("shape,load,sites", [
    ((1, 32, 8, 2048, 2048, 128), 3, PREFILL_SITES),  # tcgen05 prefill, V tile of key tile 1 withheld
    ((1, 32, 8, 512, 4096, 128), 3, PREFILL_SITES),   # prefill key split (ticket combine)
    ((1, 32, 8, 1, 16384, 128), 1, STREAM_SITES),     # split-KV decode, stage 1 withheld
    ((2, 64, 8, 3, 777, 64), 0, STREAM_SITES),        # streaming kernel, first stage withheld
], ids=["prefill", "prefill_split", "decode_split", "stream_rows"])
def test_expired_wait_reports_and_recovers(libs, shape, load, sites):
    rel, dbg = libs
    q, k, v = (t.cuda() for t in make_inputs(*shape, seed=61))
    ref = _fwd(rel, q, k, v, _workspace(rel, q, k))
    ws = _workspace(dbg, q, k)  # shared by the aborted call and the call after it
    assert _error(dbg) == (0, 0)
    assert dbg.gqa_debug_inject(0, load, LIMIT_NS) == 0
    try:
        t0 = time.perf_counter()
        _fwd(dbg, q, k, v, ws)
        elapsed = time.perf_counter() - t0
        code, site = _error(dbg)
    finally:
        assert dbg.gqa_debug_inject(-1, -1, 0) == 0
    assert code == GQA_ERR_TIMEOUT and site in sites, (code, site)
    assert elapsed >= LIMIT_NS * 1e-9, elapsed  # the wait did run to its limit
    # The context is usable, TMEM was returned, the ticket counters are back at zero:
    # the next call on the same workspace is exact and clean.
    out = _fwd(dbg, q, k, v, ws)
    assert _error(dbg) == (0, 0)
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_release_build_has_no_injection(libs):
    rel, _ = libs
    assert rel.gqa_debug_inject(0, 0, LIMIT_NS) == 2  # GQA_ERR_UNSUPPORTED
