"""The checked build (libgqa_sm100_debug.so, build.py --debug) on the GPU: its in-kernel
address and coordinate checks pass on every path (prefill, prefill key split, split-KV
decode, paged decode) and leave the results bit-identical to the release library's."""
import ctypes
import os

import pytest
import torch

from gqa_kernels import _lib
from tests._common import make_inputs

pytestmark = pytest.mark.gpu
LOG2E = 1.4426950408889634


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
    if not os.path.exists(dbg):
        pytest.skip("debug variant not built")
    return _load(lib_path), _load(dbg)


def _fwd(lib, q, k, v):
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    o = torch.full_like(q, float("nan"))
    nb = lib.gqa_fwd_workspace_bytes(B, Hq, Hkv, Sq, Skv, D)
    ws = torch.zeros(max(nb, 256), dtype=torch.uint8, device=q.device)
    rc = lib.gqa_fwd(*(ctypes.c_void_p(t.data_ptr()) for t in (q, k, v, o)), *(_lib.strides(t) for t in (q, k, v, o)),
                     B, Hq, Hkv, Sq, Skv, D, ctypes.c_float(D ** -0.5 * LOG2E), 1, _lib.dtype_code(q),
                     ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(nb), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, rc
    torch.cuda.synchronize()
    return o


def _error(lib):
    code, site = ctypes.c_int(0), ctypes.c_int(0)
    assert lib.gqa_device_error(ctypes.byref(code), ctypes.byref(site), 1) == 0
    return code.value, site.value


@pytest.mark.parametrize("shape", [(1, 32, 8, 1024, 1024, 128),   # prefill
                                   (4, 4, 1, 512, 4096, 128),     # prefill key split
                                   (2, 32, 8, 300, 300, 64),      # prefill, head_dim 64, ragged
                                   (1, 32, 8, 1, 16384, 128),     # split-KV decode
                                   (2, 64, 8, 3, 777, 64)])       # streaming, few rows
def test_debug_build_checks_pass_and_match(libs, shape):
    rel, dbg = libs
    q, k, v = (t.cuda() for t in make_inputs(*shape, seed=21))
    a = _fwd(rel, q, k, v)
    b = _fwd(dbg, q, k, v)
    assert _error(dbg) == (0, 0)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_debug_build_reports_a_length_above_max_seq_len(libs):
    """A paged call whose seq_lens[b] exceeds the host's max_seq_len is clipped to the bound
    (the plan covers max_seq_len keys); the checked build reports it as GQA_ERR_DEBUG_CHECK
    (site 906), on the streaming path (decode) and on the tcgen05 path (long chunks)."""
    rel, dbg = libs
    Hq, Hkv, D, bs = 32, 8, 128, 64
    g = torch.Generator(device="cuda").manual_seed(3)
    kc = torch.randn(8, bs, Hkv, D, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn_like(kc)
    bt = torch.arange(8, dtype=torch.int32, device="cuda").view(1, 8)
    sl = torch.tensor([500], dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for chunk in (1, 128):
        q = torch.randn(1, Hq, chunk, D, generator=g, device="cuda").to(torch.bfloat16)
        o = torch.empty_like(q)
        ws = torch.zeros(1 << 22, dtype=torch.uint8, device="cuda")
        for lib, max_len, want in ((dbg, 512, (0, 0)), (dbg, 256, (9, 906)), (rel, 256, (0, 0))):
            rc = lib.gqa_paged_fwd(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(kc.data_ptr()),
                                   ctypes.c_void_p(vc.data_ptr()), ctypes.c_void_p(o.data_ptr()), _lib.strides(q),
                                   _lib.strides(o), ctypes.c_void_p(bt.data_ptr()), 8, ctypes.c_void_p(sl.data_ptr()),
                                   1, Hq, Hkv, chunk, D, bs, 8, max_len, ctypes.c_float(D ** -0.5 * LOG2E), 1, 1,
                                   ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()), stream)
            assert rc == 0, rc
            torch.cuda.synchronize()
            assert _error(lib) == want, (chunk, max_len)
