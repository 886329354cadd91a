"""The peer exchange of the key-sharded combine on one GPU.

gqa_partial_peer stores each unit's (m, l, acc) into every rank's receive buffer
and raises that rank's counter for this source; gqa_lse_combine_peer waits in the
kernel for every source's counter, then combines (include/gqa_sm100.h, peer
exchange). With one rank (no process group) PeerExchange runs the same kernels
against its own buffer, so these cases need one GPU; the ranks-over-NVLink case
is in test_multigpu_gpu.py.

Checked here:
  * bit-identical to the all-gather form (gqa_partial + gqa_lse_combine over the
    same part) over consecutive calls, which alternate the buffer's two halves;
  * within the fp32-reference tolerance of the single-GPU forward;
  * CUDA-graph replays: the epoch lives on the device, so each replay is a new call;
  * a source that never arrives: the combine's bounded wait ends with
    GQA_ERR_TIMEOUT (site 301) in the device error word, O is left unwritten and
    the context stays usable (checked build, 20 ms wait limit).
"""
import ctypes
import os

import pytest
import torch

from gqa_kernels import _lib, gqa_flash_attn
from gqa_kernels import sharded as S
from tests._common import BASELINE_TOL, make_inputs

pytestmark = pytest.mark.gpu
GQA_ERR_TIMEOUT = 5


def _all_gather_form(q, k, v, skv):
    packed = S.partial_forward(q, k, v, True, 0, skv)
    return S.combine_partials(packed.view(1, -1), tuple(q.shape), q.dtype, q.device)


@pytest.mark.parametrize("shape", [(4, 64, 8, 1, 5000, 128), (1, 32, 8, 1, 16384, 128), (2, 32, 8, 3, 777, 64)],
                         ids=["batched_decode", "split_decode", "short_chunk_d64"])
def test_one_rank_matches_the_all_gather_form(cuda_lib, shape):
    B, Hq, Hkv, Sq, Skv, D = shape
    q, k, v = (t.cuda() for t in make_inputs(*shape, seed=71))
    ex = S.PeerExchange(q.shape, Hkv, q.device)
    try:
        for call in range(3):
            qc = q * (1.0 + 0.5 * call)
            ref = _all_gather_form(qc, k, v, Skv)
            got = ex.forward(qc, k, v, 0, Skv)
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), call
        d = (got.float() - gqa_flash_attn(qc, k, v).float()).abs()
        assert d.max().item() < BASELINE_TOL[0] and d.mean().item() < BASELINE_TOL[1]
    finally:
        ex.close()


def test_graph_replays_are_new_calls(cuda_lib):
    B, Hq, Hkv, Sq, Skv, D = 2, 32, 8, 1, 4096, 128
    q, k, v = (t.cuda() for t in make_inputs(B, Hq, Hkv, Sq, Skv, D, seed=72))
    ex = S.PeerExchange(q.shape, Hkv, q.device)
    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ex.forward(q, k, v, 0, Skv)  # caches the partial's workspace for this stream
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            out = ex.forward(q, k, v, 0, Skv)
        base = q.clone()
        for rep in range(4):
            q.copy_(base * (1.0 + 0.3 * rep))
            out.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            ref = _all_gather_form(q, k, v, Skv)
            assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), rep
        del g
    finally:
        ex.close()


def test_missing_source_times_out(cuda_lib, lib_path):
    path = os.path.join(os.path.dirname(lib_path), "libgqa_sm100_debug.so")
    assert os.path.exists(path), "build.py --debug first"
    dbg = ctypes.CDLL(path)
    for name, (res, args) in _lib.SIGNATURES.items():
        fn = getattr(dbg, name)
        fn.restype, fn.argtypes = res, args
    B, Hq, Skv, D = 1, 32, 1024, 128
    slot, parity, cnt_off, total = S.exchange_layout((B, Hq, 1, D), 1)
    buf = ctypes.c_void_p()
    assert dbg.gqa_exchange_alloc(total, ctypes.byref(buf)) == 0
    o = torch.full((B, Hq, 1, D), 7.0, dtype=torch.bfloat16, device="cuda")
    code, site = ctypes.c_int(0), ctypes.c_int(0)
    assert dbg.gqa_device_error(ctypes.byref(code), ctypes.byref(site), 1) == 0
    assert dbg.gqa_debug_inject(-1, -1, 20_000_000) == 0
    try:
        epoch = ctypes.c_void_p(buf.value + cnt_off + 8)
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        assert dbg.gqa_epoch_bump(epoch, stream) == 0
        # epoch 1 wants 1 unit from source 0; no partial kernel ran, so its counter stays 0
        rc = dbg.gqa_lse_combine_peer(buf, ctypes.c_void_p(buf.value + cnt_off), epoch, 1, slot, parity, 1,
                                      ctypes.c_void_p(o.data_ptr()), _lib.strides(o), B, Hq, 1, D,
                                      _lib.dtype_code(o), stream)
        assert rc == 0
        torch.cuda.synchronize()  # the wait ended by itself; nothing faulted
        assert dbg.gqa_device_error(ctypes.byref(code), ctypes.byref(site), 1) == 0
        assert (code.value, site.value) == (GQA_ERR_TIMEOUT, 301)
        assert (o.float() == 7.0).all()  # O unwritten
    finally:
        assert dbg.gqa_debug_inject(-1, -1, 0) == 0
        assert dbg.gqa_exchange_free(buf) == 0
    # the context is usable: a normal call afterwards is correct
    q, k, v = (t.cuda() for t in make_inputs(B, Hq, 8, 1, Skv, D, seed=73))
    ex = S.PeerExchange(q.shape, 8, q.device)
    try:
        got = ex.forward(q, k, v, 0, Skv)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), _all_gather_form(q, k, v, Skv).view(torch.int16))
    finally:
        ex.close()
