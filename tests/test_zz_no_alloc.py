"""gqa_split_fused_noalloc: the split-KV forward for callers that cannot allocate
device memory (an FFI host with no CUDA allocator of its own, or an engine whose
memory pool owns all of HBM). It must give the same output as gqa_split_fused,
which takes a caller-allocated workspace, on consecutive calls that share the
library's static scratch array.

Called through the C ABI with ctypes, as an FFI host would. This file is named
to be collected last, so a run that stops at the first failure has already run
every other test.
"""
import ctypes

import pytest
import torch

from oracle import gqa_oracle as O
from tests._common import BASELINE_TOL, compare, make_inputs, to_np

pytestmark = pytest.mark.gpu
LOG2E = 1.4426950408889634
GQA_ERR_SCRATCH_LIMIT = 8


def _args(q, k, v, o):
    st = [(ctypes.c_int64 * 4)(*t.stride()) for t in (q, k, v, o)]
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    ptrs = [ctypes.c_void_p(t.data_ptr()) for t in (q, k, v, o)]
    dims = (B, Hq, Hkv, Sq, Skv, D, ctypes.c_float((D ** -0.5) * LOG2E), 1, 1)  # causal, bf16
    return ptrs, st, dims


def _split_fused(lib, q, k, v):
    o = torch.empty_like(q)
    ptrs, st, dims = _args(q, k, v, o)
    B, Hq, Hkv, Sq, Skv, D = dims[:6]
    nbytes = lib.gqa_split_fused_workspace_bytes(B, Hq, Hkv, Sq, Skv, D)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=q.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.gqa_split_fused(*ptrs, *st, *dims, ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(nbytes), stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    return o


def _noalloc(lib, q, k, v):
    o = torch.full_like(q, float("nan"))
    ptrs, st, dims = _args(q, k, v, o)
    rc = lib.gqa_split_fused_noalloc(*ptrs, *st, *dims, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return rc, o


SHAPES = [(1, 32, 8, 1, 16384, 128),   # BASELINE split-KV decode, 16K keys
          (2, 32, 8, 3, 3000, 64),
          (1, 16, 4, 1, 5000, 128)]


def test_noalloc_matches_split_fused_on_consecutive_calls(cuda_lib):
    lib = cuda_lib
    cases = []
    for i, s in enumerate(SHAPES):
        q, k, v = (t.cuda() for t in make_inputs(*s, seed=40 + i))
        cases.append((q, k, v, _split_fused(lib, q, k, v)))
    # two calls in a row per shape, and shapes interleaved so each call finds the
    # scratch array laid out by a different previous call
    checked = set()
    for q, k, v, ref in cases + cases:
        for _ in range(2):
            rc, out = _noalloc(lib, q, k, v)
            assert rc == 0, rc
            assert not torch.isnan(out).any()
            compare(to_np(out), to_np(ref), BASELINE_TOL)
            if id(q) not in checked:  # and once per shape against the CPU oracle itself
                checked.add(id(q))
                compare(to_np(out), O.gqa_reference(to_np(q), to_np(k), to_np(v), causal=True), BASELINE_TOL)


def test_noalloc_rejects_problems_beyond_the_static_scratch(cuda_lib):
    lib = cuda_lib
    # 64 x 8 units x 4 chunks x 8 rows of fp32 partials is well beyond 4 MiB. The size
    # check comes before any kernel reads K or V, so one batch element of keys,
    # expanded over the batch (stride 0), stands in for the 8.6 GB tensor.
    q = torch.zeros(64, 64, 1, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 8, 65536, 128, dtype=torch.bfloat16, device="cuda").expand(64, -1, -1, -1)
    assert lib.gqa_split_fused_workspace_bytes(64, 64, 8, 1, 65536, 128) > (4 << 20)
    rc, _ = _noalloc(lib, q, k, k)
    assert rc == GQA_ERR_SCRATCH_LIMIT
    assert "static no-allocation buffer" in lib.gqa_strerror(rc).decode()
