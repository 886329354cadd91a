"""The prefill softmax's FMA-pipe exp2 (exp2_poly2, csrc/gqa_common.cuh) on the B200,
through the checked build's test entry gqa_debug_exp2_poly2.

Checked against CUDA's own exp2 (torch.exp2 on the same device) and against float64
exp2 of the same inputs: relative error below the 1.5e-4 bound the kernel states, over
the softmax's whole argument range [-126, 8]. Below the clamp (x < -126, -inf) and for
NaN the function returns the clamp's tiny positive value (about 2^-126), which the
kernel's comment documents: masked keys get ~1e-38 instead of 0, and NaN rows reach the
output through the MUFU columns instead.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from gqa_kernels import _lib

pytestmark = pytest.mark.gpu
BOUND = 1.5e-4


@pytest.fixture(scope="module")
def dbg(cuda_lib, lib_path):
    path = os.path.join(os.path.dirname(lib_path), "libgqa_sm100_debug.so")
    assert os.path.exists(path), "build.py --debug first"
    lib = ctypes.CDLL(path)
    for name, (res, args) in _lib.SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def _poly(lib, x):
    y = torch.full_like(x, float("nan"))
    rc = lib.gqa_debug_exp2_poly2(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), x.numel(),
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, rc
    torch.cuda.synchronize()
    return y


def test_relative_error_within_bound(dbg):
    g = torch.Generator().manual_seed(0)
    x = torch.cat([torch.linspace(-126.0, 8.0, 4_000_001),
                   -torch.rand(1_000_000, generator=g) * 30.0,  # the softmax's usual range
                   torch.arange(-126, 9, dtype=torch.float32),   # integers (f = 0)
                   torch.arange(-126, 8, dtype=torch.float32) + 0.5]).cuda()  # rounding ties
    y = _poly(dbg, x)
    cuda_ref = torch.exp2(x)  # CUDA's exp2 on the same device
    rel_cuda = ((y.double() - cuda_ref.double()) / cuda_ref.double()).abs()
    exact = torch.from_numpy(np.exp2(x.cpu().double().numpy())).cuda()
    rel_exact = ((y.double() - exact) / exact).abs()
    assert torch.isfinite(y).all() and (y > 0).all()
    assert rel_exact.max().item() < BOUND, rel_exact.max().item()
    assert rel_cuda.max().item() < BOUND + 1e-6, rel_cuda.max().item()


def test_clamp_and_nan_inputs(dbg):
    x = torch.tensor([float("-inf"), -1e30, -200.0, -126.5, float("nan"), -126.0, 0.0, 8.0], device="cuda")
    y = _poly(dbg, x).cpu()
    tiny = 2.0 ** -126
    # at and below the clamp, and NaN: about 2^-126, positive and finite (never NaN or negative)
    for i in range(6):
        assert 0.0 < y[i].item() < 2.0 * tiny, (x[i].item(), y[i].item())
    assert abs(y[6].item() - 1.0) < BOUND and abs(y[7].item() / 256.0 - 1.0) < BOUND


def test_odd_length_and_empty(dbg):
    x = torch.linspace(-3.0, 3.0, 7, device="cuda")
    y = _poly(dbg, x)
    assert ((y - torch.exp2(x)).abs() / torch.exp2(x)).max().item() < BOUND
    before = y.clone()
    assert dbg.gqa_debug_exp2_poly2(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), 0,
                                    ctypes.c_void_p(0)) == 0
    torch.cuda.synchronize()
    assert torch.equal(y, before)  # n = 0 writes nothing
