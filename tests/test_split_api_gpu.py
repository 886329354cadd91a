"""The split-KV entry points on the GPU: the reference's two-pass launch syntax
(gqa_split_first_kernel / gqa_split_reduce_kernel, through the C ABI) against
the oracle and the reference's own Triton partials, and the one-launch fused
path (split_kv_forward) with its workspace reuse."""
import os

import numpy as np
import pytest
import torch

from gqa_kernels.gqa_split import split_kv_forward, split_kv_two_pass
from oracle import gqa_oracle as O
from tests._common import BASELINE_TOL, compare, make_inputs, to_np

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEVICE = "cuda"


@pytest.fixture(autouse=True)
def _lib_ready(cuda_lib):
    yield
    torch.cuda.synchronize()


def _partials_close(mine, ref, name):
    m, l, a = (to_np(t) for t in mine)
    rm, rl, ra = ref
    assert np.array_equal(np.isinf(m), np.isinf(rm)), name
    fin = np.isfinite(rm)
    np.testing.assert_allclose(m[fin], rm[fin], rtol=2e-3, atol=2e-2, err_msg=f"{name} m")
    np.testing.assert_allclose(l, rl, rtol=1e-2, atol=2e-2, err_msg=f"{name} l")
    np.testing.assert_allclose(a, ra, rtol=1e-2, atol=5e-2, err_msg=f"{name} acc")


@pytest.mark.parametrize("shape,splits", [
    ((1, 32, 8, 1, 4096, 128), 16), ((1, 32, 8, 16, 1024, 128), 16), ((2, 8, 2, 3, 1000, 64), 8),
    ((1, 8, 2, 1, 1500, 128), 16), ((1, 16, 2, 5, 777, 64), 4)])
def test_two_pass_against_oracle(shape, splits):
    B, Hq, Hkv, Sq, Skv, D = shape
    q, k, v = (t.to(DEVICE) for t in make_inputs(B, Hq, Hkv, Sq, Skv, D, seed=Skv))
    o, parts = split_kv_two_pass(q, k, v, True, splits)
    qn, kn, vn = to_np(q), to_np(k), to_np(v)
    ref_parts = O.gqa_split_first(qn, kn, vn, True, splits, io="bf16", clean_masked=True)
    _partials_close(parts, ref_parts, str(shape))
    compare(to_np(o), O.gqa_reference(qn, kn, vn, causal=True), BASELINE_TOL)


def test_two_pass_against_reference_triton_partials():
    g = np.load(os.path.join(GOLD, "triton_f16.npz"))
    name = "split_clean_chunks"  # chunking where the reference reads exactly its chunks
    B, Hq, Hkv, Sq, Skv, D, causal, seed, splits = (int(x) for x in g[f"{name}/meta"])
    q, k, v = (torch.from_numpy(g[f"{name}/{x}"]).to(DEVICE) for x in "qkv")
    o, parts = split_kv_two_pass(q, k, v, bool(causal), splits)
    _partials_close(parts, (g[f"{name}/m_p"], g[f"{name}/l_p"], g[f"{name}/acc_p"]), name)
    compare(to_np(o), g[f"{name}/out"].astype(np.float32), BASELINE_TOL)


def test_two_pass_masked_chunk_is_clean():
    """Where the reference writes NaN partials (a non-empty chunk fully masked for a
    row) the CUDA partials are (-inf, 0, 0) and the output is finite and correct."""
    g = np.load(os.path.join(GOLD, "triton_f16.npz"))
    name = "split_masked_chunk"
    B, Hq, Hkv, Sq, Skv, D, causal, seed, splits = (int(x) for x in g[f"{name}/meta"])
    q, k, v = (torch.from_numpy(g[f"{name}/{x}"]).to(DEVICE) for x in "qkv")
    o, (m, l, a) = split_kv_two_pass(q, k, v, True, splits)
    assert not torch.isnan(m).any() and not torch.isnan(l).any() and not torch.isnan(o).any()
    qn, kn, vn = (g[f"{name}/{x}"].astype(np.float32) for x in "qkv")
    compare(to_np(o), O.gqa_reference(qn, kn, vn, causal=True), BASELINE_TOL)


@pytest.mark.parametrize("shape", [(1, 32, 8, 1, 16384, 128), (1, 32, 8, 1, 4096, 128), (2, 32, 8, 4, 3000, 128),
                                   (1, 64, 8, 1, 2048, 64), (1, 32, 8, 16, 1024, 128)])
def test_fused_split(shape):
    B, Hq, Hkv, Sq, Skv, D = shape
    q, k, v = (t.to(DEVICE) for t in make_inputs(B, Hq, Hkv, Sq, Skv, D, seed=11))
    out = split_kv_forward(q, k, v, True, 16)
    compare(to_np(out), O.gqa_reference(to_np(q), to_np(k), to_np(v), causal=True), BASELINE_TOL)


def test_fused_workspace_reuse_across_shapes():
    """Alternating shapes on one stream: ticket counters are zero at every call."""
    shapes = [(1, 32, 8, 1, 8192, 128), (2, 32, 8, 2, 3000, 128), (1, 32, 8, 1, 8192, 128), (1, 16, 4, 1, 20000, 64)]
    cases = []
    for i, s in enumerate(shapes):
        q, k, v = (t.to(DEVICE) for t in make_inputs(*s, seed=i))
        cases.append((q, k, v, O.gqa_reference(to_np(q), to_np(k), to_np(v), causal=True)))
    for _ in range(3):
        for q, k, v, ref in cases:
            compare(to_np(split_kv_forward(q, k, v, True, 16)), ref, BASELINE_TOL)
