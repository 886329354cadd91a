"""Multi-GPU partitionings on one GPU: every rank's compute (gqa_partial,
head-sharded forward) and the combine (gqa_lse_combine) run for real; the
exchange is the stacking an all-gather would produce. The NCCL exchange itself
runs in bench.py --workload long_decode at N > 1."""
import numpy as np
import pytest
import torch

from gqa_kernels import gqa_flash_attn
from gqa_kernels import sharded as S
from oracle import gqa_oracle as O
from tests._common import BASELINE_TOL, compare, make_inputs, to_np

pytestmark = pytest.mark.gpu
DEVICE = "cuda"


@pytest.fixture(autouse=True)
def _lib_ready(cuda_lib):
    yield
    torch.cuda.synchronize()


@pytest.mark.parametrize("shape,world", [((2, 64, 8, 1, 4096, 128), 4), ((1, 32, 8, 3, 1000, 128), 3),
                                         ((2, 16, 2, 2, 700, 64), 8),
                                         ((2, 32, 8, 1, 300, 128), 8)])  # 5 key blocks: 3 ranks empty
def test_partials_and_combine(shape, world):
    B, Hq, Hkv, Sq, Skv, D = shape
    q, k, v = (t.to(DEVICE) for t in make_inputs(B, Hq, Hkv, Sq, Skv, D, seed=21))
    qn, kn, vn = to_np(q), to_np(k), to_np(v)
    packed = []
    for r in range(world):
        k0, k1 = S.kv_range(Skv, world, r)
        p = S.partial_forward(q, k[:, :, k0:k1], v[:, :, k0:k1], True, k0, Skv)
        rows, acc_off, _ = S.packed_layout(q.shape)
        m, l, a = O.partial_attention(qn, kn[:, :, k0:k1], vn[:, :, k0:k1], True, k0, Skv)
        pn = to_np(p)
        fin = np.isfinite(m.reshape(-1))
        np.testing.assert_allclose(pn[:rows][fin], m.reshape(-1)[fin], rtol=1e-3, atol=2e-2)
        np.testing.assert_allclose(pn[rows:2 * rows], l.reshape(-1), rtol=2e-2, atol=2e-2)
        np.testing.assert_allclose(pn[acc_off:], a.reshape(-1), rtol=2e-2, atol=5e-2)
        packed.append(p)
    out = S.combine_partials(torch.stack(packed), tuple(q.shape), q.dtype, q.device)
    compare(to_np(out), O.gqa_reference(qn, kn, vn, causal=True), BASELINE_TOL)


@pytest.mark.parametrize("world", [2, 4, 8, 16])
def test_head_sharded_units(world):
    B, Hq, Hkv, Sq, Skv, D = 4, 32, 8, 128, 1024, 128
    q, k, v = (t.to(DEVICE) for t in make_inputs(B, Hq, Hkv, Sq, Skv, D, seed=31))
    full = gqa_flash_attn(q, k, v)
    stitched = torch.empty_like(full)
    g = Hq // Hkv
    for r in range(world):
        br, hr = S.shard_units(B, Hkv, world, r)
        ql, kl, vl = S.slice_units(q, k, v, br, hr)
        stitched[br[0]:br[1], hr[0] * g:hr[1] * g] = S.head_sharded_forward(ql, kl, vl)
    # A GPU's share has fewer units, so its launch may split key tiles across CTAs
    # (a different summation order): equal within the contract, not bit for bit.
    compare(to_np(stitched), to_np(full), BASELINE_TOL)
