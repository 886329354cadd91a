"""The BASELINE configurations at full size, through the public API.

Every configuration is run on the contract's inputs (q, k, v ~ N(0,1) in fp32
from a CUDA generator seeded 0, cast to bf16) and checked three ways:

* against the torch fp32 restatement of tests/reference.py on the GPU, over
  every output element (16K prefill: over its first and last 2048 query rows,
  the rows with the fewest and the most visible keys), with the contract's
  tolerance (max-abs 2e-2, mean-abs 2e-3);
* against the numpy oracle on a seeded sample of rows (rows are independent,
  so each sampled row is the oracle over that row's visible keys only);
* through a size-independent property: every output is a convex combination of
  the visible V rows, so each element lies within the per-column range of V
  (plus bf16 rounding of the output).
"""
import numpy as np
import pytest
import torch

from gqa_kernels import gqa_flash_attn
from oracle import gqa_oracle as O
from tests._common import BASELINE_TOL, compare, to_np

pytestmark = pytest.mark.gpu
DEVICE = "cuda"


@pytest.fixture(autouse=True)
def _lib_ready(cuda_lib):
    yield
    torch.cuda.synchronize()


def _inputs(B, Hq, Hkv, Sq, Skv, D, seed=0):
    """N(0,1) fp32 from a CUDA generator (q, k, v in that order), cast to bf16; k and
    v are drawn one batch element at a time so the fp32 staging stays small."""
    g = torch.Generator(device=DEVICE).manual_seed(seed)
    q = torch.randn(B, Hq, Sq, D, generator=g, device=DEVICE).to(torch.bfloat16)
    kv = []
    for _ in range(2):
        t = torch.empty(B, Hkv, Skv, D, dtype=torch.bfloat16, device=DEVICE)
        for b in range(B):
            t[b] = torch.randn(Hkv, Skv, D, generator=g, device=DEVICE).to(torch.bfloat16)
        kv.append(t)
    return q, kv[0], kv[1]


@torch.no_grad()
def _torch_rows(q, k, v, r0, r1):
    """fp32 attention of query rows [r0, r1) with the bottom-right causal mask (TF32 off)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        B, Hq, Sq, D = q.shape
        Hkv, Skv = k.shape[1], k.shape[2]
        G = Hq // Hkv
        out = torch.empty(B, Hq, r1 - r0, D, dtype=torch.float32, device=q.device)
        kpos = torch.arange(Skv, device=q.device)
        qpos = torch.arange(r0, r1, device=q.device) + (Skv - Sq)
        mask = qpos[:, None] < kpos[None, :]
        for b in range(B):
            for h in range(Hkv):
                kf, vf = k[b, h].float(), v[b, h].float()
                for c0 in range(r0, r1, 1024):
                    c1 = min(r1, c0 + 1024)
                    s = torch.matmul(q[b, h * G:(h + 1) * G, c0:c1].float(), kf.T) * (D ** -0.5)
                    s = s.masked_fill(mask[c0 - r0:c1 - r0], float("-inf"))
                    out[b, h * G:(h + 1) * G, c0 - r0:c1 - r0] = torch.matmul(torch.softmax(s, dim=-1), vf)
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _oracle_rows(q, k, v, out, n_rows, seed):
    """The numpy oracle on a seeded sample of (b, head, i) rows (first and last rows
    included); each row is evaluated over its visible keys, non-causally."""
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    G = Hq // Hkv
    rng = np.random.default_rng(seed)
    rows = [(0, 0, 0), (B - 1, Hq - 1, Sq - 1)]
    rows += [(int(rng.integers(B)), int(rng.integers(Hq)), int(rng.integers(Sq))) for _ in range(n_rows - 2)]
    got, ref = [], []
    for b, h, i in rows:
        lim = min(Skv, i + Skv - Sq + 1)
        qi = to_np(q[b:b + 1, h:h + 1, i:i + 1])
        ki = to_np(k[b:b + 1, h // G:h // G + 1, :lim])
        vi = to_np(v[b:b + 1, h // G:h // G + 1, :lim])
        ref.append(O.gqa_reference_rows(qi, ki, vi, [(0, 0, 0)], causal=False)[0])
        got.append(to_np(out[b, h, i]))
    return np.stack(got), np.stack(ref)


def _check_convex(q, v, out, causal_full_rows):
    """out[b, h, i, d] within [min_j v[b, kv, j, d], max_j v[b, kv, j, d]] over all keys
    (a superset of every row's visible keys), with bf16 output rounding."""
    B, Hq = q.shape[:2]
    Hkv = v.shape[1]
    G = Hq // Hkv
    vmin = v.amin(dim=2).float()  # (B, Hkv, D), exact in bf16
    vmax = v.amax(dim=2).float()
    lo = vmin.repeat_interleave(G, dim=1)[:, :, None, :]
    hi = vmax.repeat_interleave(G, dim=1)[:, :, None, :]
    o = out.float()
    slack = 2.0 ** -7 * torch.maximum(lo.abs(), hi.abs())  # one bf16 ulp at the bound
    assert bool(((o >= lo - slack) & (o <= hi + slack)).all()), "output outside the convex hull of V"
    if causal_full_rows:
        assert not torch.isnan(o).any()


CONFIGS = {
    # name: (B, Hq, Hkv, Sq, Skv, D)
    "prefill_2k": (1, 32, 8, 2048, 2048, 128),
    "prefill_8k": (1, 32, 8, 8192, 8192, 128),
    "prefill_16k": (1, 32, 8, 16384, 16384, 128),
    "decode_4k": (1, 32, 8, 1, 4096, 128),
    "decode_16k": (1, 32, 8, 1, 16384, 128),
    "decode_64k": (1, 32, 8, 1, 65536, 128),
    "chunked_b4_512x16k": (4, 32, 8, 512, 16384, 128),
    "long_decode_b64_131k": (64, 64, 8, 1, 131072, 128),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_baseline_config_full_size(name):
    B, Hq, Hkv, Sq, Skv, D = CONFIGS[name]
    q, k, v = _inputs(B, Hq, Hkv, Sq, Skv, D)
    out = gqa_flash_attn(q, k, v, causal=True)
    torch.cuda.synchronize()
    # every row sees at least one key (Sq <= Skv), so no NaN anywhere
    _check_convex(q, v, out, causal_full_rows=True)
    if B * Hq * Sq * Skv <= 32 * 8192 * 8192:
        ref = _torch_rows(q, k, v, 0, Sq)
        compare(to_np(out), to_np(ref), BASELINE_TOL)
    else:
        for r0, r1 in ((0, 2048), (Sq - 2048, Sq)):
            ref = _torch_rows(q, k, v, r0, r1)
            compare(to_np(out[:, :, r0:r1]), to_np(ref), BASELINE_TOL)
    got, ref = _oracle_rows(q, k, v, out, 24, seed=len(name))
    compare(got, ref, BASELINE_TOL)
