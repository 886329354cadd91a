"""Parity of the CUDA path (gqa_kernels -> libgqa_sm100.so) with the oracle.

* The reference's own 17 cases (tests/test_correctness.py:48-77): same shapes,
  same CUDA generator (seed 0, q/k/v order, x0.1) and tolerances, checked
  against the numpy oracle (fp32) instead of a same-dtype torch evaluation.
* The golden fixtures recorded from the reference (oracle_bf16.npz: its torch
  oracle; triton_f16.npz: its Triton kernels).
* The BASELINE contract: N(0,1) bf16 inputs, max-abs 2e-2 / mean-abs 2e-3
  against the fp32 oracle.
* Edge cases: odd lengths, seq_q > seq_kv (NaN rows), head_dim 64, group sizes
  1..64, batch > 1, non-causal, strided inputs, empty keys, poisoned outputs.
"""
import os

import numpy as np
import pytest
import torch

from gqa_kernels import gqa_flash_attn, check_device_error
from gqa_kernels.gqa_fwd import gqa_fwd_kernel
from oracle import gqa_oracle as O
from tests._common import BASELINE_TOL, REF_TOL, compare, make_inputs, to_np, torch_reference

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEVICE = "cuda"

NUM_HEADS, NUM_KV_HEADS, HEAD_DIM = 32, 8, 128  # tests/test_correctness.py:18-21


@pytest.fixture(autouse=True)
def _lib_ready(cuda_lib):
    yield
    torch.cuda.synchronize()


def _make_ref_style(seq_q, seq_kv, dtype):
    """tests/test_correctness.py:30-37: CUDA generator seeded 0, q/k/v order, randn * 0.1."""
    g = torch.Generator(device=DEVICE).manual_seed(0)
    q = torch.randn(1, NUM_HEADS, seq_q, HEAD_DIM, dtype=dtype, device=DEVICE, generator=g) * 0.1
    k = torch.randn(1, NUM_KV_HEADS, seq_kv, HEAD_DIM, dtype=dtype, device=DEVICE, generator=g) * 0.1
    v = torch.randn(1, NUM_KV_HEADS, seq_kv, HEAD_DIM, dtype=dtype, device=DEVICE, generator=g) * 0.1
    return q, k, v


def _oracle(q, k, v, causal):
    if q.shape[2] * k.shape[2] * q.shape[1] <= 32 * 1024 * 1024:
        return O.gqa_reference(to_np(q), to_np(k), to_np(v), causal=causal)
    return to_np(torch_reference(q, k, v, causal))


# ---------------------------------------------------------------- the reference's 17 cases
@pytest.mark.parametrize("seq_len", [512, 2048, 4096])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_prefill(seq_len, dtype):
    q, k, v = _make_ref_style(seq_len, seq_len, dtype)
    out = gqa_flash_attn(q, k, v, causal=True)
    compare(to_np(out), _oracle(q, k, v, True), REF_TOL[dtype])


@pytest.mark.parametrize("seq_kv", [512, 2048, 4096, 8192])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decode(seq_kv, dtype):
    q, k, v = _make_ref_style(1, seq_kv, dtype)
    out = gqa_flash_attn(q, k, v, causal=True)
    compare(to_np(out), _oracle(q, k, v, True), REF_TOL[dtype])


@pytest.mark.parametrize("seq_q,seq_kv", [(16, 1024), (64, 2048), (256, 4096)])
def test_chunked_prefill(seq_q, seq_kv):
    q, k, v = _make_ref_style(seq_q, seq_kv, torch.bfloat16)
    out = gqa_flash_attn(q, k, v, causal=True)
    compare(to_np(out), _oracle(q, k, v, True), REF_TOL[torch.bfloat16])


# ---------------------------------------------------------------- golden fixtures
def _gold(name):
    return np.load(os.path.join(GOLD, name))


def test_golden_reference_oracle_cases():
    g = _gold("oracle_bf16.npz")
    names = sorted({k.split("/")[0] for k in g.files} - {"config1"})
    for name in names:
        B, Hq, Hkv, Sq, Skv, D, causal, seed = (int(x) for x in g[f"{name}/meta"])
        q, k, v = (torch.from_numpy(g[f"{name}/{x}"].view(np.int16)).view(torch.bfloat16).to(DEVICE) for x in "qkv")
        out = gqa_flash_attn(q, k, v, causal=bool(causal))
        compare(to_np(out), g[f"{name}/out"], BASELINE_TOL)


def test_golden_config1_rows_and_sums():
    """BASELINE config 1 on the GPU: inputs regenerated from seed 0 (CPU generator)."""
    g = _gold("oracle_bf16.npz")
    B, Hq, Hkv, S, _, D, causal, seed = (int(x) for x in g["config1/meta"])
    q, k, v = (t.to(DEVICE) for t in make_inputs(B, Hq, Hkv, S, S, D, seed=seed))
    out = to_np(gqa_flash_attn(q, k, v, causal=True))
    rows = g["config1/rows"]
    compare(out[0, rows[:, 0], rows[:, 1]], g["config1/row_out"], BASELINE_TOL)
    full = O.gqa_reference(to_np(q), to_np(k), to_np(v), causal=True)
    compare(out, full, BASELINE_TOL)
    assert abs(out.astype(np.float64).sum() - g["config1/sum"][0]) < 5.0


def test_golden_reference_triton_fp16():
    """The reference's own single-pass Triton kernel (fp16, interpreter) vs ours."""
    g = _gold("triton_f16.npz")
    for name in sorted({k.split("/")[0] for k in g.files if k.startswith("fwd_")}):
        B, Hq, Hkv, Sq, Skv, D, causal, seed, BM, BN = (int(x) for x in g[f"{name}/meta"])
        q, k, v = (torch.from_numpy(g[f"{name}/{x}"]).to(DEVICE) for x in "qkv")
        out = gqa_flash_attn(q, k, v, causal=bool(causal))
        compare(to_np(out), g[f"{name}/out"].astype(np.float32), BASELINE_TOL)


# ---------------------------------------------------------------- BASELINE contract + edges
EDGE = [
    # B, Hq, Hkv, Sq, Skv, D, causal
    (1, 32, 8, 512, 512, 128, True),    # config 1 shape
    (1, 32, 8, 1, 300, 128, True),      # decode, odd length
    (1, 32, 8, 3, 65, 128, True),
    (1, 32, 8, 17, 1000, 128, True),
    (1, 32, 8, 100, 1000, 128, True),   # chunked, Sq not a multiple of the tile
    (1, 32, 8, 129, 129, 128, True),
    (1, 32, 8, 257, 300, 64, True),
    (2, 8, 8, 200, 200, 128, True),     # group size 1 (MHA)
    (1, 16, 8, 150, 150, 128, True),    # group size 2
    (1, 64, 8, 64, 700, 128, True),     # group size 8
    (1, 32, 2, 40, 90, 64, True),       # group size 16
    (1, 64, 1, 4, 333, 128, True),      # group size 64, short q (streaming kernel)
    (1, 128, 1, 3, 200, 64, True),      # group size 128 (tcgen05 kernel, 1 position per tile)
    (3, 32, 8, 300, 300, 64, True),     # batch > 1, head_dim 64
    (2, 32, 8, 200, 333, 128, False),   # non-causal
    (1, 32, 8, 1, 1, 128, True),        # one key
    (1, 8, 2, 63, 63, 128, True),
    (1, 8, 2, 65, 65, 64, True),
    (1, 8, 2, 300, 100, 128, True),     # seq_q > seq_kv: top rows see no key -> NaN
    (1, 8, 2, 5, 2, 64, True),          # seq_q > seq_kv, streaming kernel
    # few query pairs against long keys: the tcgen05 kernel splits each unit's key
    # tiles across CTAs and the unit's last CTA combines the partials
    (4, 4, 1, 512, 16384, 128, True),   # one GPU's share of config 4 at 8 GPUs (4 splits)
    (2, 8, 2, 300, 2000, 128, True),    # causal chunks past some rows' diagonal
    (1, 8, 1, 200, 3000, 64, False),    # non-causal, head_dim 64
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", EDGE, ids=lambda s: "x".join(map(str, s)))
def test_baseline_contract_edges(shape, dtype):
    B, Hq, Hkv, Sq, Skv, D, causal = shape
    q, k, v = (t.to(DEVICE) for t in make_inputs(B, Hq, Hkv, Sq, Skv, D, dtype=dtype, seed=Sq * 131 + Skv))
    out = gqa_flash_attn(q, k, v, causal=causal)
    assert out.dtype == dtype and out.shape == q.shape
    compare(to_np(out), O.gqa_reference(to_np(q), to_np(k), to_np(v), causal=causal), BASELINE_TOL)


@pytest.mark.parametrize("shape", [(1, 32, 8, 300, 300, 128, True), (2, 32, 8, 1, 5000, 128, True),
                                   (1, 32, 8, 16, 1024, 128, True)])
def test_every_row_written(shape):
    """Output poisoned with NaN before the launch: no NaN may survive."""
    B, Hq, Hkv, Sq, Skv, D, causal = shape
    q, k, v = (t.to(DEVICE) for t in make_inputs(B, Hq, Hkv, Sq, Skv, D, seed=7))
    o = torch.full_like(q, float("nan"))
    gqa_fwd_kernel[(1,)](q, k, v, o, *q.stride(), *k.stride(), *v.stride(), *o.stride(), Sq, Skv,
                         (D ** -0.5) * O.LOG2E, IS_CAUSAL=causal, GROUP_SIZE=Hq // Hkv, HEAD_DIM=D)
    assert not torch.isnan(o).any()
    compare(to_np(o), O.gqa_reference(to_np(q), to_np(k), to_np(v), causal=causal), BASELINE_TOL)


def test_strided_inputs():
    B, Hq, Hkv, Sq, Skv, D = 2, 16, 4, 130, 260, 128
    q, k, v = (t.to(DEVICE) for t in make_inputs(B, Hq, Hkv, Sq, Skv, D, seed=3))
    ref = O.gqa_reference(to_np(q), to_np(k), to_np(v), causal=True)
    # (B, S, H, D) storage viewed as (B, H, S, D): TMA-compatible strides, no copy
    qt = q.transpose(1, 2).contiguous().transpose(1, 2)
    kt = k.transpose(1, 2).contiguous().transpose(1, 2)
    vt = v.transpose(1, 2).contiguous().transpose(1, 2)
    compare(to_np(gqa_flash_attn(qt, kt, vt)), ref, BASELINE_TOL)
    # head_dim slice of a wider buffer
    wide = torch.zeros(B, Hq, Sq, 2 * D, dtype=q.dtype, device=DEVICE)
    wide[..., :D] = q
    compare(to_np(gqa_flash_attn(wide[..., :D], k, v)), ref, BASELINE_TOL)
    # not contiguous in head_dim: copied once by the shim
    kd = k.transpose(2, 3).contiguous().transpose(2, 3)
    compare(to_np(gqa_flash_attn(q, kd, v)), ref, BASELINE_TOL)


def test_empty_keys_give_nan():
    q, k, v = (t.to(DEVICE) for t in make_inputs(1, 8, 2, 4, 0, 64, seed=1))
    assert torch.isnan(gqa_flash_attn(q, k, v)).all()


def test_non_default_stream():
    q, k, v = (t.to(DEVICE) for t in make_inputs(1, 32, 8, 256, 256, 128, seed=5))
    ref = O.gqa_reference(to_np(q), to_np(k), to_np(v), causal=True)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = gqa_flash_attn(q, k, v)
    s.synchronize()
    compare(to_np(out), ref, BASELINE_TOL)


def test_unsupported_inputs_raise():
    q, k, v = (t.to(DEVICE) for t in make_inputs(1, 24, 8, 16, 16, 128, seed=1))  # group 3
    with pytest.raises(RuntimeError, match="unsupported"):
        gqa_flash_attn(q, k, v)
    q, k, v = (t.to(DEVICE) for t in make_inputs(1, 8, 2, 16, 16, 128, dtype=torch.float32, seed=1))
    with pytest.raises(RuntimeError):
        gqa_flash_attn(q, k, v)


def test_no_device_error_recorded():
    torch.cuda.synchronize()
    assert check_device_error() == (0, 0)


@pytest.mark.parametrize("shape", [(4, 4, 1, 512, 16384, 128),   # prefill key split (last-CTA combine)
                                   (1, 32, 8, 1, 16384, 128)])   # split-KV decode (last-CTA combine)
def test_split_paths_are_deterministic(shape):
    """Which CTA of a unit arrives last varies from run to run; the combine must not."""
    q, k, v = (t.to(DEVICE) for t in make_inputs(*shape, seed=31))
    first = gqa_flash_attn(q, k, v, causal=True)
    for _ in range(4):
        assert torch.equal(gqa_flash_attn(q, k, v, causal=True).view(torch.int16), first.view(torch.int16))


def test_nvtx_ranges_do_not_change_results():
    import gqa_kernels
    q, k, v = (t.to(DEVICE) for t in make_inputs(1, 32, 8, 300, 300, 128, seed=32))
    plain = gqa_flash_attn(q, k, v, causal=True)
    gqa_kernels.set_nvtx_ranges(True)
    try:
        ranged = gqa_flash_attn(q, k, v, causal=True)
    finally:
        gqa_kernels.set_nvtx_ranges(False)
    assert torch.equal(plain.view(torch.int16), ranged.view(torch.int16))
