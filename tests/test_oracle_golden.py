"""Pins the CPU oracle (oracle/gqa_oracle.py) to outputs of the reference itself.

The fixtures come from tests/golden/make_golden.py: the reference's torch
oracle (tests/reference.py) on bf16 inputs, and the reference's Triton kernels
run by Triton's CPU interpreter on fp16 inputs. No GPU needed.
"""
import json
import os
import zlib

import numpy as np
import pytest
import torch

from oracle import gqa_oracle as O
from tests._common import make_inputs

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def oracle_gold():
    return np.load(os.path.join(GOLD, "oracle_bf16.npz"))


@pytest.fixture(scope="module")
def triton_gold():
    return np.load(os.path.join(GOLD, "triton_f16.npz"))


def _cases(npz, prefix=""):
    return sorted({k.split("/")[0] for k in npz.files if k.startswith(prefix)})


def _nan_equal(a, b):
    return np.array_equal(np.isnan(a), np.isnan(b))


def test_bf16_rounding_matches_torch():
    x = torch.randn(10000) * 10
    ref = x.to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.bf16_round(x.numpy()), ref)
    bits = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(O.f32_to_bf16_bits(x.numpy()), bits)
    assert np.array_equal(O.bf16_bits_to_f32(bits), ref)


def test_oracle_matches_reference_oracle(oracle_gold):
    names = [c for c in _cases(oracle_gold) if c != "config1"]
    assert len(names) >= 9
    for name in names:
        B, Hq, Hkv, Sq, Skv, D, causal, seed = oracle_gold[f"{name}/meta"]
        q = O.bf16_bits_to_f32(oracle_gold[f"{name}/q"])
        k = O.bf16_bits_to_f32(oracle_gold[f"{name}/k"])
        v = O.bf16_bits_to_f32(oracle_gold[f"{name}/v"])
        ref = oracle_gold[f"{name}/out"]
        out = O.gqa_reference(q, k, v, causal=bool(causal))
        assert out.shape == ref.shape
        assert _nan_equal(out, ref), name
        fin = ~np.isnan(ref)
        np.testing.assert_allclose(out[fin], ref[fin], rtol=1e-5, atol=1e-5, err_msg=name)


def test_sq_gt_skv_gives_nan_rows(oracle_gold):
    ref = oracle_gold["sq_gt_skv/out"]
    B, Hq, Hkv, Sq, Skv, D, causal, seed = oracle_gold["sq_gt_skv/meta"]
    # rows i with i + (Skv - Sq) < 0 see no key
    dead = np.arange(Sq) + (Skv - Sq) < 0
    assert np.isnan(ref[:, :, dead]).all() and not np.isnan(ref[:, :, ~dead]).any()


def test_input_generator_is_the_fixtures(oracle_gold):
    """The test-suite generator (CPU torch.Generator, q/k/v order) reproduces the fixture inputs."""
    for name in ("prefill_g4_d64", "odd_17_65"):
        B, Hq, Hkv, Sq, Skv, D, causal, seed = (int(x) for x in oracle_gold[f"{name}/meta"])
        q, k, v = make_inputs(B, Hq, Hkv, Sq, Skv, D, seed=seed)
        for key, t in (("q", q), ("k", k), ("v", v)):
            assert np.array_equal(t.view(torch.int16).numpy().view(np.uint16), oracle_gold[f"{name}/{key}"])


def test_config1_summary(oracle_gold):
    """BASELINE config 1 (B=1, Hq=32, Hkv=8, D=128, S=512, causal, seed 0) in full through the oracle."""
    B, Hq, Hkv, S, _, D, causal, seed = (int(x) for x in oracle_gold["config1/meta"])
    q, k, v = make_inputs(B, Hq, Hkv, S, S, D, seed=seed)
    crc = [zlib.crc32(t.view(torch.int16).numpy().view(np.uint16).tobytes()) for t in (q, k, v)]
    assert crc == list(oracle_gold["config1/crc_qkv"])
    out = O.gqa_reference(*(t.float().numpy() for t in (q, k, v)), causal=True)
    rows = oracle_gold["config1/rows"]
    np.testing.assert_allclose(out[0, rows[:, 0], rows[:, 1]], oracle_gold["config1/row_out"], rtol=1e-5, atol=1e-5)
    s = oracle_gold["config1/sum"]
    assert abs(out.astype(np.float64).sum() - s[0]) < 1e-2
    assert abs(np.abs(out.astype(np.float64)).sum() - s[1]) < 1e-2 * max(1.0, s[1] * 1e-6)
    # the row-sampled oracle agrees with the full one
    sel = [(0, int(h), int(i)) for h, i in rows[:8]]
    rr = O.gqa_reference_rows(*(t.float().numpy() for t in (q, k, v)), sel, causal=True)
    np.testing.assert_allclose(rr, out[0, rows[:8, 0], rows[:8, 1]], rtol=1e-4, atol=1e-5)


def test_blocked_kernel_restatement_matches_triton(triton_gold):
    """oracle.gqa_fwd_blocked restates gqa_fwd.py; compare with the reference Triton kernel (fp16)."""
    names = _cases(triton_gold, "fwd_")
    assert names
    for name in names:
        B, Hq, Hkv, Sq, Skv, D, causal, seed, BM, BN = (int(x) for x in triton_gold[f"{name}/meta"])
        q, k, v = (triton_gold[f"{name}/{x}"].astype(np.float32) for x in "qkv")
        ref = triton_gold[f"{name}/out"].astype(np.float32)
        out = O.gqa_fwd_blocked(q, k, v, bool(causal), block_m=BM, block_n=BN, io="f16")
        assert _nan_equal(out, ref), name
        fin = ~np.isnan(ref)
        d = np.abs(out[fin] - ref[fin])
        # both round P and the output to fp16; accumulation order differs
        assert d.max() < 4e-3 and d.mean() < 2e-4, (name, d.max(), d.mean())
        # and the kernel restatement agrees with the naive oracle within fp16 tolerance
        naive = O.gqa_reference(q, k, v, causal=bool(causal))
        d2 = np.abs(out[fin] - naive[fin])
        assert d2.max() < 2e-2 and d2.mean() < 2e-3, (name, d2.max(), d2.mean())


SPLIT_BLOCK_N = 32  # the BLOCK_N make_golden.py ran the reference split kernel with


def test_split_restatement_matches_triton(triton_gold):
    for name in _cases(triton_gold, "split_"):
        B, Hq, Hkv, Sq, Skv, D, causal, seed, splits = (int(x) for x in triton_gold[f"{name}/meta"])
        q, k, v = (triton_gold[f"{name}/{x}"].astype(np.float32) for x in "qkv")
        m_p, l_p, acc_p = O.gqa_split_first(q, k, v, bool(causal), splits, io="f16", block_n=SPLIT_BLOCK_N)
        for key, mine in (("m_p", m_p), ("l_p", l_p), ("acc_p", acc_p)):
            ref = triton_gold[f"{name}/{key}"]
            assert _nan_equal(mine, ref), (name, key)
            fin = np.isfinite(ref)
            assert np.array_equal(np.isinf(mine), np.isinf(ref)), (name, key)
            np.testing.assert_allclose(mine[fin], ref[fin], rtol=2e-3, atol=5e-3, err_msg=f"{name}/{key}")
        out = O.gqa_split_reduce(m_p, l_p, acc_p, io="f16")
        ref = triton_gold[f"{name}/out"].astype(np.float32)
        assert _nan_equal(out, ref), name
        fin = ~np.isnan(ref)
        np.testing.assert_allclose(out[fin], ref[fin], rtol=2e-3, atol=2e-3, err_msg=name)


def test_reference_split_block_overrun(triton_gold):
    """Where ceil(seq_kv/splits) is not a multiple of BLOCK_N the reference's split
    result differs from its own oracle (keys read twice); where it is, the exact-chunk
    restatement (CUDA semantics) and the reference agree."""
    name = "split_decode"  # ceil(200/4) = 50, BLOCK_N 32
    q, k, v = (triton_gold[f"{name}/{x}"].astype(np.float32) for x in "qkv")
    naive = O.gqa_reference(q, k, v, causal=True)
    assert np.abs(triton_gold[f"{name}/out"] - naive).max() > 5e-2
    exact = O.gqa_split_reduce(*O.gqa_split_first(q, k, v, True, 4, io="f16"), io="f16")
    assert np.abs(exact - naive).max() < 2e-3
    name = "split_clean_chunks"
    B, Hq, Hkv, Sq, Skv, D, causal, seed, splits = (int(x) for x in triton_gold[f"{name}/meta"])
    q, k, v = (triton_gold[f"{name}/{x}"].astype(np.float32) for x in "qkv")
    exact = O.gqa_split_first(q, k, v, True, splits, io="f16")
    for key, mine in zip(("m_p", "l_p", "acc_p"), exact):
        np.testing.assert_allclose(mine, triton_gold[f"{name}/{key}"], rtol=2e-3, atol=5e-3)


def test_reference_split_nan_on_fully_masked_chunk(triton_gold):
    """The reference's split path gives NaN partials (and NaN output) for a row whose
    non-empty chunk is fully masked; the clean variant (the CUDA kernels' semantics)
    gives (-inf, 0, 0) and a finite output equal to the naive oracle."""
    name = "split_masked_chunk"
    B, Hq, Hkv, Sq, Skv, D, causal, seed, splits = (int(x) for x in triton_gold[f"{name}/meta"])
    q, k, v = (triton_gold[f"{name}/{x}"].astype(np.float32) for x in "qkv")
    assert np.isnan(triton_gold[f"{name}/out"]).any()
    m_p, l_p, acc_p = O.gqa_split_first(q, k, v, True, splits, io="f16", clean_masked=True)
    assert np.isfinite(l_p).all() and not np.isnan(m_p).any()
    assert np.isnan(O.gqa_split_first(q, k, v, True, splits, io="f16", block_n=SPLIT_BLOCK_N)[1]).any()
    out = O.gqa_split_reduce(m_p, l_p, acc_p, io="f16")
    naive = O.gqa_reference(q, k, v, causal=True)
    np.testing.assert_allclose(out, naive, atol=2e-3)


def test_route_matches_reference_dispatcher():
    with open(os.path.join(GOLD, "routing.json")) as f:
        table = json.load(f)["rows"]
    assert len(table) > 1000
    for sq, skv, hkv, batch, path, splits in table:
        assert O.route(sq, skv, hkv, batch) == (path, splits), (sq, skv, hkv, batch)


def test_lse_combine_equals_full_attention():
    rng = np.random.default_rng(0)
    B, Hq, Hkv, Sq, Skv, D = 2, 8, 2, 5, 300, 64
    q, k, v = (rng.standard_normal(s).astype(np.float32) for s in
               [(B, Hq, Sq, D), (B, Hkv, Skv, D), (B, Hkv, Skv, D)])
    full = O.gqa_reference(q, k, v, causal=True, dtype=np.float64)
    for cuts in ([0, 300], [0, 100, 300], [0, 64, 128, 250, 300], [0, 1, 2, 299, 300]):
        parts = [O.partial_attention(q, k[:, :, a:b], v[:, :, a:b], True, a, Skv) for a, b in zip(cuts, cuts[1:])]
        ms, ls, accs = (np.stack(x) for x in zip(*parts))
        np.testing.assert_allclose(O.lse_combine(ms, ls, accs), full, rtol=1e-9, atol=1e-10)


def test_torch_restatement_matches_reference_oracle(oracle_gold):
    """oracle/gqa_oracle_torch.py (the torch restatement used as the full-size GPU checker
    and as the timed CPU baseline) against the reference oracle's recorded outputs, both
    whole and blocked over query rows (small blocks exercise the bottom-right key prefix)."""
    from oracle import gqa_oracle_torch as T
    names = [c for c in _cases(oracle_gold) if c != "config1"]
    for name in names:
        B, Hq, Hkv, Sq, Skv, D, causal, seed = (int(x) for x in oracle_gold[f"{name}/meta"])
        q, k, v = (torch.from_numpy(O.bf16_bits_to_f32(oracle_gold[f"{name}/{x}"])) for x in "qkv")
        ref = oracle_gold[f"{name}/out"]
        for out in (T.gqa_reference(q, k, v, causal=bool(causal)).numpy(),
                    T.gqa_reference_blocked(q, k, v, causal=bool(causal), row_block=7).numpy()):
            assert out.shape == ref.shape
            assert _nan_equal(out, ref), name
            fin = ~np.isnan(ref)
            np.testing.assert_allclose(out[fin], ref[fin], rtol=1e-5, atol=1e-5, err_msg=name)


def test_torch_restatement_config1_rows(oracle_gold):
    B, Hq, Hkv, S, _, D, causal, seed = (int(x) for x in oracle_gold["config1/meta"])
    q, k, v = make_inputs(B, Hq, Hkv, S, S, D, seed=seed)
    from oracle import gqa_oracle_torch as T
    out = T.gqa_reference_blocked(q, k, v, causal=True, row_block=100).numpy()
    rows = oracle_gold["config1/rows"]
    np.testing.assert_allclose(out[0, rows[:, 0], rows[:, 1]], oracle_gold["config1/row_out"], rtol=1e-5, atol=1e-5)
