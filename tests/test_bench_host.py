"""bench.py's host-side arithmetic (no GPU): the algorithmic work per launch that the
roofline numerators use, against the per-config figures of the measurement plan, and
the bounded CPU-baseline sample."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_prefill_flops_count_causal_pairs_only(bench):
    # 4 * B * Hq * D * S (S + 1) / 2 for a square causal prefill
    assert bench.attn_flops(1, 32, 8192, 8192, 128) == 4 * 32 * 128 * 8192 * 8193 / 2  # 549.82 GFLOP
    assert bench.attn_flops(1, 32, 2048, 2048, 128) == pytest.approx(34.38e9, rel=1e-3)
    # config 4: bottom-right, 512 queries over 16384 keys
    assert bench.attn_flops(4, 32, 512, 16384, 128) == 4 * 4 * 32 * 128 * (512 * 15872 + 512 * 513 // 2)
    assert bench.attn_flops(1, 8, 10, 10, 64, causal=False) == 4 * 8 * 64 * 100


def test_decode_bytes(bench):
    assert bench.wl_bytes(bench.WORKLOADS["decode"]) == 4096 * 16384 + 16384  # 67.13 MB (K + V + Q + O)
    # e4m3 K/V count one byte per element; Q and O stay 16-bit
    bf16 = bench.wl_bytes(bench.WORKLOADS["paged_decode"])
    fp8 = bench.wl_bytes(bench.WORKLOADS["paged_decode_fp8"])
    qo = 2 * 2 * 8 * 32 * 128
    assert fp8 - qo == (bf16 - qo) / 2
    assert bench.wl_bytes(bench.WORKLOADS["long_decode"]) == pytest.approx(34.36e9, rel=1e-3)


def test_causal_pairs_edge_cases(bench):
    assert bench.causal_pairs(4, 2) == 0 + 0 + 1 + 2  # seq_q > seq_kv: top rows see nothing
    assert bench.causal_pairs(1, 100) == 100
    assert bench.causal_pairs(3, 3, causal=False) == 9


def test_cpu_sample_is_bounded_and_counts_its_work(bench):
    val, unit, sample, per = bench.cpu_sample(bench.WORKLOADS["decode"], budget_s=0.0, steps=2)
    assert unit == "GB/s" and val > 0 and len(per) == 2 and "2 step(s)" in sample
    val, unit, _, _ = bench.cpu_sample(bench.WORKLOADS["paged_decode_fp8"], budget_s=0.0, steps=1)
    assert unit == "GB/s" and val > 0
