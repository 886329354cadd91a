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
    for kind in ("torch", "numpy"):
        val, unit, sample, per, cores = bench.cpu_sample(bench.WORKLOADS["decode"], budget_s=0.0, steps=2, kind=kind)
        assert unit == "GB/s" and val > 0 and len(per) == 2 and "2 step(s)" in sample and cores >= 1
        val, unit, _, _, _ = bench.cpu_sample(bench.WORKLOADS["paged_decode_fp8"], budget_s=0.0, steps=1, kind=kind)
        assert unit == "GB/s" and val > 0
    val, unit, sample, _, _ = bench.cpu_sample(bench.WORKLOADS["prefill"], budget_s=0.0, steps=1, kind="torch")
    assert unit == "TFLOP/s" and "tests/reference.py" in sample


def test_reference_arm_config_is_the_gpu_line_config(bench):
    """The reference arm prints the config dict of the GPU line (same workload, same N)."""
    for name, wl in bench.WORKLOADS.items():
        for world in (1, 8):
            a = bench.config_of(wl, world, name)
            assert a == bench.config_of(dict(wl), world, name)
            assert a["workload"] == wl["name"] and a["seq_kv"] == wl["Skv"]


def _rows_setup(seed=0, B=2, Hq=8, Hkv=2, Sq=5, Skv=300, D=64):
    import torch
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, Sq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, Skv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, Skv, D, generator=g).to(torch.bfloat16)
    return q, k, v


def test_parity_check_accepts_the_oracle_and_rejects_a_planted_error(bench):
    import torch
    from oracle import gqa_oracle_torch as T
    q, k, v = _rows_setup()
    o = T.gqa_reference_blocked(q, k, v, causal=True).to(torch.bfloat16)
    assert bench.parity_check({"q": q, "k": k, "v": v, "o": o}, 1)["ok"]
    bad = o.clone()
    for b, h, i in bench.check_rows_sel(q.shape, 16)[:1]:
        bad[b, h, i, 3] += 0.25  # one wrong element in one checked row
    res = bench.parity_check({"q": q, "k": k, "v": v, "o": bad}, 1)
    assert not res["ok"] and res["max_abs"] >= 0.2


def test_row_partials_combine_to_the_full_rows(bench):
    """Key-range statistics of the in-run check, combined by log-sum-exp, equal the rows
    over all keys (the check of the key-sharded configuration), empty ranges included."""
    import torch
    q, k, v = _rows_setup(seed=1)
    sel = bench.check_rows_sel(q.shape, 12, seed=3)
    full = bench.fp32_row_partials(q, k, v, sel)
    ref = full[:, 2:] / full[:, 1:2]
    for cuts in ([0, 100, 300], [0, 0, 64, 300], [0, 299, 300, 300]):
        parts = torch.stack([bench.fp32_row_partials(q, k[:, :, a:b], v[:, :, a:b], sel, True, a, 300)
                             for a, b in zip(cuts, cuts[1:])])
        m = parts[:, :, 0]
        w = torch.where(torch.isinf(m), torch.zeros_like(m), torch.exp(m - m.max(0).values))
        got = (w[:, :, None] * parts[:, :, 2:]).sum(0) / (w * parts[:, :, 1]).sum(0)[:, None]
        assert torch.allclose(got, ref, rtol=1e-6, atol=1e-7)


def _sharded_parity_rank(rank, world):
    import importlib.util
    import torch
    from oracle import gqa_oracle_torch as T
    spec = importlib.util.spec_from_file_location("bench_rank", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    q, k, v = _rows_setup(seed=2, Skv=400)
    o = T.gqa_reference_blocked(q, k, v, causal=True).to(torch.bfloat16)
    a, b = (0, 128) if rank == 0 else (128, 400)
    local = {"q": q, "k": k[:, :, a:b], "v": v[:, :, a:b], "o": o, "kv_offset": a, "seq_kv_total": 400}
    good = bench.parity_check(local, world, sharded_keys=True)["ok"]
    # a wrong output on one rank fails the check on every rank
    if rank == 1:
        local["o"] = o + 0.5
    bad = bench.parity_check(local, world, sharded_keys=True)["ok"]
    return good, bad


def test_sharded_parity_check_over_gloo():
    from tests._dist import run_ranks
    out = run_ranks(_sharded_parity_rank, 2, timeout_s=60)
    assert len(out) == 2, out
    for rank, (status, res) in out.items():
        assert status == "ok", res
        assert res == (True, False), (rank, res)


def _row(workload, L, ours, fa2, sdpa):
    sq = L if workload == "prefill" else 1
    return {"workload": workload, "seq_kv": L, "ours_ms": ours, "fa2_ms": fa2, "sdpa_ms": sdpa,
            "tok_s": sq * 1000.0 / ours, "speedup_vs_fa2": fa2 / ours, "speedup_vs_sdpa": sdpa / ours,
            "peak_mem_gb": 0.1, "roofline_frac": 0.5}


def test_sweep_results_keep_the_reference_harness_schema(bench):
    """--sweep writes benchmark/run.py's results schema (commit, device, dtype, trials,
    config, rows with the same row keys) plus its own keys."""
    trials = [[_row("prefill", 2048, 0.03, 0.09, 0.04), _row("decode", 2048, 0.008, 0.02, 0.009)],
              [_row("prefill", 2048, 0.05, 0.08, 0.05), _row("decode", 2048, 0.006, 0.02, 0.01)],
              [_row("prefill", 2048, 0.04, 0.10, 0.06), _row("decode", 2048, 0.007, 0.03, 0.008)]]
    rows = bench.aggregate_median(trials)
    assert rows[0]["ours_ms"] == 0.04 and rows[1]["sdpa_ms"] == 0.009
    assert rows[0]["speedup_vs_fa2"] == pytest.approx(0.09 / 0.04)
    doc = bench.sweep_document(rows, True, [], 3, "NVIDIA B200", True, bench.measured_peaks())
    for key in ("commit", "device", "dtype", "trials", "config", "rows"):
        assert key in doc
    assert doc["config"] == {"batch": 1, "num_heads": 32, "num_kv_heads": 8, "head_dim": 128,
                             "model": "Llama 3.1 8B attention shape"}
    ref_row_keys = {"workload", "seq_kv", "ours_ms", "fa2_ms", "sdpa_ms", "tok_s", "speedup_vs_fa2",
                    "speedup_vs_sdpa", "peak_mem_gb"}
    assert all(ref_row_keys <= set(r) for r in doc["rows"])
    import json
    json.dumps(doc)  # serialisable
    table = bench.markdown_table(doc)
    assert table.count("\n") == 1 + len(rows) and "| prefill | 2048 |" in table


def test_sweep_lengths_are_the_reference_harness_lengths(bench):
    assert bench.SWEEP_PREFILL == (2048, 4096, 6144, 8192, 12288, 16384)
    assert bench.SWEEP_DECODE == (2048, 4096, 8192, 16384)
    assert bench.GATE_LENS == (512, 2048, 4096) and bench.GATE_TOL == (1e-2, 1e-3)


def test_fp32_attention_checker_matches_the_oracle(bench):
    """The harness gate's fp32 checker against the torch restatement of the reference oracle."""
    import torch
    from oracle import gqa_oracle_torch as T
    q, k, v = _rows_setup(seed=3, Sq=20, Skv=50)
    ref = T.gqa_reference_blocked(q, k, v, causal=True)
    assert torch.allclose(bench.fp32_attention(q, k, v), ref, atol=1e-6, rtol=1e-5)


def test_reference_arm_line(bench, capsys, monkeypatch):
    """--impl reference prints one line with the GPU line's config, its CPU sample and an
    e2e that moves no bytes; warm-up steps are not timed."""
    import argparse
    import json
    monkeypatch.delenv("RANK", raising=False)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    args = argparse.Namespace(workload="decode", warmup=3)
    bench.main_reference(args, bench.WORKLOADS["decode"], 3)
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "GB/s"
    assert line["config"] == bench.config_of(bench.WORKLOADS["decode"], 1, "decode")
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and "warm-up step(s) untimed" in line["cpu_baseline"]["sample"]
