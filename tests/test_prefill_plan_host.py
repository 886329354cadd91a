"""The tcgen05 prefill path's launch planner (C ABI gqa_prefill_plan; host only, no
GPU): one CTA per unit (query pair x batch x kv head); units fewer than the SMs are
split across CTAs along the key axis; the unit order is head-major when the pairs'
key counts are within a factor of two, longest-first pair-major otherwise."""
import ctypes

import pytest

from gqa_kernels import _lib

B200_SMS = 148


def plan(B, Hq, Hkv, Sq, Skv, D=128, causal=True, sms=B200_SMS):
    out = (ctypes.c_int * 5)()
    rc = _lib.load().gqa_prefill_plan(B, Hq, Hkv, Sq, Skv, D, int(causal), sms, out)
    assert rc == 0
    units, nsplit, chunk, head_major, grid = list(out)
    assert grid == units * nsplit
    return dict(units=units, nsplit=nsplit, chunk=chunk, head_major=head_major, grid=grid)


def test_full_causal_prefill_runs_longest_pairs_first():
    assert plan(1, 32, 8, 8192, 8192) == dict(units=1024, nsplit=1, chunk=0, head_major=0, grid=1024)
    assert plan(1, 32, 8, 2048, 2048)["head_major"] == 0


def test_chunked_prefill_is_head_major():
    # config 4: 8 pairs per (batch, kv head), each seeing nearly all 16K keys
    assert plan(4, 32, 8, 512, 16384) == dict(units=256, nsplit=1, chunk=0, head_major=1, grid=256)
    assert plan(1, 32, 8, 8192, 8192, causal=False)["head_major"] == 1


def test_fewer_units_than_sms_split_the_keys():
    p = plan(1, 32, 8, 512, 16384)  # 64 units: 2 splits of 64 key tiles
    assert (p["units"], p["nsplit"], p["chunk"], p["grid"]) == (64, 2, 64, 128)
    p = plan(4, 4, 1, 512, 16384)  # one GPU's share of config 4 at 8 GPUs: 32 units, 4 splits
    assert (p["units"], p["nsplit"], p["chunk"]) == (32, 4, 32)
    p = plan(1, 8, 1, 256, 600)  # few key tiles: at least two per split
    assert p["nsplit"] == 1 or p["chunk"] >= 2


@pytest.mark.parametrize("sms", [132, 148, 160])
def test_splits_never_exceed_the_sms(sms):
    for shape in [(1, 32, 8, 512, 16384), (2, 8, 2, 300, 2000), (1, 32, 8, 128, 65536)]:
        p = plan(*shape, sms=sms)
        assert p["nsplit"] == 1 or p["grid"] <= sms
        assert p["nsplit"] <= 16


def test_bad_arguments():
    out = (ctypes.c_int * 5)()
    assert _lib.load().gqa_prefill_plan(1, 32, 8, 512, 512, 128, 1, 0, out) != 0
    assert _lib.load().gqa_prefill_plan(1, 32, 8, 512, 512, 96, 1, 148, out) != 0
