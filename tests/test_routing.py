"""The shim's dispatcher routes every shape exactly as the reference's dispatcher
(golden table recorded from gqa_kernels/dispatch.py:37-49 by make_golden.py). No GPU."""
import json
import os
import types

import pytest

import gqa_kernels.dispatch as D

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "routing.json")


class _Fake:
    is_cuda = True
    dtype = "bf16"
    device = "cuda:0"

    def __init__(self, shape):
        self.shape = tuple(shape)

    def stride(self, i=None):
        return 0 if i is not None else (0, 0, 0, 0)


@pytest.fixture
def recorder(monkeypatch):
    calls = []

    class _Rec:
        def __getitem__(self, grid):
            def launch(*a, **kw):
                calls.append(("single", None, kw))
            return launch

    monkeypatch.setattr(D, "split_kv_forward", lambda q, k, v, causal, splits: calls.append(("split", splits, {})))
    monkeypatch.setattr(D, "gqa_fwd_kernel", _Rec())
    monkeypatch.setattr(D, "_layout_ok", lambda *ts: True)
    monkeypatch.setattr(D, "torch", types.SimpleNamespace(empty_like=lambda t: _Fake(t.shape)))
    return calls


def test_routing_matches_reference(recorder):
    with open(GOLD) as f:
        rows = json.load(f)["rows"]
    for sq, skv, hkv, batch, path, splits in rows:
        recorder.clear()
        D.gqa_flash_attn(_Fake((batch, hkv * 4, sq, 128)), _Fake((batch, hkv, skv, 128)),
                         _Fake((batch, hkv, skv, 128)), causal=True)
        assert (recorder[0][0], recorder[0][1]) == (path, splits), (sq, skv, hkv, batch)


def test_single_pass_launch_arguments(recorder):
    D.gqa_flash_attn(_Fake((2, 16, 100, 64)), _Fake((2, 4, 300, 64)), _Fake((2, 4, 300, 64)), causal=False)
    kind, _, kw = recorder[0]
    assert kind == "single"
    assert kw == {"IS_CAUSAL": False, "GROUP_SIZE": 4, "HEAD_DIM": 64}


def test_reference_asserts_kept():
    with pytest.raises(AssertionError, match="divisible"):
        D.gqa_flash_attn(_Fake((1, 6, 4, 64)), _Fake((1, 4, 4, 64)), _Fake((1, 4, 4, 64)))
    with pytest.raises(AssertionError, match="unsupported head_dim"):
        D.gqa_flash_attn(_Fake((1, 8, 4, 96)), _Fake((1, 2, 4, 96)), _Fake((1, 2, 4, 96)))
    cpu = _Fake((1, 8, 4, 64))
    cpu.is_cuda = False
    with pytest.raises(AssertionError):
        D.gqa_flash_attn(cpu, _Fake((1, 2, 4, 64)), _Fake((1, 2, 4, 64)))


def test_sm_count_constant_is_the_reference_one():
    assert D.SM_COUNT == 28 and D.LOG2E == 1.4426950408889634
