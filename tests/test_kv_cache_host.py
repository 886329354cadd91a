"""PrefixKVCache bookkeeping on CPU tensors (no GPU): appends land after the cached
positions, views share the cache's storage, truncation and the capacity limit."""
import pytest
import torch

from gqa_kernels.kv_cache import PrefixKVCache


def _chunk(n, seed, B=2, H=4, D=64):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, H, n, D, generator=g).to(torch.bfloat16), torch.randn(B, H, n, D, generator=g).to(torch.bfloat16)


def test_append_and_views():
    c = PrefixKVCache(2, 4, 64, capacity=100, device="cpu")
    k1, v1 = _chunk(30, 1)
    k2, v2 = _chunk(7, 2)
    assert c.append(k1, v1) == 30 and c.append(k2, v2) == 37
    assert torch.equal(c.keys(), torch.cat([k1, k2], dim=2))
    assert torch.equal(c.values(), torch.cat([v1, v2], dim=2))
    # views of the cache, not copies
    assert c.keys().data_ptr() == c.k.data_ptr() and c.keys().stride() == c.k.stride()


def test_truncate_then_append_replaces_the_tail():
    c = PrefixKVCache(2, 4, 64, capacity=64, device="cpu")
    kp, vp = _chunk(20, 3)
    c.append(kp, vp)
    c.append(*_chunk(10, 4))
    c.truncate(20)
    kb, vb = _chunk(5, 5)
    c.append(kb, vb)
    assert c.length == 25
    assert torch.equal(c.keys(), torch.cat([kp, kb], dim=2))


def test_limits_and_mismatches_raise():
    c = PrefixKVCache(2, 4, 64, capacity=16, device="cpu")
    c.append(*_chunk(10, 6))
    with pytest.raises(ValueError, match="cache full"):
        c.append(*_chunk(7, 7))
    with pytest.raises(ValueError):
        c.truncate(11)
    with pytest.raises(ValueError):
        c.append(*_chunk(2, 8, H=2))
    with pytest.raises(TypeError):
        k, v = _chunk(2, 9)
        c.append(k.float(), v.float())
    with pytest.raises(ValueError):
        PrefixKVCache(1, 1, 96, capacity=8, device="cpu")
