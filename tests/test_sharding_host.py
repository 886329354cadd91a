"""Host logic of the multi-GPU partitionings (gqa_kernels/sharded.py), on CPU.

The key-axis split is exercised end to end with gloo ranks: each rank's partial
comes from the oracle, the exchange is the product's gather_partials over the
product's packed layout, and the combine must equal full attention.
"""
import numpy as np
import pytest
import torch

from gqa_kernels import sharded as S
from oracle import gqa_oracle as O
from tests._dist import run_ranks


@pytest.mark.parametrize("n,parts", [(10, 3), (8, 8), (3, 5), (131072, 8), (0, 2)])
def test_balanced_range_partitions(n, parts):
    got = [S.balanced_range(n, parts, i) for i in range(parts)]
    assert got[0][0] == 0 and got[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
    sizes = [b - a for a, b in got]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("seq_kv,world", [(131072, 8), (16384, 3), (1000, 4), (64, 8)])
def test_kv_range_covers_keys(seq_kv, world):
    rs = [S.kv_range(seq_kv, world, r) for r in range(world)]
    assert rs[0][0] == 0 and rs[-1][1] == seq_kv
    assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
    assert all(a % 64 == 0 for a, _ in rs)


@pytest.mark.parametrize("batch,hkv,world", [(4, 8, 1), (4, 8, 2), (4, 8, 4), (4, 8, 8), (4, 8, 16), (64, 8, 32)])
def test_shard_units_cover_every_unit_once(batch, hkv, world):
    seen = np.zeros((batch, hkv), dtype=int)
    for r in range(world):
        (b0, b1), (h0, h1) = S.shard_units(batch, hkv, world, r)
        seen[b0:b1, h0:h1] += 1
    assert (seen == 1).all()


def test_slice_units_group_heads():
    q = torch.arange(2 * 8 * 3 * 4).reshape(2, 8, 3, 4)
    k = torch.arange(2 * 2 * 5 * 4).reshape(2, 2, 5, 4)
    qs, ks, vs = S.slice_units(q, k, k, (1, 2), (1, 2))
    assert torch.equal(qs, q[1:2, 4:8]) and torch.equal(ks, k[1:2, 1:2])


def test_exchange_layout():
    """The peer exchange buffer: two parities of `world` 16-byte-aligned slots of
    the packed partial, then the counters and the epoch (8-byte aligned)."""
    for shape in ((64, 64, 1, 128), (1, 32, 3, 64), (3, 5, 7, 64)):
        for world in (1, 2, 8):
            slot, parity, cnt_off, total = S.exchange_layout(shape, world)
            assert slot == S.packed_size(shape) and slot % 4 == 0
            assert parity == world * slot and cnt_off == 8 * parity
            assert cnt_off % 8 == 0 and total == cnt_off + 8 * world + 8


def test_peer_exchange_needs_keys_on_every_rank():
    """kv_range leaves ranks empty past the 64-key blocks; the peer form then does not
    apply (every rank must take the same form: the all-gather accepts empty shards)."""
    assert S.all_shards_hold_keys(131072, 8)
    assert S.all_shards_hold_keys(20000, 8)
    assert not S.all_shards_hold_keys(64, 2)
    assert not S.all_shards_hold_keys(300, 8)
    for skv, world in ((131072, 8), (20000, 8), (64, 2), (300, 8), (512, 8)):
        expect = all(b > a for a, b in (S.kv_range(skv, world, r) for r in range(world)))
        assert S.all_shards_hold_keys(skv, world) == expect


def test_packed_layout_alignment():
    for shape in [(1, 1, 1, 64), (64, 64, 1, 128), (3, 5, 7, 128)]:
        rows, acc_off, total = S.packed_layout(shape)
        assert acc_off % 4 == 0 and acc_off >= 2 * rows and total == acc_off + rows * shape[3]


def _seq_shard_rank(rank, world, B, Hq, Hkv, Sq, Skv, D, causal):
    rng = np.random.default_rng(0)
    q = rng.standard_normal((B, Hq, Sq, D))
    k = rng.standard_normal((B, Hkv, Skv, D))
    v = rng.standard_normal((B, Hkv, Skv, D))
    k0, k1 = S.kv_range(Skv, world, rank)
    m, l, acc = O.partial_attention(q, k[:, :, k0:k1], v[:, :, k0:k1], causal, k0, Skv)
    rows, acc_off, total = S.packed_layout(q.shape)
    packed = torch.zeros(total, dtype=torch.float32)
    packed[:rows] = torch.from_numpy(m.reshape(-1))
    packed[rows:2 * rows] = torch.from_numpy(l.reshape(-1))
    packed[acc_off:] = torch.from_numpy(acc.reshape(-1))
    g = S.gather_partials(packed).numpy()
    ms = g[:, :rows].reshape(world, B, Hq, Sq)
    ls = g[:, rows:2 * rows].reshape(world, B, Hq, Sq)
    accs = g[:, acc_off:].reshape(world, B, Hq, Sq, D)
    out = O.lse_combine(ms, ls, accs)
    full = O.gqa_reference(q, k, v, causal=causal, dtype=np.float64)
    return float(np.nanmax(np.abs(out - full))), bool(np.array_equal(np.isnan(out), np.isnan(full)))


@pytest.mark.parametrize("world,Sq,Skv,causal", [(2, 1, 300, True), (2, 5, 300, True), (3, 4, 300, False),
                                                 (3, 2, 100, True), (4, 1, 64, True)])
def test_seq_sharded_exchange_gloo(world, Sq, Skv, causal):
    """world > ceil(Skv / 64) leaves ranks with no keys: their (-inf, 0, 0) part joins the
    exchange like any other and weighs 0 in the combine."""
    if world > -(-Skv // 64):
        assert any(S.kv_range(Skv, world, r)[0] == S.kv_range(Skv, world, r)[1] for r in range(world))
    res = run_ranks(_seq_shard_rank, world, args=(2, 8, 2, Sq, Skv, 32, causal))
    assert len(res) == world
    for rank, (status, val) in res.items():
        assert status == "ok", val
        err, nan_ok = val
        assert nan_ok and err < 1e-5, (rank, err)
