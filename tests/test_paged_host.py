"""Argument checks of the paged-attention API (gqa_kernels.paged) on CPU tensors: every
malformed call raises before anything is launched, so these run without a GPU."""
import pytest
import torch

from gqa_kernels.paged import paged_decode, paged_prefill


def _cache(num_blocks=4, block_size=64, hkv=2, D=128, dtype=torch.bfloat16):
    return torch.zeros(num_blocks, block_size, hkv, D, dtype=dtype), torch.zeros(num_blocks, block_size, hkv, D,
                                                                                  dtype=dtype)


def _meta(n=2, max_blocks=2):
    return torch.zeros(n, max_blocks, dtype=torch.int32), torch.full((n,), 10, dtype=torch.int32)


def test_cache_shape_and_heads():
    kc, vc = _cache()
    bt, sl = _meta()
    q = torch.zeros(2, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="num_blocks, block_size"):
        paged_decode(q, kc, vc[:, :, :, :64], bt, sl)
    with pytest.raises(ValueError, match="num_blocks, block_size"):
        paged_decode(torch.zeros(2, 8, 64, dtype=torch.bfloat16), kc, vc, bt, sl)
    with pytest.raises(ValueError, match="divisible"):
        paged_decode(torch.zeros(2, 7, 128, dtype=torch.bfloat16), kc, vc, bt, sl)


def test_tensors_must_be_on_the_gpu():
    kc, vc = _cache()
    bt, sl = _meta()
    with pytest.raises(ValueError, match="CUDA"):
        paged_decode(torch.zeros(2, 8, 128, dtype=torch.bfloat16), kc, vc, bt, sl)
    with pytest.raises(ValueError, match="CUDA"):
        paged_prefill(torch.zeros(2, 8, 16, 128, dtype=torch.bfloat16), kc, vc, bt, sl)


def test_dtypes():
    kc, vc = _cache(dtype=torch.float16)
    bt, sl = _meta()
    q = torch.zeros(2, 8, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(TypeError, match="dtype"):
        paged_prefill(q, kc, vc, bt, sl)  # fp16 caches under bf16 queries
    k8, v8 = _cache(dtype=torch.float8_e4m3fn)
    with pytest.raises(TypeError, match="dtype"):
        paged_prefill(q, k8, vc, bt, sl)  # mixed cache dtypes


def test_block_table_and_lengths():
    kc, vc = _cache()
    q = torch.zeros(2, 8, 128, dtype=torch.bfloat16)
    bt, sl = _meta()
    with pytest.raises(TypeError, match="int32"):
        paged_decode(q, kc, vc, bt.long(), sl)
    with pytest.raises(TypeError, match="int32"):
        paged_decode(q, kc, vc, bt, sl.long())
    with pytest.raises(ValueError, match="num_seqs"):
        paged_decode(q, kc, vc, bt[:1], sl)
    with pytest.raises(ValueError, match="num_seqs"):
        paged_decode(q, kc, vc, bt, sl[:1])


def test_caches_must_be_contiguous():
    kc, vc = _cache()
    bt, sl = _meta()
    q = torch.zeros(2, 8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="contiguous"):
        paged_decode(q, kc.transpose(0, 1).contiguous().transpose(0, 1), vc, bt, sl)


def test_split_and_partial_entry_points_refuse_host_tensors():
    from gqa_kernels import sharded
    from gqa_kernels.gqa_split import split_kv_forward, split_kv_two_pass
    q = torch.zeros(1, 8, 1, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 2048, 128, dtype=torch.bfloat16)
    for fn in (lambda: split_kv_forward(q, k, k, True, 4), lambda: split_kv_two_pass(q, k, k, True, 4),
               lambda: sharded.partial_forward(q, k, k, True, 0, 2048)):
        with pytest.raises(ValueError, match="CUDA"):
            fn()


def test_paged_oracle_equals_the_dense_oracle_on_gathered_keys():
    """oracle.paged_reference against gqa_reference on the same keys laid out densely:
    shuffled blocks, lengths below, at and above the chunk, an empty sequence, scales."""
    import numpy as np
    from oracle import gqa_oracle as O
    rng = np.random.default_rng(0)
    bs, Hkv, Hq, D, Sq = 16, 2, 8, 32, 5
    seq_lens = [3, 5, 40, 0]
    n_blocks = sum(-(-s // bs) for s in seq_lens) + 2
    kc = rng.standard_normal((n_blocks, bs, Hkv, D)).astype(np.float32)
    vc = rng.standard_normal((n_blocks, bs, Hkv, D)).astype(np.float32)
    perm = rng.permutation(n_blocks)
    bt = np.zeros((len(seq_lens), 3), dtype=np.int32)
    c = 0
    for i, s in enumerate(seq_lens):
        for j in range(-(-s // bs)):
            bt[i, j] = perm[c]
            c += 1
    q = rng.standard_normal((len(seq_lens), Hq, Sq, D)).astype(np.float32)
    out = O.paged_reference(q, kc, vc, bt, seq_lens, causal=True, k_scale=0.5, v_scale=2.0)
    for i, s in enumerate(seq_lens):
        if s == 0:
            assert np.isnan(out[i]).all()
            continue
        k = np.concatenate([kc[bt[i, j]] for j in range(-(-s // bs))])[:s].transpose(1, 0, 2)[None] * 0.5
        v = np.concatenate([vc[bt[i, j]] for j in range(-(-s // bs))])[:s].transpose(1, 0, 2)[None] * 2.0
        ref = O.gqa_reference(q[i:i + 1], k, v, causal=True)[0]
        np.testing.assert_allclose(out[i], ref, rtol=1e-6, atol=1e-6, equal_nan=True)
    assert np.isnan(out[0, :, :2]).all() and not np.isnan(out[0, :, 2:]).any()  # 3 keys, 5 queries


def test_kv_append_argument_checks_before_the_device():
    """paged_kv_append validates shapes and dtypes on CPU tensors before any launch."""
    from gqa_kernels.paged import paged_kv_append
    k = torch.zeros(4, 2, 128, dtype=torch.bfloat16)
    kc = torch.zeros(3, 64, 2, 128, dtype=torch.bfloat16)
    slots = torch.zeros(4, dtype=torch.int64)
    with pytest.raises(ValueError):
        paged_kv_append(k, k[:, :1], kc, kc, slots)  # value shape
    with pytest.raises(ValueError):
        paged_kv_append(k, k, kc[:, :, :1], kc[:, :, :1], slots)  # cache heads
    with pytest.raises(TypeError):
        paged_kv_append(k, k, kc.half(), kc.half(), slots)  # cache dtype
    with pytest.raises(TypeError):
        paged_kv_append(k, k, kc, kc, slots.int())  # slot dtype
    with pytest.raises(ValueError):
        paged_kv_append(k, k, kc.to(torch.float8_e4m3fn), kc.to(torch.float8_e4m3fn), slots, k_scale=0.0)
    with pytest.raises(ValueError):
        paged_kv_append(k, k, kc, kc, slots)  # CPU tensors: not CUDA memory


def test_paged_attention_layer_arguments():
    from gqa_kernels.paged import PagedAttention
    with pytest.raises(ValueError):
        PagedAttention(32, 128, num_kv_heads=6)
    with pytest.raises(ValueError):
        PagedAttention(32, 128, kv_cache_dtype="fp8_e5m2")
    layer = PagedAttention(32, 128, num_kv_heads=8, kv_cache_dtype="fp8_e4m3")
    cache = layer.allocate_kv_cache(4, 64, torch.bfloat16, "cpu")
    assert cache.shape == (2, 4, 64, 8, 128) and cache.dtype == torch.float8_e4m3fn


def test_paged_attention_layer_rejects_inconsistent_query_lens():
    from gqa_kernels.paged import PagedAttention, PagedAttentionMetadata
    layer = PagedAttention(8, 64, num_kv_heads=2)
    q = torch.zeros(5, 8 * 64, dtype=torch.bfloat16)
    kv = torch.zeros(5, 2 * 64, dtype=torch.bfloat16)
    cache = layer.allocate_kv_cache(4, 64, torch.bfloat16, "cpu")
    md = PagedAttentionMetadata(slot_mapping=torch.zeros(5, dtype=torch.int64),
                                block_tables=torch.zeros(2, 2, dtype=torch.int32),
                                seq_lens=torch.tensor([3, 3], dtype=torch.int32), query_lens=[2, 2])
    with pytest.raises(ValueError):
        layer.forward(q, kv, kv, cache, md)  # 2 + 2 != 5 tokens
    md.query_lens = None
    md.query_len = 2
    with pytest.raises(ValueError):
        layer.forward(q, kv, kv, cache, md)  # 2 sequences x 2 != 5 tokens
