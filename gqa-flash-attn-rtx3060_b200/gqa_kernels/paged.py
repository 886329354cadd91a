"""Paged-KV attention with vLLM-shaped signatures.

The reference's roadmap (README.md:144) names a vLLM-compatible interface as
mostly glue over its kernel. In vLLM, keys and values live in a paged cache:
fixed-size blocks (num_blocks, block_size, num_kv_heads, head_dim) and a
per-sequence block table. The kernels here read such a cache in place, with no
gather copy: their TMA producers map every 64-key box through the block table.

- `paged_decode`: one new query token per sequence over all of that sequence's
  cached keys (the split-KV streaming kernel; the reference's
  gqa_kernels/gqa_split.py attention).
- `paged_prefill`: a chunk of new query tokens per sequence, bottom-right
  aligned to the sequence's own length (chunked prefill, speculative decoding):
  the tcgen05 prefill kernel for long chunks, the streaming kernel for short
  ones (the reference's gqa_kernels/gqa_fwd.py attention).

Cache slots past a sequence's length in its last block are read and masked, so
they must hold finite values (vLLM zero-initialises its caches).
"""
import ctypes

import torch

from . import _lib

__all__ = ["paged_decode", "paged_prefill"]

LOG2E = 1.4426950408889634


def paged_decode(query, key_cache, value_cache, block_tables, seq_lens, max_seq_len=None, scale=None,
                 k_scale=1.0, v_scale=1.0):
    """Decode attention over a paged K/V cache.

    Args:
        query: (num_seqs, num_heads, head_dim), bf16 or fp16, one token per sequence.
        key_cache, value_cache: (num_blocks, block_size, num_kv_heads, head_dim), contiguous,
            block_size a power of two >= 64; query's dtype, or torch.float8_e4m3fn (head_dim
            128) with key = stored key * k_scale and value = stored value * v_scale.
        block_tables: int32 (num_seqs, max_blocks_per_seq); sequence b's key k is in block
            block_tables[b, k // block_size] at position k % block_size.
        seq_lens: int32 (num_seqs,), keys cached per sequence (the new token's included).
        max_seq_len: an upper bound of seq_lens used to size the key split; defaults to
            max_blocks_per_seq * block_size (no host synchronisation).
        scale: softmax scale; defaults to head_dim ** -0.5.

    Returns:
        (num_seqs, num_heads, head_dim), query's dtype. Asynchronous on the current stream.
    """
    if key_cache.dtype == torch.float8_e4m3fn:  # one query position: the chunked entry point
        return paged_prefill(query.unsqueeze(2), key_cache, value_cache, block_tables, seq_lens, max_seq_len,
                             scale, causal=False, k_scale=k_scale, v_scale=v_scale)[:, :, 0]
    num_seqs, num_heads, head_dim = query.shape
    num_blocks, block_size, num_kv_heads = _check_cache(query, key_cache, value_cache, block_tables, seq_lens,
                                                        num_seqs, num_heads, head_dim)
    block_tables = block_tables.contiguous()
    seq_lens = seq_lens.contiguous()
    if max_seq_len is None:
        max_seq_len = block_tables.shape[1] * block_size
    if query.stride(-1) != 1:
        query = query.contiguous()
    scale = head_dim ** -0.5 if scale is None else float(scale)
    out = torch.empty_like(query)
    lib = _lib.load()
    with torch.cuda.device(query.device):
        ws_bytes = lib.gqa_paged_decode_workspace_bytes(num_seqs, num_heads, num_kv_heads, max_seq_len, head_dim)
        ws = _lib.WORKSPACES.get(query.device, ws_bytes,
                                 ("paged", num_seqs, num_heads, num_kv_heads, max_seq_len, head_dim))
        rc = lib.gqa_paged_decode(
            ctypes.c_void_p(query.data_ptr()), ctypes.c_void_p(key_cache.data_ptr()),
            ctypes.c_void_p(value_cache.data_ptr()), ctypes.c_void_p(out.data_ptr()),
            _lib.strides(query, 3), _lib.strides(out, 3),
            ctypes.c_void_p(block_tables.data_ptr()), block_tables.stride(0), ctypes.c_void_p(seq_lens.data_ptr()),
            num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks, max_seq_len,
            float(scale * LOG2E), _lib.dtype_code(query),
            ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()), _lib.stream_ptr(query.device))
        if rc != 0:
            _lib.WORKSPACES.drop(query.device)
        _lib.check(rc, "gqa_paged_decode")
    return out


def _check_cache(query, key_cache, value_cache, block_tables, seq_lens, num_seqs, num_heads, head_dim):
    """Shapes, dtypes and layout first, the device last, so every check runs on CPU tensors."""
    num_blocks, block_size, num_kv_heads, hd = key_cache.shape
    if hd != head_dim or value_cache.shape != key_cache.shape:
        raise ValueError("key_cache and value_cache must be (num_blocks, block_size, num_kv_heads, head_dim)")
    if num_heads % num_kv_heads:
        raise ValueError("num_heads must be divisible by num_kv_heads")
    if key_cache.dtype != value_cache.dtype or key_cache.dtype not in (query.dtype, torch.float8_e4m3fn):
        raise TypeError("the caches must share query's dtype, or both be float8_e4m3fn")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("the caches must be contiguous")
    if block_tables.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise TypeError("block_tables and seq_lens must be int32")
    if block_tables.dim() != 2 or block_tables.shape[0] != num_seqs or seq_lens.shape != (num_seqs,):
        raise ValueError("block_tables must be (num_seqs, max_blocks) and seq_lens (num_seqs,)")
    _lib.check_one_device(query, key_cache, value_cache, block_tables, seq_lens)
    return num_blocks, block_size, num_kv_heads


def paged_prefill(query, key_cache, value_cache, block_tables, seq_lens, max_seq_len=None, scale=None,
                  causal=True, k_scale=1.0, v_scale=1.0):
    """Attention of a chunk of new tokens per sequence over a paged K/V cache.

    Args:
        query: (num_seqs, num_heads, chunk_len, head_dim), bf16 or fp16 (the (B, H, S, D)
            layout of gqa_flash_attn; any strides with d stride 1). The chunk is the last
            chunk_len positions of each sequence, whose keys (the chunk's own included)
            are already in the cache.
        key_cache, value_cache: (num_blocks, block_size, num_kv_heads, head_dim), contiguous,
            block_size a power of two >= 64; query's dtype, or torch.float8_e4m3fn with
            key = stored key * k_scale and value = stored value * v_scale (head_dim 128 and
            group * chunk_len <= 64: the streaming kernel).
        block_tables: int32 (num_seqs, max_blocks_per_seq); sequence b's key k is in block
            block_tables[b, k // block_size] at position k % block_size.
        seq_lens: int32 (num_seqs,), keys cached per sequence (the chunk included).
        max_seq_len: an upper bound of seq_lens used to plan the key split; defaults to
            max_blocks_per_seq * block_size (no host synchronisation).
        scale: softmax scale; defaults to head_dim ** -0.5.
        causal: query i of sequence b sees keys [0, seq_lens[b] - chunk_len + i] (the dense
            path's bottom-right rule per sequence); False: all seq_lens[b] keys.

    Returns:
        (num_seqs, num_heads, chunk_len, head_dim), query's dtype, contiguous. Asynchronous
        on the current stream. Rows that see no key (seq_lens[b] < chunk_len) are NaN.
    """
    num_seqs, num_heads, chunk_len, head_dim = query.shape
    num_blocks, block_size, num_kv_heads = _check_cache(query, key_cache, value_cache, block_tables, seq_lens,
                                                        num_seqs, num_heads, head_dim)
    block_tables = block_tables.contiguous()
    seq_lens = seq_lens.contiguous()
    if max_seq_len is None:
        max_seq_len = block_tables.shape[1] * block_size
    if query.stride(-1) != 1:
        query = query.contiguous()
    scale = head_dim ** -0.5 if scale is None else float(scale)
    out = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    lib = _lib.load()
    with torch.cuda.device(query.device):
        ws_bytes = lib.gqa_paged_fwd_workspace_bytes(num_seqs, num_heads, num_kv_heads, chunk_len, max_seq_len,
                                                     head_dim)
        ws = _lib.WORKSPACES.get(query.device, ws_bytes,
                                 ("paged_fwd", num_seqs, num_heads, num_kv_heads, chunk_len, max_seq_len, head_dim))
        fp8 = key_cache.dtype == torch.float8_e4m3fn
        common = (ctypes.c_void_p(query.data_ptr()), ctypes.c_void_p(key_cache.data_ptr()),
                  ctypes.c_void_p(value_cache.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                  _lib.strides(query), _lib.strides(out),
                  ctypes.c_void_p(block_tables.data_ptr()), block_tables.stride(0),
                  ctypes.c_void_p(seq_lens.data_ptr()),
                  num_seqs, num_heads, num_kv_heads, chunk_len, head_dim, block_size, num_blocks, max_seq_len,
                  float(scale * LOG2E))
        tail = (1 if causal else 0, _lib.dtype_code(query), ctypes.c_void_p(ws.data_ptr()),
                ctypes.c_size_t(ws.numel()), _lib.stream_ptr(query.device))
        if fp8:
            rc = lib.gqa_paged_fwd_kv8(*common, float(k_scale), float(v_scale), *tail)
        else:
            rc = lib.gqa_paged_fwd(*common, *tail)
        if rc != 0:
            _lib.WORKSPACES.drop(query.device)
        _lib.check(rc, "gqa_paged_fwd_kv8" if fp8 else "gqa_paged_fwd")
    return out
