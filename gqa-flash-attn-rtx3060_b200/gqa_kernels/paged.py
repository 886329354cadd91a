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

- `paged_kv_append`: the cache-write half (vLLM's reshape_and_cache_flash): each
  new token's K and V rows go to its slot of the caches, 16-bit as they are or
  e4m3-quantised with the layer's k/v scale.
- `PagedAttention`: a vLLM-shaped attention layer tying them together:
  forward(query, key, value, kv_cache, attn_metadata) appends the step's K/V and
  attends over the cache.

Cache slots past a sequence's length in its last block are read but never reach
the output (the kernels zero those V rows before the PV product), so stale or
non-finite values left there by earlier sequences are harmless.

Both attention entry points take `max_seq_len`, the bound the host plans the key
split for. A sequence longer than it is silently clipped to its first max_seq_len
keys (and its queries are aligned to that length), so pass a true bound or leave
the default, the block table's capacity; the checked build (build.py --debug)
reports such a call as GQA_ERR_DEBUG_CHECK in the device error word.
"""
import ctypes
from dataclasses import dataclass

import torch

from . import _lib

__all__ = ["paged_decode", "paged_prefill", "paged_kv_append", "PagedAttention", "PagedAttentionMetadata"]

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
    with _lib.on_device(query.device):
        ws_bytes = _lib.workspace_bytes("gqa_paged_decode_workspace_bytes", num_seqs, num_heads, num_kv_heads,
                                         max_seq_len, head_dim)
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
                  causal=True, k_scale=1.0, v_scale=1.0, out=None):
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

        out: optional output of that shape and query's dtype (any strides with d stride 1
            and the others multiples of 8 elements, e.g. a (num_tokens, num_heads, head_dim)
            buffer viewed per sequence).

    Returns:
        (num_seqs, num_heads, chunk_len, head_dim), query's dtype (`out` if given, else a new
        contiguous tensor). Asynchronous on the current stream. Rows that see no key
        (seq_lens[b] < chunk_len) are NaN.
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
    if out is None:
        out = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    elif out.shape != query.shape or out.dtype != query.dtype:
        raise ValueError("out must have query's shape and dtype")
    else:
        _lib.check_one_device(query, out)
    lib = _lib.load()
    with _lib.on_device(query.device):
        ws_bytes = _lib.workspace_bytes("gqa_paged_fwd_workspace_bytes", num_seqs, num_heads, num_kv_heads, chunk_len,
                                         max_seq_len, head_dim)
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


def paged_kv_append(key, value, key_cache, value_cache, slot_mapping, k_scale=1.0, v_scale=1.0):
    """Writes new tokens' K and V rows into paged caches (vLLM's reshape_and_cache_flash).

    Args:
        key, value: (num_tokens, num_kv_heads, head_dim), bf16 or fp16, d stride 1.
        key_cache, value_cache: (num_blocks, block_size, num_kv_heads, head_dim), contiguous;
            key's dtype, or torch.float8_e4m3fn (stored = x / scale rounded to nearest even,
            saturated to +-448, so that real value = stored value x scale).
        slot_mapping: int64 (num_tokens,) on the caches' device; token t goes to block
            slot // block_size at position slot % block_size. Negative slots (padding
            tokens) are skipped. A slot past the cache is not written and is reported
            through the device error word (gqa_kernels.check_device_error()).

    Asynchronous on the current stream.
    """
    num_tokens, num_kv_heads, head_dim = key.shape
    num_blocks, block_size, hkv, hd = key_cache.shape
    if value.shape != key.shape or (hkv, hd) != (num_kv_heads, head_dim) or value_cache.shape != key_cache.shape:
        raise ValueError("key/value must be (num_tokens, num_kv_heads, head_dim) and the caches "
                         "(num_blocks, block_size, num_kv_heads, head_dim)")
    fp8 = key_cache.dtype == torch.float8_e4m3fn
    if value_cache.dtype != key_cache.dtype or key_cache.dtype not in (key.dtype, torch.float8_e4m3fn) \
            or value.dtype != key.dtype:
        raise TypeError("key and value share a dtype; the caches share it too, or are both float8_e4m3fn")
    if not (key_cache.is_contiguous() and value_cache.is_contiguous()):
        raise ValueError("the caches must be contiguous")
    if slot_mapping.dtype != torch.int64 or slot_mapping.shape != (num_tokens,):
        raise TypeError("slot_mapping must be int64 (num_tokens,)")
    if fp8 and not (k_scale > 0 and v_scale > 0):
        raise ValueError("fp8 caches need positive k_scale and v_scale")
    _lib.check_one_device(key, value, key_cache, value_cache, slot_mapping)
    key = key if _lib.tma_compatible(key) else key.contiguous()
    value = value if _lib.tma_compatible(value) else value.contiguous()
    slot_mapping = slot_mapping.contiguous()
    lib = _lib.load()
    with _lib.on_device(key.device):
        rc = lib.gqa_paged_kv_append(
            ctypes.c_void_p(key.data_ptr()), ctypes.c_void_p(value.data_ptr()), _lib.strides(key, 3),
            _lib.strides(value, 3), ctypes.c_void_p(key_cache.data_ptr()), ctypes.c_void_p(value_cache.data_ptr()),
            ctypes.c_void_p(slot_mapping.data_ptr()), num_tokens, num_kv_heads, head_dim, block_size, num_blocks,
            _lib.dtype_code(key), 1 if fp8 else 0, float(k_scale), float(v_scale), _lib.stream_ptr(key.device))
        _lib.check(rc, "gqa_paged_kv_append")


@dataclass
class PagedAttentionMetadata:
    """The per-step metadata PagedAttention.forward reads (vLLM's attention metadata).

    slot_mapping: int64 (num_tokens,), the cache slot of every new token (-1: padding).
    block_tables: int32 (num_seqs, max_blocks_per_seq).
    seq_lens: int32 (num_seqs,), keys per sequence after this step's tokens are appended.
    query_len: new tokens per sequence when every sequence has the same count (1 for
        decode); num_tokens = num_seqs * query_len, the tokens ordered by sequence.
    query_lens: for a mixed batch (chunked prefills and decodes together), the host list
        of new tokens per sequence, tokens ordered by sequence; overrides query_len.
    max_seq_len: an upper bound of seq_lens (plans the key split); None: the block
        tables' capacity.
    """
    slot_mapping: torch.Tensor
    block_tables: torch.Tensor
    seq_lens: torch.Tensor
    query_len: int = 1
    max_seq_len: int = None
    query_lens: list = None


class PagedAttention:
    """A vLLM-shaped attention layer over the paged caches: forward(query, key, value,
    kv_cache, attn_metadata) writes this step's K and V into the cache, then attends.

    Args:
        num_heads, head_size: query heads and head dim (64 or 128).
        scale: softmax scale (default head_size ** -0.5).
        num_kv_heads: key/value heads (default num_heads); num_heads a power-of-two
            multiple of it.
        kv_cache_dtype: "auto" (the caches hold the model's dtype) or "fp8_e4m3".
        k_scale, v_scale: the fp8 caches' scales (real value = stored value x scale).
        causal: the new tokens attend causally among themselves (bottom-right aligned
            to each sequence's length); decode tokens see every cached key either way.
    """

    def __init__(self, num_heads, head_size, scale=None, num_kv_heads=None, kv_cache_dtype="auto", k_scale=1.0,
                 v_scale=1.0, causal=True):
        if kv_cache_dtype not in ("auto", "fp8_e4m3"):
            raise ValueError("kv_cache_dtype must be 'auto' or 'fp8_e4m3'")
        self.num_heads = num_heads
        self.head_size = head_size
        self.num_kv_heads = num_heads if num_kv_heads is None else num_kv_heads
        if self.num_heads % self.num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        self.scale = head_size ** -0.5 if scale is None else float(scale)
        self.kv_cache_dtype = kv_cache_dtype
        self.k_scale = float(k_scale)
        self.v_scale = float(v_scale)
        self.causal = causal

    def allocate_kv_cache(self, num_blocks, block_size, dtype, device):
        """A zeroed (2, num_blocks, block_size, num_kv_heads, head_size) cache of the layer's
        cache dtype (vLLM's FlashAttention cache layout: [0] keys, [1] values)."""
        dt = torch.float8_e4m3fn if self.kv_cache_dtype == "fp8_e4m3" else dtype
        return torch.zeros(2, num_blocks, block_size, self.num_kv_heads, self.head_size, dtype=dt, device=device)

    def forward(self, query, key, value, kv_cache, attn_metadata):
        """query (num_tokens, num_heads * head_size) or (num_tokens, num_heads, head_size);
        key/value (num_tokens, num_kv_heads [* head_size][, head_size]); kv_cache as
        allocate_kv_cache returns. Returns the attention output shaped like query."""
        md = attn_metadata
        shape = query.shape
        num_tokens = shape[0]
        q = query.view(num_tokens, self.num_heads, self.head_size)
        k = key.view(num_tokens, self.num_kv_heads, self.head_size)
        v = value.view(num_tokens, self.num_kv_heads, self.head_size)
        key_cache, value_cache = kv_cache[0], kv_cache[1]
        num_seqs = md.seq_lens.shape[0]
        lens = None if md.query_lens is None else [int(x) for x in md.query_lens]
        if lens is not None:
            if len(lens) != num_seqs or sum(lens) != num_tokens or min(lens, default=0) < 0:
                raise ValueError("query_lens must give each sequence's new tokens, summing to num_tokens")
        elif num_seqs * md.query_len != num_tokens:
            raise ValueError("num_tokens must be num_seqs * query_len (or pass query_lens)")
        paged_kv_append(k, v, key_cache, value_cache, md.slot_mapping, self.k_scale, self.v_scale)
        if lens is None or len(set(lens)) == 1:
            query_len = md.query_len if lens is None else lens[0]
            out = self._attend(q, key_cache, value_cache, md.block_tables, md.seq_lens, md.max_seq_len, query_len)
            return out.view(shape)
        # Mixed batch: the kernels take one chunk length per call, so the sequences are
        # grouped by their new-token count, each group attends in one call, and the rows
        # are gathered from and scattered back to their places in the token order.
        out = torch.empty((num_tokens, self.num_heads, self.head_size), dtype=query.dtype, device=query.device)
        starts = [0]
        for n in lens:
            starts.append(starts[-1] + n)
        groups = {}
        for i, n in enumerate(lens):
            if n:
                groups.setdefault(n, []).append(i)
        for n, seqs in groups.items():
            rows = torch.tensor([starts[i] + t for i in seqs for t in range(n)], dtype=torch.int64,
                                device=query.device)
            sel = torch.tensor(seqs, dtype=torch.int64, device=query.device)
            og = self._attend(q.index_select(0, rows), key_cache, value_cache, md.block_tables.index_select(0, sel),
                              md.seq_lens.index_select(0, sel), md.max_seq_len, n)
            out.index_copy_(0, rows, og)
        return out.view(shape)

    def _attend(self, q, key_cache, value_cache, block_tables, seq_lens, max_seq_len, query_len):
        """Attention of num_seqs sequences with query_len new tokens each; q and the result
        are (num_seqs * query_len, num_heads, head_size), tokens ordered by sequence."""
        num_seqs = seq_lens.shape[0]
        if query_len == 1 and key_cache.dtype != torch.float8_e4m3fn:
            return paged_decode(q, key_cache, value_cache, block_tables, seq_lens, max_seq_len, self.scale)
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        # tokens are ordered by sequence: (num_seqs, query_len, H, D) viewed as (num_seqs, H, query_len, D)
        qv = q.view(num_seqs, query_len, self.num_heads, self.head_size).transpose(1, 2)
        ov = out.view(num_seqs, query_len, self.num_heads, self.head_size).transpose(1, 2)
        paged_prefill(qv, key_cache, value_cache, block_tables, seq_lens, max_seq_len, self.scale,
                      causal=self.causal, k_scale=self.k_scale, v_scale=self.v_scale, out=ov)
        return out
