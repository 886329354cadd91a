"""Persistent prefix K/V cache and chunked prefill over gqa_flash_attn.

The reference lists these as the natural follow-ups of its kernel
(README.md:138-146): keep the K/V of a shared prefix (system prompt, memory
block) across calls and compute attention only for the new tokens; its
`seq_q < seq_kv` bottom-right causal alignment (gqa_kernels/dispatch.py:20-24,
gqa_kernels/gqa_fwd.py:70-73) is the primitive that needs.

`PrefixKVCache` holds K and V as (batch, num_kv_heads, capacity, head_dim)
tensors on one GPU. Appending writes the new keys after the cached ones;
attention runs gqa_flash_attn on views of the first `length` keys, which the
CUDA library reads in place through TMA (the views keep head_dim contiguous and
16-byte strides), so no call copies the cache. A chunk of n new tokens
attends with query i at key position `length_before + i`: the chunked-prefill
rule, and decode for n = 1.
"""
import torch

from .dispatch import gqa_flash_attn

__all__ = ["PrefixKVCache"]


class PrefixKVCache:
    def __init__(self, batch, num_kv_heads, head_dim, capacity, dtype=torch.bfloat16, device="cuda"):
        if head_dim not in (64, 128):
            raise ValueError(f"unsupported head_dim {head_dim}")
        if capacity <= 0:
            raise ValueError("capacity must be positive")
        shape = (batch, num_kv_heads, capacity, head_dim)
        self.k = torch.empty(shape, dtype=dtype, device=device)
        self.v = torch.empty(shape, dtype=dtype, device=device)
        self._length = 0

    @property
    def capacity(self):
        return self.k.shape[2]

    @property
    def length(self):
        """Number of cached key positions."""
        return self._length

    def keys(self):
        return self.k[:, :, :self._length]

    def values(self):
        return self.v[:, :, :self._length]

    def append(self, k_new, v_new):
        """Writes (batch, num_kv_heads, n, head_dim) keys and values after the cached ones
        (asynchronously, on the current stream). Returns the new length."""
        if k_new.shape != v_new.shape:
            raise ValueError("k and v must have the same shape")
        b, h, n, d = k_new.shape
        if (b, h, d) != (self.k.shape[0], self.k.shape[1], self.k.shape[3]):
            raise ValueError(f"new keys {tuple(k_new.shape)} do not match the cache {tuple(self.k.shape)}")
        if k_new.dtype != self.k.dtype:
            raise TypeError("new keys must have the cache's dtype")
        if self._length + n > self.capacity:
            raise ValueError(f"cache full: {self._length} + {n} > capacity {self.capacity}")
        self.k[:, :, self._length:self._length + n].copy_(k_new, non_blocking=True)
        self.v[:, :, self._length:self._length + n].copy_(v_new, non_blocking=True)
        self._length += n
        return self._length

    def truncate(self, length):
        """Keeps the first `length` positions (e.g. back to a shared prefix after a turn)."""
        if not 0 <= length <= self._length:
            raise ValueError(f"cannot truncate a cache of {self._length} positions to {length}")
        self._length = length

    def attend(self, q, causal=True):
        """Attention of q (batch, num_heads, seq_q, head_dim) over the cached keys; with
        causal, the queries are the last seq_q positions (bottom-right alignment)."""
        if self._length == 0:
            raise ValueError("the cache is empty")
        if q.shape[2] > self._length and causal:
            raise ValueError("more queries than cached positions")
        return gqa_flash_attn(q, self.keys(), self.values(), causal=causal)

    def prefill(self, q, k_new, v_new, causal=True):
        """One chunked-prefill (or decode, for one token) step: append the chunk's keys and
        values, then attend its queries over the whole cache."""
        if q.shape[2] != k_new.shape[2]:
            raise ValueError("a chunk has one query per new key position")
        self.append(k_new, v_new)
        return self.attend(q, causal=causal)
