"""Public entrypoint: choose single-pass vs split-KV path per workload.

Same routing as the reference's gqa_kernels/dispatch.py:14-62, including the
SM_COUNT = 28 predicate constant. The predicate only decides which API path a
call takes; both paths size their CUDA launches for the actual device (148
SMs on B200), and every BASELINE shape routes identically at 28 or 148.
"""
import torch

from . import _lib
from .gqa_fwd import gqa_fwd_kernel
from .gqa_split import split_kv_forward

__all__ = ["gqa_flash_attn", "set_nvtx_ranges"]

SM_COUNT = 28  # routing constant of the reference (dispatch.py:10); launches use the real SM count
LOG2E = 1.4426950408889634
_NVTX = False


def set_nvtx_ranges(enabled=True):
    """Wrap every gqa_flash_attn call in an NVTX range named after its path and shape
    (visible in Nsight timelines); off by default, when a call pays one flag test."""
    global _NVTX
    _NVTX = bool(enabled)


def _cdiv(a, b):
    return -(-a // b)


def _layout_ok(*ts):
    return all(_lib.tma_compatible(t) for t in ts)


def gqa_flash_attn(q, k, v, causal=True):
    """GQA flash attention.

    Args:
        q: (batch, num_heads,    seq_q,  head_dim)  — fp16 or bf16
        k: (batch, num_kv_heads, seq_kv, head_dim)
        v: (batch, num_kv_heads, seq_kv, head_dim)
        causal: if True, q position i (in K coordinates: i + seq_kv - seq_q)
                attends to K positions [0, q_pos]. Works for prefill
                (seq_q == seq_kv) and decode / chunked-prefill (seq_q < seq_kv).

    Returns:
        (batch, num_heads, seq_q, head_dim), same dtype as q.
    """
    if not _NVTX:
        return _gqa_flash_attn(q, k, v, causal)
    b, hq, sq, d = q.shape
    torch.cuda.nvtx.range_push(f"gqa_flash_attn b{b} hq{hq} hkv{k.shape[1]} sq{sq} skv{k.shape[2]} d{d}")
    try:
        return _gqa_flash_attn(q, k, v, causal)
    finally:
        torch.cuda.nvtx.range_pop()


def _gqa_flash_attn(q, k, v, causal=True):
    """The call itself (routing and launch); see gqa_flash_attn."""
    batch, num_heads, seq_q, head_dim = q.shape
    _, num_kv_heads, seq_kv, _ = k.shape
    assert num_heads % num_kv_heads == 0, "num_heads must be divisible by num_kv_heads"
    group_size = num_heads // num_kv_heads
    assert head_dim in (64, 128), f"unsupported head_dim {head_dim}"
    assert q.is_cuda and k.is_cuda and v.is_cuda
    if not (q.device == k.device == v.device):  # one device's memory per launch
        raise ValueError("q, k and v must be on one device")
    if tuple(v.shape) != tuple(k.shape):
        raise ValueError("k and v must have the same shape")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k and v must share one dtype")
    # The CUDA library reads tensors through TMA: contiguous in head_dim with
    # 16-byte aligned strides. Other layouts are copied once here.
    if not _layout_ok(q, k, v):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()

    # Split-KV when the single-pass grid would underfill the SMs
    # (short seq_q, long seq_kv).
    if seq_q <= 16 and seq_kv >= 1024 and num_kv_heads * batch < SM_COUNT:
        target = 4 * SM_COUNT
        splits = 1
        while splits * num_kv_heads * batch < target and splits < 32:
            splits *= 2
        while splits > 1 and seq_kv // splits < 64:
            splits //= 2
        if splits > 1:
            return split_kv_forward(q, k, v, causal, splits)

    o = torch.empty_like(q)
    out = o if _layout_ok(o) else torch.empty(q.shape, dtype=q.dtype, device=q.device)
    scale_log2 = (head_dim ** -0.5) * LOG2E
    grid = lambda META: (_cdiv(seq_q, META['BLOCK_M']), num_kv_heads, batch)  # noqa: E731 (ignored)
    gqa_fwd_kernel[grid](
        q, k, v, out,
        q.stride(0), q.stride(1), q.stride(2), q.stride(3),
        k.stride(0), k.stride(1), k.stride(2), k.stride(3),
        v.stride(0), v.stride(1), v.stride(2), v.stride(3),
        out.stride(0), out.stride(1), out.stride(2), out.stride(3),
        seq_q, seq_kv,
        scale_log2,
        IS_CAUSAL=causal,
        GROUP_SIZE=group_size,
        HEAD_DIM=head_dim,
    )
    if out is not o:
        o.copy_(out)
    return o
