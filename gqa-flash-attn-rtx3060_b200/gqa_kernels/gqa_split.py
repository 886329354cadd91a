"""Split-KV GQA flash attention for decode and short-Q workloads (sm_100a).

Mirrors gqa_kernels/gqa_split.py of the reference:
  - `split_kv_forward(q, k, v, causal, splits)` (reference :153-194). Here it
    runs ONE launch: the key axis is cut into chunks sized for the device's
    SM count (the `splits` argument is accepted as the reference's hint and
    does not change the result) and the last CTA of each (batch, kv_head,
    q-block) combines the chunk partials in-kernel.
  - `gqa_split_first_kernel[grid](...)` and `gqa_split_reduce_kernel[grid](...)`
    keep the reference's two-pass launch syntax (:26-44, :115-123) and write
    / read the same (m, l, acc) partial arrays, through the C ABI entry points
    gqa_split_first and gqa_split_reduce.
"""
import ctypes
import math

import torch

from . import _lib

LOG2E = 1.4426950408889634


def split_kv_forward(q, k, v, causal, splits):
    """Split-KV forward (one fused launch). Call from dispatch when seq_q is small."""
    _lib.check_one_device(q, k, v)
    batch, num_heads, seq_q, head_dim = q.shape
    _, num_kv_heads, seq_kv, _ = k.shape
    scale_log2 = (head_dim ** -0.5) * LOG2E
    o = torch.empty_like(q)
    lib = _lib.load()
    with _lib.on_device(q.device):
        ws_bytes = _lib.workspace_bytes("gqa_split_fused_workspace_bytes", batch, num_heads, num_kv_heads, seq_q,
                                         seq_kv, head_dim)
        ws = _lib.WORKSPACES.get(q.device, ws_bytes,
                                 ("split", batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim))
        rc = lib.gqa_split_fused(
            ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(v.data_ptr()),
            ctypes.c_void_p(o.data_ptr()),
            _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(o),
            batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim,
            float(scale_log2), 1 if causal else 0, _lib.dtype_code(q),
            ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()), _lib.stream_ptr(q.device))
        if rc != 0:
            _lib.WORKSPACES.drop(q.device)
        _lib.check(rc, "gqa_split_fused")
    return o


class _SplitFirstLauncher:
    """`gqa_split_first_kernel[grid](Q, K, V, Mp, Lp, Ap, <21 strides>, seq_q, seq_kv, scale,
    IS_CAUSAL=, GROUP_SIZE=, HEAD_DIM=, BLOCK_M=, SPLITS=)` -> C ABI gqa_split_first.

    Mp/Lp: float32 (B, Hq, Sq, SPLITS); Ap: float32 (B, Hq, Sq, SPLITS, D).
    Chunk s covers keys [s*ceil(seq_kv/SPLITS), (s+1)*ceil(seq_kv/SPLITS)) as in the
    reference; BLOCK_M only affects the reference's tiling, not the partials.
    """

    def __getitem__(self, grid):
        return self._launch

    @staticmethod
    def _launch(Q, K, V, Mp, Lp, Ap, *args, IS_CAUSAL, GROUP_SIZE, HEAD_DIM, BLOCK_M, SPLITS, **_tuning):
        if len(args) != 24:
            raise TypeError("gqa_split_first_kernel expects Q, K, V, Mp, Lp, Ap, 21 strides, seq_q, seq_kv, scale")
        st = [int(x) for x in args[:21]]
        seq_q, seq_kv, scale = args[21:24]
        if (tuple(st[0:4]) != Q.stride() or tuple(st[4:8]) != K.stride() or tuple(st[8:12]) != V.stride()
                or tuple(st[12:16]) != Mp.stride() or tuple(st[16:21]) != Ap.stride()):
            raise ValueError("stride arguments must match the tensors' own strides")
        if Mp.stride() != Lp.stride():
            raise ValueError("Mp and Lp must share strides")
        batch, num_heads, _, head_dim = Q.shape
        num_kv_heads = K.shape[1]
        if num_heads != GROUP_SIZE * num_kv_heads or head_dim != HEAD_DIM:
            raise ValueError("GROUP_SIZE / HEAD_DIM must match the tensors")
        for t in (Mp, Lp, Ap):
            if t.dtype != torch.float32:
                raise TypeError("partials must be float32")
        with _lib.on_device(Q.device):
            rc = _lib.load().gqa_split_first(
                ctypes.c_void_p(Q.data_ptr()), ctypes.c_void_p(K.data_ptr()), ctypes.c_void_p(V.data_ptr()),
                ctypes.c_void_p(Mp.data_ptr()), ctypes.c_void_p(Lp.data_ptr()), ctypes.c_void_p(Ap.data_ptr()),
                _lib.strides(Q), _lib.strides(K), _lib.strides(V), _lib.strides(Mp), _lib.strides(Ap, 5),
                batch, num_heads, num_kv_heads, int(seq_q), int(seq_kv), head_dim, float(scale),
                1 if IS_CAUSAL else 0, int(SPLITS), _lib.dtype_code(Q), _lib.stream_ptr(Q.device))
            _lib.check(rc, "gqa_split_first")


class _SplitReduceLauncher:
    """`gqa_split_reduce_kernel[grid](Mp, Lp, Ap, O, <13 strides>, HEAD_DIM=, SPLITS=)` -> gqa_split_reduce."""

    def __getitem__(self, grid):
        return self._launch

    @staticmethod
    def _launch(Mp, Lp, Ap, O, *args, HEAD_DIM, SPLITS, **_tuning):
        if len(args) != 13:
            raise TypeError("gqa_split_reduce_kernel expects Mp, Lp, Ap, O and 13 strides")
        st = [int(x) for x in args]
        if tuple(st[0:4]) != Mp.stride() or tuple(st[4:9]) != Ap.stride() or tuple(st[9:13]) != O.stride():
            raise ValueError("stride arguments must match the tensors' own strides")
        batch, num_heads, seq_q, head_dim = O.shape
        if head_dim != HEAD_DIM:
            raise ValueError("HEAD_DIM must match O")
        with _lib.on_device(O.device):
            rc = _lib.load().gqa_split_reduce(
                ctypes.c_void_p(Mp.data_ptr()), ctypes.c_void_p(Lp.data_ptr()), ctypes.c_void_p(Ap.data_ptr()),
                ctypes.c_void_p(O.data_ptr()), _lib.strides(Mp), _lib.strides(Ap, 5), _lib.strides(O),
                batch, num_heads, seq_q, head_dim, int(SPLITS), _lib.dtype_code(O), _lib.stream_ptr(O.device))
            _lib.check(rc, "gqa_split_reduce")


gqa_split_first_kernel = _SplitFirstLauncher()
gqa_split_reduce_kernel = _SplitReduceLauncher()


def split_kv_two_pass(q, k, v, causal, splits):
    """The reference's two-launch split-KV forward, kept for API parity and tests:
    partials (m_p, l_p, acc_p) through gqa_split_first, combine through gqa_split_reduce."""
    _lib.check_one_device(q, k, v)
    batch, num_heads, seq_q, head_dim = q.shape
    _, num_kv_heads, seq_kv, _ = k.shape
    group_size = num_heads // num_kv_heads
    scale_log2 = (head_dim ** -0.5) * LOG2E
    m_p = torch.empty((batch, num_heads, seq_q, splits), dtype=torch.float32, device=q.device)
    l_p = torch.empty_like(m_p)
    acc_p = torch.empty((batch, num_heads, seq_q, splits, head_dim), dtype=torch.float32, device=q.device)
    o = torch.empty_like(q)
    block_m = 16 if seq_q <= 16 else 32
    grid1 = (num_kv_heads, math.ceil(seq_q / block_m), batch * splits)
    gqa_split_first_kernel[grid1](
        q, k, v, m_p, l_p, acc_p,
        *q.stride(), *k.stride(), *v.stride(), *m_p.stride(), *acc_p.stride(),
        seq_q, seq_kv, scale_log2,
        IS_CAUSAL=causal, GROUP_SIZE=group_size, HEAD_DIM=head_dim, BLOCK_M=block_m, SPLITS=splits)
    grid2 = (num_heads, seq_q, batch)
    gqa_split_reduce_kernel[grid2](
        m_p, l_p, acc_p, o,
        *m_p.stride(), *acc_p.stride(), *o.stride(),
        HEAD_DIM=head_dim, SPLITS=splits)
    return o, (m_p, l_p, acc_p)
