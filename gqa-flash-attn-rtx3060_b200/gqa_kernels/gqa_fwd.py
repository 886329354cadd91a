"""Single-pass GQA flash attention forward (host side of the sm_100a kernels).

Mirrors gqa_kernels/gqa_fwd.py of the reference: `gqa_fwd_kernel` keeps the
launch syntax `gqa_fwd_kernel[grid](Q, K, V, O, <16 strides>, seq_q, seq_kv,
scale, IS_CAUSAL=, GROUP_SIZE=, HEAD_DIM=)` of the reference's Triton kernel
(gqa_fwd.py:33-49, launched at dispatch.py:50-61). The grid argument is
accepted for source compatibility and ignored: tile shapes are fixed in the
CUDA library and the launch is sized there for the device's SM count.

Underneath, the call goes through the C ABI entry point `gqa_fwd`
(include/gqa_sm100.h): the tcgen05/TMEM prefill kernel for >= 128 packed rows,
the HBM-streaming kernel for fewer (decode-shaped calls).
"""
import ctypes

from . import _lib


def _check_tensor_args(Q, K, V, O, strides):
    if len(strides) != 16:
        raise TypeError("gqa_fwd_kernel expects 16 stride arguments (q, k, v, o x 4)")
    for t, st in zip((Q, K, V, O), (strides[0:4], strides[4:8], strides[8:12], strides[12:16])):
        if tuple(int(x) for x in st) != tuple(t.stride()):
            raise ValueError("stride arguments must match the tensors' own strides")


def launch_fwd(q, k, v, o, causal, scale_log2):
    """Enqueues O = attention(q, k, v) on the current stream of q's device."""
    batch, num_heads, seq_q, head_dim = q.shape
    _, num_kv_heads, seq_kv, _ = k.shape
    lib = _lib.load()
    dev = q.device
    ws_bytes = _lib.workspace_bytes("gqa_fwd_workspace_bytes", batch, num_heads, num_kv_heads, seq_q, seq_kv,
                                     head_dim)
    ws_ptr = None
    if ws_bytes:
        ws = _lib.WORKSPACES.get(dev, ws_bytes, ("fwd", batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim))
        ws_ptr = ctypes.c_void_p(ws.data_ptr())
    rc = lib.gqa_fwd(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(v.data_ptr()),
        ctypes.c_void_p(o.data_ptr()),
        _lib.strides(q), _lib.strides(k), _lib.strides(v), _lib.strides(o),
        batch, num_heads, num_kv_heads, seq_q, seq_kv, head_dim,
        float(scale_log2), 1 if causal else 0, _lib.dtype_code(q),
        ws_ptr, ctypes.c_size_t(ws_bytes), _lib.stream_ptr(dev))
    if rc != 0 and ws_bytes:
        _lib.WORKSPACES.drop(dev)
    _lib.check(rc, "gqa_fwd")


class _FwdLauncher:
    """`gqa_fwd_kernel[grid](...)` -> C ABI gqa_fwd."""

    def __getitem__(self, grid):
        return self._launch

    @staticmethod
    def _launch(Q, K, V, O, *args, IS_CAUSAL, GROUP_SIZE, HEAD_DIM, BLOCK_M=None, BLOCK_N=None, **_tuning):
        if len(args) != 19:
            raise TypeError("gqa_fwd_kernel expects Q, K, V, O, 16 strides, seq_q, seq_kv, scale")
        strides, (seq_q, seq_kv, scale) = args[:16], args[16:]
        _check_tensor_args(Q, K, V, O, strides)
        if Q.shape[2] != seq_q or K.shape[2] != seq_kv:
            raise ValueError("seq_q / seq_kv must match the tensors")
        if Q.shape[1] != GROUP_SIZE * K.shape[1] or Q.shape[3] != HEAD_DIM:
            raise ValueError("GROUP_SIZE / HEAD_DIM must match the tensors")
        with _lib.on_device(Q.device):
            launch_fwd(Q, K, V, O, bool(IS_CAUSAL), float(scale))


gqa_fwd_kernel = _FwdLauncher()
