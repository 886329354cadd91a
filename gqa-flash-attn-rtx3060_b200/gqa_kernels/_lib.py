"""ctypes binding of libgqa_sm100.so, the sm_100a CUDA library behind gqa_kernels.

This is the Python-side FFI of the C ABI declared in include/gqa_sm100.h.
There is no fallback: if the library is missing or the current device is not
an sm_100 GPU, calls raise RuntimeError.
"""
import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
# GQA_KERNELS_LIB=debug selects the checked build (build.py --debug), whose kernels
# report a bad address or coordinate as GQA_ERR_DEBUG_CHECK instead of faulting;
# any other value is taken as a path.
_SEL = os.environ.get("GQA_KERNELS_LIB", "")
LIB_PATH = (os.path.join(_HERE, "libgqa_sm100_debug.so") if _SEL == "debug"
            else _SEL if _SEL else os.path.join(_HERE, "libgqa_sm100.so"))

GQA_DTYPE_F16 = 0
GQA_DTYPE_BF16 = 1

_P = ctypes.c_void_p
_I64P = ctypes.POINTER(ctypes.c_int64)
_I = ctypes.c_int
_F = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/gqa_sm100.h
SIGNATURES = {
    "gqa_strerror": (ctypes.c_char_p, [_I]),
    "gqa_version": (_I, []),
    "gqa_sm_count": (_I, []),
    "gqa_fwd_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "gqa_fwd": (_I, [_P, _P, _P, _P, _I64P, _I64P, _I64P, _I64P, _I, _I, _I, _I, _I, _I, _F, _I, _I, _P, _SZ, _P]),
    "gqa_split_first": (_I, [_P, _P, _P, _P, _P, _P, _I64P, _I64P, _I64P, _I64P, _I64P,
                             _I, _I, _I, _I, _I, _I, _F, _I, _I, _I, _P]),
    "gqa_split_reduce": (_I, [_P, _P, _P, _P, _I64P, _I64P, _I64P, _I, _I, _I, _I, _I, _I, _P]),
    "gqa_split_fused_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "gqa_split_fused": (_I, [_P, _P, _P, _P, _I64P, _I64P, _I64P, _I64P, _I, _I, _I, _I, _I, _I, _F, _I, _I,
                             _P, _SZ, _P]),
    "gqa_split_fused_noalloc": (_I, [_P, _P, _P, _P, _I64P, _I64P, _I64P, _I64P, _I, _I, _I, _I, _I, _I, _F, _I, _I,
                                     _P]),
    "gqa_partial_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "gqa_partial": (_I, [_P, _P, _P, _P, _P, _P, _I64P, _I64P, _I64P, _I, _I, _I, _I, _I, _I, _I, _I, _F, _I, _I,
                         _P, _SZ, _P]),
    "gqa_lse_combine": (_I, [_P, _P, _P, _I, ctypes.c_int64, ctypes.c_int64, _P, _I64P, _I, _I, _I, _I, _I, _P]),
    "gqa_device_error": (_I, [ctypes.POINTER(_I), ctypes.POINTER(_I), _I]),
    "gqa_paged_decode_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I]),
    "gqa_paged_decode": (_I, [_P, _P, _P, _P, _I64P, _I64P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _F, _I, _P,
                              _SZ, _P]),
    "gqa_paged_fwd_workspace_bytes": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "gqa_paged_fwd": (_I, [_P, _P, _P, _P, _I64P, _I64P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _F, _I, _I,
                           _P, _SZ, _P]),
    "gqa_prefill_plan": (_I, [_I, _I, _I, _I, _I, _I, _I, _I, ctypes.POINTER(ctypes.c_int)]),
    "gqa_paged_fwd_kv8": (_I, [_P, _P, _P, _P, _I64P, _I64P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _F, _F,
                               _F, _I, _I, _P, _SZ, _P]),
    "gqa_paged_kv_append": (_I, [_P, _P, _I64P, _I64P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _F, _P]),
    "gqa_debug_inject": (_I, [_I, _I, ctypes.c_longlong]),
    "gqa_debug_exp2_poly2": (_I, [_P, _P, _I, _P]),
    "gqa_exchange_alloc": (_I, [_SZ, ctypes.POINTER(_P)]),
    "gqa_exchange_free": (_I, [_P]),
    "gqa_ipc_handle": (_I, [_P, _P]),
    "gqa_ipc_open": (_I, [_P, ctypes.POINTER(_P)]),
    "gqa_ipc_close": (_I, [_P]),
    "gqa_epoch_bump": (_I, [_P, _P]),
    "gqa_partial_units": (_I, [_I, _I, _I, _I, _I, ctypes.POINTER(_I)]),
    "gqa_partial_peer": (_I, [_P, _P, _P, _I64P, _I64P, _I64P, _I, _I, _I, _I, _I, _I, _I, _I, _F, _I, _I,
                              ctypes.POINTER(_P), ctypes.POINTER(_P), _I, _I, _P, ctypes.c_int64, ctypes.c_int64,
                              _P, _SZ, _P]),
    "gqa_lse_combine_peer": (_I, [_P, _P, _P, _I, ctypes.c_int64, ctypes.c_int64, _I, _P, _I64P, _I, _I, _I, _I, _I,
                                  _P]),
}

_lib = None
_lock = threading.Lock()


def load():
    """Loads (once) and returns the ctypes handle of libgqa_sm100.so."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with "
                        "`python gqa-flash-attn-rtx3060_b200/build.py` (nvcc, sm_100a)")
                lib = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = lib
    return _lib


def strerror(code):
    return load().gqa_strerror(int(code)).decode()


def check(code, what):
    if code != 0:
        raise RuntimeError(f"{what} failed: {strerror(code)} (status {code})")


def check_one_device(*tensors):
    """Every tensor a launch reads or writes must be CUDA memory of one device: the
    kernels take raw pointers and run on the first tensor's device."""
    dev = tensors[0].device
    if dev.type != "cuda":
        raise ValueError("tensors must be on a CUDA device")
    for t in tensors:
        if t.device != dev:
            raise ValueError("tensors must be on one device" if t.is_cuda else "tensors must be on a CUDA device")


_STRIDES = {}


def strides(t, n=4):
    """Element strides of `t` as a ctypes int64 array (one array per distinct stride
    tuple, reused: the library only reads it during the call)."""
    st = t.stride()
    if len(st) != n:
        raise ValueError(f"expected a {n}-d tensor")
    arr = _STRIDES.get(st)
    if arr is None:
        if len(_STRIDES) > 4096:
            _STRIDES.clear()
        arr = _STRIDES[st] = (ctypes.c_int64 * n)(*st)
    return arr


def dtype_code(t):
    if t.dtype == torch.bfloat16:
        return GQA_DTYPE_BF16
    if t.dtype == torch.float16:
        return GQA_DTYPE_F16
    raise RuntimeError(f"gqa_kernels supports float16 and bfloat16 tensors, got {t.dtype}")


def stream_ptr(device):
    """The raw cudaStream_t of the current stream of `device`, as an int."""
    return torch._C._cuda_getCurrentRawStream(device.index)


class _NoGuard:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


_NO_GUARD = _NoGuard()


def on_device(device):
    """Context making `device` current for a launch: a no-op when it already is (the
    usual case), torch.cuda.device(device) otherwise."""
    if device.index == torch.cuda.current_device():
        return _NO_GUARD
    return torch.cuda.device(device)


_WS_BYTES = {}


def workspace_bytes(query, *shape):
    """lib.<query>(*shape) on the current device, remembered per (device, query, shape):
    the answer depends on nothing else (the device's SM count sizes the split)."""
    key = (torch.cuda.current_device(), query, shape)
    n = _WS_BYTES.get(key)
    if n is None:
        if len(_WS_BYTES) > 4096:
            _WS_BYTES.clear()
        n = _WS_BYTES[key] = getattr(load(), query)(*shape)
    return n


def tma_compatible(t):
    """True if `t` meets the library's layout rule: contiguous in the last dim,
    other strides multiples of 8 elements, base 16-byte aligned."""
    st = t.stride()
    if st[-1] != 1 and t.shape[-1] != 1:
        return False
    if t.data_ptr() & 15:
        return False
    for s in st[:-1]:
        if s & 7:
            return False
    return True


class WorkspaceCache:
    """Per-(device, stream) scratch for the split kernels.

    The fused kernels count chunk arrivals with ticket counters that must read
    zero at the start of a call and are reset to zero by the call itself. A
    buffer is zeroed when it is (re)allocated or when the call signature
    changes (a different shape moves the counters), so steady-state calls
    launch no memset. Calls sharing a stream are ordered, so they may share
    its buffer.
    """

    def __init__(self):
        self._bufs = {}
        self._lock = threading.Lock()

    def get(self, device, nbytes, signature):
        key = (device.index, stream_ptr(device))
        with self._lock:
            ent = self._bufs.get(key)
            if ent is None or ent[0].numel() < nbytes:
                buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
                self._bufs[key] = [buf, signature]
                return buf
            if ent[1] != signature:
                ent[0].zero_()
                ent[1] = signature
            return ent[0]

    def drop(self, device):
        with self._lock:
            for key in [k for k in self._bufs if k[0] == device.index]:
                del self._bufs[key]


WORKSPACES = WorkspaceCache()


def device_error(clear=True):
    """Returns (code, site) of the current device's in-kernel error word.

    A nonzero code means some launch aborted (a bounded wait expired, or a checked
    build's check failed). The split kernels' ticket counters in a cached workspace
    are then no longer trusted: the device's cached workspaces are dropped, so the
    next call allocates zeroed ones."""
    code = ctypes.c_int(0)
    site = ctypes.c_int(0)
    check(load().gqa_device_error(ctypes.byref(code), ctypes.byref(site), 1 if clear else 0), "gqa_device_error")
    if code.value != 0:
        WORKSPACES.drop(torch.device("cuda", torch.cuda.current_device()))
    return code.value, site.value
