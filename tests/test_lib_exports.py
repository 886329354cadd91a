"""libgqa_sm100.so loads on a CPU-only machine and exports every symbol of
include/gqa_sm100.h; host-only entry points answer without a GPU."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gqa_sm100.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gqa_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_api():
    names = declared_functions()
    for n in ("gqa_fwd", "gqa_split_first", "gqa_split_reduce", "gqa_split_fused", "gqa_partial",
              "gqa_lse_combine", "gqa_strerror", "gqa_device_error"):
        assert n in names


def test_library_exports_every_declared_symbol(lib_path):
    lib = ctypes.CDLL(lib_path)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_debug_library_exports_every_declared_symbol(lib_path):
    """The checked variant (build.py --debug) has the same C ABI."""
    path = os.path.join(os.path.dirname(lib_path), "libgqa_sm100_debug.so")
    if not os.path.exists(path):
        pytest.skip("debug variant not built")
    lib = ctypes.CDLL(path)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_the_header(lib_path):
    from gqa_kernels import _lib
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_host_only_entry_points(lib_path):
    from gqa_kernels import _lib
    lib = _lib.load()
    assert lib.gqa_version() == 100
    assert _lib.strerror(0) == "success"
    for code in range(1, 8):
        assert _lib.strerror(code) and "unknown" not in _lib.strerror(code)
    assert "unknown" in _lib.strerror(99)
    # the checked build's test hooks are absent from the release library (no GPU touched)
    assert lib.gqa_debug_inject(0, 0, 1000000) == 2


def test_built_for_sm100a(lib_path):
    # the fatbin of the library names its target; no disassembly involved
    data = open(lib_path, "rb").read()
    assert b"sm_100a" in data


def test_invalid_arguments_rejected_before_any_launch(lib_path):
    """Argument validation runs on the host and needs no device."""
    from gqa_kernels import _lib
    lib = _lib.load()
    st = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    # head_dim 96 -> unsupported; Hq % Hkv != 0 -> invalid
    rc = lib.gqa_fwd(None, None, None, None, st, st, st, st, 1, 8, 2, 4, 4, 96, 0.1, 1, 1, None, 0, None)
    assert rc == 2
    rc = lib.gqa_fwd(None, None, None, None, st, st, st, st, 1, 6, 4, 4, 4, 64, 0.1, 1, 1, None, 0, None)
    assert rc == 1
    rc = lib.gqa_fwd(None, None, None, None, st, st, st, st, 1, 24, 8, 4, 4, 64, 0.1, 1, 1, None, 0, None)
    assert rc == 2  # group size 3 is not a power of two
