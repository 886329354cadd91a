"""pytest configuration: the `gpu` marker, import paths, and the library build."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gqa-flash-attn-rtx3060_b200")
for _p in (PKG, ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; run with -m gpu")


def _load_build_module():
    spec = importlib.util.spec_from_file_location("gqa_build", os.path.join(PKG, "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def lib_path():
    """Path of libgqa_sm100.so, built in-tree with nvcc if it is missing or stale."""
    return _load_build_module().build()


@pytest.fixture(scope="session")
def cuda_lib(lib_path):
    """The loaded library, on a machine with a B200; skips nothing: a GPU test
    run without CUDA fails loudly."""
    import torch
    assert torch.cuda.is_available(), "GPU tests need CUDA (run them on a B200 with -m gpu)"
    from gqa_kernels import _lib
    return _lib.load()
