"""B200 (sm_100a) GQA flash-attention forward with the reference's public API.

`gqa_flash_attn(q, k, v, causal=True)` keeps the signature, layout and routing
of tonbistudio/gqa-flash-attn-rtx3060 (gqa_kernels/__init__.py:1-4); the work
runs in hand-written sm_100a CUDA behind the C ABI of include/gqa_sm100.h.
"""
from .dispatch import gqa_flash_attn, set_nvtx_ranges
from ._lib import device_error as check_device_error

__all__ = ["gqa_flash_attn", "check_device_error", "set_nvtx_ranges"]
__version__ = "0.1.0"
