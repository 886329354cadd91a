"""The NVTX switch of gqa_flash_attn: off by default, toggled by set_nvtx_ranges, and
the public function keeps the reference's signature and docstring."""
import inspect

import gqa_kernels
from gqa_kernels import dispatch


def test_nvtx_switch_and_signature():
    assert dispatch._NVTX is False
    gqa_kernels.set_nvtx_ranges(True)
    assert dispatch._NVTX is True
    gqa_kernels.set_nvtx_ranges(False)
    assert dispatch._NVTX is False
    assert list(inspect.signature(gqa_kernels.gqa_flash_attn).parameters) == ["q", "k", "v", "causal"]
    assert "GQA flash attention" in gqa_kernels.gqa_flash_attn.__doc__
