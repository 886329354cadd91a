"""The prefill softmax's FMA-pipe exp2 (exp2_poly2 in csrc/gqa_common.cuh): its four
polynomial coefficients are the output of tests/exp2_fit.py's Lawson fit, rounded to
float32, and the float32 emulation of the kernel's instruction sequence stays within the
relative error bound the kernel's comment states (1.5e-4). No GPU needed; the device
function itself is checked by tests/test_exp2_poly_gpu.py."""
import os
import re

import numpy as np

from tests import exp2_fit as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
COMMON = os.path.join(ROOT, "gqa-flash-attn-rtx3060_b200", "csrc", "gqa_common.cuh")


def kernel_coefficients():
    text = open(COMMON).read()
    body = text[text.index("float2 exp2_poly2("):]
    body = body[:body.index("\n}\n")]
    got = {k: float(v) for k, v in re.findall(r"\b(kC[0-3])\s*=\s*([0-9.eE+-]+)f", body)}
    return np.array([got[f"kC{i}"] for i in range(4)], dtype=np.float32)


def test_kernel_constants_are_the_fit():
    fit = F.fit(3).astype(np.float32)
    assert np.array_equal(kernel_coefficients(), fit), (kernel_coefficients(), fit)


def test_emulated_kernel_sequence_meets_the_stated_bound():
    mx, mean, bad = F.max_rel_error(kernel_coefficients())
    assert mx < 1.5e-4 and bad == 0, (mx, mean, bad)
