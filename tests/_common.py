"""Shared helpers of the test suite: seeded inputs, tolerance checks, and a
torch fp32 restatement of the oracle for full-size GPU comparisons."""
import numpy as np
import torch

# BASELINE contract: bf16 outputs within max-abs 2e-2 and mean-abs 2e-3 of the fp32 oracle.
BASELINE_TOL = (2e-2, 2e-3)
# Reference test tolerances for its N(0,1)*0.1 inputs (tests/test_correctness.py:24-27).
REF_TOL = {torch.bfloat16: (1e-2, 1e-3), torch.float16: (1e-3, 1e-4)}


def make_inputs(B, Hq, Hkv, Sq, Skv, D, dtype=torch.bfloat16, seed=0, device="cpu", scale=1.0):
    """q, k, v drawn in that order, N(0,1) in fp32 from a torch.Generator seeded `seed`
    on `device`, times `scale`, then cast to `dtype` (the BASELINE convention)."""
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(B, Hq, Sq, D, generator=g, device=device)
    k = torch.randn(B, Hkv, Skv, D, generator=g, device=device)
    v = torch.randn(B, Hkv, Skv, D, generator=g, device=device)
    return tuple((t * scale).to(dtype) for t in (q, k, v))


def to_np(t):
    return t.detach().float().cpu().numpy()


def compare(out, ref, tol, allow_nan_rows=True):
    """max/mean abs error of out vs ref over finite reference entries; NaN must match NaN."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    ref_nan = np.isnan(ref)
    out_nan = np.isnan(out)
    assert np.array_equal(ref_nan, out_nan), (
        f"NaN pattern differs: ref {ref_nan.sum()} NaN, out {out_nan.sum()} NaN, "
        f"mismatch {np.sum(ref_nan != out_nan)}")
    if not allow_nan_rows:
        assert not ref_nan.any()
    fin = ~ref_nan
    if not fin.any():
        return 0.0, 0.0
    d = np.abs(out[fin] - ref[fin])
    mx, mn = float(d.max()), float(d.mean())
    assert mx < tol[0], f"max abs err {mx:.3e} >= {tol[0]:.1e}"
    assert mn < tol[1], f"mean abs err {mn:.3e} >= {tol[1]:.1e}"
    return mx, mn


def torch_reference(q, k, v, causal=True, row_block=2048):
    """tests/reference.py semantics in fp32 on the tensors' device, chunked over
    (batch, kv head, query rows) so the score matrix stays bounded. TF32 off.
    The torch restatement of the reference oracle, pinned to the reference's
    fixtures by tests/test_oracle_golden.py."""
    from oracle.gqa_oracle_torch import gqa_reference_blocked
    return gqa_reference_blocked(q, k, v, causal=causal, row_block=row_block)
