"""Fits the polynomial of the kernels' software exp2 (gqa_common.cuh: exp2_poly2).

Method: Cody-Waite style range reduction x = n + f, n = round(x), f in [-1/2, 1/2],
2^x = 2^n * 2^f, with 2^f approximated by a degree-3 polynomial whose relative
error is made near-equioscillating by Lawson's iteratively reweighted least
squares on a Chebyshev grid. The evaluation below mirrors the kernel's float32
instruction sequence (round-to-nearest via the 1.5 * 2^23 addend, Horner FMAs,
exponent add on the bit pattern) and reports its error against numpy.exp2.

    python tests/exp2_fit.py

tests/test_exp2_fit_host.py checks that the kernel's coefficients are this fit.
"""
import numpy as np


def fit(deg, iters=400):
    f = np.cos(np.linspace(0, np.pi, 4001)) * 0.5          # Chebyshev-clustered grid on [-1/2, 1/2]
    y = np.exp2(f)
    A = np.vander(f, deg + 1, increasing=True) / y[:, None]  # relative error
    w = np.ones_like(f) / len(f)
    for _ in range(iters):
        sw = np.sqrt(w)
        c, *_ = np.linalg.lstsq(A * sw[:, None], np.ones_like(f) * sw, rcond=None)
        e = np.abs(A @ c - 1)
        w = w * e
        w /= w.sum()
    return c


def kernel_exp2(x, c):
    """The kernel's float32 sequence: clamp, round via addend, Horner, exponent add."""
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    r = (t - magic).astype(np.float32)
    fr = (x - r).astype(np.float32)
    p = np.float32(c[-1])
    for ck in c[-2::-1]:
        p = (p * fr + np.float32(ck)).astype(np.float32)
    bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return bits.astype(np.uint32).view(np.float32)


def max_rel_error(c32):
    x = np.concatenate([np.linspace(-126, 8, 2_000_001, dtype=np.float32),
                        -np.random.default_rng(0).random(1_000_000, dtype=np.float32) * 30])
    got = kernel_exp2(x, c32)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got / ref - 1)
    return float(rel.max()), float(rel.mean()), int(np.sum(~(got >= 0)))


if __name__ == "__main__":
    for deg in (3, 4):
        c32 = fit(deg).astype(np.float32)
        mx, mean, bad = max_rel_error(c32)
        print(f"deg {deg}: coeffs {[float(v) for v in c32]}  max rel err {mx:.3e}  mean {mean:.3e}  neg/nan {bad}")
