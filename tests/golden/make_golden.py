"""Generates the golden fixtures in tests/golden/ from the reference project itself.

    TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/reference

Run once, where the reference checkout exists (it is not needed afterwards):
  * oracle_bf16.npz -- the reference's oracle (tests/reference.py:gqa_reference)
    evaluated in fp32 on bf16 inputs drawn N(0,1) from a CPU torch.Generator
    seeded per case (q, k, v drawn in that order), for small shapes that cover
    prefill, bottom-right chunked prefill, decode, non-causal, seq_q > seq_kv
    (NaN rows), group sizes 1/2/4/8 and head_dim 64/128. For BASELINE config 1
    (B=1, Hq=32, Hkv=8, D=128, S=512, causal, seed 0) it stores a CRC of the
    inputs' bits, output sums and 64 seeded output rows instead of the full tensors.
  * triton_f16.npz -- the reference's Triton kernels (gqa_kernels/gqa_fwd.py,
    gqa_kernels/gqa_split.py) run on CPU by Triton's interpreter in float16
    (the interpreter cannot evaluate the bf16 kernels): single-pass outputs,
    split-KV partials (m_p, l_p, acc_p) and the reduced output.
  * routing.json -- the (path, splits) the reference dispatcher
    (gqa_kernels/dispatch.py:37-49) picks for a grid of shapes, recorded by
    calling its gqa_flash_attn with the two launch targets replaced by recorders.
"""
import json
import os
import sys
import types
import zlib

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("GQA_REFERENCE_DIR", "")
if not REF or not os.path.isdir(REF):
    sys.exit("usage: make_golden.py /path/to/reference (or set GQA_REFERENCE_DIR)")
sys.path.insert(0, REF)

from tests.reference import gqa_reference  # noqa: E402  (reference oracle)
import gqa_kernels.dispatch as ref_dispatch  # noqa: E402
from gqa_kernels.gqa_fwd import gqa_fwd_kernel  # noqa: E402
from gqa_kernels.gqa_split import gqa_split_first_kernel, gqa_split_reduce_kernel  # noqa: E402

LOG2E = 1.4426950408889634

# name: (B, Hq, Hkv, Sq, Skv, D, causal, seed)
ORACLE_CASES = {
    "prefill_g4_d64": (1, 8, 2, 64, 64, 64, True, 0),
    "chunked_b2": (2, 8, 2, 16, 80, 64, True, 1),
    "decode_d128": (1, 8, 2, 1, 200, 128, True, 2),
    "noncausal_g2": (1, 4, 2, 24, 40, 64, False, 3),
    "sq_gt_skv": (1, 4, 2, 40, 24, 64, True, 4),
    "g8_d64": (1, 16, 2, 48, 48, 64, True, 5),
    "llama_s16": (1, 32, 8, 16, 16, 128, True, 6),
    "g1_s130": (1, 2, 2, 130, 130, 128, True, 7),
    "odd_17_65": (1, 8, 2, 17, 65, 128, True, 8),
}

# name: (B, Hq, Hkv, Sq, Skv, D, causal, seed, BLOCK_M, BLOCK_N)
TRITON_FWD_CASES = {
    "fwd_prefill": (1, 8, 2, 64, 64, 64, True, 10, 16, 32),
    "fwd_chunked": (2, 8, 2, 16, 80, 64, True, 11, 16, 32),
    "fwd_noncausal_d128": (1, 4, 1, 20, 20, 128, False, 12, 8, 32),
    "fwd_sq_gt_skv": (1, 4, 2, 24, 16, 64, True, 13, 16, 32),
}
# name: (B, Hq, Hkv, Sq, Skv, D, causal, seed, SPLITS)
TRITON_SPLIT_CASES = {
    "split_decode": (1, 8, 2, 1, 200, 64, True, 20, 4),
    "split_sq4_d128": (1, 8, 2, 4, 150, 128, True, 21, 4),
    # chunk [8, 10) is non-empty but fully masked for the rows at positions 6, 7:
    # the reference's partials are NaN there, and so is its reduced output.
    "split_masked_chunk": (1, 4, 2, 4, 10, 64, True, 22, 8),
    # ceil(256 / 4) = 64 is a multiple of BLOCK_N = 32: no key-block overrun
    "split_clean_chunks": (1, 8, 2, 2, 256, 64, True, 23, 4),
}


def draw(B, Hq, Hkv, Sq, Skv, D, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, Sq, D, generator=g).to(dtype)
    k = torch.randn(B, Hkv, Skv, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, Skv, D, generator=g).to(dtype)
    return q, k, v


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def oracle_fixtures():
    out = {}
    for name, (B, Hq, Hkv, Sq, Skv, D, causal, seed) in ORACLE_CASES.items():
        q, k, v = draw(B, Hq, Hkv, Sq, Skv, D, seed, torch.bfloat16)
        ref = gqa_reference(q.float(), k.float(), v.float(), causal=causal)
        out[f"{name}/q"] = bits(q)
        out[f"{name}/k"] = bits(k)
        out[f"{name}/v"] = bits(v)
        out[f"{name}/out"] = ref.numpy().astype(np.float32)
        out[f"{name}/meta"] = np.array([B, Hq, Hkv, Sq, Skv, D, int(causal), seed], dtype=np.int64)
    # BASELINE config 1 (CPU reference case), summarised.
    B, Hq, Hkv, S, D = 1, 32, 8, 512, 128
    q, k, v = draw(B, Hq, Hkv, S, S, D, 0, torch.bfloat16)
    ref = gqa_reference(q.float(), k.float(), v.float(), causal=True).numpy()
    rng = np.random.default_rng(1234)
    rows = np.stack([rng.integers(0, Hq, 64), rng.integers(0, S, 64)], axis=1)
    out["config1/meta"] = np.array([B, Hq, Hkv, S, S, D, 1, 0], dtype=np.int64)
    out["config1/crc_qkv"] = np.array([zlib.crc32(bits(t).tobytes()) for t in (q, k, v)], dtype=np.int64)
    out["config1/rows"] = rows.astype(np.int64)
    out["config1/row_out"] = ref[0, rows[:, 0], rows[:, 1]].astype(np.float32)
    out["config1/sum"] = np.array([ref.astype(np.float64).sum(), np.abs(ref.astype(np.float64)).sum()])
    return out


def triton_fixtures():
    out = {}
    for name, (B, Hq, Hkv, Sq, Skv, D, causal, seed, BM, BN) in TRITON_FWD_CASES.items():
        q, k, v = draw(B, Hq, Hkv, Sq, Skv, D, seed, torch.float16)
        o = torch.full_like(q, float("nan"))
        fn = gqa_fwd_kernel.fn  # the JIT function under the autotuner, with one explicit config
        fn[(-(-Sq // BM), Hkv, B)](
            q, k, v, o, *q.stride(), *k.stride(), *v.stride(), *o.stride(), Sq, Skv, (D ** -0.5) * LOG2E,
            IS_CAUSAL=causal, GROUP_SIZE=Hq // Hkv, HEAD_DIM=D, BLOCK_M=BM, BLOCK_N=BN)
        for key, t in (("q", q), ("k", k), ("v", v), ("out", o)):
            out[f"{name}/{key}"] = t.numpy()
        out[f"{name}/meta"] = np.array([B, Hq, Hkv, Sq, Skv, D, int(causal), seed, BM, BN], dtype=np.int64)
    for name, (B, Hq, Hkv, Sq, Skv, D, causal, seed, SPLITS) in TRITON_SPLIT_CASES.items():
        q, k, v = draw(B, Hq, Hkv, Sq, Skv, D, seed, torch.float16)
        m_p = torch.full((B, Hq, Sq, SPLITS), float("nan"))
        l_p = torch.full_like(m_p, float("nan"))
        acc_p = torch.full((B, Hq, Sq, SPLITS, D), float("nan"))
        o = torch.full_like(q, float("nan"))
        BM = 16 if Sq <= 16 else 32
        gqa_split_first_kernel.fn[(Hkv, -(-Sq // BM), B * SPLITS)](
            q, k, v, m_p, l_p, acc_p, *q.stride(), *k.stride(), *v.stride(), *m_p.stride(), *acc_p.stride(),
            Sq, Skv, (D ** -0.5) * LOG2E, IS_CAUSAL=causal, GROUP_SIZE=Hq // Hkv, HEAD_DIM=D, BLOCK_M=BM,
            SPLITS=SPLITS, BLOCK_N=32)
        gqa_split_reduce_kernel[(Hq, Sq, B)](
            m_p, l_p, acc_p, o, *m_p.stride(), *acc_p.stride(), *o.stride(), HEAD_DIM=D, SPLITS=SPLITS)
        for key, t in (("q", q), ("k", k), ("v", v), ("m_p", m_p), ("l_p", l_p), ("acc_p", acc_p), ("out", o)):
            out[f"{name}/{key}"] = t.numpy()
        out[f"{name}/meta"] = np.array([B, Hq, Hkv, Sq, Skv, D, int(causal), seed, SPLITS], dtype=np.int64)
    return out


class _Fake:
    """Shape-only stand-in for a CUDA tensor, enough for the dispatcher's host logic."""

    is_cuda = True

    def __init__(self, shape):
        self.shape = tuple(shape)

    def stride(self, i=None):
        return 0 if i is not None else (0, 0, 0, 0)


def routing_fixture():
    calls = []

    def rec_split(q, k, v, causal, splits):
        calls.append(("split", splits))

    class _Rec:
        def __getitem__(self, grid):
            def launch(*a, **kw):
                calls.append(("single", None))
            return launch

    ref_dispatch.split_kv_forward = rec_split
    ref_dispatch.gqa_fwd_kernel = _Rec()
    ref_dispatch.torch = types.SimpleNamespace(empty_like=lambda t: _Fake(t.shape))
    table = []
    for batch in (1, 2, 3, 4, 64):
        for hkv in (1, 2, 4, 8, 16):
            for sq in (1, 2, 16, 17, 512):
                for skv in (1, 63, 64, 512, 1023, 1024, 1500, 2048, 4096, 16384, 65536, 131072):
                    calls.clear()
                    ref_dispatch.gqa_flash_attn(_Fake((batch, hkv * 4, sq, 128)), _Fake((batch, hkv, skv, 128)),
                                                _Fake((batch, hkv, skv, 128)), causal=True)
                    path, splits = calls[0]
                    table.append([sq, skv, hkv, batch, path, splits])
    return table


def main():
    np.savez_compressed(os.path.join(HERE, "oracle_bf16.npz"), **oracle_fixtures())
    np.savez_compressed(os.path.join(HERE, "triton_f16.npz"), **triton_fixtures())
    with open(os.path.join(HERE, "routing.json"), "w") as f:
        json.dump({"columns": ["seq_q", "seq_kv", "num_kv_heads", "batch", "path", "splits"],
                   "rows": routing_fixture()}, f)
    for fn in ("oracle_bf16.npz", "triton_f16.npz", "routing.json"):
        print(fn, os.path.getsize(os.path.join(HERE, fn)))


if __name__ == "__main__":
    main()
