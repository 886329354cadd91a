"""Paged-KV decode (gqa_kernels.paged.paged_decode, C ABI gqa_paged_decode) against the
torch fp32 restatement of tests/reference.py on each sequence's keys, gathered dense.
Physical blocks are shuffled across sequences; lengths cover 0, 1, block edges and
long sequences that take the fused key split."""
import ctypes

import pytest
import torch

from gqa_kernels import _lib
from gqa_kernels.paged import paged_decode
from tests._common import BASELINE_TOL, compare, to_np, torch_reference

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _lib_ready(cuda_lib):
    yield
    torch.cuda.synchronize()


def _paged_case(seq_lens, Hq, Hkv, D, block_size, seed, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    n = len(seq_lens)
    max_blocks = max(1, max(-(-s // block_size) for s in seq_lens))
    need = sum(-(-s // block_size) for s in seq_lens)
    num_blocks = need + 5
    kc = torch.randn(num_blocks, block_size, Hkv, D, generator=g, device="cuda").to(dtype)
    vc = torch.randn(num_blocks, block_size, Hkv, D, generator=g, device="cuda").to(dtype)
    perm = torch.randperm(num_blocks, generator=torch.Generator().manual_seed(seed)).tolist()
    bt = torch.zeros(n, max_blocks, dtype=torch.int32)
    c = 0
    for i, s in enumerate(seq_lens):
        for j in range(-(-s // block_size)):
            bt[i, j] = perm[c]
            c += 1
    q = torch.randn(n, Hq, D, generator=g, device="cuda").to(dtype)
    return q, kc, vc, bt.cuda(), torch.tensor(seq_lens, dtype=torch.int32, device="cuda")


def _dense(kc, bt_row, s, block_size):
    """(1, Hkv, s, D) keys of one sequence, gathered from its blocks."""
    blocks = [kc[int(bt_row[j])] for j in range(-(-s // block_size))]
    return torch.cat(blocks, dim=0)[:s].permute(1, 0, 2).unsqueeze(0)


@pytest.mark.parametrize("block_size,D,dtype", [(64, 128, torch.bfloat16), (128, 128, torch.float16),
                                                (256, 64, torch.bfloat16)])
def test_paged_decode_matches_dense_reference(block_size, D, dtype):
    seq_lens = [1, 63, 64, 65, 1000, 4097, 17000]
    Hq, Hkv = 32, 8
    q, kc, vc, bt, sl = _paged_case(seq_lens, Hq, Hkv, D, block_size, seed=block_size + D, dtype=dtype)
    out = paged_decode(q, kc, vc, bt, sl)
    torch.cuda.synchronize()
    btc = bt.cpu()
    for i, s in enumerate(seq_lens):
        k = _dense(kc, btc[i], s, block_size)
        v = _dense(vc, btc[i], s, block_size)
        ref = torch_reference(q[i:i + 1, :, None, :], k, v, causal=True)[0, :, 0]
        compare(to_np(out[i]), to_np(ref), BASELINE_TOL)


def test_paged_decode_empty_sequence_is_nan_and_others_unaffected():
    seq_lens = [0, 300, 2048]
    q, kc, vc, bt, sl = _paged_case(seq_lens, 16, 2, 128, 64, seed=3)
    out = paged_decode(q, kc, vc, bt, sl, max_seq_len=2048)
    torch.cuda.synchronize()
    assert torch.isnan(out[0]).all()
    btc = bt.cpu()
    for i in (1, 2):
        k = _dense(kc, btc[i], seq_lens[i], 64)
        v = _dense(vc, btc[i], seq_lens[i], 64)
        ref = torch_reference(q[i:i + 1, :, None, :], k, v, causal=True)[0, :, 0]
        compare(to_np(out[i]), to_np(ref), BASELINE_TOL)


def test_paged_decode_in_a_cuda_graph():
    seq_lens = [5000, 12000, 700, 64]
    q, kc, vc, bt, sl = _paged_case(seq_lens, 32, 8, 128, 128, seed=9)
    ref = paged_decode(q, kc, vc, bt, sl)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        paged_decode(q, kc, vc, bt, sl)  # warm-up on the capture stream (workspace)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = paged_decode(q, kc, vc, bt, sl)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    compare(to_np(out), to_np(ref), (1e-6, 1e-7))  # the same plan: identical results


def test_paged_decode_rejects_bad_blocks():
    lib = _lib.load()
    q, kc, vc, bt, sl = _paged_case([100], 8, 2, 128, 64, seed=1)
    o = torch.empty_like(q)
    args = lambda bs: (ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(kc.data_ptr()), ctypes.c_void_p(vc.data_ptr()),  # noqa: E731
                       ctypes.c_void_p(o.data_ptr()), _lib.strides(q, 3), _lib.strides(o, 3),
                       ctypes.c_void_p(bt.data_ptr()), bt.stride(0), ctypes.c_void_p(sl.data_ptr()),
                       1, 8, 2, 128, bs, kc.shape[0], 100, 0.1, 1, None, 0, None)
    assert lib.gqa_paged_decode(*args(32)) == 2  # block_size below 64: unsupported
    assert lib.gqa_paged_decode(*args(96)) == 2  # not a power of two
