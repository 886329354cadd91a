"""Paged chunked prefill (gqa_kernels.paged.paged_prefill, C ABI gqa_paged_fwd) against
the torch fp32 restatement of tests/reference.py on each sequence's keys, gathered
dense, and against the dense path on the same keys. Physical blocks are shuffled
across sequences. Chunks of more than 64 packed rows take the tcgen05 prefill
kernel (with and without the key split), shorter ones the streaming kernel."""
import pytest
import torch

from gqa_kernels import gqa_flash_attn
from gqa_kernels.paged import paged_decode, paged_prefill
from tests._common import BASELINE_TOL, compare, to_np, torch_reference

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _lib_ready(cuda_lib):
    yield
    torch.cuda.synchronize()


def _cache(seq_lens, Hkv, D, block_size, seed, dtype, spare=5):
    """Random K/V caches and a shuffled block table holding seq_lens keys per sequence."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    n = len(seq_lens)
    max_blocks = max(1, max(-(-s // block_size) for s in seq_lens))
    num_blocks = sum(-(-s // block_size) for s in seq_lens) + spare
    kc = torch.randn(num_blocks, block_size, Hkv, D, generator=g, device="cuda").to(dtype)
    vc = torch.randn(num_blocks, block_size, Hkv, D, generator=g, device="cuda").to(dtype)
    perm = torch.randperm(num_blocks, generator=torch.Generator().manual_seed(seed)).tolist()
    bt = torch.zeros(n, max_blocks, dtype=torch.int32)
    c = 0
    for i, s in enumerate(seq_lens):
        for j in range(-(-s // block_size)):
            bt[i, j] = perm[c]
            c += 1
    return kc, vc, bt.cuda(), torch.tensor(seq_lens, dtype=torch.int32, device="cuda")


def _dense(cache, bt_row, s, block_size):
    """(1, Hkv, s, D) keys (or values) of one sequence, gathered from its blocks."""
    if s == 0:
        return cache[:0, 0].permute(1, 0, 2).unsqueeze(0)
    blocks = [cache[int(bt_row[j])] for j in range(-(-s // block_size))]
    return torch.cat(blocks, dim=0)[:s].permute(1, 0, 2).unsqueeze(0)


def _check_against_reference(out, q, kc, vc, bt, seq_lens, block_size, causal=True):
    btc = bt.cpu()
    for i, s in enumerate(seq_lens):
        k = _dense(kc, btc[i], s, block_size)
        v = _dense(vc, btc[i], s, block_size)
        if s == 0:
            assert torch.isnan(out[i]).all()
            continue
        ref = torch_reference(q[i:i + 1], k, v, causal=causal)
        compare(to_np(out[i:i + 1]), to_np(ref), BASELINE_TOL)


@pytest.mark.parametrize("block_size,D,dtype", [(64, 128, torch.bfloat16), (128, 128, torch.float16),
                                                (256, 64, torch.bfloat16)])
def test_paged_prefill_matches_reference(block_size, D, dtype):
    # 5 sequences x 8 kv heads x 5 query pairs = 200 units: one CTA per unit.
    chunk = 300
    seq_lens = [300, 301, 1000, 4097, 17000]
    Hq, Hkv = 32, 8
    kc, vc, bt, sl = _cache(seq_lens, Hkv, D, block_size, seed=block_size + D, dtype=dtype)
    q = torch.randn(len(seq_lens), Hq, chunk, D, device="cuda").to(dtype)
    out = paged_prefill(q, kc, vc, bt, sl)
    torch.cuda.synchronize()
    _check_against_reference(out, q, kc, vc, bt, seq_lens, block_size)


def test_paged_prefill_split_with_short_and_empty_sequences():
    # 4 sequences x 8 kv heads x 2 query pairs = 64 units < SMs: the key split runs.
    # The plan covers max_seq_len; the short sequences' later splits have no key
    # tile, the empty sequence none at all (NaN), and the first sequence's first 28
    # query rows see no key (NaN).
    chunk = 128
    seq_lens = [100, 700, 17000, 0]
    kc, vc, bt, sl = _cache(seq_lens, 8, 128, 64, seed=11, dtype=torch.bfloat16)
    q = torch.randn(len(seq_lens), 32, chunk, 128, device="cuda").bfloat16()
    out = paged_prefill(q, kc, vc, bt, sl)
    torch.cuda.synchronize()
    assert torch.isnan(out[0, :, :28]).all() and not torch.isnan(out[0, :, 28:]).any()
    _check_against_reference(out, q, kc, vc, bt, seq_lens, 64)


@pytest.mark.parametrize("chunk,Hq,Hkv", [(8, 32, 8), (1, 32, 8), (16, 16, 4)])
def test_paged_short_chunks_take_the_streaming_kernel(chunk, Hq, Hkv):
    seq_lens = [chunk, chunk + 1, 100, 5000, 17000]
    kc, vc, bt, sl = _cache(seq_lens, Hkv, 128, 128, seed=chunk + Hq, dtype=torch.bfloat16)
    q = torch.randn(len(seq_lens), Hq, chunk, 128, device="cuda").bfloat16()
    out = paged_prefill(q, kc, vc, bt, sl)
    torch.cuda.synchronize()
    _check_against_reference(out, q, kc, vc, bt, seq_lens, 128)
    if chunk == 1:  # one token per sequence: the decode entry point's result
        dec = paged_decode(q[:, :, 0], kc, vc, bt, sl)
        assert torch.equal(dec.view(torch.int16), out[:, :, 0].view(torch.int16))


def test_paged_prefill_non_causal():
    seq_lens = [512, 3000]
    kc, vc, bt, sl = _cache(seq_lens, 8, 128, 128, seed=5, dtype=torch.bfloat16)
    q = torch.randn(2, 32, 200, 128, device="cuda").bfloat16()
    out = paged_prefill(q, kc, vc, bt, sl, causal=False)
    torch.cuda.synchronize()
    _check_against_reference(out, q, kc, vc, bt, seq_lens, 128, causal=False)


@pytest.mark.parametrize("B,chunk,S", [(4, 512, 16384), (1, 512, 8192), (2, 384, 1000)])
def test_paged_prefill_equals_dense_path(B, chunk, S):
    # Every sequence as long as the plan's bound: the paged kernel runs the dense
    # kernel's plan (split for (1, 512, 8192)) on the same keys; boxes past the end
    # are zero in both, and masked slots (stale cache rows in the paged case) get
    # P <= 2^-126, far below one ulp of O. The outputs are bit-identical.
    block_size = 128
    kc, vc, bt, sl = _cache([S] * B, 8, 128, block_size, seed=B + chunk, dtype=torch.bfloat16, spare=0)
    q = torch.randn(B, 32, chunk, 128, device="cuda").bfloat16()
    out = paged_prefill(q, kc, vc, bt, sl, max_seq_len=S)
    btc = bt.cpu()
    k = torch.cat([_dense(kc, btc[i], S, block_size) for i in range(B)]).contiguous()
    v = torch.cat([_dense(vc, btc[i], S, block_size) for i in range(B)]).contiguous()
    dense = gqa_flash_attn(q, k, v, causal=True)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), dense.view(torch.int16))


def test_paged_prefill_in_a_cuda_graph():
    seq_lens = [5000, 12000, 700, 600]
    kc, vc, bt, sl = _cache(seq_lens, 8, 128, 64, seed=21, dtype=torch.bfloat16)
    q = torch.randn(4, 32, 512, 128, device="cuda").bfloat16()
    ref = paged_prefill(q, kc, vc, bt, sl)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        paged_prefill(q, kc, vc, bt, sl)  # warm-up on the capture stream (workspace)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = paged_prefill(q, kc, vc, bt, sl)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("chunk", [1, 8, 100])
def test_paged_against_the_numpy_oracle(chunk):
    """oracle.paged_reference (the reference attention over the gathered blocks) on a
    small case: decode, a streaming-kernel chunk and a tcgen05 chunk."""
    from oracle import gqa_oracle as O
    seq_lens = [chunk, 130, 700]
    kc, vc, bt, sl = _cache(seq_lens, 2, 128, 64, seed=chunk, dtype=torch.bfloat16)
    q = torch.randn(len(seq_lens), 8, chunk, 128, device="cuda").bfloat16()
    out = paged_prefill(q, kc, vc, bt, sl)
    torch.cuda.synchronize()
    ref = O.paged_reference(to_np(q), to_np(kc), to_np(vc), bt.cpu().numpy(), seq_lens, causal=True)
    compare(to_np(out), ref, BASELINE_TOL)
