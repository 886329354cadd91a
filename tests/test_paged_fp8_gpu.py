"""fp8 (e4m3) paged K/V for decode and short chunks (gqa_kernels.paged with
float8_e4m3fn caches, C ABI gqa_paged_fwd_kv8) against the torch fp32 restatement of
tests/reference.py on the dequantised keys and values (stored value x scale) of each
sequence, gathered dense. The quantisation is in the inputs, so the contract
tolerance applies unchanged."""
import pytest
import torch

from gqa_kernels.paged import paged_decode, paged_prefill
from tests._common import BASELINE_TOL, compare, to_np, torch_reference

pytestmark = pytest.mark.gpu

FP8 = torch.float8_e4m3fn


@pytest.fixture(autouse=True)
def _lib_ready(cuda_lib):
    yield
    torch.cuda.synchronize()


def _cache8(seq_lens, Hkv, block_size, seed, D=128):
    """Random e4m3 K/V caches and a shuffled block table holding seq_lens keys per sequence."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    n = len(seq_lens)
    max_blocks = max(1, max(-(-s // block_size) for s in seq_lens))
    num_blocks = sum(-(-s // block_size) for s in seq_lens) + 3
    kc = (torch.randn(num_blocks, block_size, Hkv, D, generator=g, device="cuda") * 2).to(FP8)
    vc = (torch.randn(num_blocks, block_size, Hkv, D, generator=g, device="cuda") * 2).to(FP8)
    perm = torch.randperm(num_blocks, generator=torch.Generator().manual_seed(seed)).tolist()
    bt = torch.zeros(n, max_blocks, dtype=torch.int32)
    c = 0
    for i, s in enumerate(seq_lens):
        for j in range(-(-s // block_size)):
            bt[i, j] = perm[c]
            c += 1
    return kc, vc, bt.cuda(), torch.tensor(seq_lens, dtype=torch.int32, device="cuda")


def _dense(cache, bt_row, s, block_size, scale):
    """(1, Hkv, s, D) dequantised fp32 keys (or values) of one sequence."""
    blocks = [cache[int(bt_row[j])] for j in range(-(-s // block_size))]
    return (torch.cat(blocks, dim=0)[:s].float() * scale).permute(1, 0, 2).unsqueeze(0)


def _check(out, q, kc, vc, bt, seq_lens, block_size, k_scale, v_scale, causal):
    btc = bt.cpu()
    for i, s in enumerate(seq_lens):
        k = _dense(kc, btc[i], s, block_size, k_scale)
        v = _dense(vc, btc[i], s, block_size, v_scale)
        ref = torch_reference(q[i:i + 1].float(), k, v, causal=causal)
        compare(to_np(out[i:i + 1]), to_np(ref), BASELINE_TOL)


@pytest.mark.parametrize("block_size,dtype", [(64, torch.bfloat16), (256, torch.float16)])
def test_fp8_paged_decode_matches_dequantised_reference(block_size, dtype):
    seq_lens = [1, 63, 64, 65, 1000, 4097, 17000]
    kc, vc, bt, sl = _cache8(seq_lens, 8, block_size, seed=block_size)
    q = torch.randn(len(seq_lens), 32, 128, device="cuda").to(dtype)
    out = paged_decode(q, kc, vc, bt, sl, k_scale=0.5, v_scale=1.5)
    torch.cuda.synchronize()
    assert out.dtype == dtype and out.shape == q.shape
    _check(out[:, :, None], q[:, :, None], kc, vc, bt, seq_lens, block_size, 0.5, 1.5, causal=True)


@pytest.mark.parametrize("chunk,Hq,Hkv", [(8, 32, 8), (16, 32, 8), (2, 64, 8)])
def test_fp8_paged_short_chunks(chunk, Hq, Hkv):
    # 32, 64 and 16 packed rows: the streaming kernel's two- and four-row-group and
    # one-row-group variants.
    seq_lens = [chunk, chunk + 5, 700, 9000]
    kc, vc, bt, sl = _cache8(seq_lens, Hkv, 128, seed=chunk + Hq)
    q = torch.randn(len(seq_lens), Hq, chunk, 128, device="cuda").bfloat16()
    out = paged_prefill(q, kc, vc, bt, sl, k_scale=0.25, v_scale=0.75)
    torch.cuda.synchronize()
    _check(out, q, kc, vc, bt, seq_lens, 128, 0.25, 0.75, causal=True)


def test_fp8_unsupported_shapes_raise():
    kc, vc, bt, sl = _cache8([300], 8, 64, seed=1)
    long_chunk = torch.randn(1, 32, 64, 128, device="cuda").bfloat16()  # 256 packed rows
    with pytest.raises(RuntimeError, match="unsupported"):
        paged_prefill(long_chunk, kc, vc, bt, sl)
    kc64, vc64, bt64, sl64 = _cache8([300], 8, 64, seed=2, D=64)
    with pytest.raises(RuntimeError, match="unsupported"):
        paged_decode(torch.randn(1, 32, 64, device="cuda").bfloat16(), kc64, vc64, bt64, sl64)


def test_fp8_against_the_numpy_oracle():
    from oracle import gqa_oracle as O
    seq_lens = [1, 300, 2000]
    kc, vc, bt, sl = _cache8(seq_lens, 2, 64, seed=77)
    q = torch.randn(len(seq_lens), 8, 128, device="cuda").bfloat16()
    out = paged_decode(q, kc, vc, bt, sl, k_scale=0.5, v_scale=1.25)
    torch.cuda.synchronize()
    ref = O.paged_reference(to_np(q[:, :, None]), kc.float().cpu().numpy(), vc.float().cpu().numpy(),
                            bt.cpu().numpy(), seq_lens, causal=True, k_scale=0.5, v_scale=1.25)
    compare(to_np(out[:, :, None]), ref, BASELINE_TOL)
