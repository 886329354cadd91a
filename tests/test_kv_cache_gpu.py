"""PrefixKVCache on the GPU: chunked prefill and prefix reuse through the CUDA path
match full causal attention (torch fp32 restatement of tests/reference.py) within the
BASELINE tolerance, and attention reads the cache in place."""
import pytest
import torch

from gqa_kernels.kv_cache import PrefixKVCache
from tests._common import BASELINE_TOL, compare, make_inputs, to_np, torch_reference

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _lib_ready(cuda_lib):
    yield
    torch.cuda.synchronize()


@pytest.mark.parametrize("chunks,D", [((512, 300, 287, 1, 1), 128), ((64, 1000, 3), 64)])
def test_chunked_prefill_equals_full_causal_attention(chunks, D):
    B, Hq, Hkv = 2, 32, 8
    S = sum(chunks)
    q, k, v = (t.cuda() for t in make_inputs(B, Hq, Hkv, S, S, D, seed=11))
    full = torch_reference(q, k, v, causal=True)
    cache = PrefixKVCache(B, Hkv, D, capacity=S + 16)
    outs, p = [], 0
    for n in chunks:
        outs.append(cache.prefill(q[:, :, p:p + n], k[:, :, p:p + n], v[:, :, p:p + n]))
        p += n
    compare(to_np(torch.cat(outs, dim=2)), to_np(full), BASELINE_TOL)


def test_prefix_reuse_across_turns():
    B, Hq, Hkv, D = 1, 32, 8, 128
    P, A, Bn = 700, 200, 150
    q, k, v = (t.cuda() for t in make_inputs(B, Hq, Hkv, P + A, P + A, D, seed=12))
    qb, kb, vb = (t.cuda() for t in make_inputs(B, Hq, Hkv, Bn, Bn, D, seed=13))
    cache = PrefixKVCache(B, Hkv, D, capacity=2048)
    cache.prefill(q[:, :, :P], k[:, :, :P], v[:, :, :P])      # shared prefix
    cache.prefill(q[:, :, P:], k[:, :, P:], v[:, :, P:])      # turn A
    cache.truncate(P)                                          # back to the prefix
    out_b = cache.prefill(qb, kb, vb)                          # turn B
    kk = torch.cat([k[:, :, :P], kb], dim=2)
    vv = torch.cat([v[:, :, :P], vb], dim=2)
    ref = torch_reference(qb, kk, vv, causal=True)
    compare(to_np(out_b), to_np(ref), BASELINE_TOL)


def test_decode_steps_read_the_cache_in_place():
    B, Hq, Hkv, D = 1, 32, 8, 128
    S = 4096
    q, k, v = (t.cuda() for t in make_inputs(B, Hq, Hkv, S + 2, S + 2, D, seed=14))
    cache = PrefixKVCache(B, Hkv, D, capacity=S + 64)
    cache.append(k[:, :, :S], v[:, :, :S])
    out1 = cache.prefill(q[:, :, S:S + 1], k[:, :, S:S + 1], v[:, :, S:S + 1])   # warm-up (workspace)
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    out2 = cache.prefill(q[:, :, S + 1:S + 2], k[:, :, S + 1:S + 2], v[:, :, S + 1:S + 2])
    torch.cuda.synchronize()
    grown = torch.cuda.memory_allocated() - before
    assert grown <= 2 * out2.numel() * out2.element_size() + 4096, grown  # the output, not a cache copy
    ref = torch_reference(q[:, :, S:S + 2], k, v, causal=True)
    compare(to_np(torch.cat([out1, out2], dim=2)), to_np(ref), BASELINE_TOL)
