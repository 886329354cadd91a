"""The cache-write half of the vLLM-shaped interface and the layer that ties it to the
attention (gqa_kernels.paged: paged_kv_append, PagedAttention; C ABI gqa_paged_kv_append).

- The cache bytes after an append are bit-exact against a host scatter through the slot
  mapping (16-bit caches), and against torch's float8_e4m3fn cast of the scaled values,
  saturated to +-448 (e4m3 caches). Padding tokens (slot -1) write nothing; a slot past
  the cache writes nothing and is reported in the device error word.
- Stale cache slots past a sequence's length that hold NaN or Inf do not reach the
  output, on the streaming path (decode, short chunks, e4m3) and on the tcgen05 path
  (long chunks, with and without the key split).
- PagedAttention.forward (append, then attend) over decode and chunked-prefill steps
  matches the torch fp32 restatement of tests/reference.py on each sequence's keys.
"""
import pytest
import torch

from gqa_kernels import check_device_error
from gqa_kernels.paged import PagedAttention, PagedAttentionMetadata, paged_decode, paged_kv_append, paged_prefill
from tests._common import BASELINE_TOL, compare, to_np, torch_reference

pytestmark = pytest.mark.gpu
GQA_ERR_INVALID_ARG = 1


@pytest.fixture(autouse=True)
def _lib_ready(cuda_lib):
    check_device_error()
    yield
    torch.cuda.synchronize()


def _e4m3(x, scale):
    """torch's float8_e4m3fn cast of x / scale saturated to +-448, the division done
    element by element in IEEE fp32 on the CPU (as the kernel divides)."""
    xf = x.float().cpu()
    return (xf / torch.full_like(xf, scale)).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)


def _tokens(n, Hkv, D, dtype, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = (torch.randn(n, Hkv, D, generator=g, device="cuda") * scale).to(dtype)
    v = (torch.randn(n, Hkv, D, generator=g, device="cuda") * scale).to(dtype)
    return k, v


def _slots(n, num_slots, seed, pad=()):
    perm = torch.randperm(num_slots, generator=torch.Generator().manual_seed(seed))[:n].to(torch.int64)
    for i in pad:
        perm[i] = -1
    return perm.cuda()


@pytest.mark.parametrize("D,dtype,block_size", [(128, torch.bfloat16, 64), (64, torch.float16, 16),
                                                (128, torch.float16, 256)])
def test_append_16bit_is_a_scatter(D, dtype, block_size):
    Hkv, num_blocks, n = 8, 40, 300
    k, v = _tokens(n, Hkv, D, dtype, seed=D)
    slots = _slots(n, num_blocks * block_size, seed=D, pad=(0, 7, 299))
    kc = torch.full((num_blocks, block_size, Hkv, D), 3.0, dtype=dtype, device="cuda")
    vc = torch.full((num_blocks, block_size, Hkv, D), -5.0, dtype=dtype, device="cuda")
    ek, ev = kc.clone().view(-1, Hkv, D), vc.clone().view(-1, Hkv, D)
    paged_kv_append(k, v, kc, vc, slots)
    torch.cuda.synchronize()
    keep = slots >= 0
    ek[slots[keep]] = k[keep]
    ev[slots[keep]] = v[keep]
    assert torch.equal(kc.view(-1, Hkv, D).view(torch.int16), ek.view(torch.int16))
    assert torch.equal(vc.view(-1, Hkv, D).view(torch.int16), ev.view(torch.int16))
    assert check_device_error() == (0, 0)


def test_append_strided_rows():
    """key/value as slices of a fused (num_tokens, 3, Hkv, D) projection: row strides of
    the slice, not of a contiguous tensor."""
    Hkv, D, bs, nb, n = 4, 128, 64, 10, 50
    g = torch.Generator(device="cuda").manual_seed(4)
    qkv = torch.randn(n, 3, Hkv, D, generator=g, device="cuda").to(torch.bfloat16)
    k, v = qkv[:, 1], qkv[:, 2]
    slots = _slots(n, nb * bs, seed=4)
    kc = torch.zeros(nb, bs, Hkv, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    paged_kv_append(k, v, kc, vc, slots)
    torch.cuda.synchronize()
    assert torch.equal(kc.view(-1, Hkv, D)[slots], k) and torch.equal(vc.view(-1, Hkv, D)[slots], v)


@pytest.mark.parametrize("D,dtype,k_scale,v_scale", [(128, torch.bfloat16, 0.05, 0.5), (128, torch.float16, 1.0, 0.013),
                                                     (64, torch.bfloat16, 0.25, 2.0)])
def test_append_fp8_matches_torch_cast(D, dtype, k_scale, v_scale):
    Hkv, bs, nb, n = 8, 64, 30, 200
    k, v = _tokens(n, Hkv, D, dtype, seed=11, scale=8.0)  # |x| / scale reaches far past 448
    k[0, 0, :8] = torch.tensor([0.0, -0.0, 1e-6, -1e-6, 30.0, -30.0, 500.0, -500.0], dtype=dtype)
    slots = _slots(n, nb * bs, seed=11, pad=(5,))
    kc = torch.zeros(nb, bs, Hkv, D, dtype=torch.float8_e4m3fn, device="cuda")
    vc = torch.zeros_like(kc)
    paged_kv_append(k, v, kc, vc, slots, k_scale=k_scale, v_scale=v_scale)
    torch.cuda.synchronize()
    keep = slots >= 0
    for cache, x, sc in ((kc, k, k_scale), (vc, v, v_scale)):
        want = _e4m3(x[keep], sc)
        got = cache.view(-1, Hkv, D)[slots[keep]].cpu()
        assert torch.equal(got.view(torch.uint8), want.view(torch.uint8))
        # the padding token's slot and every untouched slot stay zero
        untouched = torch.ones(nb * bs, dtype=torch.bool, device="cuda")
        untouched[slots[keep]] = False
        assert (cache.view(-1, Hkv, D)[untouched].view(torch.uint8) == 0).all()
    assert (kc.view(-1, Hkv, D)[slots[0]].float().abs().max() == 448.0)  # saturated, not NaN


def test_append_slot_past_the_cache_is_reported_not_written():
    Hkv, D, bs, nb = 2, 128, 64, 4
    k, v = _tokens(3, Hkv, D, torch.bfloat16, seed=2)
    slots = torch.tensor([5, nb * bs, 7], dtype=torch.int64, device="cuda")
    kc = torch.zeros(nb + 1, bs, Hkv, D, dtype=torch.bfloat16, device="cuda")  # one guard block
    vc = torch.zeros_like(kc)
    paged_kv_append(k, v, kc[:nb], vc[:nb], slots)
    torch.cuda.synchronize()
    assert check_device_error() == (GQA_ERR_INVALID_ARG, 201)
    assert (kc[nb] == 0).all() and (vc[nb] == 0).all()  # nothing past the cache
    assert torch.equal(kc.view(-1, Hkv, D)[5], k[0]) and torch.equal(kc.view(-1, Hkv, D)[7], k[2])


# ----------------------------------------------------------------------------- stale slots
def _poisoned_cache(seq_lens, Hkv, D, bs, seed, dtype, poison):
    """Caches whose slots past each sequence's length in its last block hold `poison`
    (stale values of an earlier sequence), shuffled block table."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    n = len(seq_lens)
    nblk = [max(1, -(-s // bs)) for s in seq_lens]
    num_blocks = sum(nblk) + 3
    kc = torch.randn(num_blocks, bs, Hkv, D, generator=g, device="cuda").to(dtype)
    vc = torch.randn(num_blocks, bs, Hkv, D, generator=g, device="cuda").to(dtype)
    perm = torch.randperm(num_blocks, generator=torch.Generator().manual_seed(seed)).tolist()
    bt = torch.zeros(n, max(nblk), dtype=torch.int32)
    c = 0
    for i, s in enumerate(seq_lens):
        for j in range(nblk[i]):
            bt[i, j] = perm[c]
            c += 1
        last, used = bt[i, nblk[i] - 1], s - (nblk[i] - 1) * bs
        kc[last, used:] = poison
        vc[last, used:] = poison
    return kc, vc, bt.cuda(), torch.tensor(seq_lens, dtype=torch.int32, device="cuda")


def _gather(cache, bt_row, s, bs):
    blocks = [cache[int(bt_row[j])] for j in range(-(-s // bs))]
    return torch.cat(blocks, dim=0)[:s].permute(1, 0, 2).unsqueeze(0)


@pytest.mark.parametrize("poison", [float("nan"), float("inf")])
@pytest.mark.parametrize("chunk", [1, 4, 256])  # decode; streaming chunk; tcgen05 chunk
def test_stale_nonfinite_slots_do_not_reach_the_output(poison, chunk):
    seq_lens = [300, 1000, 4097, 17000] if chunk < 256 else [300, 1000, 4097]
    Hq, Hkv, D, bs = 32, 8, 128, 64
    kc, vc, bt, sl = _poisoned_cache(seq_lens, Hkv, D, bs, seed=chunk, dtype=torch.bfloat16, poison=poison)
    g = torch.Generator(device="cuda").manual_seed(7)
    q = torch.randn(len(seq_lens), Hq, chunk, D, generator=g, device="cuda").to(torch.bfloat16)
    out = paged_decode(q[:, :, 0], kc, vc, bt, sl)[:, :, None] if chunk == 1 else paged_prefill(q, kc, vc, bt, sl)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    btc = bt.cpu()
    for i, s in enumerate(seq_lens):
        ref = torch_reference(q[i:i + 1], _gather(kc, btc[i], s, bs), _gather(vc, btc[i], s, bs), causal=True)
        compare(to_np(out[i:i + 1]), to_np(ref), BASELINE_TOL)


def test_stale_nan_slots_key_split_prefill():
    """Few long sequences: the tcgen05 path splits each unit's keys across CTAs."""
    seq_lens = [8000, 2000]
    Hq, Hkv, D, bs = 32, 8, 128, 128
    kc, vc, bt, sl = _poisoned_cache(seq_lens, Hkv, D, bs, seed=5, dtype=torch.float16, poison=float("nan"))
    q = torch.randn(2, Hq, 128, D, generator=torch.Generator(device="cuda").manual_seed(8),
                    device="cuda").to(torch.float16)
    out = paged_prefill(q, kc, vc, bt, sl)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    btc = bt.cpu()
    for i, s in enumerate(seq_lens):
        ref = torch_reference(q[i:i + 1], _gather(kc, btc[i], s, bs), _gather(vc, btc[i], s, bs), causal=True)
        compare(to_np(out[i:i + 1]), to_np(ref), BASELINE_TOL)


def test_stale_nan_bytes_in_an_fp8_cache():
    seq_lens = [100, 5000]
    Hq, Hkv, D, bs = 32, 8, 128, 64
    kc, vc, bt, sl = _poisoned_cache(seq_lens, Hkv, D, bs, seed=9, dtype=torch.bfloat16, poison=0.0)
    k8, v8 = kc.to(torch.float8_e4m3fn), vc.to(torch.float8_e4m3fn)
    btc = bt.cpu()
    for i, s in enumerate(seq_lens):  # e4m3 NaN (0x7f) bytes in the stale slots
        nb = -(-s // bs)
        last, used = int(btc[i, nb - 1]), s - (nb - 1) * bs
        k8.view(torch.uint8)[last, used:] = 0x7F
        v8.view(torch.uint8)[last, used:] = 0x7F
    q = torch.randn(2, Hq, D, generator=torch.Generator(device="cuda").manual_seed(10),
                    device="cuda").to(torch.bfloat16)
    out = paged_decode(q, k8, v8, bt, sl, k_scale=0.5, v_scale=0.25)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    for i, s in enumerate(seq_lens):
        k = _gather(k8, btc[i], s, bs).float() * 0.5
        v = _gather(v8, btc[i], s, bs).float() * 0.25
        ref = torch_reference(q[i:i + 1, :, None].float(), k, v, causal=True)[0, :, 0]
        compare(to_np(out[i]), to_np(ref), BASELINE_TOL)


# ----------------------------------------------------------------------------- the layer
@pytest.mark.parametrize("kv_cache_dtype", ["auto", "fp8_e4m3"])
def test_paged_attention_layer_prefill_then_decode(kv_cache_dtype):
    """Two sequences: a chunked prefill step of 96 tokens each, then three decode steps,
    all through forward(query, key, value, kv_cache, attn_metadata)."""
    Hq, Hkv, D, bs, nb = 32, 8, 128, 64, 16
    dt = torch.bfloat16
    layer = PagedAttention(Hq, D, num_kv_heads=Hkv, kv_cache_dtype=kv_cache_dtype,
                           k_scale=0.02 if kv_cache_dtype == "fp8_e4m3" else 1.0,
                           v_scale=0.02 if kv_cache_dtype == "fp8_e4m3" else 1.0)
    cache = layer.allocate_kv_cache(nb, bs, dt, "cuda")
    bt = torch.tensor([[3, 9, 1, 12], [7, 0, 14, 5]], dtype=torch.int32, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(12)
    lens = [0, 0]
    all_q, all_k, all_v = [[], []], [[], []], [[], []]
    for step, qlen in enumerate([96, 1, 1, 1]):
        if kv_cache_dtype == "fp8_e4m3" and qlen > 1:
            qlen = 16  # e4m3 caches serve decode and short chunks (group * chunk <= 64)
        n = 2 * qlen
        q = torch.randn(n, Hq * D, generator=g, device="cuda").to(dt)
        k = torch.randn(n, Hkv * D, generator=g, device="cuda").to(dt)
        v = torch.randn(n, Hkv * D, generator=g, device="cuda").to(dt)
        slots = []
        for s in range(2):
            for t in range(qlen):
                pos = lens[s] + t
                slots.append(int(bt[s, pos // bs]) * bs + pos % bs)
            lens[s] += qlen
        md = PagedAttentionMetadata(slot_mapping=torch.tensor(slots, dtype=torch.int64, device="cuda"),
                                    block_tables=bt, seq_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"),
                                    query_len=qlen)
        out = layer.forward(q, k, v, cache, md)
        torch.cuda.synchronize()
        assert out.shape == q.shape and torch.isfinite(out).all()
        for s in range(2):
            rows = slice(s * qlen, (s + 1) * qlen)
            all_q[s].append(q[rows].view(qlen, Hq, D))
            kk = k[rows].view(qlen, Hkv, D)
            vv = v[rows].view(qlen, Hkv, D)
            if kv_cache_dtype == "fp8_e4m3":  # the reference sees the values the cache holds
                kk = _e4m3(kk, 0.02).float().cuda() * 0.02
                vv = _e4m3(vv, 0.02).float().cuda() * 0.02
            all_k[s].append(kk)
            all_v[s].append(vv)
            qs = q[rows].view(1, qlen, Hq, D).transpose(1, 2)
            ks = torch.cat(all_k[s]).float().permute(1, 0, 2).unsqueeze(0)
            vs = torch.cat(all_v[s]).float().permute(1, 0, 2).unsqueeze(0)
            ref = torch_reference(qs.float(), ks, vs, causal=True)
            got = out[rows].view(1, qlen, Hq, D).transpose(1, 2)
            compare(to_np(got), to_np(ref), BASELINE_TOL)


def test_paged_attention_layer_mixed_batches():
    """Mixed batches (vLLM's chunked prefill and decode in one step): three sequences with
    different new-token counts per step, given as query_lens; each step appends, then
    attends, and every sequence's rows match the fp32 reference over its own history."""
    Hq, Hkv, D, bs = 32, 8, 128, 64
    dt = torch.bfloat16
    layer = PagedAttention(Hq, D, num_kv_heads=Hkv)
    cache = layer.allocate_kv_cache(64, bs, dt, "cuda")
    bt = torch.randperm(60, generator=torch.Generator().manual_seed(5))[:60].view(3, 20).to(torch.int32).cuda()
    g = torch.Generator(device="cuda").manual_seed(13)
    lens = [0, 0, 0]
    hist_k, hist_v = [[], [], []], [[], [], []]
    for step_lens in ([200, 500, 1000], [1, 1, 37], [5, 1, 1], [1, 64, 1]):
        n = sum(step_lens)
        q = torch.randn(n, Hq * D, generator=g, device="cuda").to(dt)
        k = torch.randn(n, Hkv * D, generator=g, device="cuda").to(dt)
        v = torch.randn(n, Hkv * D, generator=g, device="cuda").to(dt)
        slots = []
        for s, m in enumerate(step_lens):
            for t in range(m):
                pos = lens[s] + t
                slots.append(int(bt[s, pos // bs]) * bs + pos % bs)
            lens[s] += m
        md = PagedAttentionMetadata(slot_mapping=torch.tensor(slots, dtype=torch.int64, device="cuda"),
                                    block_tables=bt, seq_lens=torch.tensor(lens, dtype=torch.int32, device="cuda"),
                                    query_lens=step_lens)
        out = layer.forward(q, k, v, cache, md)
        torch.cuda.synchronize()
        assert out.shape == q.shape and torch.isfinite(out).all()
        r0 = 0
        for s, m in enumerate(step_lens):
            rows = slice(r0, r0 + m)
            r0 += m
            hist_k[s].append(k[rows].view(m, Hkv, D))
            hist_v[s].append(v[rows].view(m, Hkv, D))
            ks = torch.cat(hist_k[s]).float().permute(1, 0, 2).unsqueeze(0)
            vs = torch.cat(hist_v[s]).float().permute(1, 0, 2).unsqueeze(0)
            qs = q[rows].view(1, m, Hq, D).transpose(1, 2).float()
            ref = torch_reference(qs, ks, vs, causal=True)
            compare(to_np(out[rows].view(1, m, Hq, D).transpose(1, 2)), to_np(ref), BASELINE_TOL)
