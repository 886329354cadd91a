"""The multi-GPU partitionings over real NCCL ranks (one process per GPU).

Skipped unless at least two GPUs are visible. Each rank computes its share
with the CUDA path; the key-axis split exchanges partials with one NCCL
all-gather and combines them with gqa_lse_combine. Every rank's output must
match the single-GPU gqa_flash_attn of the same inputs.
"""
import datetime
import os

import pytest
import torch

from tests._common import BASELINE_TOL, compare, make_inputs, to_np
from tests._dist import free_port

pytestmark = pytest.mark.gpu


def _rank_main(rank, world, port, q_ret):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from gqa_kernels import gqa_flash_attn
        from gqa_kernels import sharded as S
        res = {}
        # key-axis split (long-context decode shape, reduced)
        B, Hq, Hkv, Sq, Skv, D = 4, 64, 8, 1, 20000, 128
        q, k, v = (t.to(dev) for t in make_inputs(B, Hq, Hkv, Sq, Skv, D, seed=5))
        full = gqa_flash_attn(q, k, v)
        k0, k1 = S.kv_range(Skv, world, rank)
        out = S.seq_sharded_forward(q, k[:, :, k0:k1].contiguous(), v[:, :, k0:k1].contiguous(), k0, Skv)
        res["seq"] = ((out.float() - full.float()).abs().max().item(), (out.float() - full.float()).abs().mean().item())
        # chunked prefill with a bottom-right causal mask, split into key shards
        B, Hq, Hkv, Sq, Skv, D = 1, 32, 8, 5, 3000, 128
        q, k, v = (t.to(dev) for t in make_inputs(B, Hq, Hkv, Sq, Skv, D, seed=6))
        full = gqa_flash_attn(q, k, v)
        k0, k1 = S.kv_range(Skv, world, rank)
        out = S.seq_sharded_forward(q, k[:, :, k0:k1].contiguous(), v[:, :, k0:k1].contiguous(), k0, Skv)
        res["seq_causal"] = ((out.float() - full.float()).abs().max().item(),
                             (out.float() - full.float()).abs().mean().item())
        # the same key split with the peer exchange (NVLink stores in the partial
        # kernel, in-kernel waits in the combine): bit-identical to the all-gather
        # form over three calls (both parities of the receive buffer, new inputs each)
        B, Hq, Hkv, Sq, Skv, D = 4, 64, 8, 1, 20000, 128
        q, k, v = (t.to(dev) for t in make_inputs(B, Hq, Hkv, Sq, Skv, D, seed=8))
        k0, k1 = S.kv_range(Skv, world, rank)
        ks, vs = k[:, :, k0:k1].contiguous(), v[:, :, k0:k1].contiguous()
        ex = S.PeerExchange(q.shape, Hkv, dev)
        same, worst = True, 0.0
        try:
            full = gqa_flash_attn(q, k, v)
            for call in range(3):
                qc = q * (1.0 + 0.25 * call)
                ref = S.seq_sharded_forward(qc, ks, vs, k0, Skv)
                got = ex.forward(qc, ks, vs, k0, Skv)
                torch.cuda.synchronize(dev)
                same = same and torch.equal(got.view(torch.int16), ref.view(torch.int16))
                if call == 0:
                    worst = (got.float() - full.float()).abs().max().item()
        finally:
            ex.close()
        res["peer_same"] = same
        res["peer"] = (worst, 0.0)
        # batch x kv-head units, no communication
        B, Hq, Hkv, Sq, Skv, D = 4, 32, 8, 512, 2048, 128
        q, k, v = (t.to(dev) for t in make_inputs(B, Hq, Hkv, Sq, Skv, D, seed=7))
        full = gqa_flash_attn(q, k, v)
        br, hr = S.shard_units(B, Hkv, world, rank)
        ql, kl, vl = S.slice_units(q, k, v, br, hr)
        g = Hq // Hkv
        d = (S.head_sharded_forward(ql, kl, vl).float() - full[br[0]:br[1], hr[0] * g:hr[1] * g].float()).abs()
        res["units"] = (d.max().item(), d.mean().item())
        dist.barrier()
        q_ret.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_sharded_paths_over_nccl():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    world = min(n, 8)
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for rank, res in results.items():
        for key in ("seq", "seq_causal", "units", "peer"):
            mx, mn = res[key]
            assert mx < BASELINE_TOL[0] and mn < BASELINE_TOL[1], (rank, key, mx, mn)
        assert res["peer_same"], rank
