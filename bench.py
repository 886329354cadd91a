"""Benchmark of the B200 GQA flash-attention forward (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|sdpa|flash_attn]
                    [--workload prefill|decode|chunked|long_decode|paged_decode|paged_decode_fp8]

Default workload (BASELINE metric "prefill TFLOP/s @8K causal; decode HBM GB/s
& us @16K KV"): Llama-3.1-8B-shape causal prefill B=1 per GPU, Hq=32, Hkv=8,
D=128, S=8192, bf16, inputs N(0,1) from a CUDA generator seeded by rank
(configs[1] of BASELINE.json); the same line carries the 16K-KV split-KV decode
(configs[2]) under "decode_16k". With N GPUs (torchrun) every rank runs its own
batch element (batch sharding, no communication: weak scaling).

A step is one gqa_flash_attn call. Prefill steps are timed one by one with CUDA
events on the launching stream, L2 (126 MB) flushed between steps by writing a
256 MB buffer (outside the events). Decode steps run as a serving loop does:
replayed back to back from CUDA graphs of up to 16 steps cycling 4 input copies
(268 MB > L2), the K timed steps between one pair of events. `value` is
algorithmic FLOPs (causal pairs only) or algorithmic bytes of all ranks /
max-over-ranks time. `e2e` repeats the metric through the public API with
pinned host inputs copied in and the output copied back inside the timed region,
double-buffered as a serving loop does (the next step's inputs copy in while a
step computes).

--impl reference times the reference's CPU path (the numpy port of
tests/reference.py in oracle/) on the host cores on a bounded sample of the
same workload; under torchrun only rank 0 runs it. --impl sdpa and --impl
flash_attn time same-box library comparators (torch SDPA, flash_attn 2) on the
same workloads and timing, the role the reference's benchmark/run.py gives
SDPA and FA2; their lines carry "impl" and report no launches of this library.

--workload paged_decode / paged_decode_fp8 time decode over a vLLM-layout paged
cache (gqa_kernels.paged) with bf16 or e4m3 K/V, config 3's shape for 8
sequences; `value` counts K/V at the cache's element size.
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "gqa-flash-attn-rtx3060_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "prefill TFLOP/s @8K causal; decode HBM GB/s & µs @16K KV (1/2/4/8 B200)"
FLUSH_BYTES = 256 << 20


# ----------------------------------------------------------------------------- workloads
def causal_pairs(sq, skv, causal=True):
    """Number of (query, key) pairs a causal (bottom-right) attention evaluates."""
    if not causal:
        return sq * skv
    off = skv - sq
    i = np.arange(sq, dtype=np.int64)
    return int(np.clip(i + off + 1, 0, skv).sum())


def attn_flops(B, Hq, Sq, Skv, D, causal=True):
    return 4.0 * B * Hq * D * causal_pairs(Sq, Skv, causal)


def attn_bytes(B, Hq, Hkv, Sq, Skv, D, elem=2):
    """Compulsory HBM bytes: K + V read once, Q read once, O written once."""
    return float(elem * (2 * B * Hkv * Skv * D + 2 * B * Hq * Sq * D))


WORKLOADS = {
    # name: (B per rank, Hq, Hkv, Sq, Skv, D, bound, scaling)
    "prefill": dict(B=1, Hq=32, Hkv=8, Sq=8192, Skv=8192, D=128, bound="tensor", scaling="weak",
                    name="llama3.1-8b-prefill-8k (config 2)"),
    "decode": dict(B=1, Hq=32, Hkv=8, Sq=1, Skv=16384, D=128, bound="hbm", scaling="weak",
                   name="split-kv-decode-16k (config 3)"),
    "chunked": dict(B=4, Hq=32, Hkv=8, Sq=512, Skv=16384, D=128, bound="tensor", scaling="strong",
                    name="chunked-prefill-b4-512x16k (config 4), batch x kv-head sharded"),
    "long_decode": dict(B=64, Hq=64, Hkv=8, Sq=1, Skv=131072, D=128, bound="hbm", scaling="strong",
                        name="long-decode-b64-131k (config 5), seq_kv sharded + NCCL LSE combine"),
    # Paged-cache decode (gqa_kernels.paged): config 3's shape for 8 sequences, vLLM
    # cache layout with 256-key blocks in shuffled order; bf16 or e4m3 K/V.
    "paged_decode": dict(B=8, Hq=32, Hkv=8, Sq=1, Skv=16384, D=128, bound="hbm", scaling="weak", kv="bf16",
                         name="paged-decode-8x16k (config 3 shape x 8 sequences, bf16 cache, block 256)"),
    "paged_decode_fp8": dict(B=8, Hq=32, Hkv=8, Sq=1, Skv=16384, D=128, bound="hbm", scaling="weak", kv="fp8",
                             name="paged-decode-fp8-8x16k (config 3 shape x 8 sequences, e4m3 cache, block 256)"),
}


def wl_bytes(wl):
    """Compulsory HBM bytes of one workload instance (K/V at the cache's element size)."""
    B, Hq, Hkv, Sq, Skv, D = wl["B"], wl["Hq"], wl["Hkv"], wl["Sq"], wl["Skv"], wl["D"]
    kv_elem = 1 if wl.get("kv") == "fp8" else 2
    return float(kv_elem * 2 * B * Hkv * Skv * D + 2 * 2 * B * Hq * Sq * D)


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return dict(hbm=p["hbm_gbs"], bf16=p["bf16_tflops"], bf16_sus=p.get("bf16_tflops_sustained"),
                    source="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sus=1400.0, source="fallback")


def profile_traffic(kernel_key):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary (profiles/*.md|txt), or None."""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for fn in sorted(os.listdir(pdir)):
        if not fn.endswith((".txt", ".md")):
            continue
        with open(os.path.join(pdir, fn)) as f:
            for line in f:
                if line.startswith(f"traffic_bytes_per_launch[{kernel_key}]:"):
                    try:
                        return float(line.split(":", 1)[1].split()[0])
                    except ValueError:
                        return None
    return None


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device):
        self.proc = None
        self.out = tempfile.NamedTemporaryFile(prefix="clocks_", suffix=".csv", delete=False)
        try:
            pr = torch.cuda.get_device_properties(device)
            self.target = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
        except Exception:
            self.target = str(device)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.target, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.close()
        rows = []
        with open(self.out.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) != 10:
                    continue
                try:
                    rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), util=float(parts[4]),
                                     reasons={n: parts[6 + i] for i, n in enumerate(self.REASONS)}))
                except ValueError:
                    continue
        os.unlink(self.out.name)
        if not rows:
            return None
        load = [r for r in rows if r["util"] >= 50] or rows
        reasons = sorted({n for r in load for n, v in r["reasons"].items() if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": max(r["smax"] for r in rows),
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(load)}


# ----------------------------------------------------------------------------- distributed plumbing
def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    elif n_gpus > 1:
        raise SystemExit("--gpus N > 1 needs torchrun (one process per GPU)")
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- timing
def timed_steps(step_fn, steps, warmup, world, device, flush=None, stream=None):
    """Runs warmup + steps; each timed step bracketed by CUDA events on `stream`.
    Returns (per-step ms list, wall ms of the whole timed loop)."""
    stream = stream or torch.cuda.current_stream(device)
    for _ in range(warmup):
        step_fn(0)
        if flush is not None:
            flush()
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    barrier(world)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for i in range(steps):
        if flush is not None:
            flush()
        torch.cuda._sleep(100000)  # ~50 us: gives the host a head start so the events bracket only the step
        pairs[i][0].record(stream)
        step_fn(i)
        pairs[i][1].record(stream)
    torch.cuda.synchronize(device)
    wall = (time.perf_counter() - t0) * 1e3
    barrier(world)
    return [a.elapsed_time(b) for a, b in pairs], wall


def timed_loop(run_steps, steps, warmup, world, device):
    """Runs warmup, then `steps` steps back to back (run_steps(n) issues n of them),
    bracketed by one pair of CUDA events with a barrier and synchronize on both
    sides. Returns ([total / K] * K, wall ms)."""
    stream = torch.cuda.current_stream(device)
    run_steps(warmup)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    a.record(stream)
    run_steps(steps)
    b.record(stream)
    torch.cuda.synchronize(device)
    wall = (time.perf_counter() - t0) * 1e3
    barrier(world)
    ms = a.elapsed_time(b)
    return [ms / steps] * steps, wall


def make_flush(device):
    buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)

    def flush():
        buf.fill_(1)
    return flush


# ----------------------------------------------------------------------------- attention arms
def make_attention(impl):
    """The attention call a step makes: this library (`ours`) or a same-box library
    comparator (`sdpa`: torch scaled_dot_product_attention; `flash_attn`: flash_attn's
    flash_attn_func), all with the reference's bottom-right causal rule."""
    if impl == "ours":
        from gqa_kernels import gqa_flash_attn
        return lambda q, k, v: gqa_flash_attn(q, k, v, causal=True)
    if impl == "sdpa":
        import torch.nn.functional as F
        masks = {}

        def sdpa(q, k, v):
            sq, skv = q.shape[2], k.shape[2]
            if sq == skv:
                return F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
            if sq == 1:  # the one query sees every key
                return F.scaled_dot_product_attention(q, k, v, enable_gqa=True)
            key = (sq, skv, q.device)
            if key not in masks:  # is_causal is top-left aligned: pass the bottom-right mask
                qpos = torch.arange(sq, device=q.device)[:, None] + (skv - sq)
                masks[key] = qpos >= torch.arange(skv, device=q.device)[None, :]
            return F.scaled_dot_product_attention(q, k, v, attn_mask=masks[key], enable_gqa=True)
        return sdpa
    if impl == "flash_attn":
        from flash_attn import flash_attn_func  # bottom-right causal, GQA by head count

        def fa(q, k, v):
            return flash_attn_func(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), causal=True).transpose(1, 2)
        return fa
    raise SystemExit(f"unknown impl {impl}")


# ----------------------------------------------------------------------------- our arm
def run_attention_workload(wl, world, rank, device, steps, warmup, args):
    from gqa_kernels import sharded as S
    attn = make_attention(args.impl)
    B, Hq, Hkv, Sq, Skv, D = wl["B"], wl["Hq"], wl["Hkv"], wl["Sq"], wl["Skv"], wl["D"]
    dt = torch.bfloat16
    gen = torch.Generator(device=device).manual_seed(rank)
    flops_total = attn_flops(B, Hq, Sq, Skv, D) * (world if wl["scaling"] == "weak" else 1)
    bytes_total = wl_bytes(wl) * (world if wl["scaling"] == "weak" else 1)

    def rnd(*shape):
        return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32).to(dt)

    name = args.workload
    local = {}
    if name == "prefill":
        local["q"], local["k"], local["v"] = rnd(B, Hq, Sq, D), rnd(B, Hkv, Skv, D), rnd(B, Hkv, Skv, D)

        def step(i):
            local["o"] = attn(local["q"], local["k"], local["v"])
        flush = make_flush(device)
        launches_per_step = 1
    elif name in ("decode", "paged_decode", "paged_decode_fp8"):
        # Dense decode: K+V (67 MB) fit in L2, so four input copies rotate (268 MB)
        # instead of a flush. Paged decode: two cache copies of 268 MB (bf16) or 134 MB
        # (e4m3) rotate. A serving loop replays its decode steps from CUDA graphs: here
        # graphs of up to 16 consecutive steps (cycling the copies), so consecutive
        # kernels overlap launch and prologue (programmatic dependent launch). Captured
        # after a warm-up on the capture stream, so the split workspace is cached and
        # none is allocated.
        if name == "decode":
            sets = [(rnd(B, Hq, Sq, D), rnd(B, Hkv, Skv, D), rnd(B, Hkv, Skv, D)) for _ in range(4)]

            def call(i):
                return attn(*sets[i % len(sets)])
            local["q"], local["k"], local["v"] = sets[0]
        else:
            if args.impl != "ours":
                raise SystemExit("the paged workloads run this library only")
            from gqa_kernels.paged import paged_decode
            bs, nb = 256, B * Skv // 256
            kv_dt = torch.float8_e4m3fn if wl["kv"] == "fp8" else dt
            sets = []
            for _ in range(2):
                bt = torch.randperm(nb, generator=gen, device=device).to(torch.int32).view(B, Skv // bs)
                sets.append((rnd(B, Hq, D), rnd(nb, bs, Hkv, D).to(kv_dt), rnd(nb, bs, Hkv, D).to(kv_dt), bt,
                             torch.full((B,), Skv, dtype=torch.int32, device=device)))

            def call(i):
                return paged_decode(*sets[i % len(sets)])
        gs = torch.cuda.Stream(device)
        gs.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(gs):
            for i in range(len(sets)):
                call(i)
        gs.synchronize()
        graphs = {}

        def graph_of(n):
            if n not in graphs:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.stream(gs), torch.cuda.graph(g, stream=gs):
                    for i in range(n):
                        local["o"] = call(i)
                graphs[n] = g
            return graphs[n]

        def step(n):  # runs n consecutive steps
            while n > 0:
                c = min(n, 16)
                graph_of(c).replay()
                n -= c
        flush = None
        launches_per_step = 1
    elif name == "chunked":
        br, hr = S.shard_units(B, Hkv, world, rank)
        g = Hq // Hkv
        nb, nh = br[1] - br[0], hr[1] - hr[0]
        q, k, v = rnd(nb, nh * g, Sq, D), rnd(nb, nh, Skv, D), rnd(nb, nh, Skv, D)

        def step(i):
            local["o"] = S.head_sharded_forward(q, k, v) if args.impl == "ours" else attn(q, k, v)
        flush = make_flush(device)
        launches_per_step = 1
    elif name == "long_decode":
        k0, k1 = S.kv_range(Skv, world, rank)
        q = torch.randn(B, Hq, Sq, D, generator=torch.Generator(device=device).manual_seed(0), device=device).to(dt)
        k, v = rnd(B, Hkv, k1 - k0, D), rnd(B, Hkv, k1 - k0, D)
        if world == 1:
            def step(i):
                local["o"] = attn(q, k, v)
            launches_per_step = 1
        elif args.impl != "ours":
            raise SystemExit("the library comparators run the seq_kv-sharded workload on one GPU only")
        else:
            packed = torch.empty(S.packed_size(q.shape), dtype=torch.float32, device=device)
            gathered = torch.empty((world, packed.numel()), dtype=torch.float32, device=device)

            def step(i):
                S.partial_forward(q, k, v, True, k0, Skv, out=packed)
                S.gather_partials(packed, out=gathered)
                local["o"] = S.combine_partials(gathered, tuple(q.shape), dt, device)
            launches_per_step = 2
        flush = None
    else:
        raise SystemExit(f"unknown workload {name}")

    clock = ClockSampler(device) if rank == 0 else None
    if clock:
        clock.start()
    if name in ("decode", "paged_decode", "paged_decode_fp8"):
        graph_of(16), graph_of(steps % 16 or 16)  # capture outside the timed region
        times, wall = timed_loop(step, steps, warmup, world, device)
    else:
        times, wall = timed_steps(step, steps, warmup, world, device, flush=flush)
    clocks = clock.stop() if clock else None
    mean_ms = statistics.mean(times)
    total_ms = max_over_ranks(sum(times), world, device)
    ms_step = total_ms / steps
    res = dict(ms_per_step=ms_step, mean_ms_rank0=mean_ms, median_ms_rank0=statistics.median(times),
               wall_ms=wall, clocks=clocks, launches=steps * launches_per_step,
               flops=flops_total, bytes=bytes_total, local=local)
    if wl["bound"] == "tensor":
        res["value"] = flops_total / (ms_step * 1e-3) / 1e12
        res["unit"] = "TFLOP/s"
    else:
        res["value"] = bytes_total / (ms_step * 1e-3) / 1e9
        res["unit"] = "GB/s"
    return res


def run_e2e(wl, world, rank, device, steps, args):
    """Same metric through the public API with pinned host buffers, as a serving loop
    runs it: every step copies its own q/k/v in (H2D), calls gqa_flash_attn and copies
    o back (D2H). Inputs are double-buffered: step i+1's H2D runs on a copy stream
    while step i computes, and step i's D2H on a third stream (PCIe is full duplex).
    The K timed steps sit between one pair of events (barrier and synchronize on both
    sides), all copies included."""
    from gqa_kernels import gqa_flash_attn
    B, Hq, Hkv, Sq, Skv, D = wl["B"], wl["Hq"], wl["Hkv"], wl["Sq"], wl["Skv"], wl["D"]
    if args.workload not in ("prefill", "decode"):
        return None
    g = torch.Generator().manual_seed(rank)

    def host(*shape):
        return torch.randn(*shape, generator=g).to(torch.bfloat16).pin_memory()
    hosts = [(host(B, Hq, Sq, D), host(B, Hkv, Skv, D), host(B, Hkv, Skv, D)) for _ in range(2)]
    outs = [torch.empty(B, Hq, Sq, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dev = [tuple(torch.empty(t.shape, dtype=t.dtype, device=device) for t in hs) for hs in hosts]
    comp = torch.cuda.current_stream(device)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in range(2)]    # inputs of buffer b landed
    ev_done = [torch.cuda.Event() for _ in range(2)]  # the step on buffer b finished computing

    def h2d(i):
        b = i % 2
        s_in.wait_event(ev_done[b])  # the step two back has finished reading buffer b
        with torch.cuda.stream(s_in):
            for d, h in zip(dev[b], hosts[b]):
                d.copy_(h, non_blocking=True)
        ev_in[b].record(s_in)

    def run_steps(n):
        if n <= 0:
            return
        h2d(0)
        for i in range(n):
            if i + 1 < n:
                h2d(i + 1)
            b = i % 2
            comp.wait_event(ev_in[b])
            o = gqa_flash_attn(*dev[b], causal=True)
            ev_done[b].record(comp)
            s_out.wait_event(ev_done[b])
            with torch.cuda.stream(s_out):
                outs[b].copy_(o, non_blocking=True)
            o.record_stream(s_out)
        comp.wait_stream(s_out)

    times, _ = timed_loop(run_steps, steps, 3, world, device)
    ms = max_over_ranks(sum(times), world, device) / steps
    # This box's pinned host<->device bandwidth (outside the timed region): the e2e
    # number is bound by it, and PCIe links differ between machines of a pool.
    link = {}
    for name, dst, src in (("h2d_gbs", dev[0][1], hosts[0][1]), ("d2h_gbs", outs[0], dev[0][0])):
        dst.copy_(src, non_blocking=True)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(device)
        a.record(comp)
        for _ in range(5):
            dst.copy_(src, non_blocking=True)
        b.record(comp)
        torch.cuda.synchronize(device)
        link[name] = round(5 * src.numel() * src.element_size() / (a.elapsed_time(b) * 1e-3) / 1e9, 1)
    mult = world if wl["scaling"] == "weak" else 1
    h2d_bytes = sum(t.numel() * t.element_size() for t in hosts[0])
    d2h_bytes = outs[0].numel() * outs[0].element_size()
    if wl["bound"] == "tensor":
        val, unit = attn_flops(B, Hq, Sq, Skv, D) * mult / (ms * 1e-3) / 1e12, "TFLOP/s"
    else:
        val, unit = attn_bytes(B, Hq, Hkv, Sq, Skv, D) * mult / (ms * 1e-3) / 1e9, "GB/s"
    return {"value": round(val, 3), "unit": unit, "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
            "pipeline": "inputs double-buffered: H2D of step i+1 and D2H of step i overlap step i",
            "link": link}


# ----------------------------------------------------------------------------- CPU baseline (oracle)
def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:
        return 1


def cpu_sample(wl, budget_s, steps=None):
    """Times the oracle port of tests/reference.py on blocks of query rows of the
    workload (one kv head's query heads at a time). Returns (value, unit, sample text, per-step s)."""
    from oracle import gqa_oracle as O
    B, Hq, Hkv, Sq, Skv, D = wl["B"], wl["Hq"], wl["Hkv"], wl["Sq"], wl["Skv"], wl["D"]
    G = Hq // Hkv
    rng = np.random.default_rng(0)
    rows = Sq if Sq <= 64 else 256  # query rows per sample step
    q = rng.standard_normal((1, G, Sq, D), dtype=np.float32)
    k = rng.standard_normal((1, 1, Skv, D), dtype=np.float32)
    v = rng.standard_normal((1, 1, Skv, D), dtype=np.float32)
    q, k, v = (O.bf16_round(x) for x in (q, k, v))
    done_flops = done_bytes = 0.0
    elapsed = 0.0
    n = 0
    per = []
    off = Skv - Sq
    kv_elem = 1 if wl.get("kv") == "fp8" else 2  # bytes per cached K/V element of the workload
    while (steps is None and (elapsed < budget_s or n == 0)) or (steps is not None and n < steps):
        r0 = (n * rows * 37) % max(1, Sq - rows + 1) if Sq > rows else 0
        r1 = min(Sq, r0 + rows)
        # rows r0..r1 of one (b, kv head): keys up to the last row's causal bound
        kend = min(Skv, r1 + off)
        t0 = time.perf_counter()
        O.gqa_reference(q[:, :, r0:r1], k[:, :, :kend], v[:, :, :kend], causal=True)
        dt = time.perf_counter() - t0
        per.append(dt)
        elapsed += dt
        pairs = int(np.clip(np.arange(r0, r1) + off + 1, 0, Skv).sum())
        done_flops += 4.0 * G * D * pairs
        done_bytes += kv_elem * 2 * kend * D + 2.0 * 2 * G * (r1 - r0) * D
        n += 1
    if wl["bound"] == "tensor":
        val, unit = done_flops / elapsed / 1e12, "TFLOP/s"
    else:
        val, unit = done_bytes / elapsed / 1e9, "GB/s"
    sample = (f"{n} step(s) of {rows} query rows x {G} query heads of one (batch, kv head) unit of the "
              f"workload, fp32 numpy oracle; {elapsed:.2f} s")
    return val, unit, sample, per


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference", "sdpa", "flash_attn"], default="ours",
                    help="reference: the reference's CPU path; sdpa / flash_attn: same-box library comparators")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="prefill")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode half of the default line")
    ap.add_argument("--decode-steps", type=int, default=5000, help="timed steps of the decode half")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    wl = WORKLOADS[args.workload]
    default_steps = {"prefill": 1000, "decode": 5000, "chunked": 500, "long_decode": 100, "paged_decode": 2000,
                     "paged_decode_fp8": 2000}[args.workload]
    steps = args.steps or default_steps

    if args.impl == "reference":
        return main_reference(args, wl, steps)

    comparator = args.impl in ("sdpa", "flash_attn")
    if comparator:
        try:
            make_attention(args.impl)
        except Exception as e:  # the comparator library is absent or cannot load here
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": args.impl, "unavailable": f"{type(e).__name__}: {e}"[:300]}), flush=True)
            return
        args.no_e2e = args.no_cpu = True
    world, rank, local = dist_setup(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    import gqa_kernels._lib as L
    L.load()
    peaks = measured_peaks()

    res = run_attention_workload(wl, world, rank, device, steps, args.warmup, args)
    line = {
        "metric": METRIC if args.workload in ("prefill", "decode") else f"{args.workload} {res['unit']}",
        "value": round(res["value"], 3),
        "unit": res["unit"],
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(res["ms_per_step"], 5),
        "higher_is_better": True,
        "scaling": wl["scaling"],
        "vs_baseline": None,
        "dtype": "e4m3 K/V, f16 MMA, bf16 Q/O" if wl.get("kv") == "fp8" else "bf16",
        "data": "synthetic (N(0,1) bf16, CUDA generator seeded by rank)",
        "config": {"workload": wl["name"], "batch_per_gpu" if wl["scaling"] == "weak" else "batch": wl["B"],
                   "num_heads": wl["Hq"], "num_kv_heads": wl["Hkv"], "seq_q": wl["Sq"], "seq_kv": wl["Skv"],
                   "head_dim": wl["D"], "causal": True,
                   "l2": "flushed between steps (256 MB write)" if args.workload in ("prefill", "chunked")
                   else "inputs larger than L2 (4 rotating copies, 268 MB); 16-step CUDA graphs back to back"
                   if args.workload == "decode"
                   else "inputs larger than L2 (2 rotating caches); 16-step CUDA graphs back to back"
                   if args.workload.startswith("paged")
                   else "inputs larger than L2 (32 GiB K/V)",
                   "parallelism": (f"batch-sharded x{world}" if wl["scaling"] == "weak" else
                                   f"kv-head/batch x{world}" if args.workload == "chunked" else
                                   f"seq_kv x{world} + NCCL all-gather LSE combine")},
        "gpu_launches": 0 if comparator else res["launches"],
    }
    # roofline of the dominant kernel, from rank 0's mean per-launch event time. Per-rank
    # work: one workload instance (weak scaling) or 1/world of it (strong scaling).
    launch_ms = res["mean_ms_rank0"]
    share = 1.0 if wl["scaling"] == "weak" else 1.0 / world
    if wl["bound"] == "tensor":
        work = attn_flops(wl["B"], wl["Hq"], wl["Sq"], wl["Skv"], wl["D"]) * share
        achieved = work / (launch_ms * 1e-3) / 1e12
        line["roofline"] = {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16"],
                            "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16"], 4),
                            "frac_of_sustained": (round(achieved / peaks["bf16_sus"], 4)
                                                  if peaks["bf16_sus"] else None),
                            "peak_source": f"{peaks['source']} bf16 dense burst (MEASURED_PEAKS.json)",
                            "work_per_launch": work, "traffic": profile_traffic(args.workload)}
    else:
        work = wl_bytes(wl) * share
        achieved = work / (launch_ms * 1e-3) / 1e9
        line["roofline"] = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm"], "unit": "GB/s",
                            "frac": round(achieved / peaks["hbm"], 4),
                            "peak_source": f"{peaks['source']} HBM copy (MEASURED_PEAKS.json)",
                            "work_per_launch": work, "traffic": profile_traffic(args.workload)}
    line["clocks"] = res["clocks"]

    # decode half of the headline metric
    if args.workload == "prefill" and not args.no_decode:
        dwl = WORKLOADS["decode"]
        dargs = argparse.Namespace(**{**vars(args), "workload": "decode"})
        dres = run_attention_workload(dwl, world, rank, device, args.decode_steps, args.warmup, dargs)
        dl_ms = dres["mean_ms_rank0"]
        dbytes = attn_bytes(1, 32, 8, 1, 16384, 128)
        line["decode_16k"] = {"value": round(dres["value"], 1), "unit": "GB/s",
                              "us_per_step": round(dres["ms_per_step"] * 1e3, 2),
                              "steps": args.decode_steps, "scaling": "weak",
                              "timing": "CUDA graphs of 16 steps replayed back to back between one "
                                        "event pair; 4 rotating input copies (268 MB > L2)",
                              "roofline": {"bound": "hbm", "achieved": round(dbytes / (dl_ms * 1e-3) / 1e9, 1),
                                           "peak": peaks["hbm"], "unit": "GB/s",
                                           "frac": round(dbytes / (dl_ms * 1e-3) / 1e9 / peaks["hbm"], 4),
                                           "traffic": profile_traffic("decode")},
                              "clocks": dres["clocks"]}
        line["gpu_launches"] += 0 if comparator else dres["launches"]

    if not args.no_e2e:
        e2e = run_e2e(wl, world, rank, device, 20 if args.workload == "prefill" else 200, args)
        if e2e is not None:
            line["e2e"] = e2e

    if rank == 0 and world == 1 and not args.no_cpu:
        val, unit, sample, _ = cpu_sample(wl, budget_s=12.0)
        line["cpu_baseline"] = {"value": round(val, 5), "unit": unit, "cores": cpu_threads(), "kind": "port",
                                "sample": sample}

    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    if comparator:
        line["impl"] = args.impl  # library kernels on the same box: context, not this library
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main_reference(args, wl, steps):
    """The reference arm: the reference's CPU path (numpy port of tests/reference.py)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    # each step is one block of query rows; run as many of the requested warmup + steps
    # as fit in about two minutes (at least 3)
    _, _, _, per = cpu_sample(wl, budget_s=0.0, steps=1)
    total = steps + args.warmup
    n_run = max(3, min(total, int(120.0 / max(per[0], 1e-3))))
    val, unit, sample, per = cpu_sample(wl, budget_s=0.0, steps=n_run)
    ms_step = statistics.mean(per) * 1e3
    line = {
        "metric": METRIC if args.workload in ("prefill", "decode") else f"{args.workload} {unit}",
        "value": round(val, 6), "unit": unit, "impl": "reference", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True,
        "scaling": wl["scaling"], "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl["name"], "num_heads": wl["Hq"], "num_kv_heads": wl["Hkv"], "seq_q": wl["Sq"],
                   "seq_kv": wl["Skv"], "head_dim": wl["D"], "causal": True},
        "cpu_baseline": {"value": round(val, 6), "unit": unit, "cores": cpu_threads(), "kind": "port",
                         "sample": sample + f"; {n_run} of {total} requested steps run (bounded)"},
        "e2e": {"value": round(val, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
