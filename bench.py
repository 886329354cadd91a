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
                        name="long-decode-b64-131k (config 5), seq_kv sharded + LSE combine"),
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


# ----------------------------------------------------------------------------- in-run parity
CHECK_TOL = (2e-2, 2e-3)  # BASELINE contract: max-abs 2e-2, mean-abs 2e-3 against fp32


def check_rows_sel(q_shape, n, seed=1234):
    """n seeded (batch, head, position) rows of an output of shape (B, Hq, Sq, D)."""
    B, Hq, Sq, _ = q_shape
    g = torch.Generator().manual_seed(seed)
    return [tuple(int(torch.randint(hi, (1,), generator=g)) for hi in (B, Hq, Sq)) for _ in range(n)]


@torch.no_grad()
def fp32_row_partials(q, k, v, sel, causal=True, kv_offset=0, seq_kv_total=None):
    """Softmax statistics of the output rows `sel` over the keys k/v hold (global key
    positions kv_offset + j of seq_kv_total), in fp32 with plain torch ops on the tensors'
    device (tests/reference.py's math: scores * head_dim^-0.5, bottom-right causal mask,
    softmax, @ V; TF32 off). Returns an (n, 2 + D) float64 tensor of rows [m | l | acc]:
    m the row max of the scores, l = sum exp(s - m), acc = sum exp(s - m) v; a row that
    sees none of these keys gets (-inf, 0, 0)."""
    B, Hq, Sq, D = q.shape
    Hkv, n = k.shape[1], k.shape[2]
    G = Hq // Hkv
    total = n if seq_kv_total is None else seq_kv_total
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        out = torch.zeros(len(sel), 2 + D, dtype=torch.float64, device=q.device)
        pos = torch.arange(n, device=q.device)
        for r, (b, h, i) in enumerate(sel):
            s = (k[b, h // G].float() @ q[b, h, i].float()) * D ** -0.5
            if causal:
                s = s.masked_fill(pos > i + total - Sq - kv_offset, float("-inf"))
            m = s.max() if n else torch.tensor(float("-inf"), device=q.device)
            if not torch.isfinite(m):
                out[r, 0] = float("-inf")
                continue
            p = torch.exp(s - m)
            out[r, 0], out[r, 1] = m.double(), p.sum().double()
            out[r, 2:] = (p @ v[b, h // G].float()).double()
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def parity_check(local, world, n_rows=16, sharded_keys=False):
    """Checks n_rows seeded output rows of this rank against an fp32 torch evaluation of
    the same rows. With sharded_keys, every rank holds a key range of every row: the
    ranks' fp32 row statistics are all-gathered and combined (log-sum-exp) before the
    comparison. The verdict is all-reduced (every rank must pass)."""
    q, k, v, o = local["q"], local["k"], local["v"], local["o"]
    sel = check_rows_sel(q.shape, n_rows)
    part = fp32_row_partials(q, k, v, sel, True, local.get("kv_offset", 0), local.get("seq_kv_total"))
    if sharded_keys and world > 1:
        import torch.distributed as dist
        gathered = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(gathered, part)
        parts = torch.stack(gathered)
    else:
        parts = part[None]
    m = parts[:, :, 0]
    M = m.max(0).values
    w = torch.where(torch.isinf(m), torch.zeros_like(m), torch.exp(m - M))
    ref = (w[:, :, None] * parts[:, :, 2:]).sum(0) / (w * parts[:, :, 1]).sum(0)[:, None]
    got = torch.stack([o[b, h, i].double() for b, h, i in sel])
    nan_ok = bool(torch.equal(torch.isnan(ref), torch.isnan(got)))
    fin = ~torch.isnan(ref)
    d = (got[fin] - ref[fin]).abs()
    mx = float(d.max()) if d.numel() else 0.0
    mn = float(d.mean()) if d.numel() else 0.0
    ok = nan_ok and mx < CHECK_TOL[0] and mn < CHECK_TOL[1]
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([0.0 if ok else 1.0, mx, mn], dtype=torch.float64, device=q.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ok, mx, mn = t[0].item() == 0.0, t[1].item(), t[2].item()
    return {"ok": bool(ok), "rows_per_rank": len(sel), "max_abs": round(mx, 6), "mean_abs": round(mn, 7),
            "tol": list(CHECK_TOL), "against": "fp32 torch rows (reference math), all ranks"
            + ("; key shards combined by log-sum-exp" if sharded_keys and world > 1 else "")}


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


# ----------------------------------------------------------------------------- harness parity (benchmark/run.py)
SWEEP_PREFILL = (2048, 4096, 6144, 8192, 12288, 16384)  # benchmark/run.py:44-46
SWEEP_DECODE = (2048, 4096, 8192, 16384)
GATE_LENS = (512, 2048, 4096)
GATE_TOL = (1e-2, 1e-3)  # the reference harness's gate: inputs N(0,1) * 0.1, max/mean abs


@torch.no_grad()
def fp32_attention(q, k, v):
    """Bottom-right causal GQA attention in fp32 torch ops on the GPU (TF32 off), per kv
    head so the scores stay bounded: the reference's oracle math, as a checker."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        B, Hq, Sq, D = q.shape
        Hkv, Skv = k.shape[1], k.shape[2]
        G = Hq // Hkv
        out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
        mask = (torch.arange(Sq, device=q.device)[:, None] + (Skv - Sq)) < torch.arange(Skv, device=q.device)[None]
        for b in range(B):
            for h in range(Hkv):
                s = q[b, h * G:(h + 1) * G].float() @ k[b, h].float().T * D ** -0.5
                out[b, h * G:(h + 1) * G] = torch.softmax(s.masked_fill(mask, float("-inf")), -1) @ v[b, h].float()
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def harness_impls():
    """The harness's kernels: this library, SDPA (K/V expanded over the group outside the
    timing, is_causal only when seq_q == seq_kv: SDPA's causal mask is top-left aligned,
    the reference harness's decode trap), and flash_attn when it loads here."""
    import torch.nn.functional as F
    from gqa_kernels import gqa_flash_attn
    impls = {"ours": (lambda q, k, v: (q, k, v), lambda q, k, v: gqa_flash_attn(q, k, v, causal=True))}

    def sdpa_prep(q, k, v):
        g = q.shape[1] // k.shape[1]
        return q, k.repeat_interleave(g, 1), v.repeat_interleave(g, 1)
    impls["sdpa"] = (sdpa_prep, lambda q, k, v: F.scaled_dot_product_attention(q, k, v,
                                                                               is_causal=q.shape[2] == k.shape[2]))
    try:
        from flash_attn import flash_attn_func
        impls["fa2"] = (lambda q, k, v: tuple(t.transpose(1, 2).contiguous() for t in (q, k, v)),
                        lambda q, k, v: flash_attn_func(q, k, v, causal=True))
    except Exception:
        pass
    return impls


def _to_bhsd(name, o):
    return o.transpose(1, 2) if name == "fa2" else o


def correctness_gate(device, impls, lens=GATE_LENS, log=sys.stderr):
    """benchmark/run.py:96-137 on this box: every kernel against fp32 attention at the
    gate lengths, prefill (S x S) and decode (1 x S), B=1, Hq=32, Hkv=8, D=128, bf16
    inputs N(0,1) * 0.1. Returns (all ok, rows)."""
    print(f"[correctness] gate: max_abs < {GATE_TOL[0]:g}, mean_abs < {GATE_TOL[1]:g}", file=log)
    g = torch.Generator(device=device).manual_seed(0)
    rows, all_ok = [], True
    for sq, sk, label in [(L, L, "prefill") for L in lens] + [(1, L, "decode") for L in lens]:
        q = (torch.randn(1, 32, sq, 128, generator=g, device=device) * 0.1).to(torch.bfloat16)
        k = (torch.randn(1, 8, sk, 128, generator=g, device=device) * 0.1).to(torch.bfloat16)
        v = (torch.randn(1, 8, sk, 128, generator=g, device=device) * 0.1).to(torch.bfloat16)
        ref = fp32_attention(q, k, v)
        for name, (prep, fn) in impls.items():
            out = _to_bhsd(name, fn(*prep(q, k, v))).float()
            d = (out - ref).abs()
            mx, mn = d.max().item(), d.mean().item()
            ok = mx < GATE_TOL[0] and mn < GATE_TOL[1]
            all_ok &= ok
            rows.append({"workload": label, "seq_kv": sk, "impl": name, "max_abs": mx, "mean_abs": mn, "ok": ok})
            print(f"[correctness] {label:<7} L={sk:>5d}  {name:>4}: max={mx:.2e} mean={mn:.2e}  "
                  f"{'ok' if ok else 'FAIL'}", file=log)
    return all_ok, rows


def _commit():
    try:
        return subprocess.check_output(["git", "rev-parse", "--short=7", "HEAD"], cwd=ROOT,
                                       stderr=subprocess.DEVNULL).decode().strip()
    except Exception:
        return "nogit00"


def run_sweep(device, trials=1, quick=False, warmup=25, iters=100, log=sys.stderr):
    """benchmark/run.py's sweep on this box: the gate, then per length the three kernels
    timed with CUDA events (warmup, then iters back to back), inputs pre-converted to each
    kernel's layout outside the timing. Returns the results document in run.py's schema
    (commit, device, dtype, trials, config, rows) plus rates, roofline fractions, GPU and
    host-core counts."""
    impls = harness_impls()
    ok, gate = correctness_gate(device, impls, log=log)
    peaks = measured_peaks()
    prefill, decode = ((8192,), (8192,)) if quick else (SWEEP_PREFILL, SWEEP_DECODE)
    per_trial = []
    for _ in range(trials):
        rows = []
        for workload, lens in (("prefill", prefill), ("decode", decode)):
            for L in lens:
                sq = L if workload == "prefill" else 1
                g = torch.Generator(device=device).manual_seed(L)
                q = (torch.randn(1, 32, sq, 128, generator=g, device=device) * 0.1).to(torch.bfloat16)
                k = (torch.randn(1, 8, L, 128, generator=g, device=device) * 0.1).to(torch.bfloat16)
                v = (torch.randn(1, 8, L, 128, generator=g, device=device) * 0.1).to(torch.bfloat16)
                ms = {}
                for name, (prep, fn) in impls.items():
                    args = prep(q, k, v)
                    for _ in range(warmup):
                        fn(*args)
                    torch.cuda.synchronize(device)
                    torch.cuda.reset_peak_memory_stats(device)
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    for _ in range(iters):
                        fn(*args)
                    b.record()
                    torch.cuda.synchronize(device)
                    ms[name] = (a.elapsed_time(b) / iters, torch.cuda.max_memory_allocated(device) / 2 ** 30)
                ours = ms["ours"][0]
                fa2 = ms["fa2"][0] if "fa2" in ms else float("nan")
                row = {"workload": workload, "seq_kv": L, "ours_ms": ours, "fa2_ms": fa2, "sdpa_ms": ms["sdpa"][0],
                       "tok_s": sq * 1000.0 / ours, "speedup_vs_fa2": fa2 / ours,
                       "speedup_vs_sdpa": ms["sdpa"][0] / ours, "peak_mem_gb": ms["ours"][1]}
                if workload == "prefill":
                    row["tflops"] = attn_flops(1, 32, sq, L, 128) / (ours * 1e-3) / 1e12
                    row["roofline_frac"] = row["tflops"] / peaks["bf16"]
                else:
                    row["gbs"] = attn_bytes(1, 32, 8, 1, L, 128) / (ours * 1e-3) / 1e9
                    row["roofline_frac"] = row["gbs"] / peaks["hbm"]
                rows.append(row)
                print(f"[{workload}] L={L:>5d}  ours={ours:7.3f}ms  fa2={fa2:7.3f}ms  sdpa={ms['sdpa'][0]:7.3f}ms  "
                      f"vs_fa2={row['speedup_vs_fa2']:.2f}x  vs_sdpa={row['speedup_vs_sdpa']:.2f}x", file=log)
        per_trial.append(rows)
    return sweep_document(aggregate_median(per_trial), ok, gate, trials, torch.cuda.get_device_name(device),
                          "fa2" in impls, peaks)


def aggregate_median(per_trial):
    """Median over trials of each (workload, seq_kv) row (benchmark/run.py:195-214)."""
    rows = [dict(r) for r in per_trial[0]]
    if len(per_trial) > 1:
        for i, r in enumerate(rows):
            for key in ("ours_ms", "fa2_ms", "sdpa_ms", "peak_mem_gb"):
                r[key] = statistics.median(t[i][key] for t in per_trial)
            sq = r["seq_kv"] if r["workload"] == "prefill" else 1
            r["tok_s"] = sq * 1000.0 / r["ours_ms"]
            r["speedup_vs_fa2"], r["speedup_vs_sdpa"] = r["fa2_ms"] / r["ours_ms"], r["sdpa_ms"] / r["ours_ms"]
            if "tflops" in r:
                r["tflops"] = attn_flops(1, 32, sq, r["seq_kv"], 128) / (r["ours_ms"] * 1e-3) / 1e12
            if "gbs" in r:
                r["gbs"] = attn_bytes(1, 32, 8, 1, r["seq_kv"], 128) / (r["ours_ms"] * 1e-3) / 1e9
    return rows


def sweep_document(rows, gate_ok, gate_rows, trials, device_name, have_fa2, peaks):
    """The results JSON: benchmark/run.py's schema (commit, device, dtype, trials, config,
    rows; :265-278) plus the environment, GPU and host-core counts, peaks and the gate."""
    return {"commit": _commit(), "device": device_name, "dtype": str(torch.bfloat16), "trials": trials,
            "config": {"batch": 1, "num_heads": 32, "num_kv_heads": 8, "head_dim": 128,
                       "model": "Llama 3.1 8B attention shape"},
            "env": {"torch": torch.__version__,
                    "flash_attn2": "flash_attn.flash_attn_func" if have_fa2 else "unavailable",
                    "sdpa": "F.scaled_dot_product_attention with pre-expanded K/V"},
            "n_gpus": 1, "host_cores": host_cores(),
            "peaks": {"bf16_tflops": peaks["bf16"], "hbm_gbs": peaks["hbm"], "source": peaks["source"]},
            "gate": {"ok": gate_ok, "tol": list(GATE_TOL), "rows": gate_rows}, "rows": rows}


def markdown_table(doc):
    lines = ["| Workload | seq_kv | ours (ms) | FA2 (ms) | SDPA (ms) | vs FA2 | vs SDPA | roofline | mem (GB) |",
             "|---|---|---|---|---|---|---|---|---|"]
    for r in doc["rows"]:
        lines.append(f"| {r['workload']} | {r['seq_kv']} | {r['ours_ms']:.3f} | {r['fa2_ms']:.3f} | "
                     f"{r['sdpa_ms']:.3f} | {r['speedup_vs_fa2']:.2f}x | {r['speedup_vs_sdpa']:.2f}x | "
                     f"{r['roofline_frac']:.3f} | {r['peak_mem_gb']:.2f} |")
    return "\n".join(lines)


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

        local.update(q=q, k=k, v=v)

        def step(i):
            local["o"] = S.head_sharded_forward(q, k, v) if args.impl == "ours" else attn(q, k, v)
        flush = make_flush(device)
        launches_per_step = 1
    elif name == "long_decode":
        k0, k1 = S.kv_range(Skv, world, rank)
        # q is replicated (seed 0 on every rank); each rank draws its own key shard, one
        # batch element at a time so the fp32 draw stays small (32 GiB of K/V at N=1)
        q = torch.randn(B, Hq, Sq, D, generator=torch.Generator(device=device).manual_seed(0), device=device).to(dt)
        k = torch.empty(B, Hkv, k1 - k0, D, dtype=dt, device=device)
        v = torch.empty(B, Hkv, k1 - k0, D, dtype=dt, device=device)
        for bb in range(B):
            k[bb], v[bb] = rnd(Hkv, k1 - k0, D), rnd(Hkv, k1 - k0, D)
        local.update(q=q, k=k, v=v, kv_offset=k0, seq_kv_total=Skv)
        if world == 1:
            def step(i):
                local["o"] = attn(q, k, v)
            launches_per_step = 1
        elif args.impl != "ours":
            raise SystemExit("the library comparators run the seq_kv-sharded workload on one GPU only")
        else:
            if args.exchange == "peer" and S.all_shards_hold_keys(Skv, world):
                # the partial kernel stores its rows into every rank's buffer over
                # NVLink; each rank's combine waits for them in the kernel
                ex = S.PeerExchange(q.shape, Hkv, device)
                o_buf = torch.empty_like(q)
                local["exchange"] = ex

                def step(i):
                    local["o"] = ex.forward(q, k, v, k0, Skv, out=o_buf)
                launches_per_step = 3
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
    elif name == "long_decode":
        # K/V far larger than L2 at every N (4.3 GB per rank at N = 8), so no flush:
        # the steps run back to back as a decode loop issues them, between one
        # barrier-and-synchronize pair, and each rank's host jitter is not inside
        # every step's all-gather
        def run_steps(n):
            for i in range(n):
                step(i)
        times, wall = timed_loop(run_steps, steps, warmup, world, device)
    else:
        times, wall = timed_steps(step, steps, warmup, world, device, flush=flush)
    clocks = clock.stop() if clock else None
    if name == "decode":  # the checked output: one eager step on the first input copy
        local["q"], local["k"], local["v"] = sets[0]
        local["o"] = call(0)
    elif name.startswith("paged"):
        local.clear()  # paged outputs are checked by the GPU test suite, not in the bench
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


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def _sample_blocks(wl, rows):
    """Row blocks of one (batch, kv head) unit for the CPU samples: (r0, r1, kend) with
    the key prefix up to the block's last causal bound (keeps the bottom-right offset)."""
    Sq, Skv = wl["Sq"], wl["Skv"]
    off = Skv - Sq
    n = 0
    while True:
        r0 = (n * rows * 37) % max(1, Sq - rows + 1) if Sq > rows else 0
        r1 = min(Sq, r0 + rows)
        yield r0, r1, min(Skv, r1 + off)
        n += 1


def _sample_work(wl, G, r0, r1, kend):
    D, Skv = wl["D"], wl["Skv"]
    pairs = int(np.clip(np.arange(r0, r1) + (Skv - wl["Sq"]) + 1, 0, Skv).sum())
    kv_elem = 1 if wl.get("kv") == "fp8" else 2  # bytes per cached K/V element of the workload
    return 4.0 * G * D * pairs, kv_elem * 2 * kend * D + 2.0 * 2 * G * (r1 - r0) * D


def cpu_sample(wl, budget_s, steps=None, kind="torch"):
    """Times the reference's CPU attention on blocks of query rows of the workload (one kv
    head's query heads at a time). kind "torch": the torch restatement of
    tests/reference.py (the reference's own torch operations, fp32, every host core);
    kind "numpy": the numpy port. Returns (value, unit, sample text, per-step s)."""
    B, Hq, Hkv, Sq, Skv, D = wl["B"], wl["Hq"], wl["Hkv"], wl["Sq"], wl["Skv"], wl["D"]
    G = Hq // Hkv
    rng = np.random.default_rng(0)
    rows = Sq if Sq <= 64 else 256  # query rows per sample step
    from oracle import gqa_oracle as O
    q = rng.standard_normal((1, G, Sq, D), dtype=np.float32)
    k = rng.standard_normal((1, 1, Skv, D), dtype=np.float32)
    v = rng.standard_normal((1, 1, Skv, D), dtype=np.float32)
    q, k, v = (O.bf16_round(x) for x in (q, k, v))
    if kind == "torch":
        from oracle import gqa_oracle_torch as T
        torch.set_num_threads(host_cores())
        qt, kt, vt = (torch.from_numpy(x) for x in (q, k, v))

        def run(r0, r1, kend):
            T.gqa_reference(qt[:, :, r0:r1], kt[:, :, :kend], vt[:, :, :kend], causal=True)
        what, cores = f"torch {torch.__version__} fp32 restatement of tests/reference.py", torch.get_num_threads()
    else:
        def run(r0, r1, kend):
            O.gqa_reference(q[:, :, r0:r1], k[:, :, :kend], v[:, :, :kend], causal=True)
        what, cores = "fp32 numpy port of tests/reference.py", cpu_threads()
    done_flops = done_bytes = elapsed = 0.0
    per = []
    blocks = _sample_blocks(wl, rows)
    while (steps is None and (elapsed < budget_s or not per)) or (steps is not None and len(per) < steps):
        r0, r1, kend = next(blocks)
        t0 = time.perf_counter()
        run(r0, r1, kend)
        dt = time.perf_counter() - t0
        per.append(dt)
        elapsed += dt
        fl, by = _sample_work(wl, G, r0, r1, kend)
        done_flops += fl
        done_bytes += by
    if wl["bound"] == "tensor":
        val, unit = done_flops / elapsed / 1e12, "TFLOP/s"
    else:
        val, unit = done_bytes / elapsed / 1e9, "GB/s"
    sample = (f"{len(per)} step(s) of {rows} query rows x {G} query heads of one (batch, kv head) unit of the "
              f"workload, {what}, {cores} threads; {elapsed:.2f} s")
    return val, unit, sample, per, cores


def config_of(wl, world, workload, exchange="nccl"):
    """The `config` of a bench line; the reference arm prints the same dict."""
    return {"workload": wl["name"], "batch_per_gpu" if wl["scaling"] == "weak" else "batch": wl["B"],
            "num_heads": wl["Hq"], "num_kv_heads": wl["Hkv"], "seq_q": wl["Sq"], "seq_kv": wl["Skv"],
            "head_dim": wl["D"], "causal": True,
            "l2": "flushed between steps (256 MB write)" if workload in ("prefill", "chunked")
            else "inputs larger than L2 (4 rotating copies, 268 MB); 16-step CUDA graphs back to back"
            if workload == "decode"
            else "inputs larger than L2 (2 rotating caches); 16-step CUDA graphs back to back"
            if workload.startswith("paged")
            else "inputs larger than L2 (32 GiB K/V)",
            "parallelism": (f"batch-sharded x{world}" if wl["scaling"] == "weak" else
                            f"kv-head/batch x{world}" if workload == "chunked" else
                            f"seq_kv x{world} + " + ("peer-exchange LSE combine (partials stored over NVLink by the "
                                                     "partial kernel, in-kernel waits in the combine)"
                                                     if exchange == "peer" else "NCCL all-gather LSE combine"))}


def roofline_of(wl, res, world, peaks, workload):
    """Roofline of the dominant kernel from rank 0's mean per-step event time. Per-rank
    work: one workload instance (weak scaling) or 1/world of it (strong scaling)."""
    launch_ms = res["mean_ms_rank0"]
    share = 1.0 if wl["scaling"] == "weak" else 1.0 / world
    if wl["bound"] == "tensor":
        work = attn_flops(wl["B"], wl["Hq"], wl["Sq"], wl["Skv"], wl["D"]) * share
        achieved = work / (launch_ms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16"], "unit": "TFLOP/s",
                "frac": round(achieved / peaks["bf16"], 4),
                "frac_of_sustained": round(achieved / peaks["bf16_sus"], 4) if peaks["bf16_sus"] else None,
                "peak_source": f"{peaks['source']} bf16 dense burst (MEASURED_PEAKS.json)",
                "work_per_launch": work, "traffic": profile_traffic(workload)}
    work = wl_bytes(wl) * share
    achieved = work / (launch_ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm"], 4),
            "peak_source": f"{peaks['source']} HBM copy (MEASURED_PEAKS.json)",
            "work_per_launch": work, "traffic": profile_traffic(workload)}


def sharded_object(key, args, world, rank, device, peaks, comparator):
    """One of the sharded configurations of the default line (config 4 or 5) at this N:
    timed like its standalone workload, then checked row by row."""
    wname, nsteps = {"chunked_b4": ("chunked", args.chunked_steps),
                     "long_decode": ("long_decode", args.long_steps)}[key]
    swl = WORKLOADS[wname]
    sargs = argparse.Namespace(**{**vars(args), "workload": wname})
    res = run_attention_workload(swl, world, rank, device, nsteps, args.warmup, sargs)
    par = parity_check(res["local"], world, sharded_keys=(wname == "long_decode"))
    ex = res["local"].pop("exchange", None)
    exchange = "peer" if ex is not None else "nccl"
    if ex is not None:
        ex.close()  # collective: every rank reaches it after the same steps
    res["local"].clear()
    torch.cuda.empty_cache()
    peak = peaks["bf16"] if swl["bound"] == "tensor" else peaks["hbm"]
    obj = {"value": round(res["value"], 3), "unit": res["unit"], "ms_per_step": round(res["ms_per_step"], 5),
           "steps": nsteps, "scaling": swl["scaling"], "n_gpus": world,
           "frac_of_n_peak": round(res["value"] / (world * peak), 4),
           "config": config_of(swl, world, wname, exchange if world > 1 else "nccl"),
           "roofline": roofline_of(swl, res, world, peaks, wname),
           "parity": par, "clocks": res["clocks"]}
    if world > 1:
        import torch.distributed as dist
        obj["nccl"] = {"backend": dist.get_backend(), "ranks": dist.get_world_size(),
                       "collectives_per_step": 1 if (wname == "long_decode" and exchange == "nccl") else 0}
        if wname == "long_decode":
            obj["exchange"] = exchange
    return obj, (0 if comparator else res["launches"])


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
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the sharded configurations (4 and 5) of the default line")
    ap.add_argument("--decode-steps", type=int, default=5000, help="timed steps of the decode half")
    ap.add_argument("--chunked-steps", type=int, default=200, help="timed steps of the config-4 object")
    ap.add_argument("--long-steps", type=int, default=40, help="timed steps of the config-5 object")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="config 5 at N>1: partials stored over NVLink by the kernels, or one NCCL all-gather")
    ap.add_argument("--sweep", action="store_true",
                    help="the reference harness on this box (benchmark/run.py): correctness gate of this library, "
                         "SDPA and flash_attn, then the prefill/decode sweep; prints a table, writes --results")
    ap.add_argument("--trials", type=int, default=1, help="--sweep: median over this many trials")
    ap.add_argument("--quick", action="store_true", help="--sweep: the gate and 8K only")
    ap.add_argument("--results", default=None, help="--sweep: write the results JSON here")
    args = ap.parse_args()
    if args.sweep:
        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
        doc = run_sweep(device, trials=args.trials, quick=args.quick)
        if args.results:
            with open(args.results, "w") as f:
                json.dump(doc, f, indent=2)
        print(markdown_table(doc))
        sys.exit(0 if doc["gate"]["ok"] else 1)
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
    gate = None
    if comparator and rank == 0:  # the reference harness's gate before any timing (on stderr)
        dev0 = torch.device("cuda", local)
        torch.cuda.set_device(dev0)
        impls = harness_impls()
        gok, grows = correctness_gate(dev0, {k: impls[k] for k in ("ours", "fa2" if args.impl == "flash_attn"
                                                                       else "sdpa") if k in impls})
        gate = {"ok": gok, "tol": list(GATE_TOL), "cases": len(grows)}
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
        "config": config_of(wl, world, args.workload),
        "gpu_launches": 0 if comparator else res["launches"],
    }
    line["roofline"] = roofline_of(wl, res, world, peaks, args.workload)
    line["clocks"] = res["clocks"]
    if res["local"]:
        line["parity"] = parity_check(res["local"], world, sharded_keys=(args.workload == "long_decode"))
    ex = res["local"].pop("exchange", None)
    if ex is not None:
        line["config"] = config_of(wl, world, args.workload, "peer")
        ex.close()  # collective: every rank reaches it after the same steps
    res["local"].clear()

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
                              "parity": parity_check(dres["local"], world),
                              "clocks": dres["clocks"]}
        dres["local"].clear()
        line["gpu_launches"] += 0 if comparator else dres["launches"]

    # the sharded configurations (BASELINE configs 4 and 5), strong-scaled over the N ranks
    if args.workload == "prefill" and not args.no_sharded:
        for key in ("chunked_b4", "long_decode"):
            if comparator and key == "long_decode" and world > 1:
                continue  # the library comparators have no key-sharded path
            torch.cuda.empty_cache()
            obj, launches = sharded_object(key, args, world, rank, device, peaks, comparator)
            line[key] = obj
            line["gpu_launches"] += launches

    if not args.no_e2e:
        # 60 prefill steps: the pipeline's fill (the first inputs' copy) and drain (the last
        # output's copy) are not overlapped, so fewer steps would understate the steady state
        e2e = run_e2e(wl, world, rank, device, 60 if args.workload == "prefill" else 200, args)
        if e2e is not None:
            line["e2e"] = e2e

    if rank == 0 and world == 1 and not args.no_cpu:
        val, unit, sample, _, cores = cpu_sample(wl, budget_s=10.0, kind="torch")
        nval, nunit, nsample, _, ncores = cpu_sample(wl, budget_s=4.0, kind="numpy")
        line["cpu_baseline"] = {"value": round(val, 5), "unit": unit, "cores": cores, "kind": "port",
                                "sample": sample,
                                "numpy_port": {"value": round(nval, 5), "unit": nunit, "cores": ncores,
                                               "sample": nsample}}

    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    if comparator:
        line["impl"] = args.impl  # library kernels on the same box: context, not this library
        line["gate"] = gate
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main_reference(args, wl, steps):
    """The reference arm: the reference's CPU path, its torch attention
    (tests/reference.py, restated in oracle/gqa_oracle_torch.py) in fp32 on every host core.
    A step is a bounded sample of the workload: enough row blocks of one (batch, kv head)
    unit for about a quarter second of CPU work. The warm-up steps run untimed (the thread
    pool spins up there); the timed steps are capped at about two minutes in total."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    _, _, _, per, _ = cpu_sample(wl, budget_s=0.0, steps=3, kind="torch")  # thread pool up, block cost
    blocks = max(1, int(0.25 / max(min(per), 1e-4)))
    warm = min(args.warmup, max(1, int(10.0 / (blocks * min(per)))))
    cpu_sample(wl, budget_s=0.0, steps=warm * blocks, kind="torch")
    n_timed = max(3, min(steps, int(120.0 / (blocks * min(per)))))
    val, unit, sample, per, cores = cpu_sample(wl, budget_s=0.0, steps=n_timed * blocks, kind="torch")
    ms_step = sum(per) / n_timed * 1e3
    line = {
        "metric": METRIC if args.workload in ("prefill", "decode") else f"{args.workload} {unit}",
        "value": round(val, 6), "unit": unit, "impl": "reference", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True,
        "scaling": wl["scaling"], "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (N(0,1) bf16-rounded, numpy generator seeded 0)",
        "config": config_of(wl, world, args.workload),
        "cpu_baseline": {"value": round(val, 6), "unit": unit, "cores": cores, "kind": "port",
                         "sample": sample + f"; a step is {blocks} such blocks; {warm} warm-up step(s) untimed, "
                                   f"{n_timed} of {steps} requested steps timed (bounded)"},
        "e2e": {"value": round(val, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
