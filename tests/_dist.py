"""Spawning helpers for multi-process CPU (gloo) tests."""
import datetime
import multiprocessing as mp
import os
import socket
import traceback


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(fn, rank, world, port, timeout_s, q, args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        import torch.distributed as dist
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s))
        res = fn(rank, world, *args)
        q.put((rank, "ok", res))
    except BaseException as e:  # report every failure to the parent
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))
    finally:
        try:
            import torch.distributed as dist
            if dist.is_initialized():
                dist.destroy_process_group()
        except Exception:
            pass


def run_ranks(fn, world, args=(), timeout_s=30, join_s=120):
    """Runs fn(rank, world, *args) in `world` spawned gloo ranks; returns {rank: (status, result)}
    for the ranks that reported (a rank that exits without reporting is absent)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, timeout_s, q, args)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    import queue as _queue
    import time as _time
    deadline = _time.time() + join_s
    try:
        while len(out) < world and _time.time() < deadline:
            try:
                rank, status, res = q.get(timeout=1.0)
                out[rank] = (status, res)
            except _queue.Empty:
                if all(not p.is_alive() for p in procs):
                    # drain what the exited ranks left in the queue
                    try:
                        while True:
                            rank, status, res = q.get(timeout=0.5)
                            out[rank] = (status, res)
                    except _queue.Empty:
                        break
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return out
