"""Multi-GPU partitioning of the GQA forward on one node (one process per GPU).

The reference is single-GPU (README.md:131); these are the two partitionings
of its forward that BASELINE's multi-GPU configurations name:

* Batch x KV-head sharding (`shard_units`, `head_sharded_forward`): the
  (batch, kv_head) units of attention are independent, so each rank computes
  its units with the single-GPU path and no data crosses GPUs.

* Key-axis sharding (`seq_sharded_forward`): each rank holds a contiguous
  range of the keys for every (batch, kv_head). It computes the partial
  softmax statistics (m, l, acc) of its range with `gqa_partial`, the ranks
  exchange them in ONE all-gather of a packed [m | l | acc] fp32 buffer
  (torch.distributed, NCCL over NVLink on GPUs), and each rank combines the
  parts with `gqa_lse_combine` -- the algebra of gqa_kernels/gqa_split.py:137-144
  applied across GPUs instead of across key chunks.

* The same exchange without a collective library (`PeerExchange`): the partial
  kernel stores each unit's rows straight into every rank's receive buffer over
  NVLink (CUDA IPC mappings made once), and each rank's combine kernel waits in
  the kernel (bounded) for every source's rows. Three launches per call, no
  collective call; every rank must hold keys.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib

LOG2E = 1.4426950408889634


# ----------------------------------------------------------------------------- partition plans
def balanced_range(n, parts, index):
    """[start, stop) of part `index` when n items are cut into `parts` contiguous near-equal ranges."""
    if parts <= 0 or not 0 <= index < parts:
        raise ValueError("need 0 <= index < parts")
    base, extra = divmod(n, parts)
    start = index * base + min(index, extra)
    return start, start + base + (1 if index < extra else 0)


def kv_range(seq_kv, world, rank, align=64):
    """Contiguous key range of `rank`: cuts fall on multiples of `align` keys where possible."""
    blocks = -(-seq_kv // align)
    b0, b1 = balanced_range(blocks, world, rank)
    return min(seq_kv, b0 * align), min(seq_kv, b1 * align)


def shard_units(batch, num_kv_heads, world, rank):
    """(batch range, kv-head range) owned by `rank` for batch x KV-head sharding.

    KV heads are split first (each rank keeps every batch element of its heads,
    and the matching num_heads/num_kv_heads query heads); when there are more
    ranks than KV heads, the batch is split among the ranks that share a head.
    """
    if world <= num_kv_heads:
        return (0, batch), balanced_range(num_kv_heads, world, rank)
    if world % num_kv_heads:
        raise ValueError("world size must divide num_kv_heads or be a multiple of it")
    per_head = world // num_kv_heads
    head = rank // per_head
    return balanced_range(batch, per_head, rank % per_head), (head, head + 1)


def slice_units(q, k, v, batch_range, head_range):
    """The q/k/v slices of one rank's units (views)."""
    g = q.shape[1] // k.shape[1]
    (b0, b1), (h0, h1) = batch_range, head_range
    return q[b0:b1, h0 * g:h1 * g], k[b0:b1, h0:h1], v[b0:b1, h0:h1]


def head_sharded_forward(q_local, k_local, v_local, causal=True):
    """Batch x KV-head sharded forward: the local units through the single-GPU path."""
    from .dispatch import gqa_flash_attn
    return gqa_flash_attn(q_local, k_local, v_local, causal=causal)


# ----------------------------------------------------------------------------- key-axis sharding
def partial_forward(q, k_shard, v_shard, causal, kv_offset, seq_kv_total, out=None):
    """(m, l, acc) of this rank's key shard, packed as one fp32 buffer [m | l | pad | acc].

    m, l: batch*num_heads*seq_q values each; acc: rows x head_dim (packed_layout
    gives the offsets). `out` may be a preallocated buffer of packed_size() elements.
    """
    _lib.check_one_device(q, k_shard, v_shard, *(() if out is None else (out,)))
    batch, num_heads, seq_q, head_dim = q.shape
    _, num_kv_heads, n_local, _ = k_shard.shape
    rows, acc_off, total = packed_layout(q.shape)
    if out is None:
        out = torch.empty(total, dtype=torch.float32, device=q.device)
    m, l, acc = out[:rows], out[rows:2 * rows], out[acc_off:]
    lib = _lib.load()
    with _lib.on_device(q.device):
        ws_bytes = _lib.workspace_bytes("gqa_partial_workspace_bytes", batch, num_heads, num_kv_heads, seq_q,
                                         n_local, head_dim)
        ws = _lib.WORKSPACES.get(q.device, ws_bytes,
                                 ("partial", batch, num_heads, num_kv_heads, seq_q, n_local, head_dim))
        rc = lib.gqa_partial(
            ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k_shard.data_ptr()), ctypes.c_void_p(v_shard.data_ptr()),
            ctypes.c_void_p(m.data_ptr()), ctypes.c_void_p(l.data_ptr()), ctypes.c_void_p(acc.data_ptr()),
            _lib.strides(q), _lib.strides(k_shard), _lib.strides(v_shard),
            batch, num_heads, num_kv_heads, seq_q, n_local, int(kv_offset), int(seq_kv_total), head_dim,
            float((head_dim ** -0.5) * LOG2E), 1 if causal else 0, _lib.dtype_code(q),
            ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()), _lib.stream_ptr(q.device))
        if rc != 0:
            _lib.WORKSPACES.drop(q.device)
        _lib.check(rc, "gqa_partial")
    return out


def packed_layout(q_shape):
    """(rows, acc offset, total floats) of the packed partial buffer [m | l | pad | acc];
    acc starts on a 16-byte boundary."""
    batch, num_heads, seq_q, head_dim = q_shape
    rows = batch * num_heads * seq_q
    acc_off = -(-2 * rows // 4) * 4
    return rows, acc_off, acc_off + rows * head_dim


def packed_size(q_shape):
    return packed_layout(q_shape)[2]


def gather_partials(packed, group=None, out=None):
    """All-gather of every rank's packed partials -> (world, packed_size) on each rank.

    One collective: NCCL all_gather_into_tensor on GPUs; gloo (CPU) gets the
    list form it supports.
    """
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world, packed.numel()), dtype=packed.dtype, device=packed.device)
    if packed.is_cuda:
        dist.all_gather_into_tensor(out, packed, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), packed, group=group)
    return out


def combine_partials(gathered, q_shape, dtype, device, out=None):
    """O from the gathered per-rank partials (gqa_lse_combine, one launch)."""
    batch, num_heads, seq_q, head_dim = q_shape
    rows, acc_off, _ = packed_layout(q_shape)
    nparts, stride = gathered.shape
    if out is None:
        out = torch.empty(q_shape, dtype=dtype, device=device)
    with _lib.on_device(device):
        rc = _lib.load().gqa_lse_combine(
            ctypes.c_void_p(gathered.data_ptr()), ctypes.c_void_p(gathered.data_ptr() + 4 * rows),
            ctypes.c_void_p(gathered.data_ptr() + 4 * acc_off), nparts, stride, stride,
            ctypes.c_void_p(out.data_ptr()), _lib.strides(out), batch, num_heads, seq_q, head_dim,
            _lib.dtype_code(out), _lib.stream_ptr(device))
        _lib.check(rc, "gqa_lse_combine")
    return out


def seq_sharded_forward(q, k_shard, v_shard, kv_offset, seq_kv_total, causal=True, group=None):
    """Key-axis sharded forward: q is replicated, k/v hold this rank's key range.

    Every rank returns the full output (batch, num_heads, seq_q, head_dim).
    """
    packed = partial_forward(q, k_shard, v_shard, causal, kv_offset, seq_kv_total)
    gathered = gather_partials(packed, group)
    return combine_partials(gathered, tuple(q.shape), q.dtype, q.device)


# ----------------------------------------------------------------------------- peer exchange
def all_shards_hold_keys(seq_kv_total, world):
    """True when kv_range gives every rank at least one key (the peer exchange needs it)."""
    return all(b > a for a, b in (kv_range(seq_kv_total, world, r) for r in range(world)))


def exchange_layout(q_shape, world):
    """(slot floats, parity floats, counters byte offset, total bytes) of one rank's
    exchange buffer: [2 parities][world slots][packed partial], then `world` uint64
    counters and the uint64 epoch (include/gqa_sm100.h, peer exchange)."""
    slot = packed_size(q_shape)  # a multiple of 4 floats: every slot starts on 16 bytes
    parity = world * slot
    cnt_off = 2 * parity * 4
    return slot, parity, cnt_off, cnt_off + 8 * world + 8


class PeerExchange:
    """Key-sharded forward with the partials exchanged over NVLink by the kernels.

    Construct it on every rank of `group` with the same q shape (a collective: the
    ranks' CUDA IPC handles are all-gathered once); then `forward` on every rank, in
    the same order, gives what `seq_sharded_forward` gives, as gqa_epoch_bump +
    gqa_partial_peer + gqa_lse_combine_peer on the current stream. `close()` is a
    collective too: it waits for every rank's work before any buffer is unmapped or
    freed, since another rank's kernel may still write into this rank's buffer.
    With one rank (no process group) it runs the same kernels on this GPU alone.
    """

    def __init__(self, q_shape, num_kv_heads, device, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("the peer exchange spans the GPUs of one node (at most 8 ranks)")
        self.q_shape = tuple(int(x) for x in q_shape)
        self.device = torch.device(device)
        batch, num_heads, seq_q, head_dim = self.q_shape
        self.slot, self.parity, cnt_off, total = exchange_layout(self.q_shape, self.world)
        lib = _lib.load()
        self._opened = []
        self._own = None
        with _lib.on_device(self.device):
            units = ctypes.c_int(0)
            _lib.check(lib.gqa_partial_units(batch, num_heads, num_kv_heads, seq_q, head_dim, ctypes.byref(units)),
                       "gqa_partial_units")
            self.units = units.value
            ptr = ctypes.c_void_p()
            _lib.check(lib.gqa_exchange_alloc(total, ctypes.byref(ptr)), "gqa_exchange_alloc")
            self._own = ptr.value
            bases = [self._own]
            if self.world > 1:
                handle = (ctypes.c_uint8 * 64)()
                _lib.check(lib.gqa_ipc_handle(ctypes.c_void_p(self._own), handle), "gqa_ipc_handle")
                mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
                every = torch.empty((self.world, 64), dtype=torch.uint8, device=self.device)
                dist.all_gather_into_tensor(every, mine, group=group)
                every = every.cpu()
                bases = []
                for i in range(self.world):
                    if i == self.rank:
                        bases.append(self._own)
                        continue
                    h = (ctypes.c_uint8 * 64).from_buffer_copy(bytes(every[i].tolist()))
                    peer = ctypes.c_void_p()
                    _lib.check(lib.gqa_ipc_open(h, ctypes.byref(peer)), "gqa_ipc_open")
                    self._opened.append(peer.value)
                    bases.append(peer.value)
        self._bases = (ctypes.c_void_p * self.world)(*bases)
        self._cnts = (ctypes.c_void_p * self.world)(*[b + cnt_off for b in bases])
        self._cnt_local = self._own + cnt_off
        self._epoch = self._own + cnt_off + 8 * self.world

    def forward(self, q, k_shard, v_shard, kv_offset, seq_kv_total, causal=True, out=None):
        """O (batch, num_heads, seq_q, head_dim) from this rank's key shard and every
        other rank's, as seq_sharded_forward computes it."""
        if tuple(q.shape) != self.q_shape:
            raise ValueError(f"q shape {tuple(q.shape)} != the exchange's {self.q_shape}")
        _lib.check_one_device(q, k_shard, v_shard, *(() if out is None else (out,)))
        batch, num_heads, seq_q, head_dim = q.shape
        _, num_kv_heads, n_local, _ = k_shard.shape
        if out is None:
            out = torch.empty_like(q)
        lib = _lib.load()
        stream = _lib.stream_ptr(q.device)
        with _lib.on_device(q.device):
            ws_bytes = _lib.workspace_bytes("gqa_partial_workspace_bytes", batch, num_heads, num_kv_heads, seq_q,
                                             n_local, head_dim)
            ws = _lib.WORKSPACES.get(q.device, ws_bytes,
                                     ("partial", batch, num_heads, num_kv_heads, seq_q, n_local, head_dim))
            _lib.check(lib.gqa_epoch_bump(ctypes.c_void_p(self._epoch), stream), "gqa_epoch_bump")
            rc = lib.gqa_partial_peer(
                ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k_shard.data_ptr()), ctypes.c_void_p(v_shard.data_ptr()),
                _lib.strides(q), _lib.strides(k_shard), _lib.strides(v_shard),
                batch, num_heads, num_kv_heads, seq_q, n_local, int(kv_offset), int(seq_kv_total), head_dim,
                float((head_dim ** -0.5) * LOG2E), 1 if causal else 0, _lib.dtype_code(q),
                self._bases, self._cnts, self.world, self.rank, ctypes.c_void_p(self._epoch),
                self.slot, self.parity, ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel()), stream)
            if rc:
                _lib.WORKSPACES.drop(q.device)
            _lib.check(rc, "gqa_partial_peer")
            _lib.check(lib.gqa_lse_combine_peer(
                ctypes.c_void_p(self._own), ctypes.c_void_p(self._cnt_local), ctypes.c_void_p(self._epoch),
                self.world, self.slot, self.parity, self.units, ctypes.c_void_p(out.data_ptr()), _lib.strides(out),
                batch, num_heads, seq_q, head_dim, _lib.dtype_code(out), stream), "gqa_lse_combine_peer")
        return out

    def close(self):
        """Collective: every rank's exchange work is done before mappings and buffers go."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        lib = _lib.load()
        with _lib.on_device(self.device):
            for ptr in self._opened:
                lib.gqa_ipc_close(ctypes.c_void_p(ptr))
            self._opened = []
            if self.world > 1:
                dist.barrier(group=self.group)  # no rank frees while another still maps it
            _lib.check(lib.gqa_exchange_free(ctypes.c_void_p(self._own)), "gqa_exchange_free")
        self._own = None
