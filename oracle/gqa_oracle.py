"""CPU oracle for the GQA flash-attention forward path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only as the checker (or the timed CPU baseline); the product
path (gqa_kernels + libgqa_sm100.so) never calls it.

It restates, in numpy, the reference project's algorithms for this path:

  gqa_reference          tests/reference.py:6-34           naive GQA attention (the correctness oracle)
  gqa_reference_rows     tests/reference.py:6-34           same math, selected output rows only
  gqa_fwd_blocked        gqa_kernels/gqa_fwd.py:36-109     group-packed online-softmax kernel
  gqa_split_first        gqa_kernels/gqa_split.py:46-112   per-chunk partials (m, l, acc)
  gqa_split_reduce       gqa_kernels/gqa_split.py:124-147  log-sum-exp combine
  route                  gqa_kernels/dispatch.py:37-45     single-pass vs split-KV choice
  partial_attention      (new) partials of one key shard, the multi-GPU split of the key axis
  lse_combine            gqa_kernels/gqa_split.py:137-144 applied across shards
  paged_reference        (new) the reference attention over a vLLM-layout paged cache:
                         each sequence's keys gathered through its block table, its
                         queries bottom-right aligned to its own length

Parity pins: tests/test_oracle_golden.py checks these functions against
tests/golden/*.npz, produced by tests/golden/make_golden.py from the
reference's own code (its torch oracle, and its Triton kernels run on CPU by
Triton's interpreter in float16).
"""
import numpy as np

LOG2E = 1.4426950408889634


# ----------------------------------------------------------------------------- number formats
def bf16_round(x):
    """Round float32 values to bfloat16 (round-to-nearest-even), returned as float32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16
    r = np.where(np.isnan(x), np.uint32(0x7FC00000), r.astype(np.uint32))
    return r.astype(np.uint32).view(np.float32)


def f16_round(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def bf16_bits_to_f32(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x):
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


ROUNDERS = {"bf16": bf16_round, "f16": f16_round, "f32": lambda x: np.asarray(x, dtype=np.float32)}


# ----------------------------------------------------------------------------- oracle
def _softmax_rows(s):
    # torch.softmax semantics: a row of all -inf gives NaN (0/0).
    m = np.max(s, axis=-1, keepdims=True)
    with np.errstate(invalid="ignore"):
        e = np.exp(s - m)
        return e / np.sum(e, axis=-1, keepdims=True)


def gqa_reference(q, k, v, causal=True, dtype=np.float32, row_block=1024):
    """tests/reference.py:6-34 in numpy.

    q: (B, Hq, Sq, D); k, v: (B, Hkv, Skv, D) float arrays. Computes in `dtype`
    (float32 like the reference's fp32 oracle, or float64). The S x S score
    matrix is materialised per (batch, kv head, block of query rows) to bound
    memory; the math is that of the reference: K/V expanded over the group,
    scores * D^-0.5, bottom-right causal mask, softmax, @ V.
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    B, Hq, Sq, D = q.shape
    _, Hkv, Skv, _ = k.shape
    assert Hq % Hkv == 0
    G = Hq // Hkv
    scale = dtype(D ** -0.5)
    out = np.empty((B, Hq, Sq, D), dtype=dtype)
    k_pos = np.arange(Skv)
    for b in range(B):
        for kv in range(Hkv):
            kt = k[b, kv].T
            vv = v[b, kv]
            for r0 in range(0, Sq, row_block):
                r1 = min(Sq, r0 + row_block)
                qs = q[b, kv * G:(kv + 1) * G, r0:r1]            # (G, rows, D)
                s = np.matmul(qs, kt) * scale                    # (G, rows, Skv)
                if causal:
                    q_pos = np.arange(r0, r1) + (Skv - Sq)
                    mask = q_pos[:, None] < k_pos[None, :]
                    s = np.where(mask[None], -np.inf, s)
                out[b, kv * G:(kv + 1) * G, r0:r1] = np.matmul(_softmax_rows(s), vv)
    return out


def gqa_reference_rows(q, k, v, rows, causal=True, dtype=np.float64):
    """Oracle output for selected rows only: rows = iterable of (b, head, i).

    Rows are independent in attention, so a seeded sample of rows checks a
    full-size call against the oracle at a cost of O(seq_kv * D) per row.
    Returns an array (len(rows), D).
    """
    B, Hq, Sq, D = q.shape
    _, Hkv, Skv, _ = k.shape
    G = Hq // Hkv
    scale = D ** -0.5
    res = np.empty((len(rows), D), dtype=dtype)
    for n, (b, h, i) in enumerate(rows):
        kv = h // G
        s = (np.asarray(k[b, kv], dtype=dtype) @ np.asarray(q[b, h, i], dtype=dtype)) * scale
        if causal:
            s = np.where(np.arange(Skv) > i + (Skv - Sq), -np.inf, s)
        res[n] = _softmax_rows(s[None])[0] @ np.asarray(v[b, kv], dtype=dtype)
    return res


# ----------------------------------------------------------------------------- kernel restatements
def _pack_rows(G, block_m, pid_m, kv):
    """Group packing (gqa_fwd.py:57-65): packed row r -> (head, position)."""
    r = np.arange(G * block_m)
    g = r // block_m
    return kv * G + g, pid_m * block_m + (r % block_m)


def gqa_fwd_blocked(q, k, v, causal, block_m=16, block_n=32, io="f16"):
    """gqa_kernels/gqa_fwd.py:36-109 restated: one program per (m-tile, kv head, batch),
    group-packed rows, Q pre-scaled by scale*log2(e) and re-rounded to the input
    type (:75-78), online softmax in exp2 over key blocks up to the causal bound
    (:70-73), P rounded to the input type before P @ V (:103), acc / l (:106)."""
    rnd = ROUNDERS[io]
    B, Hq, Sq, D = q.shape
    _, Hkv, Skv, _ = k.shape
    G = Hq // Hkv
    scale = np.float32((D ** -0.5) * LOG2E)
    out = np.full((B, Hq, Sq, D), np.nan, dtype=np.float32)
    n_m = -(-Sq // block_m)
    for b in range(B):
        for kv in range(Hkv):
            for pid_m in range(n_m):
                heads, pos = _pack_rows(G, block_m, pid_m, kv)
                valid = pos < Sq
                q_pos = pos + (Skv - Sq)
                kv_end = min((pid_m + 1) * block_m + (Skv - Sq), Skv) if causal else Skv
                qt = np.zeros((G * block_m, D), dtype=np.float32)
                qt[valid] = q[b, heads[valid], pos[valid]]
                qt = rnd(qt * scale)
                m_i = np.full(G * block_m, -np.inf, dtype=np.float32)
                l_i = np.zeros(G * block_m, dtype=np.float32)
                acc = np.zeros((G * block_m, D), dtype=np.float32)
                with np.errstate(invalid="ignore"):
                    for n0 in range(0, max(kv_end, 0), block_n):
                        n = n0 + np.arange(block_n)
                        n_ok = n < Skv
                        kt = np.zeros((block_n, D), dtype=np.float32)
                        vt = np.zeros((block_n, D), dtype=np.float32)
                        kt[n_ok] = k[b, kv, n[n_ok]]
                        vt[n_ok] = v[b, kv, n[n_ok]]
                        qk = qt @ kt.T
                        qk = np.where(n_ok[None, :], qk, -np.inf)
                        if causal:
                            qk = np.where(q_pos[:, None] >= n[None, :], qk, -np.inf)
                        m_new = np.maximum(m_i, qk.max(axis=1))
                        alpha = np.exp2(m_i - m_new)
                        p = np.exp2(qk - m_new[:, None])
                        l_i = alpha * l_i + p.sum(axis=1)
                        acc = acc * alpha[:, None] + rnd(p) @ vt
                        m_i = m_new
                    o = acc / l_i[:, None]
                out[b, heads[valid], pos[valid]] = rnd(o[valid])
    return out


def gqa_split_first(q, k, v, causal, splits, block_m=None, io="f16", clean_masked=False, block_n=None):
    """gqa_kernels/gqa_split.py:46-112 restated. Returns m_p, l_p (B, Hq, Sq, splits)
    and acc_p (B, Hq, Sq, splits, D) in float32.

    Chunk s covers keys [s*ceil(Skv/splits), min((s+1)*ceil(Skv/splits), Skv)),
    clipped under causal at the m-tile's last query position (:58-60). m is in
    log2 units (Q pre-scaled by scale*log2 e and re-rounded, :77), l = sum exp2(qk - m),
    acc = sum round(p) v. A chunk that is empty after clipping gives (-inf, 0, 0).
    A non-empty chunk in which one row sees no key gives NaN in the reference
    (exp2(-inf - -inf)); with clean_masked=True such rows get (-inf, 0, 0) instead,
    which is what the CUDA kernels write.

    block_n=None uses exactly the chunk's keys (the CUDA kernels' semantics).
    With block_n given, the reference's loop is followed literally (:83-93): key
    blocks of block_n start at the chunk start while n_start < chunk_end and are
    masked only by n < seq_kv, so when the chunk size is not a multiple of
    block_n the last block also reads keys of the next chunk, which the
    combine then counts twice. The two agree when ceil(Skv/splits) % block_n == 0.
    """
    rnd = ROUNDERS[io]
    B, Hq, Sq, D = q.shape
    _, Hkv, Skv, _ = k.shape
    G = Hq // Hkv
    if block_m is None:
        block_m = 16 if Sq <= 16 else 32
    scale = np.float32((D ** -0.5) * LOG2E)
    cs = -(-Skv // splits)
    m_p = np.full((B, Hq, Sq, splits), np.nan, dtype=np.float32)
    l_p = np.full((B, Hq, Sq, splits), np.nan, dtype=np.float32)
    acc_p = np.full((B, Hq, Sq, splits, D), np.nan, dtype=np.float32)
    n_m = -(-Sq // block_m)
    for b in range(B):
        for kv in range(Hkv):
            for pid_m in range(n_m):
                heads, pos = _pack_rows(G, block_m, pid_m, kv)
                valid = pos < Sq
                q_pos = pos + (Skv - Sq)
                qt = np.zeros((G * block_m, D), dtype=np.float32)
                qt[valid] = q[b, heads[valid], pos[valid]]
                qt = rnd(qt * scale)
                for s in range(splits):
                    c0 = s * cs
                    c1 = min(c0 + cs, Skv)
                    if causal:
                        c1 = min(c1, (pid_m + 1) * block_m + (Skv - Sq))
                    m_i = np.full(G * block_m, -np.inf, dtype=np.float32)
                    l_i = np.zeros(G * block_m, dtype=np.float32)
                    acc = np.zeros((G * block_m, D), dtype=np.float32)
                    if c1 > c0:
                        hi = c1 if block_n is None else min(Skv, c0 + -(-(c1 - c0) // block_n) * block_n)
                        n = np.arange(c0, hi)
                        qk = qt @ k[b, kv, n].astype(np.float32).T
                        if causal:
                            qk = np.where(q_pos[:, None] >= n[None, :], qk, -np.inf)
                        m_i = qk.max(axis=1)
                        with np.errstate(invalid="ignore"):
                            p = np.exp2(qk - m_i[:, None])
                        if clean_masked:
                            dead = m_i == -np.inf
                            p[dead] = 0.0
                        l_i = p.sum(axis=1)
                        acc = rnd(p) @ v[b, kv, n].astype(np.float32)
                    m_p[b, heads[valid], pos[valid], s] = m_i[valid]
                    l_p[b, heads[valid], pos[valid], s] = l_i[valid]
                    acc_p[b, heads[valid], pos[valid], s] = acc[valid]
    return m_p, l_p, acc_p


def gqa_split_reduce(m_p, l_p, acc_p, io="f16"):
    """gqa_kernels/gqa_split.py:134-147: m = max_s m_s, alpha_s = exp2(m_s - m),
    o = sum_s alpha_s acc_s / sum_s alpha_s l_s, rounded to the output type."""
    with np.errstate(invalid="ignore"):
        m = np.max(m_p, axis=-1, keepdims=True)
        alpha = np.exp2(m_p - m)
        l = np.sum(alpha * l_p, axis=-1)
        o = np.sum(alpha[..., None] * acc_p, axis=-2) / l[..., None]
    return ROUNDERS[io](o)


def route(seq_q, seq_kv, num_kv_heads, batch, sm_count=28):
    """gqa_kernels/dispatch.py:37-45: ('split', splits) or ('single', None)."""
    if seq_q <= 16 and seq_kv >= 1024 and num_kv_heads * batch < sm_count:
        target = 4 * sm_count
        splits = 1
        while splits * num_kv_heads * batch < target and splits < 32:
            splits *= 2
        while splits > 1 and seq_kv // splits < 64:
            splits //= 2
        if splits > 1:
            return ("split", splits)
    return ("single", None)


# ----------------------------------------------------------------------------- key-axis sharding
def partial_attention(q, k_shard, v_shard, causal, kv_offset, seq_kv_total, dtype=np.float64):
    """Exact (m, l, acc) of one contiguous key shard [kv_offset, kv_offset + n):
    m in log2 units (scores * D^-0.5 * log2 e), l = sum exp2(s - m), acc = sum exp2(s - m) v.
    Rows that see no key of the shard get (-inf, 0, 0). Shapes: m, l (B, Hq, Sq);
    acc (B, Hq, Sq, D)."""
    q = np.asarray(q, dtype=dtype)
    k_shard = np.asarray(k_shard, dtype=dtype)
    v_shard = np.asarray(v_shard, dtype=dtype)
    B, Hq, Sq, D = q.shape
    _, Hkv, n, _ = k_shard.shape
    G = Hq // Hkv
    sc = (D ** -0.5) * LOG2E
    m = np.empty((B, Hq, Sq), dtype=dtype)
    l = np.empty((B, Hq, Sq), dtype=dtype)
    acc = np.empty((B, Hq, Sq, D), dtype=dtype)
    if n == 0:  # an empty shard: every row sees none of its keys
        m.fill(-np.inf)
        l.fill(0.0)
        acc.fill(0.0)
        return m, l, acc
    keys = kv_offset + np.arange(n)
    for b in range(B):
        for h in range(Hq):
            s = (q[b, h] @ k_shard[b, h // G].T) * sc
            if causal:
                q_pos = np.arange(Sq) + (seq_kv_total - Sq)
                s = np.where(q_pos[:, None] >= keys[None, :], s, -np.inf)
            mm = s.max(axis=1)
            mu = np.where(mm == -np.inf, 0.0, mm)
            p = np.exp2(s - mu[:, None])
            m[b, h], l[b, h], acc[b, h] = mm, p.sum(axis=1), p @ v_shard[b, h // G]
    return m, l, acc


def lse_combine(ms, ls, accs):
    """Combine partials stacked on axis 0 (parts): the algebra of gqa_split.py:137-144."""
    ms, ls, accs = np.asarray(ms), np.asarray(ls), np.asarray(accs)
    M = ms.max(axis=0)
    Mu = np.where(M == -np.inf, 0.0, M)
    w = np.exp2(ms - Mu[None])
    with np.errstate(invalid="ignore", divide="ignore"):
        return (w[..., None] * accs).sum(axis=0) / (w * ls).sum(axis=0)[..., None]


def paged_reference(q, k_cache, v_cache, block_tables, seq_lens, causal=True, k_scale=1.0, v_scale=1.0):
    """Attention of each sequence's chunk over a paged cache, by gathering.

    q: (num_seqs, Hq, Sq, D); k_cache, v_cache: (num_blocks, block_size, Hkv, D);
    block_tables: (num_seqs, max_blocks) int; seq_lens: (num_seqs,) int. Key k of
    sequence b is k_cache[block_tables[b, k // block_size], k % block_size] * k_scale
    (values likewise with v_scale); its Sq queries are its last Sq positions
    (tests/reference.py:6-34's bottom-right rule per sequence). Returns float32
    (num_seqs, Hq, Sq, D); rows that see no key are NaN.
    """
    q = np.asarray(q, dtype=np.float32)
    kc = np.asarray(k_cache, dtype=np.float32)
    vc = np.asarray(v_cache, dtype=np.float32)
    n, Hq, Sq, D = q.shape
    bs = kc.shape[1]
    out = np.empty((n, Hq, Sq, D), dtype=np.float32)
    for b in range(n):
        s = int(seq_lens[b])
        idx = np.arange(s)
        blocks = np.asarray(block_tables[b])[idx // bs]
        k = (kc[blocks, idx % bs] * np.float32(k_scale)).transpose(1, 0, 2)[None]  # (1, Hkv, s, D)
        v = (vc[blocks, idx % bs] * np.float32(v_scale)).transpose(1, 0, 2)[None]
        if s == 0:
            out[b] = np.nan
        else:
            out[b] = gqa_reference(q[b:b + 1], k, v, causal=causal)[0]
    return out
