"""PyTorch restatement of the reference's CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU-baseline leg (and its `--impl reference` arm)
import this module: as the checker of GPU results, and as the timed CPU
baseline, the reference's own PyTorch attention run on the host cores. The
product path (gqa_kernels + libgqa_sm100.so) never calls it.

  gqa_reference          tests/reference.py:6-34   the reference's naive GQA attention:
                         K/V repeated over the group (repeat_interleave), scores
                         scaled by head_dim^-0.5, bottom-right causal mask
                         (masked_fill with -inf), softmax, @ V -- the same torch
                         operations in the same order, so it computes what the
                         reference's oracle computes on the same inputs and device
  gqa_reference_blocked  the same math per (batch, kv head, block of query rows), so
                         the materialised score matrix stays bounded for full-size
                         shapes; rows are independent, so the result is the same

Parity pin: tests/test_oracle_golden.py checks both against
tests/golden/oracle_bf16.npz, which tests/golden/make_golden.py recorded from the
reference's own tests/reference.py.
"""
import torch
import torch.nn.functional as F


def gqa_reference(q, k, v, causal=True):
    """tests/reference.py:6-34 in torch: q (B, Hq, Sq, D), k/v (B, Hkv, Skv, D), any float dtype
    and device; computes in the inputs' dtype, like the reference."""
    batch, num_heads, seq_q, head_dim = q.shape
    _, num_kv_heads, seq_kv, _ = k.shape
    assert num_heads % num_kv_heads == 0
    group = num_heads // num_kv_heads
    scores = torch.matmul(q, k.repeat_interleave(group, dim=1).transpose(-2, -1)) * head_dim ** -0.5
    if causal:
        q_pos = torch.arange(seq_q, device=q.device) + (seq_kv - seq_q)
        k_pos = torch.arange(seq_kv, device=q.device)
        scores = scores.masked_fill(q_pos[:, None] < k_pos[None, :], float("-inf"))
    return torch.matmul(F.softmax(scores, dim=-1), v.repeat_interleave(group, dim=1))


@torch.no_grad()
def gqa_reference_blocked(q, k, v, causal=True, row_block=2048):
    """gqa_reference in fp32 on the tensors' device, evaluated per (batch, kv head,
    block of query rows) with TF32 off. Returns float32 (B, Hq, Sq, D)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        B, Hq, Sq, D = q.shape
        _, Hkv, Skv, _ = k.shape
        G = Hq // Hkv
        out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
        for b in range(B):
            for kv in range(Hkv):
                kf = k[b:b + 1, kv:kv + 1].float()
                vf = v[b:b + 1, kv:kv + 1].float()
                for r0 in range(0, Sq, row_block):
                    r1 = min(Sq, r0 + row_block)
                    # rows r0..r1 see keys [0, r + Skv - Sq]: the key prefix up to the last
                    # row's bound keeps the reference's bottom-right offset for the block
                    kend = Skv if not causal else max(0, min(Skv, r1 + Skv - Sq))
                    qs = q[b:b + 1, kv * G:(kv + 1) * G, r0:r1].float()
                    if kend == 0:
                        out[b, kv * G:(kv + 1) * G, r0:r1] = float("nan")
                        continue
                    out[b:b + 1, kv * G:(kv + 1) * G, r0:r1] = gqa_reference(qs, kf[:, :, :kend], vf[:, :, :kend],
                                                                              causal)
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
