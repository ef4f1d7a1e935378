"""PyTorch (CPU, fp32) restatement of the reference's attention oracle -- TEST / BENCH
INFRASTRUCTURE ONLY (tests/, __graft_entry__.smoke() and bench.py's CPU baseline and
reference arm may use it; the product path never does).

Same computation as ``pytorch_gqa_ref`` (tests/test_gqa_paged.py:19-45 of the
reference): GQA expansion by unsqueeze/expand/reshape (:37-38), fp32 einsum scores
times scale (:40), bottom-right causal mask tril(ones(M, N), diagonal=N-M) (:41-43,
here on the tensor's own device instead of 'cuda'), fp32 softmax (:44) and P V (:45),
without the final fp16 cast so autograd gives fp32 gradients.  This is what the
reference's own CPU-runnable path computes; bench.py times it on the host cores as
the CPU baseline.  tests/test_oracle_golden.py checks it against the numpy oracle.
"""
import math

import torch
import torch.nn.functional as F


def gqa_attention(q, k, v, causal, scale=None):
    """q [B, Hq, M, D], k/v [B, Hkv, N, D] (any float dtype) -> fp32 [B, Hq, M, D]."""
    b, hq, m, d = q.shape
    hkv, n = k.shape[1], k.shape[2]
    ratio = hq // hkv
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    k_exp = k.unsqueeze(2).expand(b, hkv, ratio, n, d).reshape(b, hq, n, d)
    v_exp = v.unsqueeze(2).expand(b, hkv, ratio, n, d).reshape(b, hq, n, d)
    scores = torch.einsum("bhqd,bhkd->bhqk", q.float(), k_exp.float()) * scale
    if causal:
        mask = torch.tril(torch.ones(m, n, device=q.device), diagonal=n - m)
        scores = scores.masked_fill(mask == 0, float("-inf"))
    attn = F.softmax(scores, dim=-1, dtype=torch.float32)
    return torch.einsum("bhqk,bhkd->bhqd", attn, v_exp.float())


def fwd_bwd(q, k, v, do, causal):
    """One forward + backward step on CPU fp32 tensors; returns (out, dq, dk, dv)."""
    q = q.detach().float().requires_grad_(True)
    k = k.detach().float().requires_grad_(True)
    v = v.detach().float().requires_grad_(True)
    out = gqa_attention(q, k, v, causal)
    out.backward(do.float())
    return out.detach(), q.grad, k.grad, v.grad
