"""fp32 torch reference for one (batch, head) slice of a large dense problem, on the
GPU (TEST INFRASTRUCTURE ONLY).

The BASELINE configurations are too large for the numpy oracle as a whole, so the
full-size tests compute the same function as ``oracle.attention_ref`` /
``oracle.attention_bwd_ref`` (the reference's ``pytorch_gqa_ref``,
tests/test_gqa_paged.py:19-45, and its gradients) in fp32 torch on the GPU with TF32
off, one (batch, query head) slice at a time, and check that restatement against the
numpy oracle on one slice.  Everything here is the checker, never the thing measured.
"""
import torch


def slice_ref(q, k, v, do, out, causal, bi, hi, unit_roundoff, scale=None):
    """Reference for query head ``hi`` of batch row ``bi`` of BSHD tensors.

    Returns a dict of fp32 tensors on q's device:
      out [Sq, D], lse [Sq]                       -- the exact function
      dq [Sq, D], dk / dv [Skv, D]                -- its exact gradients; dk / dv are this
                                                     query head's contribution only when
                                                     several query heads share a kv head
      dq_f, dk_f, dv_f                            -- the gradients with the row dot
                                                     D = rowsum(dO * O) taken from ``out``
                                                     (the output the backward is given, as
                                                     the reference's backward does,
                                                     _kernels_backward.py:203)
      bq, bk, bv, bo                              -- operand-rounding bounds (see
                                                     oracle.attention_bwd_ref and
                                                     oracle.attention_out_bound)
    """
    h, hk = q.shape[2], k.shape[2]
    hki = hi // (h // hk)
    return slice_ref_2d(q[bi, :, hi], k[bi, :, hki], v[bi, :, hki], do[bi, :, hi],
                        out[bi, :, hi], causal, unit_roundoff, scale)


def slice_ref_2d(qs, ks, vs, dos, os_, causal, unit_roundoff, scale=None):
    """slice_ref on one head's 2-D tensors: q / dO / out [Sq, D], k / v [Skv, D]."""
    torch.backends.cuda.matmul.allow_tf32 = False
    d = qs.shape[-1]
    scale = d ** -0.5 if scale is None else scale
    qs, ks, vs, dos, os_ = (t.float() for t in (qs, ks, vs, dos, os_))
    s = (qs @ ks.T) * scale
    m, n = s.shape
    if causal:
        vis = torch.ones(m, n, device=s.device, dtype=torch.bool).tril(diagonal=n - m)
        s = s.masked_fill(~vis, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))[:, None])
    p = torch.where(torch.isfinite(lse)[:, None], p, torch.zeros_like(p))
    o = p @ vs
    dp = dos @ vs.T
    r = {"out": o, "lse": lse}
    u = float(unit_roundoff)
    for tag, orow in (("", o), ("_f", os_)):
        ds = p * (dp - (dos * orow).sum(-1, keepdim=True))
        r["dq" + tag] = (ds @ ks) * scale
        r["dk" + tag] = (ds.T @ qs) * scale
        if tag == "_f":
            ads = ds.abs() * scale
            r["bq"] = u * (ads @ ks.abs() + r["dq_f"].abs())
            r["bk"] = u * (ads.T @ qs.abs() + r["dk_f"].abs())
    r["dv"] = p.T @ dos
    r["dv_f"] = r["dv"]
    r["bv"] = u * (p.T @ dos.abs() + r["dv"].abs())
    r["bo"] = u * (p @ vs.abs() + o.abs())
    return r


def sequence_ref(q, k, v, prefix, causal, scale=None):
    """fp32 torch reference of one paged sequence (oracle.paged_prefill_ref semantics,
    reference kernel _kernels_paged.py:296-303): q [ql, H, D] are the sequence's last ql
    query rows, k / v [L, Hkv, D] its keys in order; query row i sees key j iff, when
    causal, j <= prefix + i.  Decode is ql = 1 with every key visible.  Returns out
    [ql, H, D] and lse [H, ql]."""
    torch.backends.cuda.matmul.allow_tf32 = False
    ql, h, d = q.shape
    n, hkv = k.shape[0], k.shape[1]
    scale = d ** -0.5 if scale is None else scale
    qh = q.float().permute(1, 0, 2)                                   # [H, ql, D]
    kh = k.float().permute(1, 0, 2).repeat_interleave(h // hkv, 0)    # [H, L, D]
    vh = v.float().permute(1, 0, 2).repeat_interleave(h // hkv, 0)
    s = torch.einsum("hqd,hkd->hqk", qh, kh) * scale
    if causal:
        i = torch.arange(ql, device=q.device)[:, None]
        j = torch.arange(n, device=q.device)[None, :]
        s = s.masked_fill(~(j <= prefix + i)[None], float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.softmax(s, dim=-1).nan_to_num(0.0)
    return torch.einsum("hqk,hkd->hqd", p, vh).permute(1, 0, 2), lse
