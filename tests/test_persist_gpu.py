"""The persistent forward schedule (paged prefill and dense D = 64): many more work items
than SMs, so every CTA runs several items through its Q buffer sets and item slots;
ragged and empty query chunks; two launches in flight on different streams at once."""
import numpy as np
import pytest
import torch

import tilelang_fa_v100 as fa
from helpers import assert_close, assert_out_close, unit_roundoff
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu


def _paged_case(rng, q_lens, ctx_lens, h, hkv, d, page, dtype):
    kv_lens = [c + q for c, q in zip(ctx_lens, q_lens)]
    pps = [-(-n // page) if n > 0 else 0 for n in kv_lens]
    total = sum(pps) + 2
    perm = rng.permutation(total)
    bt = np.zeros((len(q_lens), max(max(pps), 1)), np.int32)
    c = 0
    for b, n in enumerate(pps):
        bt[b, :n] = perm[c:c + n]
        c += n
    kc = rng.standard_normal((total, page, hkv, d)).astype(np.float32)
    vc = rng.standard_normal((total, page, hkv, d)).astype(np.float32)
    q = rng.standard_normal((max(sum(q_lens), 1), h, d)).astype(np.float32)[:sum(q_lens)]
    qsl = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    sl = np.array(kv_lens, np.int32)
    pkl = np.array(ctx_lens, np.int32)
    cast = lambda x: torch.from_numpy(x).to(dtype)
    return cast(q), cast(kc), cast(vc), bt, sl, qsl, pkl


@pytest.mark.parametrize("d,dtype", [(64, torch.float16), (128, torch.bfloat16)])
def test_paged_many_items(cuda_dev, d, dtype):
    rng = np.random.default_rng(d)
    n = 300
    q_lens = rng.integers(0, 160, n).tolist()
    q_lens[5] = 0
    q_lens[77] = 0
    ctx = rng.integers(0, 300, n).tolist()
    h, hkv, page = 8, 2, 16
    q, kc, vc, bt, sl, qsl, pkl = _paged_case(rng, q_lens, ctx, h, hkv, d, page, dtype)
    t = lambda x: torch.as_tensor(x).to(cuda_dev)
    out, lse = fa.tilelang_paged_forward(t(q), t(kc), t(vc), t(bt), t(sl), t(qsl), t(pkl),
                                         block_size=page, num_kv_heads=hkv, causal=True)
    torch.cuda.synchronize()
    ref_out, ref_lse, bound = R.paged_prefill_ref(q.float().numpy(), kc.float().numpy(),
                                                  vc.float().numpy(), bt, sl, qsl, pkl, causal=True,
                                                  unit_roundoff=unit_roundoff(dtype))
    assert_out_close(out.float().cpu().numpy(), ref_out, dtype, bound, what="out")
    assert_close(lse.cpu().numpy(), ref_lse, what="lse")


def _torch_ref(q, k, v, causal):
    """fp32 attention per (batch, head); q, k, v [B, S, H, D]."""
    qf, kf, vf = (x.float().transpose(1, 2) for x in (q, k, v))
    s = qf @ kf.transpose(-1, -2) * q.shape[-1] ** -0.5
    if causal:
        m, n = s.shape[-2:]
        s = s.masked_fill(torch.ones(m, n, device=s.device, dtype=torch.bool).tril(n - m).logical_not(),
                          float("-inf"))
    return (torch.softmax(s, -1) @ vf).transpose(1, 2)


@pytest.mark.parametrize("causal", [True, False])
def test_dense_d64_many_items(cuda_dev, causal):
    g = torch.Generator(device=cuda_dev).manual_seed(7)
    b, s, h, d = 2, 2048, 16, 64
    q, k, v = (torch.randn(b, s, h, d, generator=g, device=cuda_dev).half() for _ in range(3))
    out = fa.tilelang_flash_attn_func(q, k, v, causal=causal)
    ref = _torch_ref(q, k, v, causal)
    torch.cuda.synchronize()
    assert_close(out.float().cpu().numpy(), ref.cpu().numpy(), what="out")


def test_paged_two_streams_at_once(cuda_dev):
    """Two paged launches in flight together draw different work-item counters."""
    rng = np.random.default_rng(3)
    cases = []
    for _ in range(2):
        q_lens = rng.integers(1, 200, 40).tolist()
        ctx = rng.integers(0, 200, 40).tolist()
        cases.append(_paged_case(rng, q_lens, ctx, 8, 2, 128, 16, torch.float16))
    t = lambda x: torch.as_tensor(x).to(cuda_dev)
    dev_cases = [[t(x) for x in c] for c in cases]
    streams = [torch.cuda.Stream(cuda_dev) for _ in range(2)]
    outs = [None, None]
    torch.cuda.synchronize()
    for i, (c, st) in enumerate(zip(dev_cases, streams)):
        with torch.cuda.stream(st):
            outs[i] = fa.tilelang_paged_forward(*c, block_size=16, num_kv_heads=2, causal=True)
    torch.cuda.synchronize()
    for (q, kc, vc, bt, sl, qsl, pkl), (out, lse) in zip(cases, outs):
        ref_out, ref_lse = R.paged_prefill_ref(q.float().numpy(), kc.float().numpy(),
                                               vc.float().numpy(), bt, sl, qsl, pkl, causal=True)
        assert_close(out.float().cpu().numpy(), ref_out, what="out")
        assert_close(lse.cpu().numpy(), ref_lse, what="lse")
