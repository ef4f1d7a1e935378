"""Dense attention on the GPU against the CPU oracle (pinned to the reference) and
against the reference's own golden vectors."""
import numpy as np
import pytest
import torch

import tilelang_fa_v100 as fa
from helpers import (assert_close, assert_grad_close, assert_out_close, bwd_refs, golden,
                     golden_names, max_abs, unit_roundoff)
from oracle import attention_ref as R
from slice_ref import slice_ref

pytestmark = pytest.mark.gpu


def _to_bhsd(x):
    return x.float().permute(0, 2, 1, 3).cpu().numpy()


def _rand(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


def _fwd(q, k, v, causal, scale=None):
    out, lse, _ = fa.tilelang_flash_attn_func(q, k, v, causal=causal, softmax_scale=scale,
                                              return_attn_probs=True)
    torch.cuda.synchronize()
    return out, lse


@pytest.mark.parametrize("name", golden_names("dense_"))
def test_golden_forward(cuda_dev, name):
    g = golden(name)
    q, k, v = (torch.from_numpy(g[x]).permute(0, 2, 1, 3).contiguous().to(cuda_dev)
               for x in ("q", "k", "v"))
    out, lse = _fwd(q, k, v, bool(g["causal"]))
    ref_out, ref_lse = R.attention_ref(g["q"], g["k"], g["v"], bool(g["causal"]))
    assert_close(_to_bhsd(out), ref_out, what=name + " out")
    assert_close(lse.cpu().numpy(), ref_lse, what=name + " lse")
    # and the reference's own fp16 output within its bar (max-abs < 0.01)
    assert max_abs(_to_bhsd(out), g["out"].astype(np.float32)) < 1e-2


FWD_CASES = [
    # B, Sq, Skv, H, Hk, D, causal, dtype
    (1, 128, 128, 2, 2, 64, False, torch.float16),
    (2, 200, 200, 3, 3, 128, True, torch.bfloat16),
    (1, 64, 300, 2, 2, 128, True, torch.float16),    # non-square causal (bottom-right)
    (1, 300, 64, 2, 2, 64, True, torch.bfloat16),    # Sq > Skv: leading rows fully masked
    (1, 257, 257, 4, 1, 128, True, torch.bfloat16),  # MQA
    (1, 190, 190, 8, 2, 64, True, torch.float16),    # GQA 4:1
    (1, 100, 100, 2, 2, 256, False, torch.float16),  # D = 256
    (1, 1, 77, 2, 2, 64, False, torch.bfloat16),     # single query row
    (2, 512, 512, 2, 2, 64, True, torch.float16),
    (1, 1000, 1000, 1, 1, 128, True, torch.bfloat16),
    (1, 384, 1024, 2, 2, 128, False, torch.float16),
    # long keys: work items of more than 12 KV tiles take the one-CTA-per-item kernel
    (1, 64, 4096, 2, 2, 128, True, torch.bfloat16),     # non-square causal
    (1, 3300, 3300, 4, 1, 128, True, torch.bfloat16),   # MQA
    (1, 4200, 4100, 2, 2, 128, True, torch.float16),    # Sq > Skv
    (1, 2000, 2000, 8, 2, 128, False, torch.float16),   # GQA 4:1, non-causal
    (1, 1700, 1700, 2, 2, 256, False, torch.bfloat16),  # D = 256 non-causal
    # head_dim 32 / 96 on the 64 / 128 kernels (zero-filled columns, clipped stores)
    (2, 300, 300, 4, 2, 32, True, torch.bfloat16),
    (1, 200, 520, 2, 2, 32, False, torch.float16),
    (1, 1000, 1000, 4, 4, 96, True, torch.float16),
    (2, 77, 300, 8, 1, 96, True, torch.bfloat16),
    (1, 2500, 2500, 2, 2, 96, True, torch.bfloat16),   # long items: one-CTA-per-item kernel
]


@pytest.mark.parametrize("case", FWD_CASES, ids=lambda c: "-".join(map(str, c[:7])))
def test_forward_vs_oracle(cuda_dev, case):
    b, sq, skv, h, hk, d, causal, dt = case
    q = _rand((b, sq, h, d), dt, 1)
    k = _rand((b, skv, hk, d), dt, 2)
    v = _rand((b, skv, hk, d), dt, 3)
    out, lse = _fwd(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), causal)
    ref_out, ref_lse = R.attention_ref(_to_bhsd(q), _to_bhsd(k), _to_bhsd(v), causal)
    bound = R.attention_out_bound(_to_bhsd(q), _to_bhsd(k), _to_bhsd(v), causal, unit_roundoff(dt))
    assert_out_close(_to_bhsd(out), ref_out, dt, bound, what="out")
    assert_close(lse.cpu().numpy(), ref_lse, what="lse")


def test_custom_softmax_scale(cuda_dev):
    q, k, v = (_rand((1, 130, 2, 64), torch.float16, s) for s in (4, 5, 6))
    out, lse = _fwd(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), True, scale=0.3)
    ref_out, ref_lse = R.attention_ref(_to_bhsd(q), _to_bhsd(k), _to_bhsd(v), True, scale=0.3)
    assert_close(_to_bhsd(out), ref_out, what="out")
    assert_close(lse.cpu().numpy(), ref_lse, what="lse")


def test_noncontiguous_inputs(cuda_dev):
    # BHSD storage viewed as BSHD (what a caller holding [B,H,S,D] tensors passes)
    q, k, v = (_rand((1, 2, 96, 64), torch.bfloat16, s).to(cuda_dev).permute(0, 2, 1, 3)
               for s in (7, 8, 9))
    out, lse = _fwd(q, k, v, True)
    ref_out, _ = R.attention_ref(_to_bhsd(q), _to_bhsd(k), _to_bhsd(v), True)
    bound = R.attention_out_bound(_to_bhsd(q), _to_bhsd(k), _to_bhsd(v), True, 2.0 ** -8)
    assert_out_close(_to_bhsd(out), ref_out, torch.bfloat16, bound, what="out")


def test_repeated_calls_are_deterministic(cuda_dev):
    q, k, v = (_rand((2, 333, 4, 128), torch.bfloat16, s).to(cuda_dev) for s in (10, 11, 12))
    o1, _ = _fwd(q, k, v, True)
    o2, _ = _fwd(q, k, v, True)
    assert torch.equal(o1, o2)


BWD_CASES = [
    (1, 128, 128, 2, 2, 64, False, torch.float16),
    (2, 200, 200, 3, 3, 128, True, torch.bfloat16),
    (1, 96, 300, 2, 2, 128, True, torch.float16),
    (1, 257, 257, 4, 1, 128, True, torch.bfloat16),
    (1, 190, 190, 4, 2, 64, True, torch.float16),
    (1, 512, 512, 2, 2, 64, True, torch.bfloat16),
    # causal with seqlen_q > seqlen_k + 128: query tile 0 sees no key (dq = 0 from prep)
    (1, 400, 150, 2, 2, 128, True, torch.bfloat16),
    # several KV tiles add into each query tile; ragged last tile; GQA 4:2
    (2, 1000, 1000, 4, 2, 128, True, torch.float16),
    (1, 300, 700, 2, 1, 64, False, torch.bfloat16),
    # D = 128, one query head per kv head, short items: the persistent dK/dV kernel with
    # 300-500 work items, so each CTA runs two to four of them.
    (40, 300, 300, 4, 4, 128, True, torch.bfloat16),
    (24, 700, 900, 2, 2, 128, False, torch.bfloat16),
    (30, 1000, 400, 3, 3, 128, True, torch.bfloat16),
    (16, 500, 500, 2, 2, 128, True, torch.float16),
    # D = 256: split-D dK / dV kernel + dQ kernel (64-query / 64-key steps)
    (1, 200, 200, 2, 2, 256, True, torch.bfloat16),
    (1, 300, 520, 4, 2, 256, False, torch.float16),    # GQA 2:1, non-causal, ragged
    (2, 130, 90, 2, 2, 256, True, torch.float16),      # Sq > Skv: leading rows fully masked
    (1, 1000, 1000, 2, 2, 256, True, torch.bfloat16),  # several KV tiles and query steps
    (3, 64, 300, 8, 1, 256, True, torch.bfloat16),     # MQA 8:1, non-square causal
    # head_dim 32 / 96 on the 64 / 128 kernels
    (1, 300, 300, 4, 2, 32, True, torch.bfloat16),
    (2, 200, 333, 2, 2, 32, False, torch.float16),
    (1, 700, 700, 2, 2, 96, True, torch.float16),
    (6, 300, 300, 2, 2, 96, True, torch.bfloat16),     # persistent dK/dV kernel
    (1, 190, 250, 4, 1, 96, False, torch.bfloat16),
]


@pytest.mark.parametrize("deterministic", [False, True])
@pytest.mark.parametrize("case", BWD_CASES, ids=lambda c: "-".join(map(str, c[:7])))
def test_backward_vs_oracle(cuda_dev, case, deterministic):
    b, sq, skv, h, hk, d, causal, dt = case
    q = _rand((b, sq, h, d), dt, 21)
    k = _rand((b, skv, hk, d), dt, 22)
    v = _rand((b, skv, hk, d), dt, 23)
    do = _rand((b, sq, h, d), dt, 24)
    qd, kd, vd = (x.to(cuda_dev).requires_grad_(True) for x in (q, k, v))
    out = fa.tilelang_flash_attn_func(qd, kd, vd, causal=causal, deterministic=deterministic)
    out.backward(do.to(cuda_dev))
    torch.cuda.synchronize()
    args = (_to_bhsd(q), _to_bhsd(k), _to_bhsd(v), _to_bhsd(do), causal)
    exact, faithful, bounds = bwd_refs(args, _to_bhsd(out.detach()), unit_roundoff(dt))
    for got, want, want_f, bnd, w in zip((qd.grad, kd.grad, vd.grad), exact, faithful, bounds,
                                         ("dq", "dk", "dv")):
        assert_grad_close(_to_bhsd(got), want, dt, w, bound=bnd, want_faithful=want_f)


@pytest.mark.parametrize("name", golden_names("dense_"))
def test_golden_backward(cuda_dev, name):
    g = golden(name)
    q, k, v = (torch.from_numpy(g[x]).permute(0, 2, 1, 3).contiguous().to(cuda_dev)
               .requires_grad_(True) for x in ("q", "k", "v"))
    do = torch.from_numpy(g["do"]).permute(0, 2, 1, 3).to(torch.float16).contiguous().to(cuda_dev)
    out = fa.tilelang_flash_attn_func(q, k, v, causal=bool(g["causal"]))
    out.backward(do)
    torch.cuda.synchronize()
    dq, dk, dv = R.attention_bwd_ref(g["q"], g["k"], g["v"],
                                     _to_bhsd(do.cpu()), bool(g["causal"]))
    for got, want, w in ((q.grad, dq, "dq"), (k.grad, dk, "dk"), (v.grad, dv, "dv")):
        assert_grad_close(_to_bhsd(got), want, torch.float16, name + " " + w)


def test_deterministic_backward_is_bitwise_reproducible(cuda_dev):
    q, k, v, do = (_rand((1, 700, 2, 128), torch.bfloat16, s).to(cuda_dev) for s in (31, 32, 33, 34))
    grads = []
    for _ in range(2):
        qd, kd, vd = (x.clone().requires_grad_(True) for x in (q, k, v))
        fa.tilelang_flash_attn_func(qd, kd, vd, causal=True, deterministic=True).backward(do)
        grads.append((qd.grad, kd.grad, vd.grad))
    for a, b in zip(*grads):
        assert torch.equal(a, b)


@pytest.mark.parametrize("cfg", [(4, 2048, 2048, 16, 64, torch.float16),
                                 (8, 4096, 4096, 32, 128, torch.bfloat16),
                                 (8, 1024, 4096, 32, 128, torch.bfloat16)],
                         ids=["cfg2", "cfg3", "cfg3-nonsquare"])
@pytest.mark.parametrize("deterministic", [False, True])
def test_full_size_fwd_bwd_sampled(cuda_dev, cfg, deterministic):
    """BASELINE configs at full size, forward + backward through the API as the benchmark
    runs them; out, lse, dQ, dK and dV of sampled (batch, head) slices against the fp32
    torch reference on the GPU (tests/slice_ref.py, checked against the numpy oracle by
    test_slice_ref_matches_oracle)."""
    b, sq, skv, h, d, dt = cfg
    g = torch.Generator(device=cuda_dev).manual_seed(0)
    q = torch.randn(b, sq, h, d, generator=g, device=cuda_dev).to(dt)
    k = torch.randn(b, skv, h, d, generator=g, device=cuda_dev).to(dt)
    v = torch.randn(b, skv, h, d, generator=g, device=cuda_dev).to(dt)
    do = torch.randn(b, sq, h, d, generator=g, device=cuda_dev).to(dt)
    qd, kd, vd = (x.clone().requires_grad_(True) for x in (q, k, v))
    out, lse, _ = fa.tilelang_flash_attn_func(qd, kd, vd, causal=True, deterministic=deterministic,
                                              return_attn_probs=True)
    out.backward(do)
    torch.cuda.synchronize()
    u = unit_roundoff(dt)
    cpu = lambda t: t.detach().float().cpu().numpy()
    for bi, hi in ((0, 0), (b - 1, h - 1), (b // 2, h // 3)):
        r = slice_ref(q, k, v, do, out.detach(), True, bi, hi, u)
        assert_out_close(cpu(out[bi, :, hi]), cpu(r["out"]), dt, cpu(r["bo"]), what="out")
        assert_close(cpu(lse[bi, hi]), cpu(r["lse"]), what="lse")
        for nm, got in (("dq", qd.grad), ("dk", kd.grad), ("dv", vd.grad)):
            assert_grad_close(cpu(got[bi, :, hi]), cpu(r[nm]), dt, "%s (%d, %d)" % (nm, bi, hi),
                              bound=cpu(r["b" + nm[1]]), want_faithful=cpu(r[nm + "_f"]))


def test_slice_ref_matches_oracle(cuda_dev):
    """The GPU fp32 slice reference used at full size equals the numpy oracle."""
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    q, k, v, do = (torch.randn(2, 700, 3, 64, generator=g, device=cuda_dev).to(torch.float16)
                   for _ in range(4))
    out, _ = _fwd(q, k, v, True)
    r = slice_ref(q, k, v, do, out, True, 1, 2, 2.0 ** -11)
    sl = lambda t: t[1:2, :, 2:3].float().permute(0, 2, 1, 3).cpu().numpy()
    ro, rl = R.attention_ref(sl(q), sl(k), sl(v), True)
    exact = R.attention_bwd_ref(sl(q), sl(k), sl(v), sl(do), True)
    faithful, bounds = R.attention_bwd_ref(sl(q), sl(k), sl(v), sl(do), True, o=sl(out),
                                           unit_roundoff=2.0 ** -11)
    bo = R.attention_out_bound(sl(q), sl(k), sl(v), True, 2.0 ** -11)
    close = lambda a, b_: np.testing.assert_allclose(a.detach().cpu().numpy(), b_[0, 0],
                                                     rtol=1e-4, atol=1e-5)
    close(r["out"], ro)
    close(r["lse"], rl)
    close(r["bo"], bo)
    for i, nm in enumerate(("dq", "dk", "dv")):
        close(r[nm], exact[i])
        close(r[nm + "_f"], faithful[i])
        close(r["b" + nm[1]], bounds[i])
