"""FA2 softcap through tilelang_flash_attn_func, forward and backward, against the
oracle's softcapped attention (scores = c tanh(scale q k^T / c), unit-scale softmax, dS
times 1 - tanh^2).  The reference raises NotImplementedError for softcap != 0
(interface.py:29-30); this is the next-row extension the C-ABI's softcap field carries.
Bars: the rounding bounds of the same tests without a cap (the cap's own arithmetic is
fp32, a few units of 2^-23 of the cap)."""
import pytest
import torch

import tilelang_fa_v100 as fa
from helpers import assert_close, assert_grad_close, assert_out_close, bwd_refs, unit_roundoff
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu


def _rand(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32).to(dtype)


def _to_bhsd(x):
    return x.detach().float().cpu().permute(0, 2, 1, 3).numpy()


# (batch, Sq, Skv, H, Hk, D, causal, window_size, softcap, softmax_scale, dtype)
CASES = [
    (1, 1000, 1000, 4, 2, 128, True, (-1, -1), 5.0, None, torch.bfloat16),     # mild cap
    (1, 900, 900, 2, 2, 128, True, (-1, -1), 2.0, 0.3, torch.bfloat16),        # saturating
    (1, 700, 1100, 2, 2, 128, False, (-1, -1), 1.0, 0.25, torch.float16),      # Sq < Skv
    (1, 1300, 1000, 2, 1, 128, True, (-1, -1), 3.0, 0.2, torch.bfloat16),      # empty rows
    (1, 1000, 1000, 4, 4, 128, True, (200, -1), 4.0, 0.2, torch.float16),      # with a window
    (2, 600, 600, 4, 4, 64, True, (-1, -1), 1.5, 0.3, torch.float16),          # D = 64
    (1, 500, 500, 2, 1, 256, False, (-1, -1), 3.0, 0.15, torch.bfloat16),      # D = 256
    (1, 3300, 3300, 2, 2, 256, False, (-1, -1), 50.0, None, torch.bfloat16),   # D = 256, long
]


def _inputs(case):
    b, sq, skv, h, hk, d = case[:6]
    dt = case[-1]
    return (_rand((b, sq, h, d), dt, 51), _rand((b, skv, hk, d), dt, 52),
            _rand((b, skv, hk, d), dt, 53), _rand((b, sq, h, d), dt, 54))


def _scale(case):
    return case[9] if case[9] is not None else case[5] ** -0.5


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c[:10])))
def test_softcap_forward_vs_oracle(cuda_dev, case):
    b, sq, skv, h, hk, d, causal, window, cap, scale, dt = case
    q, k, v, _ = _inputs(case)
    out, lse, _ = fa.tilelang_flash_attn_func(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev),
                                              softmax_scale=scale, causal=causal,
                                              window_size=window, softcap=cap,
                                              return_attn_probs=True)
    torch.cuda.synchronize()
    args = (_to_bhsd(q), _to_bhsd(k), _to_bhsd(v), causal)
    kw = dict(scale=_scale(case), window=window, softcap=cap)
    ref_out, ref_lse = R.attention_ref(*args, **kw)
    bound = R.attention_out_bound(*args, unit_roundoff(dt), **kw)
    assert_out_close(_to_bhsd(out), ref_out, dt, bound, what="out")
    assert_close(lse.cpu().numpy(), ref_lse, what="lse")


@pytest.mark.parametrize("deterministic", [False, True])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c[:10])))
def test_softcap_backward_vs_oracle(cuda_dev, case, deterministic):
    b, sq, skv, h, hk, d, causal, window, cap, scale, dt = case
    q, k, v, do = _inputs(case)
    qd, kd, vd = (x.to(cuda_dev).requires_grad_(True) for x in (q, k, v))
    out = fa.tilelang_flash_attn_func(qd, kd, vd, softmax_scale=scale, causal=causal,
                                      window_size=window, softcap=cap,
                                      deterministic=deterministic)
    out.backward(do.to(cuda_dev))
    torch.cuda.synchronize()
    args = (_to_bhsd(q), _to_bhsd(k), _to_bhsd(v), _to_bhsd(do), causal)
    kw = dict(scale=_scale(case), window=window, softcap=cap)
    exact, faithful, bounds = bwd_refs(args, _to_bhsd(out), unit_roundoff(dt), **kw)
    for got, want, want_f, bnd, w in zip((qd.grad, kd.grad, vd.grad), exact, faithful, bounds,
                                         ("dq", "dk", "dv")):
        assert_grad_close(_to_bhsd(got), want, dt, w, bound=bnd, want_faithful=want_f)


def test_softcap_off_is_the_uncapped_call(cuda_dev):
    # 0 and negative values switch the cap off (FA2: softcap > 0 enables it)
    q, k, v, _ = _inputs((1, 900, 900, 2, 2, 128, torch.bfloat16))
    q, k, v = q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev)
    a = fa.tilelang_flash_attn_func(q, k, v, causal=True)
    b_ = fa.tilelang_flash_attn_func(q, k, v, causal=True, softcap=0.0)
    c = fa.tilelang_flash_attn_func(q, k, v, causal=True, softcap=-3.0)
    assert torch.equal(a, b_) and torch.equal(a, c)


def test_softcap_c_abi_rejects_bad_caps(cuda_dev):
    from tilelang_fa_v100 import _ext
    q = torch.zeros(1, 128, 2, 64, dtype=torch.float16, device=cuda_dev)
    for bad in (float("inf"), float("nan")):
        with pytest.raises(ValueError, match="invalid argument"):
            _ext.dense_forward(q, q, q, 0.125, False, (-1, -1), bad)
