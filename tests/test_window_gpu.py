"""Dense sliding window (FA2 window_size) through tilelang_flash_attn_func, forward and
backward, against the oracle's visible_mask.  The reference accepts window_size and
ignores it (interface.py:33); this is the next-row extension the C-ABI's window_q /
window_k fields carry.  Bars: the rounding bounds of the same tests without a window."""
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


# (batch, Sq, Skv, H, Hk, D, causal, window_size, dtype)
CASES = [
    (1, 1000, 1000, 4, 2, 128, True, (256, -1), torch.bfloat16),   # causal sliding window
    (1, 700, 900, 2, 2, 128, False, (100, 50), torch.float16),     # both sides, Sq < Skv
    (1, 1300, 1000, 2, 2, 128, True, (300, -1), torch.bfloat16),   # Sq > Skv: rows with no key
    (1, 600, 300, 2, 2, 128, False, (-1, 5), torch.float16),       # right side only, empty rows
    (2, 600, 600, 4, 4, 64, True, (64, -1), torch.float16),        # D = 64
    (1, 500, 500, 2, 1, 256, False, (128, 128), torch.bfloat16),   # D = 256, persistent kernel
    (1, 3300, 3300, 2, 2, 256, False, (-1, 200), torch.bfloat16),  # D = 256, one CTA per item
]


def _inputs(case):
    b, sq, skv, h, hk, d, causal, window, dt = case
    return (_rand((b, sq, h, d), dt, 41), _rand((b, skv, hk, d), dt, 42),
            _rand((b, skv, hk, d), dt, 43), _rand((b, sq, h, d), dt, 44))


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c[:8])))
def test_window_forward_vs_oracle(cuda_dev, case):
    b, sq, skv, h, hk, d, causal, window, dt = case
    q, k, v, _ = _inputs(case)
    out, lse, _ = fa.tilelang_flash_attn_func(q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev),
                                              causal=causal, window_size=window,
                                              return_attn_probs=True)
    torch.cuda.synchronize()
    args = (_to_bhsd(q), _to_bhsd(k), _to_bhsd(v), causal)
    ref_out, ref_lse = R.attention_ref(*args, window=window)
    bound = R.attention_out_bound(*args, unit_roundoff(dt), window=window)
    assert_out_close(_to_bhsd(out), ref_out, dt, bound, what="out")
    assert_close(lse.cpu().numpy(), ref_lse, what="lse")


@pytest.mark.parametrize("deterministic", [False, True])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c[:8])))
def test_window_backward_vs_oracle(cuda_dev, case, deterministic):
    b, sq, skv, h, hk, d, causal, window, dt = case
    q, k, v, do = _inputs(case)
    qd, kd, vd = (x.to(cuda_dev).requires_grad_(True) for x in (q, k, v))
    out = fa.tilelang_flash_attn_func(qd, kd, vd, causal=causal, window_size=window,
                                      deterministic=deterministic)
    out.backward(do.to(cuda_dev))
    torch.cuda.synchronize()
    args = (_to_bhsd(q), _to_bhsd(k), _to_bhsd(v), _to_bhsd(do), causal)
    exact, faithful, bounds = bwd_refs(args, _to_bhsd(out), unit_roundoff(dt), window=window)
    for got, want, want_f, bnd, w in zip((qd.grad, kd.grad, vd.grad), exact, faithful, bounds,
                                         ("dq", "dk", "dv")):
        assert_grad_close(_to_bhsd(got), want, dt, w, bound=bnd, want_faithful=want_f)


def test_default_window_is_the_unwindowed_call(cuda_dev):
    q, k, v, _ = _inputs((1, 900, 900, 2, 2, 128, True, None, torch.bfloat16))
    q, k, v = q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev)
    a = fa.tilelang_flash_attn_func(q, k, v, causal=True)
    b_ = fa.tilelang_flash_attn_func(q, k, v, causal=True, window_size=(-1, -1))
    c = fa.tilelang_flash_attn_func(q, k, v, causal=True, window_size=(2000, -1))  # covers all
    assert torch.equal(a, b_) and torch.equal(a, c)
