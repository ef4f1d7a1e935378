"""Dense varlen (FA2's flash_attn_varlen_func over packed sequences) forward and backward,
checked sequence by sequence against the oracle's dense attention on that sequence alone
(its own bottom-right causal / window alignment), at the rounding bounds of the dense
tests.  No reference counterpart: the reference's dense API takes equal-length batches."""
import numpy as np
import pytest
import torch

import tilelang_fa_v100 as fa
from helpers import assert_close, assert_grad_close, assert_out_close, bwd_refs, unit_roundoff
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu

# (q_lens, k_lens, H, Hk, D, causal, window, softcap, dtype)
CASES = [
    ([100, 1, 513, 64], [100, 1, 513, 64], 4, 2, 128, True, (-1, -1), 0.0, torch.bfloat16),
    ([50, 200, 77], [120, 200, 300], 4, 4, 64, True, (-1, -1), 0.0, torch.float16),  # prefix
    ([300, 129], [260, 400], 2, 1, 256, False, (-1, -1), 0.0, torch.bfloat16),
    ([200, 90], [100, 90], 2, 2, 128, True, (-1, -1), 0.0, torch.float16),  # rows with no key
    ([10, 64, 40], [0, 64, 40], 2, 2, 128, True, (-1, -1), 0.0, torch.bfloat16),  # no keys at all
    ([400, 130], [400, 200], 4, 2, 128, True, (64, -1), 5.0, torch.bfloat16),  # window + softcap
    ([257, 3], [257, 3], 2, 1, 64, False, (-1, -1), 0.0, torch.float16),
    ([333, 150], [400, 150], 4, 2, 256, True, (100, 20), 3.0, torch.bfloat16),  # D = 256 EXT
    ([190, 70, 260], [190, 300, 260], 8, 2, 64, False, (-1, 40), 1.5, torch.float16),
]


def _ids(c):
    return "q%s-k%s-H%d-%d-D%d-%s-w%s-c%s" % ("_".join(map(str, c[0])), "_".join(map(str, c[1])),
                                            c[2], c[3], c[4], c[5], c[6][0], c[7])


def _inputs(case, seed=61):
    q_lens, k_lens, h, hk, d, causal, window, cap, dt = case
    g = torch.Generator().manual_seed(seed)
    mk = lambda n, heads: torch.randn((n, heads, d), generator=g).to(dt)
    tq, tk = sum(q_lens), sum(k_lens)
    cu = lambda ls: torch.tensor(np.concatenate([[0], np.cumsum(ls)]), dtype=torch.int32)
    return mk(tq, h), mk(tk, hk), mk(tk, hk), mk(tq, h), cu(q_lens), cu(k_lens)


def _seq(x, a, b):
    """rows [a, b) of a packed [total, heads, D] tensor as oracle [1, heads, L, D]"""
    return x[a:b].float().numpy().transpose(1, 0, 2)[None]


def _unseq(y):
    return np.asarray(y)[0].transpose(1, 0, 2)


@pytest.mark.parametrize("case", CASES, ids=_ids)
def test_varlen_forward_vs_oracle(cuda_dev, case):
    q_lens, k_lens, h, hk, d, causal, window, cap, dt = case
    q, k, v, _, cq, ck = _inputs(case)
    out, lse, _ = fa.tilelang_flash_attn_varlen_func(
        q.to(cuda_dev), k.to(cuda_dev), v.to(cuda_dev), cq.to(cuda_dev), ck.to(cuda_dev),
        max(q_lens), max(k_lens), causal=causal, window_size=window, softcap=cap,
        return_attn_probs=True)
    torch.cuda.synchronize()
    out, lse = out.float().cpu().numpy(), lse.cpu().numpy()
    for s in range(len(q_lens)):
        qa, qb, ka, kb = int(cq[s]), int(cq[s + 1]), int(ck[s]), int(ck[s + 1])
        if qb == qa:
            continue
        args = (_seq(q, qa, qb), _seq(k, ka, kb), _seq(v, ka, kb), causal)
        kw = dict(window=window, softcap=cap)
        ro, rl = R.attention_ref(*args, **kw)
        bound = R.attention_out_bound(*args, unit_roundoff(dt), **kw)
        assert_out_close(out[qa:qb], _unseq(ro), dt, _unseq(bound), what="out seq %d" % s)
        assert_close(lse[:, qa:qb], rl[0], what="lse seq %d" % s)


@pytest.mark.parametrize("deterministic", [False, True])
@pytest.mark.parametrize("case", CASES, ids=_ids)
def test_varlen_backward_vs_oracle(cuda_dev, case, deterministic):
    q_lens, k_lens, h, hk, d, causal, window, cap, dt = case
    q, k, v, do, cq, ck = _inputs(case)
    qd, kd, vd = (x.to(cuda_dev).requires_grad_(True) for x in (q, k, v))
    out = fa.tilelang_flash_attn_varlen_func(qd, kd, vd, cq.to(cuda_dev), ck.to(cuda_dev),
                                             max(q_lens), max(k_lens), causal=causal,
                                             window_size=window, softcap=cap,
                                             deterministic=deterministic)
    out.backward(do.to(cuda_dev))
    torch.cuda.synchronize()
    got = [x.grad.float().cpu().numpy() for x in (qd, kd, vd)]
    o_all = out.detach().float().cpu()
    for s in range(len(q_lens)):
        qa, qb, ka, kb = int(cq[s]), int(cq[s + 1]), int(ck[s]), int(ck[s + 1])
        rows = (slice(qa, qb), slice(ka, kb), slice(ka, kb))
        if qb == qa or kb == ka:
            # nothing attends: every gradient row of the sequence is zero
            for g_, r_ in zip(got, rows):
                assert not np.any(g_[r_]), "seq %d: gradients of an empty attention" % s
            continue
        args = (_seq(q, qa, qb), _seq(k, ka, kb), _seq(v, ka, kb), _seq(do, qa, qb), causal)
        kw = dict(window=window, softcap=cap)
        exact, faithful, bounds = bwd_refs(args, _seq(o_all, qa, qb), unit_roundoff(dt), **kw)
        for g_, r_, want, want_f, bnd, w in zip(got, rows, exact, faithful, bounds,
                                                ("dq", "dk", "dv")):
            assert_grad_close(g_[r_], _unseq(want), dt, "%s seq %d" % (w, s),
                              bound=_unseq(bnd), want_faithful=_unseq(want_f))


def test_varlen_equal_lengths_match_dense(cuda_dev):
    """Equal-length packed sequences: the same values as the dense call on [B, S, H, D]
    within the rounding bound (different kernels, so not bit-identical)."""
    b, s_, h, d = 3, 300, 4, 128
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn((b, s_, h, d), generator=g).to(torch.bfloat16).to(cuda_dev)
               for _ in range(3))
    dense = fa.tilelang_flash_attn_func(q, k, v, causal=True)
    cu = torch.arange(0, (b + 1) * s_, s_, dtype=torch.int32, device=cuda_dev)
    packed = fa.tilelang_flash_attn_varlen_func(q.reshape(-1, h, d), k.reshape(-1, h, d),
                                                v.reshape(-1, h, d), cu, cu, s_, s_, causal=True)
    torch.cuda.synchronize()
    diff = (packed.reshape(b, s_, h, d).float() - dense.float()).abs().max().item()
    assert diff <= 2 ** -6, diff


@pytest.mark.parametrize("deterministic", [False, True])
def test_varlen_many_short_sequences(cuda_dev, deterministic):
    """70 packed sequences of 1-60 tokens (prefix keys too): the forward's item scan over
    sequences crosses two 32-sequence chunks and the backward grids span 70 batch
    entries, most of them shorter than one tile."""
    rng = np.random.default_rng(72)
    q_lens = [int(x) for x in rng.integers(1, 61, size=70)]
    k_lens = [ql + int(x) for ql, x in zip(q_lens, rng.integers(0, 30, size=70))]
    case = (q_lens, k_lens, 4, 2, 64, True, (-1, -1), 0.0, torch.float16)
    q, k, v, do, cq, ck = _inputs(case, seed=73)
    qd, kd, vd = (x.to(cuda_dev).requires_grad_(True) for x in (q, k, v))
    out, lse, _ = fa.tilelang_flash_attn_varlen_func(qd, kd, vd, cq.to(cuda_dev), ck.to(cuda_dev),
                                                     max(q_lens), max(k_lens), causal=True,
                                                     deterministic=deterministic,
                                                     return_attn_probs=True)
    out.backward(do.to(cuda_dev))
    torch.cuda.synchronize()
    o_all, lse = out.detach().float().cpu(), lse.detach().cpu().numpy()
    got = [x.grad.float().cpu().numpy() for x in (qd, kd, vd)]
    dt = torch.float16
    for s in range(0, 70, 3):  # every third sequence: both chunks of the scan and the tail
        qa, qb, ka, kb = int(cq[s]), int(cq[s + 1]), int(ck[s]), int(ck[s + 1])
        args = (_seq(q, qa, qb), _seq(k, ka, kb), _seq(v, ka, kb), True)
        ro, rl = R.attention_ref(*args)
        bound = R.attention_out_bound(*args, unit_roundoff(dt))
        assert_out_close(o_all[qa:qb].numpy(), _unseq(ro), dt, _unseq(bound), what="out seq %d" % s)
        assert_close(lse[:, qa:qb], rl[0], what="lse seq %d" % s)
        bargs = args[:3] + (_seq(do, qa, qb), True)
        exact, faithful, bounds = bwd_refs(bargs, _seq(o_all, qa, qb), unit_roundoff(dt))
        rows = (slice(qa, qb), slice(ka, kb), slice(ka, kb))
        for g_, r_, want, want_f, bnd, w in zip(got, rows, exact, faithful, bounds,
                                                ("dq", "dk", "dv")):
            assert_grad_close(g_[r_], _unseq(want), dt, "%s seq %d" % (w, s),
                              bound=_unseq(bnd), want_faithful=_unseq(want_f))


def test_empty_inputs_give_the_fully_masked_result(cuda_dev):
    """No key at all (dense Skv = 0, varlen total_k = 0) gives the library's fully masked
    rows -- out 0, lse -inf, zero gradients -- and no rows gives empty results, instead of
    handing the C ABI the null data pointers of empty tensors."""
    mk = lambda *s: torch.randn(*s, device=cuda_dev, dtype=torch.float16).requires_grad_(True)
    q, k, v = mk(2, 5, 2, 64), mk(2, 0, 2, 64), mk(2, 0, 2, 64)
    out, lse, _ = fa.tilelang_flash_attn_func(q, k, v, causal=True, return_attn_probs=True)
    out.sum().backward()
    assert not out.any() and torch.isneginf(lse).all() and not q.grad.any()
    q0 = mk(2, 0, 2, 64)
    out0 = fa.tilelang_flash_attn_func(q0, mk(2, 7, 2, 64), mk(2, 7, 2, 64))
    assert out0.shape == (2, 0, 2, 64)
    cq = torch.tensor([0, 3, 5], dtype=torch.int32, device=cuda_dev)
    ck = torch.zeros(3, dtype=torch.int32, device=cuda_dev)
    qv, kv_, vv = mk(5, 2, 64), mk(0, 2, 64), mk(0, 2, 64)
    out, lse, _ = fa.tilelang_flash_attn_varlen_func(qv, kv_, vv, cq, ck, 3, 0, causal=True,
                                                     return_attn_probs=True)
    out.sum().backward()
    assert not out.any() and torch.isneginf(lse).all() and not qv.grad.any()
