"""The oracle's rounding bounds on the CPU: an emulation that rounds exactly the operands a
FlashAttention kernel rounds (P before P V and P^T dO, dS before dS K and dS^T Q, and the
outputs) to fp16 / bf16 stays inside them, and the bound is not vacuous (the rounded
result does differ from the fp32 one by a sizeable fraction of it)."""
import numpy as np
import pytest
import torch

from oracle import attention_ref as R


def _round(x, dtype):
    return torch.from_numpy(np.asarray(x, np.float32)).to(dtype).double().numpy()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [True, False])
def test_emulated_rounding_stays_inside_bound(dtype, causal):
    rng = np.random.default_rng(4)
    b, hq, hk, m, n, d = 1, 4, 2, 96, 130, 64
    q, k, v, do = (_round(rng.standard_normal(s), dtype) for s in
                   ((b, hq, m, d), (b, hk, n, d), (b, hk, n, d), (b, hq, m, d)))
    u = R.UNIT_ROUNDOFF[str(dtype).split(".")[-1]]
    scale = d ** -0.5
    out, _, p = R.attention_ref(q, k, v, causal, return_p=True)
    ve, ke = (np.repeat(x, hq // hk, axis=1) for x in (v, k))
    out_q = _round(np.einsum("bhqk,bhkd->bhqd", _round(p, dtype), ve), dtype)
    bo = R.attention_out_bound(q, k, v, causal, u)
    err = np.abs(out_q - out)
    assert (err <= 1e-6 + bo).all()
    assert err.max() > 0.05 * bo.max()  # the emulated rounding uses a good part of it

    o_q = out_q  # the backward is given the rounded output, as the kernels are
    (dq, dk, dv), (bq, bk, bv) = R.attention_bwd_ref(q, k, v, do, causal, o=o_q, unit_roundoff=u)
    dp = np.einsum("bhqd,bhkd->bhqk", do, ve)
    dsum = np.sum(do * o_q, axis=-1, keepdims=True)
    ds_q = _round(p * (dp - dsum) * scale, dtype)
    p_q = _round(p, dtype)
    g = hq // hk
    dq_q = _round(np.einsum("bhqk,bhkd->bhqd", ds_q, ke), dtype)
    dk_q = _round(np.einsum("bhqk,bhqd->bhkd", ds_q, q).reshape(b, hk, g, n, d).sum(2), dtype)
    dv_q = _round(np.einsum("bhqk,bhqd->bhkd", p_q, do).reshape(b, hk, g, n, d).sum(2), dtype)
    for got, want, bnd in ((dq_q, dq, bq), (dk_q, dk, bk), (dv_q, dv, bv)):
        e = np.abs(got - want)
        assert (e <= 1e-5 + bnd).all()
        assert e.max() > 0.05 * bnd.max()


def test_paged_and_decode_bounds_match_dense():
    """The paged / decode oracles' bounds equal the dense one on the same sequence."""
    rng = np.random.default_rng(6)
    hq, hk, n, d = 4, 2, 50, 64
    q = rng.standard_normal((1, hq, n, d)).astype(np.float32)
    k = rng.standard_normal((1, hk, n, d)).astype(np.float32)
    v = rng.standard_normal((1, hk, n, d)).astype(np.float32)
    kc, vc, bt = R.make_paged_cache(k, v, page_size=16, shuffle_seed=1)
    qf = q[0].transpose(1, 0, 2)
    sl = np.array([n], np.int32)
    qsl = np.array([0, n], np.int32)
    _, _, bp = R.paged_prefill_ref(qf, kc, vc, bt, sl, qsl, np.zeros(1, np.int32), causal=True,
                                   unit_roundoff=2.0 ** -8)
    bd = R.attention_out_bound(q, k, v, True, 2.0 ** -8)
    np.testing.assert_allclose(bp, bd[0].transpose(1, 0, 2), rtol=1e-6, atol=1e-9)
    _, _, bdec = R.decode_ref(qf[-1:], kc, vc, bt, sl, unit_roundoff=2.0 ** -8)
    np.testing.assert_allclose(bdec[0], bd[0, :, -1], rtol=1e-6, atol=1e-9)
