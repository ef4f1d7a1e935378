"""The oracle's softcap path against torch autograd through a direct statement of FA2's
definition: scores = c tanh(scale q k^T / c), masked, unit-scale softmax, P V.  The
reference has no softcap (interface.py:29-30), so this pins the oracle's forward, LSE
and hand-derived backward (dS times 1 - tanh^2) on small cases."""
import numpy as np
import pytest
import torch

from oracle import attention_ref as R


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("window", [(-1, -1), (3, -1), (2, 1)])
@pytest.mark.parametrize("cap,scale", [(0.7, 0.4), (5.0, 0.25), (30.0, 1.0)])
def test_softcap_oracle_matches_autograd(causal, window, cap, scale):
    g = np.random.default_rng(7)
    m, n, d = 7, 9, 16
    q = g.standard_normal((1, 4, m, d))
    k = g.standard_normal((1, 2, n, d))
    v = g.standard_normal((1, 2, n, d))
    do = g.standard_normal((1, 4, m, d))
    qt, kt, vt = (torch.tensor(x, requires_grad=True) for x in (q, k, v))
    ke, ve = kt.repeat_interleave(2, 1), vt.repeat_interleave(2, 1)
    s = cap * torch.tanh(torch.einsum("bhqd,bhkd->bhqk", qt, ke) * scale / cap)
    vis = R.visible_mask(m, n, causal, window)
    if vis is not None:
        s = s.masked_fill(~torch.tensor(vis), -float("inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.softmax(s, -1) @ ve
    o.backward(torch.tensor(do))
    out, ref_lse = R.attention_ref(q, k, v, causal, scale=scale, window=window, softcap=cap)
    np.testing.assert_allclose(out, o.detach().numpy(), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(ref_lse, lse.detach().numpy(), rtol=1e-5, atol=1e-6)
    dq, dk, dv = R.attention_bwd_ref(q, k, v, do, causal, scale=scale, window=window,
                                     softcap=cap)
    for got, want in ((dq, qt.grad), (dk, kt.grad), (dv, vt.grad)):
        np.testing.assert_allclose(got, want.numpy(), rtol=1e-5, atol=1e-6)


def test_softcap_zero_is_the_plain_oracle():
    g = np.random.default_rng(8)
    q, k, v = (g.standard_normal((1, 2, 6, 8)) for _ in range(3))
    a = R.attention_ref(q, k, v, True)
    b = R.attention_ref(q, k, v, True, softcap=0.0)
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
