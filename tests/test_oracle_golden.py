"""Pins the CPU oracle (oracle/attention_ref.py) to golden vectors produced by the
reference's own PyTorch functions (tests/golden/make_golden.py)."""
import numpy as np
import pytest

from helpers import golden, golden_names, assert_close, max_abs
from oracle import attention_ref as R


@pytest.mark.parametrize("name", golden_names("dense_"))
def test_dense_forward_matches_reference(name):
    g = golden(name)
    out, lse = R.attention_ref(g["q"].astype(np.float32), g["k"].astype(np.float32),
                               g["v"].astype(np.float32), bool(g["causal"]))
    # the reference returns fp16 (pytorch_gqa_ref ends in .half()): compare at fp16 resolution
    assert_close(out, g["out"].astype(np.float32), atol=1e-3, rtol=1e-3, what=name + " out")
    assert_close(lse, g["lse"], atol=1e-4, rtol=1e-5, what=name + " lse")


@pytest.mark.parametrize("name", golden_names("dense_"))
def test_dense_backward_matches_reference_autograd(name):
    g = golden(name)
    dq, dk, dv = R.attention_bwd_ref(g["q"].astype(np.float32), g["k"].astype(np.float32),
                                     g["v"].astype(np.float32), g["do"], bool(g["causal"]))
    # reference autograd runs through the fp16 cast of the output: ~1e-3 relative
    for got, want, w in ((dq, g["dq"], "dq"), (dk, g["dk"], "dk"), (dv, g["dv"], "dv")):
        assert max_abs(got, want) < 2e-3 * max(1.0, float(np.abs(want).max())), (name, w)


@pytest.mark.parametrize("name", golden_names("paged_") + golden_names("decode_"))
def test_paged_matches_reference(name):
    g = golden(name)
    out, lse = R.paged_prefill_ref(g["q_flat"].astype(np.float32), g["k_cache"], g["v_cache"],
                                   g["block_table"], g["seq_lens"], g["query_start_loc"],
                                   g["prefix_kv_lens"], causal=bool(g["causal"]))
    assert_close(out, g["out"].astype(np.float32), atol=1e-3, rtol=1e-3, what=name + " out")
    assert_close(lse, g["lse"], atol=1e-4, rtol=1e-5, what=name + " lse")


@pytest.mark.parametrize("name", golden_names("paged_"))
def test_kv_cache_write_reproduces_reference_caches(name):
    """Writing each golden sequence's tokens through slot = block_table[pos // page] * page
    + pos % page rebuilds the cache the reference's make_paged_gqa laid out."""
    g = golden(name)
    kc, vc, bt, sl = g["k_cache"], g["v_cache"], g["block_table"], g["seq_lens"]
    page = kc.shape[1]
    k2, v2 = np.zeros_like(kc), np.zeros_like(vc)
    for b in range(bt.shape[0]):
        n = int(sl[b])
        key = R.gather_pages(kc, bt[b], n).transpose(1, 0, 2)   # [n, Hkv, D]
        val = R.gather_pages(vc, bt[b], n).transpose(1, 0, 2)
        slots = R.slots_for(bt[b], np.arange(n), page)
        slots[::7] = -1  # padding tokens are skipped ...
        R.kv_cache_write_ref(key, val, k2, v2, slots)
        slots = R.slots_for(bt[b], np.arange(n), page)[::7]
        R.kv_cache_write_ref(key[::7], val[::7], k2, v2, slots)  # ... and written later
        np.testing.assert_array_equal(R.gather_pages(k2, bt[b], n), R.gather_pages(kc, bt[b], n))
        np.testing.assert_array_equal(R.gather_pages(v2, bt[b], n), R.gather_pages(vc, bt[b], n))


def test_decode_ref_equals_prefill_with_one_query():
    g = golden("decode_gqa_16_4_d128")
    out, lse = R.decode_ref(g["q_flat"].astype(np.float32), g["k_cache"], g["v_cache"],
                            g["block_table"], g["seq_lens"])
    assert_close(out, g["out"].astype(np.float32), atol=1e-3, rtol=1e-3, what="decode out")
    assert_close(lse.T, g["lse"], atol=1e-4, rtol=1e-5, what="decode lse")


def test_make_paged_cache_roundtrip():
    rng = np.random.default_rng(0)
    k = rng.standard_normal((3, 2, 37, 8)).astype(np.float32)
    v = rng.standard_normal((3, 2, 37, 8)).astype(np.float32)
    kc, vc, bt = R.make_paged_cache(k, v, page_size=16, shuffle_seed=5)
    assert sorted(bt.ravel().tolist()) == list(range(bt.size))  # a permutation of pages
    for b in range(3):
        np.testing.assert_array_equal(R.gather_pages(kc, bt[b], 37), k[b])
        np.testing.assert_array_equal(R.gather_pages(vc, bt[b], 37), v[b])


def test_fully_masked_rows_are_zero_with_neg_inf_lse():
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 1, 6, 8))
    k = rng.standard_normal((1, 1, 3, 8))
    out, lse = R.attention_ref(q, k, k, causal=True)  # Sq > Skv: rows 0..2 see nothing
    assert np.all(out[0, 0, :3] == 0) and np.all(np.isneginf(lse[0, 0, :3]))
    assert np.all(np.isfinite(lse[0, 0, 3:]))


def test_visible_pairs_counts():
    assert R.visible_pairs(1, 1, 4, 4, True) == 10
    assert R.visible_pairs(1, 1, 2, 4, True) == 3 + 4
    assert R.visible_pairs(2, 3, 5, 7, False) == 2 * 3 * 5 * 7


def test_torch_restatement_matches_numpy_oracle():
    import torch
    from oracle import attention_ref_torch as RT
    g = golden("dense_nonsquare_causal")
    q, k, v, do = (torch.from_numpy(g[x]).float() for x in ("q", "k", "v", "do"))
    out, dq, dk, dv = RT.fwd_bwd(q, k, v, do, True)
    ro, _ = R.attention_ref(g["q"], g["k"], g["v"], True)
    rq, rk, rv = R.attention_bwd_ref(g["q"], g["k"], g["v"], g["do"], True)
    assert max_abs(out.numpy(), ro) < 1e-4
    for a, b_ in ((dq, rq), (dk, rk), (dv, rv)):
        assert max_abs(a.numpy(), b_) < 1e-3
