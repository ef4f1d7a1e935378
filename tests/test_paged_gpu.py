"""Paged (vLLM layout) prefill on the GPU against the pinned CPU oracle and the
reference's golden vectors: GQA ratios, chunked prefill, scattered pages, varlen."""
import numpy as np
import pytest
import torch

import tilelang_fa_v100 as fa
from helpers import assert_close, assert_out_close, golden, golden_names, max_abs, unit_roundoff
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu


def _run(cuda_dev, q, kc, vc, bt, sl, qsl, pkl, causal, page, **kw):
    t = lambda x: torch.as_tensor(x).to(cuda_dev)
    out, lse = fa.tilelang_paged_forward(t(q), t(kc), t(vc), t(bt), t(sl), t(qsl), t(pkl),
                                         block_size=page, num_kv_heads=kc.shape[2],
                                         causal=causal, **kw)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy()


@pytest.mark.parametrize("name", golden_names("paged_") + golden_names("decode_"))
def test_golden_paged(cuda_dev, name):
    g = golden(name)
    out, lse = _run(cuda_dev, g["q_flat"], g["k_cache"], g["v_cache"], g["block_table"],
                    g["seq_lens"], g["query_start_loc"], g["prefix_kv_lens"], bool(g["causal"]), 16)
    ref_out, ref_lse = R.paged_prefill_ref(g["q_flat"], g["k_cache"], g["v_cache"],
                                           g["block_table"], g["seq_lens"], g["query_start_loc"],
                                           g["prefix_kv_lens"], causal=bool(g["causal"]))
    assert_close(out, ref_out, what=name + " out")
    assert_close(lse, ref_lse, what=name + " lse")
    assert max_abs(out, g["out"].astype(np.float32)) < 1e-2  # the reference's own bar


def _varlen_case(seed, q_lens, kv_lens, h, hkv, d, page, dtype, shuffle=True):
    rng = np.random.default_rng(seed)
    bsz = len(q_lens)
    pps = [-(-n // page) for n in kv_lens]
    total = sum(pps) + 3  # a few unused pages
    perm = rng.permutation(total) if shuffle else np.arange(total)
    max_blocks = max(pps) + 1
    bt = np.zeros((bsz, max_blocks), np.int32)
    c = 0
    for b in range(bsz):
        bt[b, :pps[b]] = perm[c:c + pps[b]]
        c += pps[b]
    npdt = np.float16
    kc = rng.standard_normal((total, page, hkv, d)).astype(npdt)
    vc = rng.standard_normal((total, page, hkv, d)).astype(npdt)
    q = rng.standard_normal((sum(q_lens), h, d)).astype(npdt)
    qsl = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    sl = np.array(kv_lens, np.int32)
    pkl = (sl - np.array(q_lens)).astype(np.int32)
    tq = torch.from_numpy(q).to(dtype)
    tk = torch.from_numpy(kc).to(dtype)
    tv = torch.from_numpy(vc).to(dtype)
    return tq, tk, tv, bt, sl, qsl, pkl


PAGED_CASES = [
    # q_lens, kv_lens, H, Hkv, D, page, dtype, causal
    ([64, 1, 200, 33], [64, 50, 450, 33], 8, 2, 128, 16, torch.float16, True),
    ([128, 128], [128, 300], 32, 8, 128, 16, torch.bfloat16, True),
    ([100, 7], [100, 7], 16, 1, 64, 32, torch.float16, True),
    ([77, 130], [77, 130], 4, 4, 128, 64, torch.bfloat16, False),
    ([40, 40], [40, 200], 16, 2, 256, 16, torch.float16, True),
    ([300], [1000], 8, 8, 64, 128, torch.bfloat16, True),
    ([96, 0, 31], [96, 10, 31], 12, 4, 128, 16, torch.float16, True),  # an empty query chunk
]


@pytest.mark.parametrize("case", PAGED_CASES, ids=lambda c: "H%d-Hkv%d-D%d-p%d-%s" % (c[2], c[3], c[4], c[5], c[7]))
def test_varlen_paged_vs_oracle(cuda_dev, case):
    q_lens, kv_lens, h, hkv, d, page, dt, causal = case
    q, kc, vc, bt, sl, qsl, pkl = _varlen_case(hash(str(case)) % 1000, q_lens, kv_lens, h, hkv,
                                               d, page, dt)
    out, lse = _run(cuda_dev, q, kc, vc, bt, sl, qsl, pkl, causal, page)
    ref_out, ref_lse, bound = R.paged_prefill_ref(q.float().numpy(), kc.float().numpy(),
                                                  vc.float().numpy(), bt, sl, qsl, pkl,
                                                  causal=causal, unit_roundoff=unit_roundoff(dt))
    assert_out_close(out, ref_out, dt, bound, what="out")
    assert_close(lse, ref_lse, what="lse")


@pytest.mark.parametrize("swq,swk", [(64, -1), (-1, 48), (40, 40)])
def test_sliding_window(cuda_dev, swq, swk):
    q, kc, vc, bt, sl, qsl, pkl = _varlen_case(11, [300], [300], 8, 2, 128, 16, torch.float16)
    out, lse = _run(cuda_dev, q, kc, vc, bt, sl, qsl, pkl, True, 16, sliding_window_q=swq,
                    sliding_window_k=swk)
    ref_out, ref_lse = R.paged_prefill_ref(q.float().numpy(), kc.float().numpy(),
                                           vc.float().numpy(), bt, sl, qsl, pkl, causal=True,
                                           sliding_window_q=swq, sliding_window_k=swk)
    assert_close(out, ref_out, what="out")
    assert_close(lse, ref_lse, what="lse")


def test_out_tensor_written_in_place(cuda_dev):
    q, kc, vc, bt, sl, qsl, pkl = _varlen_case(5, [50], [80], 4, 2, 64, 16, torch.float16)
    t = lambda x: torch.as_tensor(x).to(cuda_dev)
    out = torch.full(q.shape, 7.0, dtype=q.dtype, device=cuda_dev)
    ret, _ = fa.tilelang_paged_forward(t(q), t(kc), t(vc), t(bt), t(sl), t(qsl), t(pkl), out=out)
    assert ret is out
    ref_out, _ = R.paged_prefill_ref(q.float().numpy(), kc.float().numpy(), vc.float().numpy(),
                                     bt, sl, qsl, pkl, causal=True)
    assert_close(out.float().cpu().numpy(), ref_out, what="out")


def test_benchmark_config_sampled(cuda_dev):
    """BASELINE paged config (16 x 1024 tokens, 32/8 heads, D 128, shuffled pages) at full
    size, checked on two sequences against the oracle."""
    rng = np.random.default_rng(0)
    n_seq, L, h, hkv, d = 16, 1024, 32, 8, 128
    kc = torch.from_numpy(rng.standard_normal((1024, 16, hkv, d)).astype(np.float16))
    vc = torch.from_numpy(rng.standard_normal((1024, 16, hkv, d)).astype(np.float16))
    bt = rng.permutation(1024).astype(np.int32).reshape(n_seq, 64)
    q = torch.from_numpy(rng.standard_normal((n_seq * L, h, d)).astype(np.float16))
    qsl = np.arange(0, n_seq * L + 1, L).astype(np.int32)
    sl = np.full(n_seq, L, np.int32)
    pkl = np.zeros(n_seq, np.int32)
    out, lse = _run(cuda_dev, q, kc, vc, bt, sl, qsl, pkl, True, 16)
    for b in (0, 13):
        sel = slice(b * L, (b + 1) * L)
        ro, rl = R.paged_prefill_ref(q[sel].float().numpy(), kc.float().numpy(),
                                     vc.float().numpy(), bt[b:b + 1], sl[b:b + 1],
                                     np.array([0, L], np.int32), pkl[b:b + 1], causal=True)
        assert_close(out[sel], ro, what="out seq %d" % b)
        assert_close(lse[:, sel], rl, what="lse seq %d" % b)


def test_seq_len_past_block_table_is_clamped_and_reported(cuda_dev):
    """Paged prefill with seq_lens[b] beyond max_blocks * page_size: keys are clamped to
    the mapped pages and device error 4 is recorded (non-causal, so every mapped key is
    visible to every query row)."""
    from tilelang_fa_v100 import _ext
    q, kc, vc, bt, sl, qsl, pkl = _varlen_case(93, [20, 33], [20, 200], 8, 2, 128, 16,
                                               torch.float16)
    bt = bt[:, :-1].copy()                      # drop the spare column: row 1 maps 208 keys
    cap = bt.shape[1] * 16
    claimed = sl.copy()
    claimed[1] = cap + 64
    _ext.read_device_error(clear=True)
    out, lse = _run(cuda_dev, q, kc, vc, bt, claimed, qsl, np.zeros_like(pkl), False, 16)
    code, _, _ = _ext.read_device_error(clear=True)
    assert code == 4
    clamped = np.minimum(claimed, cap).astype(np.int32)
    ref_out, ref_lse = R.paged_prefill_ref(q.float().numpy(), kc.float().numpy(),
                                           vc.float().numpy(), bt, clamped, qsl,
                                           np.zeros_like(pkl), causal=False)
    assert_close(out, ref_out, what="out")
    assert_close(lse, ref_lse, what="lse")


def test_many_sequences_cross_the_item_scan(cuda_dev):
    """70 ragged sequences: the persistent kernel finds an item's sequence with a
    warp-wide scan 32 sequences at a time, so this crosses two chunk boundaries (and
    holds empty query chunks and single-token ones)."""
    rng = np.random.default_rng(70)
    q_lens = [int(x) for x in rng.integers(0, 40, size=70)]
    q_lens[5], q_lens[40] = 0, 1
    kv_lens = [ql + int(x) for ql, x in zip(q_lens, rng.integers(0, 90, size=70))]
    kv_lens = [max(1, n) for n in kv_lens]
    q, kc, vc, bt, sl, qsl, pkl = _varlen_case(71, q_lens, kv_lens, 8, 2, 128, 16, torch.float16)
    out, lse = _run(cuda_dev, q, kc, vc, bt, sl, qsl, pkl, True, 16)
    ref_out, ref_lse, bound = R.paged_prefill_ref(q.float().numpy(), kc.float().numpy(),
                                                  vc.float().numpy(), bt, sl, qsl, pkl,
                                                  causal=True,
                                                  unit_roundoff=unit_roundoff(torch.float16))
    assert_out_close(out, ref_out, torch.float16, bound, what="out")
    assert_close(lse, ref_lse, what="lse")
