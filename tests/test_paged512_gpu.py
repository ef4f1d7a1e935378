"""Paged prefill at head_dim 512 (the reference's _BEST_CONFIGS[512] entry,
_kernels_paged.py:357-363, over the generic paged kernel :193-344) against the oracle:
GQA ratios that do and do not divide 128 rows, chunked prefill, scattered pages, page
sizes below and above the 128-key tile, an empty query chunk, the paged sliding window.
Each work item computes half of the output columns, so every case also checks that the
two halves agree on the softmax (one LSE, written by the first half)."""
import numpy as np
import pytest
import torch

import tilelang_fa_v100 as fa
from helpers import assert_close, assert_out_close, unit_roundoff
from oracle import attention_ref as R
from test_paged_gpu import _run, _varlen_case

pytestmark = pytest.mark.gpu

CASES = [
    # q_lens, kv_lens, H, Hkv, D, page, dtype, causal
    ([64, 1, 200, 33], [64, 50, 450, 33], 8, 2, 512, 16, torch.float16, True),
    ([128, 128], [128, 300], 8, 8, 512, 16, torch.bfloat16, True),
    ([77, 130], [77, 130], 4, 1, 512, 64, torch.bfloat16, False),
    ([300], [1000], 6, 2, 512, 128, torch.float16, True),     # G = 3: 42 tokens x 3 heads
    ([40, 0, 31], [40, 10, 31], 16, 1, 512, 32, torch.float16, True),  # empty query chunk
    ([257], [700], 4, 4, 512, 256, torch.bfloat16, True),    # pages larger than a KV tile
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "H%d-Hkv%d-p%d-%s-%s" % (
    c[2], c[3], c[5], str(c[6]).split(".")[-1], c[7]))
def test_paged512_vs_oracle(cuda_dev, case):
    q_lens, kv_lens, h, hkv, d, page, dt, causal = case
    q, kc, vc, bt, sl, qsl, pkl = _varlen_case(sum(q_lens) + 7 * h, q_lens, kv_lens, h, hkv, d,
                                               page, dt)
    out, lse = _run(cuda_dev, q, kc, vc, bt, sl, qsl, pkl, causal, page)
    ref_out, ref_lse, bound = R.paged_prefill_ref(q.float().numpy(), kc.float().numpy(),
                                                  vc.float().numpy(), bt, sl, qsl, pkl,
                                                  causal=causal, unit_roundoff=unit_roundoff(dt))
    assert_out_close(out, ref_out, dt, bound, what="out")
    assert_close(lse, ref_lse, what="lse")


@pytest.mark.parametrize("swq,swk", [(64, -1), (-1, 48), (150, 40)])
def test_paged512_sliding_window(cuda_dev, swq, swk):
    q, kc, vc, bt, sl, qsl, pkl = _varlen_case(12, [300], [420], 8, 2, 512, 16, torch.float16)
    out, lse = _run(cuda_dev, q, kc, vc, bt, sl, qsl, pkl, True, 16, sliding_window_q=swq,
                    sliding_window_k=swk)
    ref_out, ref_lse = R.paged_prefill_ref(q.float().numpy(), kc.float().numpy(),
                                           vc.float().numpy(), bt, sl, qsl, pkl, causal=True,
                                           sliding_window_q=swq, sliding_window_k=swk)
    assert_close(out, ref_out, what="out")
    assert_close(lse, ref_lse, what="lse")


def test_paged512_out_written_in_place(cuda_dev):
    q, kc, vc, bt, sl, qsl, pkl = _varlen_case(6, [50], [80], 4, 2, 512, 16, torch.bfloat16)
    t = lambda x: torch.as_tensor(x).to(cuda_dev)
    out = torch.full(q.shape, 7.0, dtype=q.dtype, device=cuda_dev)
    ret, _ = fa.tilelang_paged_forward(t(q), t(kc), t(vc), t(bt), t(sl), t(qsl), t(pkl), out=out)
    torch.cuda.synchronize()
    assert ret is out
    ref_out, _, bound = R.paged_prefill_ref(q.float().numpy(), kc.float().numpy(),
                                            vc.float().numpy(), bt, sl, qsl, pkl, causal=True,
                                            unit_roundoff=unit_roundoff(torch.bfloat16))
    assert_out_close(out.float().cpu().numpy(), ref_out, torch.bfloat16, bound, what="out")
    assert np.isfinite(out.float().cpu().numpy()).all()
