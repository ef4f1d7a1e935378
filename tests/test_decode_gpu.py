"""Split-KV paged decode on the GPU against the pinned CPU oracle."""
import numpy as np
import pytest
import torch

import tilelang_fa_v100 as fa
from tilelang_fa_v100 import _ext
from helpers import assert_close, assert_out_close, golden, golden_names, max_abs, unit_roundoff
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu


def _case(seed, lens, h, hkv, d, page, dtype, extra_cols=2):
    rng = np.random.default_rng(seed)
    pps = [-(-n // page) for n in lens]
    total = max(1, sum(pps))
    perm = rng.permutation(total)
    bt = np.zeros((len(lens), max(pps + [1]) + extra_cols), np.int32)
    c = 0
    for b, n in enumerate(pps):
        bt[b, :n] = perm[c:c + n]
        c += n
    kc = torch.from_numpy(rng.standard_normal((total, page, hkv, d)).astype(np.float32)).to(dtype)
    vc = torch.from_numpy(rng.standard_normal((total, page, hkv, d)).astype(np.float32)).to(dtype)
    q = torch.from_numpy(rng.standard_normal((len(lens), h, d)).astype(np.float32)).to(dtype)
    return q, kc, vc, bt, np.array(lens, np.int32)


def _check(cuda_dev, q, kc, vc, bt, sl, page, num_splits=0):
    t = lambda x: torch.as_tensor(x).to(cuda_dev)
    lse = torch.empty(q.shape[0], q.shape[1], dtype=torch.float32, device=cuda_dev)
    out = _ext.decode(t(q), t(kc), t(vc), t(bt), t(sl), page, kc.shape[2],
                      _ext.default_scale(q.shape[-1]), num_splits=num_splits, lse=lse)
    torch.cuda.synchronize()
    ref_out, ref_lse, bound = R.decode_ref(q.float().numpy(), kc.float().numpy(),
                                           vc.float().numpy(), bt, sl,
                                           unit_roundoff=unit_roundoff(q.dtype))
    assert_out_close(out.float().cpu().numpy(), ref_out, q.dtype, bound, what="out")
    assert_close(lse.cpu().numpy(), ref_lse, what="lse")


@pytest.mark.parametrize("name", golden_names("decode_"))
def test_golden_decode(cuda_dev, name):
    g = golden(name)
    t = lambda x: torch.from_numpy(x).to(cuda_dev)
    out = fa.tilelang_decode_forward(t(g["q_flat"]), t(g["k_cache"]), t(g["v_cache"]),
                                     t(g["block_table"]), t(g["seq_lens"]))
    torch.cuda.synchronize()
    ref, _ = R.decode_ref(g["q_flat"], g["k_cache"], g["v_cache"], g["block_table"], g["seq_lens"])
    assert_close(out.float().cpu().numpy(), ref, what="out")
    assert max_abs(out.float().cpu().numpy(), g["out"].astype(np.float32)) < 1e-2


DECODE_CASES = [
    # lens, H, Hkv, D, page, dtype, splits
    ([100, 1, 17, 515, 4096], 32, 8, 128, 16, torch.bfloat16, 0),
    ([100, 1, 17, 515, 4096], 32, 8, 128, 16, torch.bfloat16, 1),
    ([100, 1, 17, 515, 4096], 32, 8, 128, 16, torch.float16, 3),
    ([33, 64, 700], 16, 1, 64, 16, torch.float16, 0),     # MQA, 16 q heads per kv head
    ([200, 300], 8, 8, 128, 32, torch.bfloat16, 0),       # MHA, page 32
    ([129, 1000], 24, 4, 64, 64, torch.bfloat16, 5),      # 6 q heads per kv head, page 64
    ([0, 50], 8, 2, 128, 16, torch.float16, 1),           # an empty sequence, single split
    ([0, 50], 8, 2, 128, 16, torch.float16, 4),           # an empty sequence, split path
    ([64, 129, 1000, 5000], 48, 3, 256, 16, torch.bfloat16, 0),  # D = 256, 16 q heads per kv head
    ([64, 129, 1000, 5000], 8, 1, 256, 16, torch.bfloat16, 0),   # D = 256 MQA 8:1 (reference synthetic row)
    ([300, 1, 0], 8, 1, 256, 16, torch.float16, 3),       # D = 256 MQA 8:1, explicit splits
    ([17, 4096], 16, 4, 256, 32, torch.bfloat16, 1),      # D = 256, 4 kv heads per CTA, direct
    ([2000], 8, 8, 256, 64, torch.float16, 0),            # D = 256 MHA, 8 kv heads in 2 CTAs
    ([64, 129, 1000, 3000], 16, 4, 512, 16, torch.bfloat16, 0),  # D = 512 (paged prefill's
    ([300, 1, 0], 8, 1, 512, 32, torch.float16, 3),       # companion), explicit splits, MQA
    ([17, 2000], 4, 4, 512, 16, torch.bfloat16, 1),       # D = 512 MHA, direct
]


@pytest.mark.parametrize("case", DECODE_CASES, ids=lambda c: "H%d-Hkv%d-D%d-p%d-s%d" % (c[1], c[2], c[3], c[4], c[6]))
def test_decode_vs_oracle(cuda_dev, case):
    lens, h, hkv, d, page, dt, splits = case
    q, kc, vc, bt, sl = _case(len(lens) * 7 + d, lens, h, hkv, d, page, dt)
    _check(cuda_dev, q, kc, vc, bt, sl, page, splits)


def test_benchmark_config_sampled(cuda_dev):
    """BASELINE decode config (256 sequences, L ~ U[512, 8192], 32/8 heads, D 128, bf16)
    at full size (inputs generated on the device); sampled sequences are checked
    against the oracle on their own gathered pages."""
    rng = np.random.default_rng(0)
    lens = rng.integers(512, 8193, size=256).astype(np.int32)
    pps = (lens + 15) // 16
    total = int(pps.sum())
    perm = rng.permutation(total).astype(np.int32)
    bt = np.zeros((256, int(pps.max())), np.int32)
    c = 0
    for b in range(256):
        bt[b, :pps[b]] = perm[c:c + pps[b]]
        c += pps[b]
    g = torch.Generator(device=cuda_dev).manual_seed(0)
    kc = torch.randn(total, 16, 8, 128, generator=g, device=cuda_dev).to(torch.bfloat16)
    vc = torch.randn(total, 16, 8, 128, generator=g, device=cuda_dev).to(torch.bfloat16)
    q = torch.randn(256, 32, 128, generator=g, device=cuda_dev).to(torch.bfloat16)
    out = fa.tilelang_decode_forward(q, kc, vc, torch.from_numpy(bt).to(cuda_dev),
                                     torch.from_numpy(lens).to(cuda_dev))
    torch.cuda.synchronize()
    for b in (0, 77, 255):
        idx = torch.from_numpy(bt[b, :pps[b]].astype(np.int64)).to(cuda_dev)
        kb = kc[idx].float().cpu().numpy()
        vb = vc[idx].float().cpu().numpy()
        ro, _, bnd = R.decode_ref(q[b:b + 1].float().cpu().numpy(), kb, vb,
                                  np.arange(pps[b], dtype=np.int32)[None], lens[b:b + 1],
                                  unit_roundoff=2.0 ** -8)
        assert_out_close(out[b:b + 1].float().cpu().numpy(), ro, torch.bfloat16, bnd,
                         what="seq %d" % b)


@pytest.mark.parametrize("num_splits", [0, 1, 3])
def test_seq_len_past_block_table_is_clamped_and_reported(cuda_dev, num_splits):
    """seq_lens[b] larger than the keys its block-table row maps (max_blocks * page): the
    kernels clamp it to the mapped keys (instead of counting zero-filled out-of-range
    loads as keys) and record device error 4."""
    q, kc, vc, bt, sl = _case(91, [40, 300], 8, 2, 128, 16, torch.bfloat16, extra_cols=0)
    cap = bt.shape[1] * 16
    claimed = sl.copy()
    claimed[1] = cap + 100  # sequence 1 claims 100 keys more than its row maps
    t = lambda x: torch.as_tensor(x).to(cuda_dev)
    _ext.read_device_error(clear=True)
    out = _ext.decode(t(q), t(kc), t(vc), t(bt), t(claimed), 16, kc.shape[2],
                      _ext.default_scale(q.shape[-1]), num_splits=num_splits)
    torch.cuda.synchronize()
    code, _, _ = _ext.read_device_error(clear=True)
    assert code == 4
    clamped = np.minimum(claimed, cap).astype(np.int32)
    ref_out, _, bound = R.decode_ref(q.float().numpy(), kc.float().numpy(), vc.float().numpy(),
                                     bt, clamped, unit_roundoff=unit_roundoff(q.dtype))
    assert_out_close(out.float().cpu().numpy(), ref_out, q.dtype, bound, what="out")
