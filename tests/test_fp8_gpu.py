"""fp8 (e4m3) KV caches with per-tensor scales: the cache write quantises bit-exactly
like the oracle (x / scale, round to nearest even, saturate to +-448) and paged decode
over such caches matches the oracle run on the dequantised caches.  The reference has
no fp8 cache; this is the layout of vLLM's fp8 KV cache."""
import numpy as np
import pytest
import torch

import tilelang_fa_v100 as fa
from tilelang_fa_v100 import _ext
from tilelang_fa_v100.cache import write_kv_cache
from helpers import assert_close, assert_out_close, unit_roundoff
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu

K_SCALE, V_SCALE = 0.0125, 0.02


def _fp8_case(seed, lens, h, hkv, d, page, dtype):
    rng = np.random.default_rng(seed)
    pps = [-(-n // page) for n in lens]
    total = max(1, sum(pps))
    perm = rng.permutation(total)
    bt = np.zeros((len(lens), max(pps + [1]) + 1), np.int32)
    c = 0
    for b, n in enumerate(pps):
        bt[b, :n] = perm[c:c + n]
        c += n
    kraw = R.quantize_e4m3(rng.standard_normal((total, page, hkv, d)), K_SCALE)
    vraw = R.quantize_e4m3(rng.standard_normal((total, page, hkv, d)), V_SCALE)
    q = torch.from_numpy(rng.standard_normal((len(lens), h, d)).astype(np.float32)).to(dtype)
    return q, kraw, vraw, bt, np.array(lens, np.int32)


def _as_fp8(raw, dev):
    return torch.from_numpy(raw).to(dev).view(torch.float8_e4m3fn)


DECODE_FP8_CASES = [
    # lens, H, Hkv, D, page, dtype, splits
    ([100, 1, 17, 515, 4096], 32, 8, 128, 16, torch.bfloat16, 0),
    ([100, 1, 17, 515, 4096], 32, 8, 128, 16, torch.float16, 1),
    ([33, 700, 0], 16, 2, 128, 32, torch.bfloat16, 3),
    ([64, 129, 1000, 3000], 8, 1, 256, 16, torch.bfloat16, 0),
    ([300, 2000], 16, 4, 256, 64, torch.float16, 2),
    ([100, 1500], 8, 2, 512, 16, torch.bfloat16, 0),
]


@pytest.mark.parametrize("case", DECODE_FP8_CASES,
                         ids=lambda c: "H%d-Hkv%d-D%d-p%d-s%d" % (c[1], c[2], c[3], c[4], c[6]))
def test_decode_fp8_cache_vs_oracle(cuda_dev, case):
    lens, h, hkv, d, page, dt, splits = case
    q, kraw, vraw, bt, sl = _fp8_case(len(lens) * 11 + d, lens, h, hkv, d, page, dt)
    t = lambda x: torch.as_tensor(x).to(cuda_dev)
    lse = torch.empty(q.shape[0], q.shape[1], dtype=torch.float32, device=cuda_dev)
    out = _ext.decode(t(q), _as_fp8(kraw, cuda_dev), _as_fp8(vraw, cuda_dev), t(bt), t(sl), page,
                      hkv, d ** -0.5, num_splits=splits, lse=lse, k_scale=K_SCALE,
                      v_scale=V_SCALE)
    torch.cuda.synchronize()
    kd, vd = R.dequantize_e4m3(kraw, K_SCALE), R.dequantize_e4m3(vraw, V_SCALE)
    ref_out, ref_lse, bound = R.decode_ref(q.float().numpy(), kd, vd, bt, sl,
                                           unit_roundoff=unit_roundoff(dt))
    assert_out_close(out.float().cpu().numpy(), ref_out, dt, bound, what="out")
    assert_close(lse.cpu().numpy(), ref_lse, what="lse")


@pytest.mark.parametrize("q_scale", [3.0e5, 1.0e-6])
@pytest.mark.parametrize("d", [128, 256])
def test_decode_fp8_bf16_query_outside_f16_range(cuda_dev, q_scale, d):
    """Over fp8 caches a bf16 query enters f16 MMAs after a power-of-two scaling chosen
    per kv-head group.  Groups far above the f16 maximum (3e5) or below its normal range
    (1e-6), next to unscaled groups, give the oracle's result."""
    lens, h, hkv, page = [100, 1, 515, 2000], 32, 8, 16
    q, kraw, vraw, bt, sl = _fp8_case(5 + d, lens, h, hkv, d, page, torch.bfloat16)
    group = torch.arange(h) // (h // hkv)
    q = (q.float() * torch.where(group % 2 == 0, q_scale, 1.0)[None, :, None]).to(torch.bfloat16)
    t = lambda x: torch.as_tensor(x).to(cuda_dev)
    lse = torch.empty(q.shape[0], q.shape[1], dtype=torch.float32, device=cuda_dev)
    out = _ext.decode(t(q), _as_fp8(kraw, cuda_dev), _as_fp8(vraw, cuda_dev), t(bt), t(sl), page,
                      hkv, d ** -0.5, lse=lse, k_scale=K_SCALE, v_scale=V_SCALE)
    torch.cuda.synchronize()
    kd, vd = R.dequantize_e4m3(kraw, K_SCALE), R.dequantize_e4m3(vraw, V_SCALE)
    ref_out, ref_lse, bound = R.decode_ref(q.float().numpy(), kd, vd, bt, sl,
                                           unit_roundoff=unit_roundoff(torch.bfloat16))
    assert_out_close(out.float().cpu().numpy(), ref_out, torch.bfloat16, bound, what="out")
    assert_close(lse.cpu().numpy(), ref_lse, what="lse")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_kv_cache_write_fp8_is_bit_exact(cuda_dev, dtype):
    rng = np.random.default_rng(7)
    n, hkv, d, page, pages = 300, 8, 128, 16, 40
    key = torch.from_numpy(rng.standard_normal((n, hkv, d)).astype(np.float32) * 3).to(dtype)
    value = torch.from_numpy(rng.standard_normal((n, hkv, d)).astype(np.float32) * 3).to(dtype)
    key[0, 0, :4] = torch.tensor([1e4, -1e4, 5.0, 0.0]).to(dtype)  # saturates at +-448 x scale
    slots = rng.permutation(pages * page)[:n].astype(np.int64)
    slots[5] = -1  # padding token
    kc = torch.zeros(pages, page, hkv, d, dtype=torch.float8_e4m3fn, device=cuda_dev)
    vc = torch.zeros_like(kc)
    write_kv_cache(key.to(cuda_dev), value.to(cuda_dev), kc, vc, torch.from_numpy(slots).to(cuda_dev),
                   k_scale=K_SCALE, v_scale=V_SCALE)
    torch.cuda.synchronize()
    kr = np.zeros((pages, page, hkv, d), np.uint8)
    vr = np.zeros_like(kr)
    R.kv_cache_write_ref(R.quantize_e4m3(key.float().numpy(), K_SCALE),
                         R.quantize_e4m3(value.float().numpy(), V_SCALE), kr, vr, slots)
    np.testing.assert_array_equal(kc.view(torch.uint8).cpu().numpy(), kr)
    np.testing.assert_array_equal(vc.view(torch.uint8).cpu().numpy(), vr)


def test_fp8_write_then_decode_through_the_api(cuda_dev):
    """A serving step: new tokens quantised into fp8 caches, then decode over them."""
    rng = np.random.default_rng(9)
    lens, h, hkv, d, page = [40, 333, 1000], 16, 4, 128, 16
    pps = [-(-n // page) for n in lens]
    total = sum(pps)
    perm = rng.permutation(total)
    bt = np.zeros((len(lens), max(pps)), np.int32)
    c = 0
    for b, n in enumerate(pps):
        bt[b, :n] = perm[c:c + n]
        c += n
    keys = torch.from_numpy(rng.standard_normal((sum(lens), hkv, d)).astype(np.float32)).to(torch.bfloat16)
    vals = torch.from_numpy(rng.standard_normal((sum(lens), hkv, d)).astype(np.float32)).to(torch.bfloat16)
    slots = np.concatenate([R.slots_for(bt[b], np.arange(n), page) for b, n in enumerate(lens)])
    kc = torch.zeros(total, page, hkv, d, dtype=torch.float8_e4m3fn, device=cuda_dev)
    vc = torch.zeros_like(kc)
    write_kv_cache(keys.to(cuda_dev), vals.to(cuda_dev), kc, vc, torch.from_numpy(slots).to(cuda_dev),
                   k_scale=K_SCALE, v_scale=V_SCALE)
    q = torch.from_numpy(rng.standard_normal((len(lens), h, d)).astype(np.float32)).to(torch.bfloat16)
    t = lambda x: torch.as_tensor(x).to(cuda_dev)
    out = fa.tilelang_decode_forward(t(q), kc, vc, t(bt), t(np.array(lens, np.int32)),
                                     k_scale=K_SCALE, v_scale=V_SCALE)
    torch.cuda.synchronize()
    kd = R.dequantize_e4m3(kc.view(torch.uint8).cpu().numpy(), K_SCALE)
    vd = R.dequantize_e4m3(vc.view(torch.uint8).cpu().numpy(), V_SCALE)
    ref, _, bound = R.decode_ref(q.float().numpy(), kd, vd, bt, np.array(lens), unit_roundoff=2.0 ** -8)
    assert_out_close(out.float().cpu().numpy(), ref, torch.bfloat16, bound, what="out")


def test_fp8_cache_rejections(cuda_dev):
    q = torch.zeros(2, 4, 64, dtype=torch.bfloat16, device=cuda_dev)
    kc = torch.zeros(4, 16, 1, 64, dtype=torch.float8_e4m3fn, device=cuda_dev)
    bt = torch.zeros(2, 2, dtype=torch.int32, device=cuda_dev)
    sl = torch.tensor([3, 5], dtype=torch.int32, device=cuda_dev)
    with pytest.raises(NotImplementedError):  # fp8 rows of 64 dims are not built
        fa.tilelang_decode_forward(q, kc, kc, bt, sl, k_scale=0.1, v_scale=0.1)
    q = torch.zeros(2, 4, 128, dtype=torch.bfloat16, device=cuda_dev)
    kc = torch.zeros(4, 16, 1, 128, dtype=torch.float8_e4m3fn, device=cuda_dev)
    with pytest.raises(ValueError):  # scales must be positive
        fa.tilelang_decode_forward(q, kc, kc, bt, sl, k_scale=0.0, v_scale=0.1)
