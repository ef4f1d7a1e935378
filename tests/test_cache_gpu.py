"""Paged KV-cache write and the vLLM-style backend step on the GPU, against the CPU
oracle (bit-exact for the cache write, attention tolerances for the step)."""
import numpy as np
import pytest
import torch

from tilelang_fa_v100 import _ext
from tilelang_fa_v100.backend import AttentionMetadata, TileLangFAAttentionImpl
from tilelang_fa_v100.cache import write_kv_cache
from helpers import assert_close, assert_out_close, unit_roundoff
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu


def _rand(rng, shape, dtype):
    return torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).to(dtype)


CACHE_CASES = [
    # tokens, Hkv, D, page, pages, dtype
    (1, 1, 64, 16, 4, torch.float16),
    (37, 8, 128, 16, 40, torch.bfloat16),
    (1000, 2, 256, 32, 80, torch.float16),
    (513, 4, 64, 128, 8, torch.bfloat16),
    (300, 1, 128, 16, 40, torch.bfloat16),   # 256-byte rows: two rows per warp
    (77, 3, 64, 16, 10, torch.float16),      # 384-byte rows: 24 of 32 lanes busy
]


@pytest.mark.parametrize("case", CACHE_CASES, ids=lambda c: "T%d-Hkv%d-D%d-p%d" % c[:4])
def test_cache_write_bit_exact(cuda_dev, case):
    n, hkv, d, page, pages, dt = case
    rng = np.random.default_rng(n + d)
    slots = rng.permutation(pages * page)[:n].astype(np.int64)
    slots[rng.random(n) < 0.1] = -1  # padding tokens
    key, value = _rand(rng, (n, hkv, d), dt), _rand(rng, (n, hkv, d), dt)
    kc0, vc0 = _rand(rng, (pages, page, hkv, d), dt), _rand(rng, (pages, page, hkv, d), dt)
    kc, vc = kc0.to(cuda_dev), vc0.to(cuda_dev)
    write_kv_cache(key.to(cuda_dev), value.to(cuda_dev), kc, vc, torch.from_numpy(slots).to(cuda_dev))
    torch.cuda.synchronize()
    kr, vr = kc0.view(torch.int16).numpy().copy(), vc0.view(torch.int16).numpy().copy()
    R.kv_cache_write_ref(key.view(torch.int16).numpy(), value.view(torch.int16).numpy(), kr, vr, slots)
    np.testing.assert_array_equal(kc.cpu().view(torch.int16).numpy(), kr)
    np.testing.assert_array_equal(vc.cpu().view(torch.int16).numpy(), vr)


def test_cache_write_from_fused_qkv_view(cuda_dev):
    """key / value as strided slices of a [T, H + 2 Hkv, D] projection output."""
    rng = np.random.default_rng(3)
    n, h, hkv, d, page, pages = 70, 8, 2, 128, 16, 8
    qkv = _rand(rng, (n, h + 2 * hkv, d), torch.bfloat16).to(cuda_dev)
    key, value = qkv[:, h:h + hkv], qkv[:, h + hkv:]
    slots = torch.arange(n, dtype=torch.int64, device=cuda_dev) + 5
    kc = torch.zeros(pages, page, hkv, d, dtype=torch.bfloat16, device=cuda_dev)
    vc = torch.zeros_like(kc)
    write_kv_cache(key, value, kc, vc, slots)
    torch.cuda.synchronize()
    flat_k, flat_v = kc.view(-1, hkv, d), vc.view(-1, hkv, d)
    assert torch.equal(flat_k[5:5 + n], key) and torch.equal(flat_v[5:5 + n], value)
    assert not flat_k[:5].any() and not flat_k[5 + n:].any()


def test_cache_write_out_of_range_slot_reported(cuda_dev):
    hkv, d, page, pages = 2, 64, 16, 4
    key = torch.ones(3, hkv, d, dtype=torch.float16, device=cuda_dev)
    kc = torch.zeros(pages, page, hkv, d, dtype=torch.float16, device=cuda_dev)
    vc = torch.zeros_like(kc)
    slots = torch.tensor([0, pages * page, 7], dtype=torch.int64, device=cuda_dev)
    write_kv_cache(key, key, kc, vc, slots)
    code, site, _ = _ext.read_device_error(clear=True)
    assert code == 3  # the library's "slot out of range" code; nothing written for it
    assert int(kc.view(-1, hkv, d).sum(dim=(1, 2)).ne(0).sum()) == 2


def test_cache_write_rejects_bad_shapes(cuda_dev):
    k = torch.zeros(4, 2, 64, dtype=torch.float16, device=cuda_dev)
    kc = torch.zeros(2, 16, 2, 64, dtype=torch.float16, device=cuda_dev)
    with pytest.raises(ValueError):
        write_kv_cache(k, k, kc, kc, torch.zeros(3, dtype=torch.int64, device=cuda_dev))
    with pytest.raises(ValueError):
        write_kv_cache(k, k, kc.to(torch.bfloat16), kc, torch.zeros(4, dtype=torch.int64, device=cuda_dev))


def _step_case(rng, ctx, new, h, hkv, d, page, dt):
    """Sequences with `ctx` cached tokens and `new` tokens in this step; pages shuffled."""
    lens = [c + q for c, q in zip(ctx, new)]
    pps = [-(-n // page) for n in lens]
    perm = rng.permutation(sum(pps) + 3)
    bt = np.zeros((len(lens), max(pps) + 1), np.int32)
    c = 0
    for b, n in enumerate(pps):
        bt[b, :n] = perm[c:c + n]
        c += n
    pages = sum(pps) + 3
    kc = rng.standard_normal((pages, page, hkv, d)).astype(np.float32)
    vc = rng.standard_normal((pages, page, hkv, d)).astype(np.float32)
    slots = np.concatenate([R.slots_for(bt[b], np.arange(ctx[b], lens[b]), page) for b in range(len(lens))])
    nt = int(sum(new))
    q = rng.standard_normal((nt, h, d)).astype(np.float32)
    k = rng.standard_normal((nt, hkv, d)).astype(np.float32)
    v = rng.standard_normal((nt, hkv, d)).astype(np.float32)
    cast = lambda x: torch.from_numpy(x).to(dt)
    return [cast(x) for x in (q, k, v, kc, vc)], bt, np.array(lens, np.int32), slots


@pytest.mark.parametrize("dt,h,hkv,d", [(torch.bfloat16, 32, 8, 128), (torch.float16, 32, 8, 128),
                                        (torch.bfloat16, 8, 2, 512)])
def test_backend_mixed_decode_and_chunked_prefill(cuda_dev, dt, h, hkv, d):
    rng = np.random.default_rng(11)
    page = 16
    ctx = [100, 1000, 17, 0, 250]   # cached tokens per sequence
    new = [1, 1, 1, 300, 64]        # three decodes first, then a prefill and a chunked prefill
    (q, k, v, kc, vc), bt, sl, slots = _step_case(rng, ctx, new, h, hkv, d, page, dt)
    qsl = np.concatenate([[0], np.cumsum(new)]).astype(np.int32)
    t = lambda x: torch.as_tensor(x).to(cuda_dev)
    kv_cache = torch.stack([kc, vc]).to(cuda_dev)
    md = AttentionMetadata(num_actual_tokens=int(sum(new)), max_query_len=max(new),
                           query_start_loc=t(qsl), max_seq_len=int(sl.max()), seq_lens=t(sl),
                           block_table=t(bt), slot_mapping=t(slots), num_decodes=3)
    impl = TileLangFAAttentionImpl(h, d, num_kv_heads=hkv)
    out = impl.forward(t(q), t(k), t(v), kv_cache, md)
    torch.cuda.synchronize()
    # oracle: write the new tokens, then attention of each new token over its sequence
    kr, vr = kc.float().numpy().copy(), vc.float().numpy().copy()
    R.kv_cache_write_ref(k.float().numpy(), v.float().numpy(), kr, vr, slots)
    np.testing.assert_array_equal(kv_cache[0].float().cpu().numpy(), kr)
    np.testing.assert_array_equal(kv_cache[1].float().cpu().numpy(), vr)
    pkl = (sl - np.array(new, np.int32)).astype(np.int32)
    ref, _, bound = R.paged_prefill_ref(q.float().numpy(), kr, vr, bt, sl, qsl, pkl, causal=True,
                                        unit_roundoff=unit_roundoff(dt))
    assert_out_close(out.float().cpu().numpy(), ref, dt, bound, what="step out")


def test_backend_decode_only_and_unsupported_options(cuda_dev):
    rng = np.random.default_rng(5)
    h, hkv, d, page = 16, 4, 64, 16
    ctx, new = [30, 500], [1, 1]
    (q, k, v, kc, vc), bt, sl, slots = _step_case(rng, ctx, new, h, hkv, d, page, torch.float16)
    t = lambda x: torch.as_tensor(x).to(cuda_dev)
    kv_cache = torch.stack([kc, vc]).to(cuda_dev)
    md = AttentionMetadata(2, 1, t(np.array([0, 1, 2], np.int32)), int(sl.max()), t(sl), t(bt),
                           t(slots), num_decodes=2)
    out = TileLangFAAttentionImpl(h, d, num_kv_heads=hkv).forward(t(q), t(k), t(v), kv_cache, md)
    torch.cuda.synchronize()
    kr, vr = kc.float().numpy().copy(), vc.float().numpy().copy()
    R.kv_cache_write_ref(k.float().numpy(), v.float().numpy(), kr, vr, slots)
    ref, _ = R.decode_ref(q.float().numpy(), kr, vr, bt, sl)
    assert_close(out.float().cpu().numpy(), ref, what="decode step")
    with pytest.raises(NotImplementedError):
        TileLangFAAttentionImpl(h, d, sliding_window=128)
