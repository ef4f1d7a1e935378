"""fa_decode_noalloc: the decode entry point for callers that cannot give the library
any device memory (a serving engine whose free HBM all belongs to its KV-cache pool,
or a plain C caller without a device allocator).  Called straight through the C ABI,
twice in a row, and compared with the CPU oracle and with the allocating entry point
fa_decode -- including a batch whose split partials do not fit the fixed scratch at the
heuristic split count, so the entry point must lower it."""
import ctypes

import numpy as np
import pytest
import torch

from tilelang_fa_v100 import _ext
from helpers import assert_close, assert_out_close
from oracle import attention_ref as R

pytestmark = pytest.mark.gpu


def _problem(dev, lens, heads, hkv, seed):
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, np.int32)
    pps = (lens + 15) // 16
    total = int(pps.sum())
    perm = rng.permutation(total).astype(np.int32)
    bt = np.zeros((len(lens), int(pps.max()) + 1), np.int32)
    c = 0
    for b, n in enumerate(pps):
        bt[b, :n] = perm[c:c + n]
        c += n
    g = torch.Generator(device=dev).manual_seed(seed)
    kc = torch.randn(total, 16, hkv, 128, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(total, 16, hkv, 128, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(len(lens), heads, 128, generator=g, device=dev).to(torch.bfloat16)
    return q, kc, vc, torch.from_numpy(bt).to(dev), torch.from_numpy(lens).to(dev)


def _args(q, kc, vc, bt, sl, out, lse, num_splits):
    return _ext.DecodeArgs(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(),
                           sl.data_ptr(), out.data_ptr(), lse.data_ptr(), q.shape[0], q.shape[1],
                           kc.shape[2], q.shape[2], kc.shape[1], kc.shape[0], bt.shape[1],
                           _ext.FA_DTYPE_BF16, num_splits, 128 ** -0.5)


def _decode_alloc(lib, q, kc, vc, bt, sl, num_splits, stream, dev):
    """The allocating entry point with a caller workspace."""
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[0], q.shape[1], device=dev)
    a = _args(q, kc, vc, bt, sl, out, lse, num_splits)
    nbytes = int(lib.fa_decode_workspace_size(ctypes.byref(a)))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    assert lib.fa_decode(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), nbytes, stream) == 0
    torch.cuda.synchronize(dev)
    return out, lse


def _oracle_check(out, lse, q, kc, vc, bt, sl, seqs):
    """Sampled sequences against the CPU oracle on their own gathered pages."""
    bt_h, sl_h = bt.cpu().numpy(), sl.cpu().numpy()
    for b in seqs:
        n = int((sl_h[b] + 15) // 16)
        idx = torch.from_numpy(bt_h[b, :n].astype(np.int64)).to(kc.device)
        ro, rl, bnd = R.decode_ref(q[b:b + 1].float().cpu().numpy(),
                                   kc[idx].float().cpu().numpy(), vc[idx].float().cpu().numpy(),
                                   np.arange(n, dtype=np.int32)[None], sl_h[b:b + 1],
                                   unit_roundoff=2.0 ** -8)
        assert_out_close(out[b:b + 1].float().cpu().numpy(), ro, torch.bfloat16, bnd,
                         what="seq %d out" % b)
        assert_close(lse[b:b + 1].cpu().numpy(), rl, what="seq %d lse" % b)


def test_decode_noalloc_matches_oracle_and_allocating_decode(cuda_dev):
    lib = _ext.load()
    q, kc, vc, bt, sl = _problem(cuda_dev, [1, 17, 300, 1000, 2048, 3001, 64, 777], 16, 4, 5)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream)
    ref_out, ref_lse = _decode_alloc(lib, q, kc, vc, bt, sl, 0, stream, cuda_dev)
    for _ in range(2):  # two calls in a row share (and reuse) the static scratch
        out = torch.full_like(q, float("nan"))
        lse = torch.full((q.shape[0], q.shape[1]), float("nan"), device=cuda_dev)
        b = _args(q, kc, vc, bt, sl, out, lse, 0)
        assert lib.fa_decode_noalloc(ctypes.byref(b), stream) == 0
        torch.cuda.synchronize(cuda_dev)
        _oracle_check(out, lse, q, kc, vc, bt, sl, range(q.shape[0]))
        # same split count, same kernels: the allocating entry point's exact result
        assert torch.equal(out, ref_out)
        assert torch.equal(lse, ref_lse)


def test_decode_noalloc_lowers_split_count_to_fit(cuda_dev):
    """The benchmark decode shape (256 sequences, L ~ U[512, 8192], 32 / 8 heads, D 128):
    the heuristic's 17 splits (one per 512 keys of the block table) need 17 x 4.2 MB of
    partials, more than the 16 MiB scratch, so the entry point runs 3 splits.  Two calls
    in a row; sampled sequences against the oracle and every sequence against fa_decode
    at the same 3 splits."""
    lib = _ext.load()
    lens = np.random.default_rng(0).integers(512, 8193, size=256)
    q, kc, vc, bt, sl = _problem(cuda_dev, lens, 32, 8, 7)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream)
    cap = int(lib.fa_decode_noalloc_scratch_bytes())
    per_split = q.shape[0] * q.shape[1] * (q.shape[2] + 1) * 4
    probe = _args(q, kc, vc, bt, sl, q, q, 0)
    heuristic = int(lib.fa_decode_workspace_size(ctypes.byref(probe)) - 256) // per_split
    fits = cap // per_split
    assert heuristic > fits >= 2, (heuristic, fits)
    ref_out, ref_lse = _decode_alloc(lib, q, kc, vc, bt, sl, fits, stream, cuda_dev)
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        lse = torch.full((q.shape[0], q.shape[1]), float("nan"), device=cuda_dev)
        b = _args(q, kc, vc, bt, sl, out, lse, 0)
        assert lib.fa_decode_noalloc(ctypes.byref(b), stream) == 0
        torch.cuda.synchronize(cuda_dev)
        assert torch.equal(out, ref_out)
        assert torch.equal(lse, ref_lse)
        _oracle_check(out, lse, q, kc, vc, bt, sl, (0, 101, 255))


def test_decode_noalloc_rejects_oversized_split_request(cuda_dev):
    lib = _ext.load()
    q, kc, vc, bt, sl = _problem(cuda_dev, [1, 17, 300, 1000, 2048, 3001, 64, 777], 16, 4, 5)
    cap = int(lib.fa_decode_noalloc_scratch_bytes())
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[0], q.shape[1], device=cuda_dev)
    per_split = q.shape[0] * q.shape[1] * (q.shape[2] + 1) * 4
    too_many = cap // per_split + 2
    b = _args(q, kc, vc, bt, sl, out, lse, too_many)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream)
    assert lib.fa_decode_noalloc(ctypes.byref(b), stream) == _ext.FA_ERR_WORKSPACE
    assert b"static scratch" in lib.fa_last_error_detail()
