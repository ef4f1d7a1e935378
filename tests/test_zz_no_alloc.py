"""fa_decode_noalloc: the decode entry point for callers that cannot give the library
any device memory (a serving engine whose free HBM all belongs to its KV-cache pool,
or a plain C caller without a device allocator).  Called straight through the C ABI,
twice in a row, and compared with the allocating entry point fa_decode."""
import ctypes

import numpy as np
import pytest
import torch

from tilelang_fa_v100 import _ext
from helpers import assert_close

pytestmark = pytest.mark.gpu


def _problem(dev):
    rng = np.random.default_rng(123)
    lens = np.array([1, 17, 300, 1000, 2048, 3001, 64, 777], np.int32)
    pps = (lens + 15) // 16
    total = int(pps.sum())
    perm = rng.permutation(total).astype(np.int32)
    bt = np.zeros((len(lens), int(pps.max()) + 1), np.int32)
    c = 0
    for b, n in enumerate(pps):
        bt[b, :n] = perm[c:c + n]
        c += n
    g = torch.Generator(device=dev).manual_seed(5)
    kc = torch.randn(total, 16, 4, 128, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(total, 16, 4, 128, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(len(lens), 16, 128, generator=g, device=dev).to(torch.bfloat16)
    return q, kc, vc, torch.from_numpy(bt).to(dev), torch.from_numpy(lens).to(dev)


def _args(q, kc, vc, bt, sl, out, lse, num_splits):
    return _ext.DecodeArgs(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(),
                           sl.data_ptr(), out.data_ptr(), lse.data_ptr(), q.shape[0], q.shape[1],
                           kc.shape[2], q.shape[2], kc.shape[1], kc.shape[0], bt.shape[1],
                           _ext.FA_DTYPE_BF16, num_splits, 128 ** -0.5)


def test_decode_noalloc_matches_allocating_decode(cuda_dev):
    lib = _ext.load()
    q, kc, vc, bt, sl = _problem(cuda_dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream)

    # reference: the allocating entry point with a caller workspace
    ref_out = torch.empty_like(q)
    ref_lse = torch.empty(q.shape[0], q.shape[1], device=cuda_dev)
    a = _args(q, kc, vc, bt, sl, ref_out, ref_lse, 0)
    nbytes = int(lib.fa_decode_workspace_size(ctypes.byref(a)))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=cuda_dev)
    assert lib.fa_decode(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), nbytes, stream) == 0
    torch.cuda.synchronize(cuda_dev)

    for _ in range(2):  # two calls in a row share (and reuse) the static scratch
        out = torch.full_like(q, float("nan"))
        lse = torch.full((q.shape[0], q.shape[1]), float("nan"), device=cuda_dev)
        b = _args(q, kc, vc, bt, sl, out, lse, 0)
        assert lib.fa_decode_noalloc(ctypes.byref(b), stream) == 0
        torch.cuda.synchronize(cuda_dev)
        assert_close(out.float().cpu().numpy(), ref_out.float().cpu().numpy(), what="out",
                     dtype=torch.bfloat16)
        assert_close(lse.cpu().numpy(), ref_lse.cpu().numpy(), what="lse")


def test_decode_noalloc_rejects_oversized_split_request(cuda_dev):
    lib = _ext.load()
    q, kc, vc, bt, sl = _problem(cuda_dev)
    cap = int(lib.fa_decode_noalloc_scratch_bytes())
    out = torch.empty_like(q)
    lse = torch.empty(q.shape[0], q.shape[1], device=cuda_dev)
    per_split = q.shape[0] * q.shape[1] * (q.shape[2] + 1) * 4
    too_many = cap // per_split + 2
    b = _args(q, kc, vc, bt, sl, out, lse, too_many)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream)
    assert lib.fa_decode_noalloc(ctypes.byref(b), stream) == _ext.FA_ERR_WORKSPACE
    assert b"static scratch" in lib.fa_last_error_detail()
