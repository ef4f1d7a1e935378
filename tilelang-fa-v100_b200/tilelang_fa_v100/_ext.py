"""ctypes binding of libfa_b200.so (the sm_100a kernels behind this package).

Mirrors include/fa_b200.h.  Every call passes raw device pointers, element strides
and the caller's current CUDA stream; the library never allocates, so outputs and
workspaces are allocated here with torch.  There is no CPU or fallback path: if the
library is missing or the tensors are not on a CUDA device, the call raises.
"""
import ctypes
import math
import os
import threading

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libfa_b200.so")
_lib = None
_lock = threading.Lock()

FA_OK = 0
FA_ERR_INVALID_ARG = -1
FA_ERR_UNSUPPORTED = -2
FA_ERR_ALIGNMENT = -3
FA_ERR_WORKSPACE = -4
FA_ERR_CUDA = -5
FA_ERR_DEVICE_TIMEOUT = -6
FA_ERR_NOT_SM100 = -7

FA_DTYPE_F16 = 0
FA_DTYPE_BF16 = 1
FA_DTYPE_E4M3 = 2

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float


class FwdArgs(ctypes.Structure):
    _fields_ = [("q", _vp), ("k", _vp), ("v", _vp), ("out", _vp), ("lse", _vp),
                ("q_stride", _i64 * 3), ("k_stride", _i64 * 3), ("v_stride", _i64 * 3),
                ("o_stride", _i64 * 3),
                ("batch", _i32), ("seqlen_q", _i32), ("seqlen_k", _i32), ("num_heads", _i32),
                ("num_heads_k", _i32), ("head_dim", _i32), ("dtype", _i32), ("causal", _i32),
                ("softmax_scale", _f32), ("window_q", _i32), ("window_k", _i32),
                ("softcap", _f32)]


class BwdArgs(ctypes.Structure):
    _fields_ = [("q", _vp), ("k", _vp), ("v", _vp), ("out", _vp), ("dout", _vp), ("lse", _vp),
                ("dq", _vp), ("dk", _vp), ("dv", _vp),
                ("q_stride", _i64 * 3), ("k_stride", _i64 * 3), ("v_stride", _i64 * 3),
                ("o_stride", _i64 * 3), ("do_stride", _i64 * 3), ("dq_stride", _i64 * 3),
                ("dk_stride", _i64 * 3), ("dv_stride", _i64 * 3),
                ("batch", _i32), ("seqlen_q", _i32), ("seqlen_k", _i32), ("num_heads", _i32),
                ("num_heads_k", _i32), ("head_dim", _i32), ("dtype", _i32), ("causal", _i32),
                ("deterministic", _i32), ("softmax_scale", _f32), ("window_q", _i32),
                ("window_k", _i32), ("softcap", _f32)]


class VarlenFwdArgs(ctypes.Structure):
    _fields_ = [("q", _vp), ("k", _vp), ("v", _vp), ("out", _vp), ("lse", _vp),
                ("cu_seqlens_q", _vp), ("cu_seqlens_k", _vp),
                ("q_stride", _i64 * 2), ("k_stride", _i64 * 2), ("v_stride", _i64 * 2),
                ("o_stride", _i64 * 2),
                ("batch", _i32), ("total_q", _i32), ("total_k", _i32), ("max_seqlen_q", _i32),
                ("max_seqlen_k", _i32), ("num_heads", _i32), ("num_heads_k", _i32),
                ("head_dim", _i32), ("dtype", _i32), ("causal", _i32), ("softmax_scale", _f32),
                ("window_q", _i32), ("window_k", _i32), ("softcap", _f32)]


class VarlenBwdArgs(ctypes.Structure):
    _fields_ = [("q", _vp), ("k", _vp), ("v", _vp), ("out", _vp), ("dout", _vp), ("lse", _vp),
                ("dq", _vp), ("dk", _vp), ("dv", _vp),
                ("cu_seqlens_q", _vp), ("cu_seqlens_k", _vp),
                ("q_stride", _i64 * 2), ("k_stride", _i64 * 2), ("v_stride", _i64 * 2),
                ("o_stride", _i64 * 2), ("do_stride", _i64 * 2), ("dq_stride", _i64 * 2),
                ("dk_stride", _i64 * 2), ("dv_stride", _i64 * 2),
                ("batch", _i32), ("total_q", _i32), ("total_k", _i32), ("max_seqlen_q", _i32),
                ("max_seqlen_k", _i32), ("num_heads", _i32), ("num_heads_k", _i32),
                ("head_dim", _i32), ("dtype", _i32), ("causal", _i32), ("deterministic", _i32),
                ("softmax_scale", _f32), ("window_q", _i32), ("window_k", _i32),
                ("softcap", _f32)]


class PagedArgs(ctypes.Structure):
    _fields_ = [("q", _vp), ("k_cache", _vp), ("v_cache", _vp), ("block_table", _vp),
                ("seq_lens", _vp), ("query_start_loc", _vp), ("prefix_kv_lens", _vp),
                ("out", _vp), ("lse", _vp),
                ("num_tokens", _i32), ("num_seqs", _i32), ("num_heads", _i32),
                ("num_kv_heads", _i32), ("head_dim", _i32), ("page_size", _i32),
                ("num_pages", _i32), ("max_blocks", _i32), ("dtype", _i32), ("causal", _i32),
                ("sliding_window_q", _i32), ("sliding_window_k", _i32),
                ("softmax_scale", _f32)]


class DecodeArgs(ctypes.Structure):
    _fields_ = [("q", _vp), ("k_cache", _vp), ("v_cache", _vp), ("block_table", _vp),
                ("seq_lens", _vp), ("out", _vp), ("lse", _vp),
                ("batch", _i32), ("num_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
                ("page_size", _i32), ("num_pages", _i32), ("max_blocks", _i32), ("dtype", _i32),
                ("num_splits", _i32), ("softmax_scale", _f32),
                ("kv_dtype", _i32), ("k_scale", _f32), ("v_scale", _f32)]


class KvWriteArgs(ctypes.Structure):
    _fields_ = [("key", _vp), ("value", _vp), ("k_cache", _vp), ("v_cache", _vp),
                ("slot_mapping", _vp), ("key_stride", _i64), ("value_stride", _i64),
                ("num_tokens", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
                ("page_size", _i32), ("num_pages", _i32), ("dtype", _i32),
                ("cache_dtype", _i32), ("k_scale", _f32), ("v_scale", _f32)]


# Exported symbols and their (restype, argtypes); the CPU test checks this list
# against include/fa_b200.h.
SIGNATURES = {
    "fa_fwd": (_i32, [ctypes.POINTER(FwdArgs), _vp]),
    "fa_bwd_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(BwdArgs)]),
    "fa_bwd": (_i32, [ctypes.POINTER(BwdArgs), _vp, ctypes.c_size_t, _vp]),
    "fa_varlen_fwd": (_i32, [ctypes.POINTER(VarlenFwdArgs), _vp]),
    "fa_varlen_bwd_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(VarlenBwdArgs)]),
    "fa_varlen_bwd": (_i32, [ctypes.POINTER(VarlenBwdArgs), _vp, ctypes.c_size_t, _vp]),
    "fa_paged_prefill": (_i32, [ctypes.POINTER(PagedArgs), _vp]),
    "fa_decode_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(DecodeArgs)]),
    "fa_decode": (_i32, [ctypes.POINTER(DecodeArgs), _vp, ctypes.c_size_t, _vp]),
    "fa_decode_noalloc": (_i32, [ctypes.POINTER(DecodeArgs), _vp]),
    "fa_decode_noalloc_scratch_bytes": (ctypes.c_size_t, []),
    "fa_kv_cache_write": (_i32, [ctypes.POINTER(KvWriteArgs), _vp]),
    "fa_status_string": (ctypes.c_char_p, [_i32]),
    "fa_read_device_error": (_i32, [ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                                    ctypes.POINTER(_i32), _i32]),
    "fa_version": (ctypes.c_char_p, []),
    "fa_last_error_detail": (ctypes.c_char_p, []),
    "fa_launch_count": (_i64, []),
    "fa_selftest_umma": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp]),
    "fa_profile_next_launch": (_i32, [_i32, _vp, _vp]),
    "fa_selftest_umma_rate": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp]),
}

PROF_FWD, PROF_BWD_DKDV, PROF_PAGED, PROF_DECODE = 1, 2, 3, 4


def profile_next_launch(kind, ev_begin, ev_end):
    """Arms torch.cuda.Event pair around the next launch of one main kernel."""
    for ev in (ev_begin, ev_end):
        if ev.cuda_event == 0:  # torch creates the CUDA event lazily, on first record
            ev.record()
    check(load().fa_profile_next_launch(kind, ctypes.c_void_p(ev_begin.cuda_event),
                                        ctypes.c_void_p(ev_end.cuda_event)))


def lib_path():
    return _LIB_PATH


def load():
    """Loads libfa_b200.so once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise RuntimeError(
                    "libfa_b200.so is not built (expected at %s); run "
                    "`python tilelang-fa-v100_b200/build.py` or __graft_entry__.build()" % _LIB_PATH)
            lib = ctypes.CDLL(_LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


class FaError(RuntimeError):
    pass


def check(status):
    if status == FA_OK:
        return
    msg = load().fa_status_string(status).decode()
    if status == FA_ERR_UNSUPPORTED:
        raise NotImplementedError("libfa_b200: " + msg)
    if status == FA_ERR_INVALID_ARG:
        raise ValueError("libfa_b200: " + msg)
    detail = load().fa_last_error_detail().decode() if status == FA_ERR_CUDA else ""
    raise FaError("libfa_b200 error %d: %s%s" % (status, msg, (" (" + detail + ")") if detail else ""))


def read_device_error(clear=True):
    """(code, site, block) of the first device-side error since the last clear."""
    c, s, b = _i32(0), _i32(0), _i32(0)
    check(load().fa_read_device_error(ctypes.byref(c), ctypes.byref(s), ctypes.byref(b),
                                      1 if clear else 0))
    return c.value, s.value, b.value


def launch_count():
    return int(load().fa_launch_count())


def _dtype_code(t):
    if t == torch.float16:
        return FA_DTYPE_F16
    if t == torch.bfloat16:
        return FA_DTYPE_BF16
    raise NotImplementedError("dtype %s not supported (fp16 / bf16 only)" % t)


def _require_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise ValueError("tilelang_fa_v100 (B200 build) needs CUDA tensors; got %s" % t.device)


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _strides3(t):
    """(batch, seq, head) element strides of a [B, S, H, D] view with a unit last stride."""
    return (_i64 * 3)(t.stride(0), t.stride(1), t.stride(2))


def _bshd(t):
    """A view the kernels accept: last dim contiguous, other strides 16-byte multiples."""
    if t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:3]) or t.data_ptr() % 16:
        t = t.contiguous()
    return t


def window_fields(window_size):
    """FA2 window_size (left, right), -1 = unbounded, as the C-ABI's (window_q, window_k)."""
    left, right = (int(window_size[0]), int(window_size[1])) if window_size is not None else (-1, -1)
    return (left + 1 if left >= 0 else 0), (right + 1 if right >= 0 else 0)


def dense_forward(q, k, v, softmax_scale, causal, window_size=(-1, -1), softcap=0.0):
    """out [B,Sq,H,D] and lse [B,H,Sq] fp32 for BSHD q/k/v."""
    _require_cuda(q, k, v)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k, v must be [B, S, H, D]")
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k, v dtypes differ")
    b, sq, h, d = q.shape
    skv, hk = k.shape[1], k.shape[2]
    if tuple(v.shape) != tuple(k.shape) or k.shape[0] != b or k.shape[3] != d:
        raise ValueError("k/v shape %s incompatible with q %s" % (tuple(k.shape), tuple(q.shape)))
    q, k, v = _bshd(q), _bshd(k), _bshd(v)
    out = torch.empty((b, sq, h, d), dtype=q.dtype, device=q.device)
    lse = torch.empty((b, h, sq), dtype=torch.float32, device=q.device)
    if out.numel() == 0 or skv == 0:
        # nothing to compute, or no key at all: the library's fully masked rows (out 0,
        # lse -inf); empty tensors have no data pointer to hand the C ABI
        load()
        return out.zero_(), lse.fill_(float("-inf"))
    a = FwdArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr(),
                _strides3(q), _strides3(k), _strides3(v), _strides3(out),
                b, sq, skv, h, hk, d, _dtype_code(q.dtype), 1 if causal else 0,
                float(softmax_scale), *window_fields(window_size), float(softcap))
    with torch.cuda.device(q.device):
        check(load().fa_fwd(ctypes.byref(a), _stream(q.device)))
    return out, lse


def dense_backward(q, k, v, out, dout, lse, softmax_scale, causal, deterministic=False,
                   window_size=(-1, -1), softcap=0.0):
    """dq, dk, dv (BSHD, q/k/v dtype) for the forward that produced out / lse."""
    _require_cuda(q, k, v, out, dout, lse)
    b, sq, h, d = q.shape
    skv, hk = k.shape[1], k.shape[2]
    q, k, v, out = _bshd(q), _bshd(k), _bshd(v), _bshd(out)
    dout = _bshd(dout.to(q.dtype))
    lse = lse.contiguous()
    dq = torch.empty((b, sq, h, d), dtype=q.dtype, device=q.device)
    dk = torch.empty((b, skv, hk, d), dtype=q.dtype, device=q.device)
    dv = torch.empty((b, skv, hk, d), dtype=q.dtype, device=q.device)
    if dq.numel() == 0 or dk.numel() == 0:
        load()  # nothing attends: every gradient is zero
        return dq.zero_(), dk.zero_(), dv.zero_()
    a = BwdArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dout.data_ptr(),
                lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                _strides3(q), _strides3(k), _strides3(v), _strides3(out), _strides3(dout),
                _strides3(dq), _strides3(dk), _strides3(dv),
                b, sq, skv, h, hk, d, _dtype_code(q.dtype), 1 if causal else 0,
                1 if deterministic else 0, float(softmax_scale), *window_fields(window_size),
                float(softcap))
    lib = load()
    nbytes = int(lib.fa_bwd_workspace_size(ctypes.byref(a)))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        check(lib.fa_bwd(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), nbytes,
                         _stream(q.device)))
    return dq, dk, dv


def _tokens_heads(t, what):
    """[total, heads, D] with a contiguous last dim; (token, head) strides in elements."""
    if t.dim() != 3:
        raise ValueError("%s must be [total_tokens, heads, head_dim]" % what)
    if t.stride(-1) != 1 or t.stride(0) % 8 or t.stride(1) % 8:
        t = t.contiguous()
    return t


def _cu(t, dev, n):
    t = t.to(device=dev, dtype=torch.int32).contiguous()
    if t.dim() != 1 or t.numel() != n:
        raise ValueError("cu_seqlens must be [batch + 1]")
    return t


def varlen_forward(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                   softmax_scale, causal, window_size=(-1, -1), softcap=0.0):
    """out [total_q, H, D] and lse [H, total_q] fp32 for packed sequences (FA2 varlen)."""
    _require_cuda(q, k, v)
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k, v dtypes differ")
    q, k, v = _tokens_heads(q, "q"), _tokens_heads(k, "k"), _tokens_heads(v, "v")
    if tuple(v.shape) != tuple(k.shape) or k.shape[2] != q.shape[2]:
        raise ValueError("k/v shape %s incompatible with q %s" % (tuple(k.shape), tuple(q.shape)))
    batch = cu_seqlens_q.numel() - 1
    cq, ck = _cu(cu_seqlens_q, q.device, batch + 1), _cu(cu_seqlens_k, q.device, batch + 1)
    tq, h, d = q.shape
    tk, hk = k.shape[0], k.shape[1]
    out = torch.empty((tq, h, d), dtype=q.dtype, device=q.device)
    lse = torch.empty((h, tq), dtype=torch.float32, device=q.device)
    if out.numel() == 0 or tk == 0:
        load()  # no rows, or no key in any sequence: out 0, lse -inf
        return out.zero_(), lse.fill_(float("-inf"))
    st2 = lambda t: (_i64 * 2)(t.stride(0), t.stride(1))
    a = VarlenFwdArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr(),
                      cq.data_ptr(), ck.data_ptr(), st2(q), st2(k), st2(v), st2(out),
                      batch, tq, tk, int(max_seqlen_q), int(max_seqlen_k), h, hk, d,
                      _dtype_code(q.dtype), 1 if causal else 0, float(softmax_scale),
                      *window_fields(window_size), float(softcap))
    with torch.cuda.device(q.device):
        check(load().fa_varlen_fwd(ctypes.byref(a), _stream(q.device)))
    return out, lse


def varlen_backward(q, k, v, out, dout, lse, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                    max_seqlen_k, softmax_scale, causal, deterministic=False,
                    window_size=(-1, -1), softcap=0.0):
    """dq, dk, dv in the packed layouts of q / k / v."""
    _require_cuda(q, k, v, out, dout, lse)
    q, k, v, out = (_tokens_heads(t, w) for t, w in ((q, "q"), (k, "k"), (v, "v"), (out, "out")))
    dout = _tokens_heads(dout.to(q.dtype), "dout")
    lse = lse.contiguous()
    batch = cu_seqlens_q.numel() - 1
    cq, ck = _cu(cu_seqlens_q, q.device, batch + 1), _cu(cu_seqlens_k, q.device, batch + 1)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    if dq.numel() == 0 or dk.numel() == 0:
        load()  # nothing attends: every gradient is zero
        return dq.zero_(), dk.zero_(), dv.zero_()
    st2 = lambda t: (_i64 * 2)(t.stride(0), t.stride(1))
    tq, h, d = q.shape
    a = VarlenBwdArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dout.data_ptr(),
                      lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                      cq.data_ptr(), ck.data_ptr(), st2(q), st2(k), st2(v), st2(out), st2(dout),
                      st2(dq), st2(dk), st2(dv), batch, tq, k.shape[0], int(max_seqlen_q),
                      int(max_seqlen_k), h, k.shape[1], d, _dtype_code(q.dtype),
                      1 if causal else 0, 1 if deterministic else 0, float(softmax_scale),
                      *window_fields(window_size), float(softcap))
    lib = load()
    nbytes = int(lib.fa_varlen_bwd_workspace_size(ctypes.byref(a)))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        check(lib.fa_varlen_bwd(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), nbytes,
                                _stream(q.device)))
    return dq, dk, dv


def _i32_on(t, dev):
    return t.to(device=dev, dtype=torch.int32).contiguous()


def paged_prefill(q, k_cache, v_cache, block_table, seq_lens, query_start_loc, prefix_kv_lens,
                  out, lse, page_size, num_kv_heads, softmax_scale, causal, swq, swk):
    """Writes out [T,H,D] (and lse [H,T] when given) for the vLLM paged layout."""
    _require_cuda(q, k_cache, v_cache, out)
    dev = q.device
    t, h, d = q.shape
    # int32 index tensors on the device (no-ops when they already are); the locals
    # keep them alive until the launch has been enqueued.
    bt = _i32_on(block_table, dev)
    sl = _i32_on(seq_lens, dev)
    qsl = _i32_on(query_start_loc, dev)
    pkl = _i32_on(prefix_kv_lens, dev)
    a = PagedArgs(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), bt.data_ptr(),
                  sl.data_ptr(), qsl.data_ptr(), pkl.data_ptr(), out.data_ptr(),
                  lse.data_ptr() if lse is not None else None,
                  t, bt.shape[0], h, num_kv_heads, d, page_size, k_cache.shape[0], bt.shape[1],
                  _dtype_code(q.dtype), 1 if causal else 0, int(swq), int(swk),
                  float(softmax_scale))
    with torch.cuda.device(dev):
        check(load().fa_paged_prefill(ctypes.byref(a), _stream(dev)))
    return out, lse


def _kv_code(cache, q_dtype):
    """0 when the cache holds the query dtype, FA_DTYPE_E4M3 for an fp8 (e4m3) cache."""
    if cache.dtype == q_dtype:
        return 0
    if cache.dtype == torch.float8_e4m3fn:
        return FA_DTYPE_E4M3
    raise ValueError("cache dtype %s: must be the query dtype or torch.float8_e4m3fn" % cache.dtype)


def decode(q, k_cache, v_cache, block_table, seq_lens, page_size, num_kv_heads, softmax_scale,
           num_splits=0, out=None, lse=None, k_scale=1.0, v_scale=1.0):
    _require_cuda(q, k_cache, v_cache)
    dev = q.device
    bsz, h, d = q.shape
    q = q.contiguous()
    bt = _i32_on(block_table, dev)
    sl = _i32_on(seq_lens, dev)
    if out is None:
        out = torch.empty_like(q)
    kv = _kv_code(k_cache, q.dtype)
    if _kv_code(v_cache, q.dtype) != kv:
        raise ValueError("k_cache and v_cache dtypes differ")
    a = DecodeArgs(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), bt.data_ptr(),
                   sl.data_ptr(), out.data_ptr(), lse.data_ptr() if lse is not None else None,
                   bsz, h, num_kv_heads, d, page_size, k_cache.shape[0], bt.shape[1],
                   _dtype_code(q.dtype), int(num_splits), float(softmax_scale),
                   kv, float(k_scale), float(v_scale))
    lib = load()
    nbytes = int(lib.fa_decode_workspace_size(ctypes.byref(a)))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        check(lib.fa_decode(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), nbytes, _stream(dev)))
    return out


def kv_cache_write(key, value, k_cache, v_cache, slot_mapping, k_scale=1.0, v_scale=1.0):
    """Scatters key/value [num_tokens, Hkv, D] into the paged caches at slot_mapping
    (quantised to e4m3 with the scales when the caches are torch.float8_e4m3fn)."""
    _require_cuda(key, value, k_cache, v_cache)
    dev = key.device
    n, hkv, d = key.shape
    sm = slot_mapping.to(device=dev, dtype=torch.int64).contiguous()
    a = KvWriteArgs(key.data_ptr(), value.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                    sm.data_ptr(), key.stride(0), value.stride(0), n, hkv, d,
                    k_cache.shape[1], k_cache.shape[0], _dtype_code(key.dtype),
                    _kv_code(k_cache, key.dtype), float(k_scale), float(v_scale))
    with torch.cuda.device(dev):
        check(load().fa_kv_cache_write(ctypes.byref(a), _stream(dev)))


def selftest_umma(a, b, n, k, b_mn, a_tmem):
    """C[128, n] = A[128, k] B^T through one tcgen05 UMMA (see include/fa_b200.h)."""
    _require_cuda(a, b)
    c = torch.empty((128, n), dtype=torch.float32, device=a.device)
    with torch.cuda.device(a.device):
        check(load().fa_selftest_umma(ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                                      ctypes.c_void_p(c.data_ptr()), n, k, _dtype_code(a.dtype),
                                      1 if b_mn else 0, 1 if a_tmem else 0, _stream(a.device)))
    return c


def default_scale(d):
    return 1.0 / math.sqrt(d)
