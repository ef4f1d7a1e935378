"""FA2-compatible API (mirror of the reference's tilelang_fa_v100/interface.py).

Same names, signatures, defaults and error behaviour as the reference:
``tilelang_flash_attn_func`` / ``tilelang_flash_attn_gpu`` (interface.py:59-80, 101)
with a torch.autograd forward/backward (interface.py:12-56), ``tilelang_paged_forward``
(interface.py:83-98) and ``tilelang_decode_forward`` (interface.py:104-117).

Differences that keep results identical: the kernels read and write the BSHD layout
directly, so the reference's permute/contiguous copies (interface.py:19-21, 38, 51)
are gone, and gradients come back as contiguous BSHD tensors (the reference returns
permuted views of the same values, interface.py:53-55).  ``softmax_scale`` is
honoured (the reference kernels hard-code 1/sqrt(D), _kernels_forward.py:96; equal
for the default).  ``deterministic=True`` selects the dQ kernel without atomics.
``window_size`` and ``softcap`` follow FA2 (the reference ignores the first and rejects
the second, interface.py:29-33; with their defaults the results agree).
"""
import math

import torch

from . import _ext
from ._paged_adapter import paged_forward as _paged_forward
from ._decode_adapter import decode_forward as _decode_forward


class FlashAttnTileLangVFunc(torch.autograd.Function):
    """Autograd function for the B200 FlashAttention kernels (training)."""

    @staticmethod
    def forward(ctx, q, k, v, dropout_p, softmax_scale, causal, window_size,
                softcap, alibi_slopes, deterministic, return_softmax):
        D = q.shape[-1]
        if dropout_p != 0.0:
            raise NotImplementedError("dropout not supported")
        if alibi_slopes is not None:
            raise NotImplementedError("alibi not supported")

        scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
        # window_size is honoured (FA2 semantics, bottom-right aligned; (-1, -1) = none).
        # The reference accepts it and ignores it (interface.py:33): with the default the
        # two agree.
        window = tuple(window_size) if window_size is not None else (-1, -1)
        # softcap is honoured (FA2 semantics: score = softcap * tanh(scale * q.k / softcap),
        # > 0 enables it, lse is over the capped scores).  The reference raises
        # NotImplementedError for softcap != 0 (interface.py:29-30).
        cap = float(softcap) if softcap > 0 else 0.0
        out, lse = _ext.dense_forward(q, k, v, scale, causal, window, cap)

        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal = causal
        ctx.window = window
        ctx.softcap = cap
        ctx.softmax_scale = scale
        ctx.deterministic = bool(deterministic)

        if return_softmax:
            return out, lse, None
        return out

    @staticmethod
    def backward(ctx, dout, *args):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = _ext.dense_backward(q, k, v, out, dout, lse, ctx.softmax_scale,
                                         ctx.causal, ctx.deterministic, ctx.window,
                                         ctx.softcap)
        return dq, dk, dv, None, None, None, None, None, None, None, None, None


def tilelang_flash_attn_func(q, k, v, dropout_p=0.0, softmax_scale=None,
                             causal=False, window_size=(-1, -1), softcap=0.0,
                             alibi_slopes=None, deterministic=False,
                             return_attn_probs=False):
    """FA2-compatible flash attention function.

    Args:
        q: [B, M, H, D]; k, v: [B, N, Hk, D] (FA2 layout, H % Hk == 0), fp16 or bf16
        causal: bottom-right aligned causal mask (key j visible to row i iff j <= i + N - M)
        softmax_scale: (default: 1/sqrt(D))
        window_size: FA2 (left, right) sliding window, -1 = unbounded on that side
        softcap: > 0: scores become softcap * tanh(scale * q.k / softcap) (FA2 softcapping)
        deterministic: compute dQ without atomics (bit-reproducible backward)
        return_attn_probs: return (out, lse, None) instead of just out

    Returns:
        out: [B, M, H, D] in the input dtype, or (out, lse [B, H, M] fp32, None)
    """
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** -0.5
    return FlashAttnTileLangVFunc.apply(
        q, k, v, dropout_p, softmax_scale, causal,
        window_size, softcap, alibi_slopes, deterministic, return_attn_probs,
    )


def tilelang_paged_forward(q, k_cache, v_cache, block_table, seq_lens,
                           query_start_loc, prefix_kv_lens, out=None,
                           block_size=16, num_kv_heads=None,
                           softmax_scale=None, causal=True,
                           sliding_window_q=-1, sliding_window_k=-1):
    """Paged FlashAttention forward for vLLM integration.

    Args match the reference FA-V100 paged_fwd API.  Returns (out, softmax_lse) with
    softmax_lse [num_heads, num_tokens] fp32 (filled, unlike the reference).
    """
    return _paged_forward(
        q, k_cache, v_cache, block_table, seq_lens,
        query_start_loc, prefix_kv_lens, out=out,
        block_size=block_size, num_kv_heads=num_kv_heads,
        softmax_scale=softmax_scale, causal=causal,
        sliding_window_q=sliding_window_q, sliding_window_k=sliding_window_k,
    )


tilelang_flash_attn_gpu = tilelang_flash_attn_func


def tilelang_decode_forward(q, k_cache, v_cache, block_table, seq_lens,
                            block_size=16, num_kv_heads=None,
                            softmax_scale=None, k_scale=1.0, v_scale=1.0):
    """Paged decode forward for vLLM integration.

    Args match the reference FA-V100 decode_fwd API; k_scale / v_scale (defaults 1)
    dequantise torch.float8_e4m3fn caches, which the reference does not accept.
    Returns:
        output: [batch, heads, dim] in the input dtype
    """
    return _decode_forward(
        q, k_cache, v_cache, block_table, seq_lens,
        block_size=block_size, num_kv_heads=num_kv_heads,
        softmax_scale=softmax_scale, k_scale=k_scale, v_scale=v_scale,
    )


class FlashAttnVarlenFunc(torch.autograd.Function):
    """Autograd function for packed variable-length sequences (FA2's varlen path)."""

    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                dropout_p, softmax_scale, causal, window_size, softcap, alibi_slopes,
                deterministic, return_softmax):
        if dropout_p != 0.0:
            raise NotImplementedError("dropout not supported")
        if alibi_slopes is not None:
            raise NotImplementedError("alibi not supported")
        scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
        window = tuple(window_size) if window_size is not None else (-1, -1)
        cap = float(softcap) if softcap > 0 else 0.0
        out, lse = _ext.varlen_forward(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                       max_seqlen_k, scale, causal, window, cap)
        ctx.save_for_backward(q, k, v, out, lse, cu_seqlens_q, cu_seqlens_k)
        ctx.max_seqlen = (int(max_seqlen_q), int(max_seqlen_k))
        ctx.causal, ctx.window, ctx.softcap, ctx.softmax_scale = causal, window, cap, scale
        ctx.deterministic = bool(deterministic)
        if return_softmax:
            return out, lse, None
        return out

    @staticmethod
    def backward(ctx, dout, *args):
        q, k, v, out, lse, cu_q, cu_k = ctx.saved_tensors
        dq, dk, dv = _ext.varlen_backward(q, k, v, out, dout, lse, cu_q, cu_k, *ctx.max_seqlen,
                                          ctx.softmax_scale, ctx.causal, ctx.deterministic,
                                          ctx.window, ctx.softcap)
        return (dq, dk, dv) + (None,) * 12


def tilelang_flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                    max_seqlen_k, dropout_p=0.0, softmax_scale=None,
                                    causal=False, window_size=(-1, -1), softcap=0.0,
                                    alibi_slopes=None, deterministic=False,
                                    return_attn_probs=False):
    """FA2-compatible ``flash_attn_varlen_func`` over packed sequences (no reference
    counterpart: the reference's dense API takes equal-length batches).

    Args:
        q: [total_q, H, D]; k, v: [total_k, Hk, D] (H % Hk == 0), fp16 or bf16, D 64/128/256
        cu_seqlens_q / cu_seqlens_k: [batch + 1] int32 offsets of each sequence's rows
        max_seqlen_q / max_seqlen_k: upper bounds of the sequences' lengths
        causal, window_size, softcap: as tilelang_flash_attn_func, per sequence
            (bottom-right aligned on that sequence's own lengths)

    Returns:
        out: [total_q, H, D], or (out, lse [H, total_q] fp32, None)
    """
    return FlashAttnVarlenFunc.apply(
        q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, dropout_p,
        softmax_scale, causal, window_size, softcap, alibi_slopes, deterministic,
        return_attn_probs,
    )
