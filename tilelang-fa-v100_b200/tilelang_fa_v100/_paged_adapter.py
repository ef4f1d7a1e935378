"""Adapter: vLLM 4D paged K/V cache -> the sm_100a paged prefill kernel.

Mirror of the reference's _paged_adapter.py:15-52 (same signature, defaults and
return value).  The kernel writes straight into ``out`` (no extra ``out.copy_``,
reference :48-49) and fills the real LSE [num_heads, num_tokens] (the reference
returns an uninitialised tensor, :51).
"""
import math

import torch

from . import _ext


def paged_forward(q, k_cache, v_cache, block_table, seq_lens,
                  query_start_loc, prefix_kv_lens, out=None,
                  block_size=16, num_kv_heads=None, softmax_scale=None,
                  causal=True, sliding_window_q=-1, sliding_window_k=-1):
    num_tokens, num_heads, D = q.shape
    heads_kv = num_kv_heads or k_cache.shape[2]
    B = block_table.shape[0]

    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(D)
    if k_cache.shape[1] != block_size or v_cache.shape != k_cache.shape:
        raise ValueError("k/v cache must be [num_pages, block_size=%d, kv_heads, dim]; got %s / %s"
                         % (block_size, tuple(k_cache.shape), tuple(v_cache.shape)))
    if k_cache.shape[2] != heads_kv or k_cache.shape[3] != D:
        raise ValueError("cache heads/dim %s do not match num_kv_heads=%d, dim=%d"
                         % (tuple(k_cache.shape[2:]), heads_kv, D))
    if query_start_loc.numel() != B + 1 or seq_lens.numel() != B or prefix_kv_lens.numel() != B:
        raise ValueError("query_start_loc must have B+1 entries and seq_lens / prefix_kv_lens B")
    if q.dtype != k_cache.dtype or q.dtype != v_cache.dtype:
        raise ValueError("q and cache dtypes differ")

    q_c = q.contiguous()
    k_c = k_cache.contiguous()
    v_c = v_cache.contiguous()
    if out is None:
        out = torch.empty_like(q_c)
    target = out if (out.is_contiguous() and out.dtype == q.dtype) else torch.empty_like(q_c)
    softmax_lse = torch.empty(num_heads, num_tokens, dtype=torch.float32, device=q.device)

    _ext.paged_prefill(q_c, k_c, v_c, block_table, seq_lens, query_start_loc, prefix_kv_lens,
                       target, softmax_lse, block_size, heads_kv, softmax_scale, causal,
                       sliding_window_q, sliding_window_k)
    if target is not out:
        out.copy_(target)
    return out, softmax_lse
