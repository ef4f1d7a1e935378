"""Adapter: paged decode (one query token per sequence) on the sm_100a kernels.

Mirror of the reference's _decode_adapter.py:15-47 (same signature and return).
``softmax_scale`` is passed to the kernel (the reference computes it and then lets
the kernel use 1/sqrt(dim), _kernels_paged.py:396; equal for the default).

Beyond the reference (fp16 caches only): the caches may be torch.float8_e4m3fn holding
key / k_scale and value / v_scale (vLLM's fp8 KV cache with per-tensor scales, head_dim
128, 256 or 512); ``k_scale`` / ``v_scale`` default to 1.
"""
import math

import torch

from . import _ext


def decode_forward(q, k_cache, v_cache, block_table, seq_lens,
                   block_size=16, num_kv_heads=None, softmax_scale=None,
                   k_scale=1.0, v_scale=1.0):
    """Paged decode forward.

    Args:
        q: [batch, heads, dim] fp16/bf16 -- one query token per sequence
        k_cache: [num_blocks, block_size, num_kv_heads, head_dim]
        v_cache: [num_blocks, block_size, num_kv_heads, head_dim]
        block_table: [batch, max_blocks_per_seq] int32
        seq_lens: [batch] int32 -- total KV cache lengths
        block_size: int -- page block size (vLLM default 16)
        num_kv_heads: int -- number of KV heads
        softmax_scale: float -- scale factor (default: 1/sqrt(dim))
        k_scale, v_scale: float -- dequantisation scales of fp8 (e4m3) caches

    Returns:
        output: [batch, heads, dim] -- attention output
    """
    batch, num_heads, dim = q.shape
    heads_kv = num_kv_heads or k_cache.shape[2]

    if softmax_scale is None:
        softmax_scale = 1.0 / math.sqrt(dim)
    if k_cache.shape[1] != block_size or v_cache.shape != k_cache.shape:
        raise ValueError("k/v cache must be [num_pages, block_size=%d, kv_heads, dim]; got %s / %s"
                         % (block_size, tuple(k_cache.shape), tuple(v_cache.shape)))
    if k_cache.shape[2] != heads_kv or k_cache.shape[3] != dim:
        raise ValueError("cache heads/dim %s do not match num_kv_heads=%d, dim=%d"
                         % (tuple(k_cache.shape[2:]), heads_kv, dim))
    if k_cache.dtype != v_cache.dtype or k_cache.dtype not in (q.dtype, torch.float8_e4m3fn):
        raise ValueError("caches must both hold q's dtype or both torch.float8_e4m3fn")

    return _ext.decode(q, k_cache.contiguous(), v_cache.contiguous(), block_table, seq_lens,
                       block_size, heads_kv, softmax_scale, k_scale=k_scale, v_scale=v_scale)
