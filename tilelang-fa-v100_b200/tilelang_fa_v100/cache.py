"""Paged KV-cache write: the step that fills the vLLM-layout caches the paged prefill
and decode paths read.

No counterpart in the reference API (its paged kernels read caches their caller filled,
_kernels_paged.py:265-272 and :441-448); it stands in for the cache-write call a vLLM
attention backend makes before attention (reshape_and_cache_flash).
"""
import torch

from . import _ext


def write_kv_cache(key, value, k_cache, v_cache, slot_mapping, k_scale=1.0, v_scale=1.0):
    """Copies key[t] and value[t] ([Hkv, D] each) into k_cache / v_cache
    [num_pages, page_size, Hkv, D] at slot slot_mapping[t] = page * page_size + offset.

    Negative slots mark padding tokens and are skipped.  key / value may be views with a
    token stride (e.g. slices of a fused QKV projection) but each token's [Hkv, D] block
    must be contiguous.  A slot past the cache is not written and is reported by
    tilelang_fa_v100._ext.read_device_error() (code 3).

    fp8 caches (torch.float8_e4m3fn): the kernel stores key / k_scale and value / v_scale
    rounded to nearest and saturated to +-448, the layout tilelang_decode_forward reads
    with the same scales."""
    if key.dim() != 3 or value.shape != key.shape:
        raise ValueError("key and value must be [num_tokens, num_kv_heads, head_dim] of one shape")
    n, hkv, d = key.shape
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape or tuple(k_cache.shape[2:]) != (hkv, d):
        raise ValueError("caches must be [num_pages, page_size, %d, %d]" % (hkv, d))
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("caches must be contiguous")
    for t in (key, value):
        if t.stride(2) != 1 or t.stride(1) != d:
            raise ValueError("each token's [num_kv_heads, head_dim] block must be contiguous")
    if key.dtype != value.dtype or k_cache.dtype != v_cache.dtype or \
            k_cache.dtype not in (key.dtype, torch.float8_e4m3fn):
        raise ValueError("key / value share one dtype; the caches hold it or torch.float8_e4m3fn")
    if slot_mapping.dim() != 1 or slot_mapping.shape[0] != n:
        raise ValueError("slot_mapping must be [num_tokens]")
    if n == 0:
        return
    _ext.kv_cache_write(key, value, k_cache, v_cache, slot_mapping, k_scale, v_scale)
