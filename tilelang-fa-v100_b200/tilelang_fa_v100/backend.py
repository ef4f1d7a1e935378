"""vLLM-style attention backend over the B200 kernels: the caller side of
tilelang_paged_forward / tilelang_decode_forward (interface.py:83-117 of the
reference).

A serving engine hands one forward step of a continuous batch: the new tokens' q/k/v,
the paged KV cache and the scheduler's metadata.  The step (1) writes the new keys and
values into the cache at their slots (tilelang_fa_v100.cache.write_kv_cache), then
(2) runs attention of every new token over its sequence's cached context plus the new
tokens: the leading ``num_decodes`` sequences have one new token each and go to the
split-KV decode kernel, the rest (prefill and chunked prefill) to the paged prefill
kernel with ``prefix_kv_lens = seq_lens - query_lens``.

The metadata fields are the subset of vLLM's FlashAttentionMetadata this path needs,
with the same names and meaning (vllm/v1/attention/backends/flash_attn.py); the cache
is vLLM's flash layout [2, num_blocks, block_size, num_kv_heads, head_size].
"""
from dataclasses import dataclass
from typing import Optional

import torch

from . import _ext
from ._paged_adapter import paged_forward
from .cache import write_kv_cache


@dataclass
class AttentionMetadata:
    num_actual_tokens: int          # new tokens in the step, padding excluded
    max_query_len: int
    query_start_loc: torch.Tensor   # [num_seqs + 1] int32: new-token offsets
    max_seq_len: int
    seq_lens: torch.Tensor          # [num_seqs] int32: cached context + new tokens
    block_table: torch.Tensor       # [num_seqs, max_blocks] int32
    slot_mapping: torch.Tensor      # [num_tokens] int64 cache slot of each new token
    num_decodes: int = 0            # leading sequences with exactly one new token


class TileLangFAAttentionImpl:
    """Attention layer implementation: ``forward(query, key, value, kv_cache, metadata)``."""

    def __init__(self, num_heads: int, head_size: int, scale: Optional[float] = None,
                 num_kv_heads: Optional[int] = None, sliding_window: Optional[int] = None,
                 logits_soft_cap: Optional[float] = None, alibi_slopes=None):
        if sliding_window is not None:
            raise NotImplementedError("sliding_window is not supported by this backend")
        if logits_soft_cap:
            raise NotImplementedError("logits_soft_cap is not supported")
        if alibi_slopes is not None:
            raise NotImplementedError("alibi_slopes is not supported")
        self.num_heads = num_heads
        self.head_size = head_size
        self.num_kv_heads = num_kv_heads or num_heads
        if num_heads % self.num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        self.scale = float(scale) if scale is not None else head_size ** -0.5

    def forward(self, query, key, value, kv_cache, attn_metadata: AttentionMetadata,
                output=None):
        """query [T, H, D], key / value [T, Hkv, D], kv_cache [2, P, page, Hkv, D].
        Returns (or fills) output [T, H, D]; rows past num_actual_tokens are untouched."""
        md = attn_metadata
        n = md.num_actual_tokens
        if kv_cache.dim() != 5 or kv_cache.shape[0] != 2:
            raise ValueError("kv_cache must be [2, num_blocks, block_size, num_kv_heads, head_size]")
        k_cache, v_cache = kv_cache[0], kv_cache[1]
        page = k_cache.shape[1]
        if output is None:
            output = torch.empty_like(query)
        if n == 0:
            return output
        write_kv_cache(key[:n], value[:n], k_cache, v_cache, md.slot_mapping[:n])

        num_seqs = md.block_table.shape[0]
        nd = int(md.num_decodes)
        if nd:  # decode requests come first: token i belongs to sequence i
            _ext.decode(query[:nd], k_cache, v_cache, md.block_table[:nd], md.seq_lens[:nd],
                        page, self.num_kv_heads, self.scale, out=output[:nd])
        if nd < num_seqs:
            qsl = md.query_start_loc[nd:]
            qsl = (qsl - qsl[:1]).to(torch.int32)
            sl = md.seq_lens[nd:]
            prefix = (sl - (qsl[1:] - qsl[:-1])).to(torch.int32)
            paged_forward(query[nd:n], k_cache, v_cache, md.block_table[nd:], sl, qsl, prefix,
                          out=output[nd:n], block_size=page, num_kv_heads=self.num_kv_heads,
                          softmax_scale=self.scale, causal=True)
        return output
