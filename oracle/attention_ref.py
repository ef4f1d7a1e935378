"""CPU oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may
import this module, and only as the checker or the timed CPU baseline.  The
product path (tilelang_fa_v100 + libfa_b200.so) never calls it.

It restates, in numpy (float64 arithmetic, float32 results), the reference
repository's pure-PyTorch attention oracles and the semantics of its kernels:

* ``attention_ref``  -- ``pytorch_gqa_ref`` (tests/test_gqa_paged.py:19-45) and
  ``pytorch_ref`` (tests/test_compare_ref.py:15-25): GQA head expansion
  (test_gqa_paged.py:37-38), scores = q k^T * scale (:40), bottom-right causal mask
  ``tril(ones(M, N), diagonal=N-M)`` (:41-43), softmax (:44), P V (:45).  The LSE
  is the natural-log ``m * scale + ln(l)`` the kernels write
  (_kernels_forward.py:170).
* ``visible_mask`` -- that causal mask combined with FA2's dense sliding window
  (window_size = (left, right), bottom-right aligned), which the reference accepts and
  ignores (interface.py:33); the default (-1, -1) leaves the reference's mask.
* ``softcap`` arguments -- FA2's score softcapping, scores = c tanh(scale q k^T / c)
  with a unit-scale softmax on top (its backward multiplies dS by 1 - tanh^2).  The
  reference raises NotImplementedError for softcap != 0 (interface.py:29-30); 0 leaves
  the reference's function.
* ``attention_bwd_ref`` -- gradients of the same function, i.e. what the reference
  backward computes (_kernels_backward.py): D = rowsum(dO * O) (:203),
  dP = dO V^T (:55), dS = P * (dP - D) (:72-74), dQ = scale dS K (:80),
  dV = P^T dO (:166), dK = scale dS^T Q (:170).
* ``paged_prefill_ref`` -- the paged kernel's masking (_kernels_paged.py:296-303):
  query i of sequence b sees key j iff j < seq_lens[b] and, when causal,
  j <= prefix_kv_lens[b] + i, plus the sliding window of :275-294; K/V gathered
  page by page through block_table (:265-272).
* ``decode_ref`` -- the decode kernel (_kernels_paged.py:393-489): one query per
  sequence, every key j < seq_lens[b] visible.

* ``kv_cache_write_ref`` -- the cache-write step before the paged path (no reference
  counterpart): token t's [Hkv, D] key / value rows land at cache[slot // page_size,
  slot % page_size] for slot = slot_mapping[t] >= 0 (the slot addressing the paged
  kernels read back through block_table, _kernels_paged.py:265-272); negative slots
  are padding.  Pinned by the paged golden vectors: writing a golden sequence's tokens
  through this function reproduces the golden cache.

* rounding bounds (``unit_roundoff`` arguments, ``attention_out_bound``) -- per-element
  worst cases of what rounding the MMA operands that every FlashAttention kernel rounds
  to the 16-bit input type (P, dS) and the outputs can change.  The reference rounds
  the same operands (_kernels_forward.py:162-165, _kernels_backward.py:77).  A kernel
  inside the bound differs from this fp32 oracle by rounding alone; bf16 tests use it
  as their bar, since bf16's 8-bit significand puts single rounding errors at the
  size of the fp16-oriented absolute bars.

Pinning: tests/test_oracle_golden.py checks every function here against golden
vectors produced by running the reference's own ``pytorch_gqa_ref`` and
``make_paged_gqa`` (tests/golden/make_golden.py).
"""
import numpy as np

NEG_INF = -np.inf


def _softmax_lse(scores):
    """Row softmax and natural-log LSE; fully masked rows give P = 0, LSE = -inf."""
    if scores.shape[-1] == 0:
        return np.zeros_like(scores), np.full(scores.shape[:-1], NEG_INF)
    m = np.max(scores, axis=-1, keepdims=True)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    e = np.exp(scores - m_safe)
    l = np.sum(e, axis=-1, keepdims=True)
    with np.errstate(divide="ignore", invalid="ignore"):
        p = np.where(l > 0, e / np.where(l > 0, l, 1.0), 0.0)
        lse = np.where(l > 0, m_safe + np.log(np.where(l > 0, l, 1.0)), NEG_INF)
    return p, lse[..., 0]


def causal_mask(m, n):
    """Bottom-right aligned causal mask: key j visible to query i iff j <= i + n - m."""
    i = np.arange(m)[:, None]
    j = np.arange(n)[None, :]
    return j <= i + (n - m)


def visible_mask(m, n, causal, window=(-1, -1)):
    """Key visibility [m, n] of a dense call, or None when every key is visible: the
    causal mask above and FA2's sliding window ``window_size = (left, right)``, bottom-right
    aligned like it -- key j visible to query i iff i + n - m - left <= j (left >= 0) and
    j <= i + n - m + right (right >= 0).  The window has no reference counterpart (the
    reference accepts window_size and ignores it, interface.py:33); with the default
    (-1, -1) this is the reference's mask."""
    left, right = (-1, -1) if window is None else (int(window[0]), int(window[1]))
    if not causal and left < 0 and right < 0:
        return None
    a = np.arange(m)[:, None] + (n - m)
    j = np.arange(n)[None, :]
    vis = np.ones((m, n), dtype=bool)
    if causal:
        vis &= j <= a
    if left >= 0:
        vis &= j >= a - left
    if right >= 0:
        vis &= j <= a + right
    return vis


def _expand_kv(x, hq):
    hkv = x.shape[1]
    return np.repeat(x, hq // hkv, axis=1)


def _scores(q, k, scale, softcap):
    """scale q k^T, softcapped to c tanh(. / c) when softcap = c > 0; also returns the
    factor d(capped)/d(scaled) = 1 - tanh^2 (1 without softcap)."""
    s = (q @ k.swapaxes(-1, -2)) * scale
    if softcap is None or softcap <= 0:
        return s, 1.0
    t = np.tanh(s / softcap)
    return softcap * t, 1.0 - t * t


def attention_ref(q, k, v, causal, scale=None, return_p=False, window=(-1, -1), softcap=0.0):
    """q [B, Hq, M, D], k/v [B, Hkv, N, D] -> out [B, Hq, M, D] f32, lse [B, Hq, M] f32."""
    q = np.asarray(q, dtype=np.float64)
    k = _expand_kv(np.asarray(k, dtype=np.float64), q.shape[1])
    v = _expand_kv(np.asarray(v, dtype=np.float64), q.shape[1])
    d = q.shape[-1]
    scale = 1.0 / np.sqrt(d) if scale is None else scale
    s, _ = _scores(q, k, scale, softcap)
    vis = visible_mask(q.shape[2], k.shape[2], causal, window)
    if vis is not None:
        s = np.where(vis, s, NEG_INF)
    p, lse = _softmax_lse(s)
    out = p @ v
    if return_p:
        return out.astype(np.float32), lse.astype(np.float32), p
    return out.astype(np.float32), lse.astype(np.float32)


def attention_bwd_ref(q, k, v, do, causal, scale=None, o=None, unit_roundoff=None,
                      window=(-1, -1), softcap=0.0):
    """Gradients (dq [B,Hq,M,D], dk/dv [B,Hkv,N,D]) of attention_ref w.r.t. q, k, v.

    ``o``: the forward output the backward is given ([B,Hq,M,D]); when passed, the row
    dot D = rowsum(dO * O) uses it, as the reference backward does with the fp16 output
    its forward stored (_kernels_backward.py:203).  Without it D uses the exact output
    (the gradient of the fp32 function).

    ``unit_roundoff`` u (2**-8 for bf16, 2**-11 for fp16): also return per-element
    bounds (bq, bk, bv) on what rounding the operands that every FlashAttention backward
    rounds to the input type can change: P before dV = P^T dO (:166), dS before
    dQ = dS K and dK = dS^T Q (:77, :80, :170), and the three outputs themselves:
        bv = u (sum_i P_ij |dO_id| + |dV_jd|)
        bq = u (sum_j |dS_ij| |K_jd| + |dQ_id|)      (dS including the softmax scale)
        bk = u (sum_i |dS_ij| |Q_id| + |dK_jd|)
    Each is a worst case (all roundings of one sum in the same direction), so a kernel
    that rounds exactly those operands stays inside it up to fp32 accumulation error."""
    q64 = np.asarray(q, dtype=np.float64)
    k64 = np.asarray(k, dtype=np.float64)
    v64 = np.asarray(v, dtype=np.float64)
    do64 = np.asarray(do, dtype=np.float64)
    hq, hkv = q64.shape[1], k64.shape[1]
    d = q64.shape[-1]
    scale = 1.0 / np.sqrt(d) if scale is None else scale
    ke = _expand_kv(k64, hq)
    ve = _expand_kv(v64, hq)
    s, dcap = _scores(q64, ke, scale, softcap)
    vis = visible_mask(q64.shape[2], ke.shape[2], causal, window)
    if vis is not None:
        s = np.where(vis, s, NEG_INF)
    p, _ = _softmax_lse(s)
    if o is None:
        o = p @ ve
    dsum = np.sum(do64 * np.asarray(o, np.float64), axis=-1, keepdims=True)  # row-dot D
    dp = do64 @ ve.swapaxes(-1, -2)  # dO V^T
    ds = p * (dp - dsum) * dcap
    dq = (ds @ ke) * scale
    dke = (ds.swapaxes(-1, -2) @ q64) * scale
    dve = p.swapaxes(-1, -2) @ do64
    g = hq // hkv
    b, _, n, _ = dke.shape
    dk = dke.reshape(b, hkv, g, n, d).sum(axis=2)
    dv = dve.reshape(b, hkv, g, n, d).sum(axis=2)
    grads = (dq.astype(np.float32), dk.astype(np.float32), dv.astype(np.float32))
    if unit_roundoff is None:
        return grads
    u = float(unit_roundoff)
    ads = np.abs(ds) * scale
    bq = u * (ads @ np.abs(ke) + np.abs(dq))
    bk = (ads.swapaxes(-1, -2) @ np.abs(q64)).reshape(b, hkv, g, n, d).sum(axis=2)
    bk = u * (bk + np.abs(dk))
    bv = (p.swapaxes(-1, -2) @ np.abs(do64)).reshape(b, hkv, g, n, d).sum(axis=2)
    bv = u * (bv + np.abs(dv))
    return grads, (bq, bk, bv)


def attention_out_bound(q, k, v, causal, unit_roundoff, scale=None, window=(-1, -1),
                        softcap=0.0):
    """Per-element bound [B,Hq,M,D] on what rounding P to the input type before the P V
    product (_kernels_forward.py:162-165) and rounding the output can change:
    u (sum_j P_ij |v_jd| + |out_id|), a worst case over the rounding directions."""
    _, _, p = attention_ref(q, k, v, causal, scale=scale, return_p=True, window=window,
                            softcap=softcap)
    ve = _expand_kv(np.asarray(v, np.float64), np.asarray(q).shape[1])
    out = p @ ve
    return float(unit_roundoff) * (p @ np.abs(ve) + np.abs(out))


# Unit roundoff of the 16-bit input types (round to nearest: |fl(x) - x| <= u |x|).
UNIT_ROUNDOFF = {"float16": 2.0 ** -11, "bfloat16": 2.0 ** -8}


def gather_pages(cache, block_table_row, length):
    """Tokens [0, length) of one sequence from a [P, page, Hkv, D] cache -> [Hkv, length, D]."""
    page = cache.shape[1]
    idx = np.arange(length)
    pages = np.asarray(block_table_row)[idx // page]
    return np.asarray(cache)[pages, idx % page].transpose(1, 0, 2)


def paged_prefill_ref(q, k_cache, v_cache, block_table, seq_lens, query_start_loc,
                      prefix_kv_lens, causal=True, scale=None, sliding_window_q=-1,
                      sliding_window_k=-1, unit_roundoff=None):
    """q [T, H, D] -> out [T, H, D] f32, lse [H, T] f32 (reference kernel semantics).
    With ``unit_roundoff`` also the output's rounding bound [T, H, D] (see
    attention_out_bound)."""
    q = np.asarray(q, dtype=np.float64)
    t, h, d = q.shape
    hkv = k_cache.shape[2]
    scale = 1.0 / np.sqrt(d) if scale is None else scale
    out = np.zeros((t, h, d), np.float64)
    bound = np.zeros((t, h, d), np.float64)
    lse = np.full((h, t), NEG_INF, np.float64)
    for b in range(len(seq_lens)):
        q0, q1 = int(query_start_loc[b]), int(query_start_loc[b + 1])
        if q1 <= q0:
            continue
        length = int(seq_lens[b])
        kb = gather_pages(k_cache, block_table[b], length).astype(np.float64)
        vb = gather_pages(v_cache, block_table[b], length).astype(np.float64)
        kb = np.repeat(kb, h // hkv, axis=0)
        vb = np.repeat(vb, h // hkv, axis=0)
        qb = q[q0:q1].transpose(1, 0, 2)                      # [H, ql, D]
        s = (qb @ kb.swapaxes(-1, -2)) * scale
        i = np.arange(q1 - q0)[:, None]
        j = np.arange(length)[None, :]
        vis = np.ones((q1 - q0, length), bool)
        if causal:
            vis &= j <= int(prefix_kv_lens[b]) + i
            if sliding_window_q > 0:
                vis &= i < j + sliding_window_q
            if sliding_window_k > 0:
                vis &= j < i + sliding_window_k
        s = np.where(vis[None], s, NEG_INF)
        p, l_ = _softmax_lse(s)
        out[q0:q1] = (p @ vb).transpose(1, 0, 2)
        lse[:, q0:q1] = l_
        if unit_roundoff is not None:
            bound[q0:q1] = (p @ np.abs(vb)).transpose(1, 0, 2)
    if unit_roundoff is not None:
        bound = float(unit_roundoff) * (bound + np.abs(out))
        return out.astype(np.float32), lse.astype(np.float32), bound
    return out.astype(np.float32), lse.astype(np.float32)


def decode_ref(q, k_cache, v_cache, block_table, seq_lens, scale=None, unit_roundoff=None):
    """q [B, H, D] -> out [B, H, D] f32, lse [B, H] f32; all keys < seq_lens[b] visible.
    With ``unit_roundoff`` also the output's rounding bound [B, H, D]."""
    q = np.asarray(q, dtype=np.float64)
    bsz, h, d = q.shape
    qsl = np.arange(bsz + 1)
    r = paged_prefill_ref(q, k_cache, v_cache, block_table, seq_lens, qsl,
                          np.zeros(bsz, np.int64), causal=False, scale=scale,
                          unit_roundoff=unit_roundoff)
    if unit_roundoff is not None:
        return r[0], np.ascontiguousarray(r[1].T), r[2]
    return r[0], np.ascontiguousarray(r[1].T)


def make_paged_cache(k, v, page_size=16, shuffle_seed=None, num_pages=None):
    """Dense k/v [B, Hkv, N, D] -> (k_cache, v_cache, block_table) in the vLLM layout.

    Sequence b's logical page p holds tokens [p*page, (p+1)*page); physical pages are
    a seeded permutation when ``shuffle_seed`` is given (scattered allocation)."""
    bsz, hkv, n, d = k.shape
    pps = -(-n // page_size)
    total = bsz * pps if num_pages is None else num_pages
    perm = np.arange(total)
    if shuffle_seed is not None:
        perm = np.random.default_rng(shuffle_seed).permutation(total)
    kc = np.zeros((total, page_size, hkv, d), k.dtype)
    vc = np.zeros((total, page_size, hkv, d), v.dtype)
    bt = np.zeros((bsz, pps), np.int32)
    for b in range(bsz):
        for p in range(pps):
            phys = perm[b * pps + p]
            bt[b, p] = phys
            t0, t1 = p * page_size, min(n, (p + 1) * page_size)
            kc[phys, : t1 - t0] = k[b, :, t0:t1].transpose(1, 0, 2)
            vc[phys, : t1 - t0] = v[b, :, t0:t1].transpose(1, 0, 2)
    return kc, vc, bt


def kv_cache_write_ref(key, value, k_cache, v_cache, slot_mapping):
    """In-place scatter of key / value [T, Hkv, D] into the paged caches (numpy)."""
    page = k_cache.shape[1]
    for t, slot in enumerate(np.asarray(slot_mapping).tolist()):
        if slot < 0:
            continue
        k_cache[slot // page, slot % page] = key[t]
        v_cache[slot // page, slot % page] = value[t]


def quantize_e4m3(x, scale):
    """x / scale rounded to nearest even e4m3 and saturated to +-448 (the rounding of
    cvt.rn.satfinite.e4m3x2.f32), as raw bytes (uint8 array of x's shape).  fp8 caches
    have no reference counterpart; this restates vLLM's per-tensor-scale fp8 KV cache."""
    import torch
    y = np.clip(np.asarray(x, np.float32) / np.float32(scale), -448.0, 448.0)
    return torch.from_numpy(y).to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def dequantize_e4m3(raw, scale):
    """e4m3 bytes (uint8) -> float32 values times scale."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(raw)).view(torch.float8_e4m3fn).float().numpy()
    return t * np.float32(scale)


def slots_for(block_table_row, positions, page_size):
    """Slot ids of token positions of one sequence under its block table row."""
    pos = np.asarray(positions)
    return np.asarray(block_table_row)[pos // page_size].astype(np.int64) * page_size + pos % page_size


def flops_dense(b, h, sq, skv, d, causal):
    """Algorithmic forward FLOPs on visible (query, key) pairs: 4 * D per pair."""
    return 4.0 * d * visible_pairs(b, h, sq, skv, causal)


def visible_pairs(b, h, sq, skv, causal):
    if not causal:
        return float(b) * h * sq * skv
    off = skv - sq
    i = np.arange(sq, dtype=np.int64)
    per_row = np.clip(i + off + 1, 0, skv)
    return float(b) * h * float(per_row.sum())
