/*
 * fa_b200.h -- C ABI of libfa_b200.so, the sm_100a (B200) FlashAttention kernels
 * behind the tilelang_fa_v100 Python API.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t (passed
 * as void*), returns 0 on success or a negative fa_status_t, never allocates
 * device memory (outputs and workspaces belong to the caller) and never
 * synchronises the stream.  Layouts are those of the reference API:
 *   dense  q [B, Sq, H, D], k/v [B, Skv, Hk, D]   (last dim contiguous)
 *   lse    [B, H, Sq] fp32                          (dense)
 *   cache  [num_pages, page_size, Hkv, D]          (vLLM paged KV cache)
 *   paged  q/out [num_tokens, H, D], lse [H, num_tokens] fp32
 *   decode q/out [B, H, D]
 * Supported: fp16 and bf16 inputs, H % Hk == 0; head_dim 32/64/96/128/256 (dense
 * forward and backward; 32 and 96 run the 64 and 128 kernels on zero-filled columns),
 * 64/128/256/512 (paged prefill; decode with H / Hkv <= 16).
 * Pointers 16-byte aligned, strides multiples of 8 elements.
 */
#ifndef FA_B200_H_
#define FA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  FA_OK = 0,
  FA_ERR_INVALID_ARG = -1,       /* null pointer, bad size, H % Hk != 0, ... */
  FA_ERR_UNSUPPORTED = -2,       /* head_dim / dtype / page_size not supported  */
  FA_ERR_ALIGNMENT = -3,         /* pointer or stride not 16-byte aligned       */
  FA_ERR_WORKSPACE = -4,         /* workspace missing or too small              */
  FA_ERR_CUDA = -5,              /* a CUDA runtime/driver call failed           */
  FA_ERR_DEVICE_TIMEOUT = -6,    /* a kernel's bounded wait expired (device)    */
  FA_ERR_NOT_SM100 = -7          /* current device is not compute capability 10.x */
} fa_status_t;

typedef enum { FA_DTYPE_F16 = 0, FA_DTYPE_BF16 = 1, FA_DTYPE_E4M3 = 2 } fa_dtype_t;

/* Dense forward.  Replaces tilelang_forward_lse(...)(q_, k_, v_) at
 * tilelang_fa_v100/interface.py:35-36 (kernel: _kernels_forward.py:94-172), minus
 * the BSHD<->BHSD permute copies (interface.py:19-21, 38): the kernel reads BSHD. */
typedef struct {
  const void* q;          /* [B, Sq, H, D]  */
  const void* k;          /* [B, Skv, Hk, D] */
  const void* v;          /* [B, Skv, Hk, D] */
  void* out;              /* [B, Sq, H, D]  */
  float* lse;             /* [B, H, Sq] (required) */
  int64_t q_stride[3];    /* batch, seq, head strides in elements */
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int32_t batch, seqlen_q, seqlen_k, num_heads, num_heads_k, head_dim;
  int32_t dtype;          /* fa_dtype_t */
  int32_t causal;         /* bottom-right aligned: key j visible to row i iff j <= i + Skv - Sq */
  float softmax_scale;
  /* Sliding window (FA2 window_size = (left, right) as window_q = left + 1,
   * window_k = right + 1; <= 0: unbounded on that side, so a zero-filled struct has
   * none): key j visible to row i iff i + Skv - Sq - window_q < j (window_q > 0) and
   * j < i + Skv - Sq + window_k (window_k > 0), on top of the causal bound.  No reference
   * counterpart: the reference accepts window_size and ignores it. */
  int32_t window_q, window_k;
  /* FA2 softcap: each score becomes softcap * tanh(softmax_scale * q.k / softcap) and
   * the softmax runs on those with unit scale; lse is their log-sum-exp.  0: off (a
   * zero-filled struct has none); otherwise finite and > 0 (FA_ERR_INVALID_ARG if not).
   * The reference raises NotImplementedError for softcap != 0 (interface.py:29-30). */
  float softcap;
} fa_fwd_args_t;

int fa_fwd(const fa_fwd_args_t* args, void* stream);

/* Dense backward.  Replaces tilelang_backward (_kernels_backward.py:200-208): the
 * row-dot (:203), the dQ kernel (:10-85) and the dK/dV kernel (:88-176).
 * Gradients are written in the BSHD layout of q/k/v.  Workspace (caller-owned,
 * fa_bwd_workspace_size bytes, 256-byte aligned): the fp32 row-dot [B,H,Sq] and,
 * in atomic mode at head_dim 64/128, the fp32 dQ accumulator [B,H,Sq,D].  At head_dim
 * 256 both modes run the same atomic-free kernels (bit-reproducible). */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  const void* out;
  const void* dout;       /* [B, Sq, H, D] */
  const float* lse;       /* [B, H, Sq] from fa_fwd */
  void* dq;               /* [B, Sq, H, D] */
  void* dk;               /* [B, Skv, Hk, D] */
  void* dv;               /* [B, Skv, Hk, D] */
  int64_t q_stride[3];
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int64_t do_stride[3];
  int64_t dq_stride[3];
  int64_t dk_stride[3];
  int64_t dv_stride[3];
  int32_t batch, seqlen_q, seqlen_k, num_heads, num_heads_k, head_dim;
  int32_t dtype;
  int32_t causal;
  int32_t deterministic;  /* 1: dQ by a separate per-Q-tile kernel (bit-reproducible);
                             0: dQ by fp32 atomics from the dK/dV kernel */
  float softmax_scale;
  int32_t window_q, window_k; /* as in fa_fwd_args_t; must match the forward's */
  float softcap;              /* as in fa_fwd_args_t; must match the forward's */
} fa_bwd_args_t;

size_t fa_bwd_workspace_size(const fa_bwd_args_t* args);
int fa_bwd(const fa_bwd_args_t* args, void* workspace, size_t workspace_bytes, void* stream);

/* Dense variable-length ("varlen") forward: FA2's flash_attn_varlen_func over packed
 * sequences.  No reference counterpart (the reference's dense API takes equal-length
 * batches).  Sequence b owns query rows [cu_seqlens_q[b], cu_seqlens_q[b + 1]) of q / out
 * and key rows [cu_seqlens_k[b], cu_seqlens_k[b + 1]) of k / v; causal and the window
 * are bottom-right aligned per sequence (key j visible to row i iff j <= i + Lk - Lq),
 * exactly as a dense call on that sequence alone.  lse is [H, total_q] (FA2's varlen
 * layout).  head_dim 64 / 128 / 256. */
typedef struct {
  const void* q;              /* [total_q, H, D]  */
  const void* k;              /* [total_k, Hk, D] */
  const void* v;              /* [total_k, Hk, D] */
  void* out;                  /* [total_q, H, D]  */
  float* lse;                 /* [H, total_q] (required) */
  const int32_t* cu_seqlens_q; /* [batch + 1], device, non-decreasing, cu[0] = 0 */
  const int32_t* cu_seqlens_k; /* [batch + 1], device */
  int64_t q_stride[2];        /* token, head strides in elements */
  int64_t k_stride[2];
  int64_t v_stride[2];
  int64_t o_stride[2];
  int32_t batch, total_q, total_k, max_seqlen_q, max_seqlen_k;
  int32_t num_heads, num_heads_k, head_dim;
  int32_t dtype;
  int32_t causal;
  float softmax_scale;
  int32_t window_q, window_k; /* as in fa_fwd_args_t */
  float softcap;              /* as in fa_fwd_args_t */
} fa_varlen_fwd_args_t;

int fa_varlen_fwd(const fa_varlen_fwd_args_t* args, void* stream);

/* Dense varlen backward (FA2's varlen backward): gradients in the packed layouts of
 * q / k / v.  max_seqlen_q / max_seqlen_k must bound every sequence (they size the
 * grids and the workspace); workspace as fa_bwd's for batch x max_seqlen_q rows. */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  const void* out;
  const void* dout;           /* [total_q, H, D] */
  const float* lse;           /* [H, total_q] from fa_varlen_fwd */
  void* dq;                   /* [total_q, H, D] */
  void* dk;                   /* [total_k, Hk, D] */
  void* dv;
  const int32_t* cu_seqlens_q;
  const int32_t* cu_seqlens_k;
  int64_t q_stride[2];
  int64_t k_stride[2];
  int64_t v_stride[2];
  int64_t o_stride[2];
  int64_t do_stride[2];
  int64_t dq_stride[2];
  int64_t dk_stride[2];
  int64_t dv_stride[2];
  int32_t batch, total_q, total_k, max_seqlen_q, max_seqlen_k;
  int32_t num_heads, num_heads_k, head_dim;
  int32_t dtype;
  int32_t causal;
  int32_t deterministic;
  float softmax_scale;
  int32_t window_q, window_k;
  float softcap;
} fa_varlen_bwd_args_t;

size_t fa_varlen_bwd_workspace_size(const fa_varlen_bwd_args_t* args);
int fa_varlen_bwd(const fa_varlen_bwd_args_t* args, void* workspace, size_t workspace_bytes,
                  void* stream);

/* Paged (vLLM-layout) prefill / chunked prefill forward.  Replaces
 * get_paged_kernel(...)(q, k_cache, v_cache, block_table, seq_lens,
 * query_start_loc, prefix_kv_lens, num_tokens, sm_scale) at
 * _paged_adapter.py:40-46 (kernel: _kernels_paged.py:193-344).  Query row i of
 * sequence b attends key j iff j < seq_lens[b] and, when causal,
 * j <= prefix_kv_lens[b] + i (plus the optional sliding window of
 * _kernels_paged.py:275-294).  Writes the real LSE [H, num_tokens]. */
typedef struct {
  const void* q;                  /* [num_tokens, H, D] */
  const void* k_cache;            /* [num_pages, page_size, Hkv, D] */
  const void* v_cache;
  const int32_t* block_table;     /* [num_seqs, max_blocks] */
  const int32_t* seq_lens;        /* [num_seqs] total KV length */
  const int32_t* query_start_loc; /* [num_seqs + 1] */
  const int32_t* prefix_kv_lens;  /* [num_seqs] */
  void* out;                      /* [num_tokens, H, D] */
  float* lse;                     /* [H, num_tokens] (may be NULL) */
  int32_t num_tokens, num_seqs, num_heads, num_kv_heads, head_dim;
  int32_t page_size, num_pages, max_blocks;
  int32_t dtype;
  int32_t causal;
  int32_t sliding_window_q, sliding_window_k; /* <= 0: off (only honoured when causal) */
  float softmax_scale;
} fa_paged_args_t;

int fa_paged_prefill(const fa_paged_args_t* args, void* stream);

/* Paged decode (one query token per sequence), split-KV + LSE combine.  Replaces
 * get_decode_kernel(...)(q, k_cache, v_cache, block_table, seq_lens) at
 * _decode_adapter.py:46 (kernel: _kernels_paged.py:393-489).  Workspace
 * (caller-owned, fa_decode_workspace_size bytes) holds the per-split partial
 * outputs and LSEs. */
typedef struct {
  const void* q;                  /* [B, H, D] */
  const void* k_cache;            /* [num_pages, page_size, Hkv, D] */
  const void* v_cache;
  const int32_t* block_table;     /* [B, max_blocks] */
  const int32_t* seq_lens;        /* [B] */
  void* out;                      /* [B, H, D] */
  float* lse;                     /* [B, H] (may be NULL) */
  int32_t batch, num_heads, num_kv_heads, head_dim;
  int32_t page_size, num_pages, max_blocks;
  int32_t dtype;
  int32_t num_splits;             /* 0: heuristic from max_blocks and the SM count */
  float softmax_scale;
  /* KV-cache element type: 0 = the query dtype, FA_DTYPE_E4M3 = fp8 (e4m3) caches
   * holding key / k_scale and value / v_scale (head_dim 128, 256 or 512); the kernel folds
   * k_scale into the scores and v_scale into the output.  Over fp8 caches the products
   * run in f16 for either query dtype (a bf16 query group enters them scaled by a power
   * of two, exact), so P is rounded to f16.  No counterpart in the reference (fp16
   * caches only); the layout of vLLM's fp8 KV cache with per-tensor scales. */
  int32_t kv_dtype;
  float k_scale, v_scale;
} fa_decode_args_t;

size_t fa_decode_workspace_size(const fa_decode_args_t* args);
int fa_decode(const fa_decode_args_t* args, void* workspace, size_t workspace_bytes, void* stream);

/* Paged KV-cache write (the step before the paged path): for each token t with
 * slot_mapping[t] >= 0, copies key[t] and value[t] (each [Hkv, D], contiguous) to
 * k_cache / v_cache[slot / page_size][slot % page_size].  Negative slots are padding
 * and are skipped; a slot beyond num_pages * page_size is not written and sets the
 * device error word (code 3).  No counterpart in the reference, which reads caches
 * that its caller filled (_kernels_paged.py:265-272, :441-448); it replaces the
 * cache-write call a vLLM attention backend makes before attention
 * (reshape_and_cache_flash, vllm/_custom_ops.py). */
typedef struct {
  const void* key;                /* [num_tokens, Hkv, D], token stride key_stride */
  const void* value;              /* [num_tokens, Hkv, D], token stride value_stride */
  void* k_cache;                  /* [num_pages, page_size, Hkv, D] */
  void* v_cache;
  const int64_t* slot_mapping;    /* [num_tokens] */
  int64_t key_stride;             /* elements between consecutive tokens */
  int64_t value_stride;
  int32_t num_tokens, num_kv_heads, head_dim, page_size, num_pages;
  int32_t dtype;                  /* fa_dtype_t of key / value (and of the caches when
                                     cache_dtype is 0) */
  /* 0: the caches hold `dtype`; FA_DTYPE_E4M3: they hold fp8 e4m3 and the kernel writes
   * key / k_scale and value / v_scale, rounded to nearest and saturated to +-448. */
  int32_t cache_dtype;
  float k_scale, v_scale;
} fa_kv_write_args_t;

int fa_kv_cache_write(const fa_kv_write_args_t* args, void* stream);

/* Decode that allocates nothing, not even a caller workspace.  No counterpart in the
 * reference: it exists for callers that cannot hand the library any device memory
 * at decode time -- e.g. a serving engine that gives all free HBM to its KV-cache
 * pool and forbids allocations inside a decode step, or a plain C/FFI caller with no
 * device allocator of its own -- and for latency-critical loops that must not call
 * cudaMalloc/cudaFree, which can synchronise the device and stall other streams.
 * Same arguments and results as fa_decode; the split partials go to a fixed
 * 16 MiB scratch array inside the library (fa_decode_noalloc_scratch_bytes) that
 * each GPU holds until the process exits.  With num_splits = 0 the split count is
 * reduced until the partials fit; an explicit num_splits whose partials
 * (batch * splits * num_heads * (head_dim + 1) * 4 bytes) exceed the scratch is
 * rejected with FA_ERR_WORKSPACE (fa_last_error_detail says why).  The first call
 * on a device looks up the scratch's device address, so make that first call
 * before any stream capture.  All calls share the one array: calls that overlap on
 * the GPU (different streams, no ordering between them) race on it. */
int fa_decode_noalloc(const fa_decode_args_t* args, void* stream);
size_t fa_decode_noalloc_scratch_bytes(void);

/* Diagnostics. */
const char* fa_status_string(int status);
/* Reads (and optionally clears) the library's device error word on the current
 * device: code, site and block index of the first error recorded.  Codes: 0 = none,
 * 1 = a bounded wait expired, 3 = fa_kv_cache_write got a slot past the cache,
 * 4 = a paged / decode call got seq_lens[b] > max_blocks * page_size (the keys were
 * clamped to the pages the block-table row maps).  Synchronises the device. */
int fa_read_device_error(int32_t* code, int32_t* site, int32_t* block, int32_t clear);
/* Text of the last CUDA call that made an entry point return FA_ERR_CUDA on this
 * host thread (call, source line, CUDA error string); "" if none. */
const char* fa_last_error_detail(void);
/* Library version and the number of kernels launched by this process so far. */
const char* fa_version(void);
int64_t fa_launch_count(void);

/* Benchmark hook: record ev_begin / ev_end (cudaEvent_t, created by the caller) on the
 * launch stream immediately around the NEXT launch of one main kernel:
 * 1 = dense forward, 2 = dense backward dK/dV kernel, 3 = paged prefill,
 * 4 = decode split kernel.  One shot and process-wide: the first matching launch
 * from any host thread takes the request (a new request replaces an unused one);
 * safe to call from several threads. */
int fa_profile_next_launch(int32_t kind, void* ev_begin, void* ev_end);

/* Self-test of the tcgen05 building blocks used by the attention kernels: one
 * 128 x N x K UMMA with the given operand majorness (0 = K-major, 1 = MN-major for
 * B) and A from shared memory (a_tmem = 0) or tensor memory (a_tmem = 1).
 * a: [128, K] row-major, b: [N, K] row-major (b_mn = 0) or [K, N] row-major
 * (b_mn = 1), c: [128, N] fp32.  K in {16..256, multiple of 64}, N in {64, 128, 256}. */
int fa_selftest_umma(const void* a, const void* b, float* c, int32_t n, int32_t k,
                     int32_t dtype, int32_t b_mn, int32_t a_tmem, void* stream);

/* Diagnostic: tcgen05 MMA throughput.  `ctas` CTAs each issue reps x (k/16)
 * back-to-back bf16 UMMAs of 128 x n x 16 on shared-memory operands (A from TMEM when
 * a_tmem = 1; a_mn / b_mn select MN-major layouts); time it with events on `stream`.
 * Used to justify the tile shapes of the attention kernels. */
int fa_selftest_umma_rate(int32_t n, int32_t k, int32_t reps, int32_t a_tmem, int32_t a_mn,
                          int32_t b_mn, int32_t ctas, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FA_B200_H_ */
