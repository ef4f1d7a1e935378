// Host-side internals shared by the kernel translation units and the C ABI.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>
#include "../../include/fa_b200.h"

namespace fa {

// Forward-kernel parameters shared by the dense and the paged (varlen) modes.
struct FwdParams {
  int Sq;            // dense: query length; paged: unused
  int Skv;           // dense: key length; paged: unused
  int H, Hk, G;      // query heads, kv heads, G = H / Hk (rows of a kv head packed per Q tile)
  int causal;
  float scale;       // softmax scale
  float scale_log2;  // scale * log2(e)
  void* out;
  float* lse;
  int64_t o_sb, o_st, o_sh;        // out strides (elements): batch, token, head
  int64_t lse_sb, lse_sh;          // lse strides (elements): batch, head (token stride 1)
  // paged mode
  const int32_t* block_table;
  const int32_t* seq_lens;
  const int32_t* qsl;
  const int32_t* pkl;
  int num_seqs, max_blocks, page_size, num_pages;
  // varlen (dense packed sequences through the paged pipeline): sequence b's K / V rows
  // are [cu_k[b], cu_k[b + 1]) of [total_k, Hk, D] tensors; null for paged and dense
  const int32_t* cu_k;
  int swq, swk;
  // softcap (dense only): sc_a = softcap / scale (0: off), sc_k = 2 log2(e) / sc_a
  float sc_a, sc_k;
  // persistent scheduling: the work list is nbx q-block slots x kv heads (x batch, dense)
  int nbx, n_items;
  int* sched;  // device counter of claimed work-list entries (zeroed before the launch)
  int* err;
};

// Dense visibility (forward and backward): key j is visible to query row i iff, with the
// anchor a = i + Skv - Sq (bottom-right alignment), j <= a when causal, a - swq < j when
// swq > 0 and j < a + swk when swk > 0 (FA2 window_size (left, right) as swq = left + 1,
// swk = right + 1; <= 0: unbounded on that side).
__host__ __device__ __forceinline__ bool dense_visible(int key, int qi, int off, int causal,
                                                      int swq, int swk) {
  const int a = qi + off;
  return (!causal || key <= a) && (swq <= 0 || a - swq < key) && (swk <= 0 || key < a + swk);
}
// Query tiles [t0, t1) (bm rows each, Sq rows in all) holding a row that sees a key of
// [k0, k0 + bn).
__host__ __device__ __forceinline__ void dense_q_tiles(int k0, int bn, int bm, int Sq, int off,
                                                      int causal, int swq, int swk, int& t0,
                                                      int& t1) {
  const int nq = (Sq + bm - 1) / bm;
  int lo = 0, hi = Sq - 1;
  if (causal) lo = max(lo, k0 - off);
  if (swk > 0) lo = max(lo, k0 - off - swk + 1);
  if (swq > 0) hi = min(hi, k0 + bn - 2 - off + swq);
  t0 = min(nq, lo / bm);
  t1 = hi < lo ? t0 : min(nq, hi / bm + 1);
}
// Key tiles [j0, j1) (bn keys each, Skv keys in all) holding a key that a row of
// [q0, q0 + bm) sees.
__host__ __device__ __forceinline__ void dense_k_tiles(int q0, int bm, int bn, int Sq, int Skv,
                                                      int off, int causal, int swq, int swk,
                                                      int& j0, int& j1) {
  const int q1 = min(q0 + bm, Sq) - 1;
  int lo = 0, hi = Skv - 1;
  if (causal) hi = min(hi, q1 + off);
  if (swk > 0) hi = min(hi, q1 + off + swk - 1);
  if (swq > 0) lo = max(lo, q0 + off - swq + 1);
  j0 = min(lo / bn, (Skv + bn - 1) / bn);
  j1 = hi < lo ? j0 : hi / bn + 1;
}

// Lengths and packed-row offsets of batch entry b: dense launches use the call's Sq / Skv
// and TMA batch coordinate b; varlen launches (EXT kernels) the sequence's own lengths,
// its first packed rows and batch coordinate 0.  A varlen length is capped at the call's
// longest (Sq / Skv = max_seqlen_q / _k), which sizes the grids and the padded per-row
// workspace: a sequence longer than its max_seqlen loses its excess rows, it never reads
// or writes past the workspace.
struct BwdSeq {
  int Sq, Skv;  // query / key rows of this batch entry
  int qr, kr;   // first packed query / key row (0 for dense)
  int tb;       // TMA batch coordinate
};
template <bool EXT, typename Params>
__device__ __forceinline__ BwdSeq bwd_seq(const Params& p, int b) {
  if (EXT && p.cu_q != nullptr) {
    const int qr = p.cu_q[b], kr = p.cu_k[b];
    return {min(p.cu_q[b + 1] - qr, p.Sq), min(p.cu_k[b + 1] - kr, p.Skv), qr, kr, 0};
  }
  return {p.Sq, p.Skv, 0, 0, b};
}

constexpr int kFwdBN = 128;  // keys per forward KV tile

// Sliding window: dense and varlen launches take FA2's window_size, bottom-right aligned
// like the causal mask (anchor = row's token + Skv - Sq); paged launches the reference's
// paged window, anchored on the row's token and honoured only with causal
// (_kernels_paged.py:275-294).  Key j is visible iff anchor - swq < j (swq > 0) and
// j < anchor + swk (swk > 0).
// VARLEN: a varlen launch of the paged pipeline (compile-time, so paged launches keep
// their code unchanged).
template <bool PAGED, bool VARLEN = false>
__device__ __forceinline__ constexpr bool fwd_paged_window() {
  return PAGED && !VARLEN;
}
template <bool PAGED, bool VARLEN = false>
__device__ __forceinline__ bool fwd_window_on(const FwdParams& p) {
  return (fwd_paged_window<PAGED, VARLEN>() ? p.causal != 0 : true) && (p.swq > 0 || p.swk > 0);
}
// KV tiles [j0, j1) that the rows of tokens [tok0, tok0 + TPB) of a work item can see:
// keys below kv_len, the causal bound and the sliding window.
template <bool PAGED, bool VARLEN = false>
__device__ __forceinline__ void fwd_kv_range(const FwdParams& p, int tok0, int TPB, int q_len,
                                             int kv_len, int off, int& j0, int& j1) {
  j0 = 0;
  j1 = (kv_len + kFwdBN - 1) / kFwdBN;
  const int last_lt = min(tok0 + TPB, q_len) - 1;
  if (p.causal) {
    const int max_key = last_lt + off;
    j1 = min(j1, max_key >= 0 ? max_key / kFwdBN + 1 : 0);
  }
  if (fwd_window_on<PAGED, VARLEN>(p)) {
    constexpr bool pw = fwd_paged_window<PAGED, VARLEN>();
    const int a0 = pw ? tok0 : tok0 + off, a1 = pw ? last_lt : last_lt + off;
    if (p.swq > 0) j0 = max(0, a0 - p.swq + 1) / kFwdBN;
    if (p.swk > 0) {
      const int max_key = a1 + p.swk - 1;
      j1 = min(j1, max_key >= 0 ? max_key / kFwdBN + 1 : 0);
    }
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
CUresult encode_tmap(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                     const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                     CUtensorMapSwizzle swizzle);
inline CUtensorMapDataType tmap_dtype(int dtype) {
  return dtype == FA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

int num_sms();
void count_launch(int n = 1);

// Whatever the library caches (module-global addresses, kernel attributes) is kept per
// CUDA context: a module global has its own address in every context.  The entry
// point binds the caller's context and records its slot (0 .. kMaxContexts - 1) for
// the launchers of the same call.
constexpr int kMaxContexts = 64;
int call_context_slot();
enum { FA_PROF_FWD = 1, FA_PROF_BWD_DKDV = 2, FA_PROF_PAGED = 3, FA_PROF_DECODE = 4 };
// Records the armed begin/end events around a launch of the given kind (see
// fa_profile_next_launch); no-ops when nothing is armed.
void prof_begin(int kind, cudaStream_t st);
void prof_end(int kind, cudaStream_t st);

int launch_fwd_dense(const fa_fwd_args_t* a, int* err, cudaStream_t st);
int launch_paged_prefill(const fa_paged_args_t* a, int* err, cudaStream_t st);
int launch_varlen_fwd(const fa_varlen_fwd_args_t* a, int* err, cudaStream_t st);
// Paged prefill at head_dim 512 (fa_paged512.cu); called by launch_paged_prefill.
int launch_paged512(const fa_paged_args_t* a, int* err, cudaStream_t st);
// Varlen backward: `a` describes the packed tensors as one batch entry of total_q / total_k
// rows; this adds the sequences' row offsets and the longest lengths.
struct BwdVarlen {
  const int32_t* cu_q;
  const int32_t* cu_k;
  int batch, max_q, max_k;
};
int launch_bwd(const fa_bwd_args_t* a, void* ws, size_t ws_bytes, int* err, cudaStream_t st,
               const BwdVarlen* vl = nullptr);
// Dense backward at head_dim 256 (fa_bwd256.cu) after the prep kernel has written lse2 / dsum.
int launch_bwd_d256(const fa_bwd_args_t* a, const float* lse2, const float* dsum, int sq_pad,
                    int* err, cudaStream_t st, const BwdVarlen* vl = nullptr);
size_t bwd_workspace_bytes(const fa_bwd_args_t* a, const BwdVarlen* vl = nullptr);
int launch_decode(const fa_decode_args_t* a, void* ws, size_t ws_bytes, int* err, cudaStream_t st);
size_t decode_workspace_bytes(const fa_decode_args_t* a);
int launch_decode_noalloc(const fa_decode_args_t* a, int* err, cudaStream_t st);
int launch_kv_cache_write(const fa_kv_write_args_t* a, int* err, cudaStream_t st);
size_t decode_noalloc_scratch_bytes();
int decode_num_splits(const fa_decode_args_t* a);
int launch_umma_rate(int n, int k, int reps, int a_tmem, int a_mn, int b_mn, int ctas, int* err,
                     cudaStream_t st);
int launch_selftest_umma(const void* a, const void* b, float* c, int n, int k, int dtype, int b_mn,
                         int a_tmem, int* err, cudaStream_t st);

// Records the failing call (text, file:line, CUDA error) for fa_last_error_detail().
void set_error_detail(const char* what, const char* file, int line, const char* err);

#define FA_CUDA_TRY(x)                                                        \
  do {                                                                        \
    cudaError_t e_ = (x);                                                     \
    if (e_ != cudaSuccess) {                                                  \
      ::fa::set_error_detail(#x, __FILE__, __LINE__, cudaGetErrorString(e_)); \
      return FA_ERR_CUDA;                                                     \
    }                                                                         \
  } while (0)

#define FA_TMAP_TRY(x)                                                        \
  do {                                                                        \
    CUresult r_ = (x);                                                        \
    if (r_ != CUDA_SUCCESS) {                                                 \
      ::fa::set_error_detail(#x, __FILE__, __LINE__, "cuTensorMapEncodeTiled failed"); \
      return FA_ERR_CUDA;                                                     \
    }                                                                         \
  } while (0)

// Raises a kernel's dynamic shared-memory limit once per context (`done` is a static
// array of kMaxContexts flags that belongs to that kernel).
template <typename K>
inline int smem_attr_once(K kern, int bytes, std::atomic<bool>* done) {
  const int slot = call_context_slot();
  if (slot < 0 || slot >= kMaxContexts) return FA_ERR_CUDA;
  if (!done[slot].load(std::memory_order_acquire)) {
    FA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done[slot].store(true, std::memory_order_release);
  }
  return FA_OK;
}

// setmaxnreg.inc waits until the block's own launch allocation can supply the raised
// count, so a split whose total exceeds (registers per thread at launch) x threads
// would never proceed.  Checked against the compiled kernel before every first launch.
template <typename K>
inline int check_reg_split(K kern, int threads, int needed_total) {
  cudaFuncAttributes fa_attr;
  FA_CUDA_TRY(cudaFuncGetAttributes(&fa_attr, kern));
  if (fa_attr.numRegs * threads < needed_total) {
    set_error_detail("register split", __FILE__, __LINE__,
                     "setmaxnreg split exceeds the kernel's launch register allocation");
    return FA_ERR_CUDA;
  }
  return FA_OK;
}
}  // namespace fa
