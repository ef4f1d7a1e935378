// C ABI of libfa_b200.so: argument validation, the device error word, tensor-map
// encoding and dispatch to the kernel launchers.  Nothing here allocates device
// memory; outputs and workspaces are owned by the caller.
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <cudaTypedefs.h>
#include "fa_internal.h"

namespace fa {

// Device error word: [0] code (0 = none, 1 = bounded wait expired), [1] site, [2] block.
__device__ int g_fa_device_error[4];


static std::mutex g_mu;
static int* g_err_ptr[kMaxContexts] = {nullptr};  // per context slot
static int g_sm_count[64] = {0};                  // per device
static int g_cc_ok[64] = {0};  // per device: 0 unknown, 1 ok, -1 not sm_100
static std::atomic<int64_t> g_launches{0};

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

static thread_local char g_err_detail[512] = "";
void set_error_detail(const char* what, const char* file, int line, const char* err) {
  const char* base = strrchr(file, '/');
  snprintf(g_err_detail, sizeof(g_err_detail), "%s at %s:%d: %s", what, base ? base + 1 : file,
           line, err);
}

// Benchmark hook state (fa_profile_next_launch).  The armed request is taken by the
// first matching launch from any thread: prof_begin claims it under the mutex and
// hands the end event to the same thread's prof_end, so two threads never record
// the same request.
static std::mutex g_prof_mu;
static std::atomic<int> g_prof_kind{0};
static cudaEvent_t g_prof_begin = nullptr, g_prof_end = nullptr;
static thread_local cudaEvent_t t_prof_end = nullptr;
static thread_local int t_prof_kind = 0;
void prof_begin(int kind, cudaStream_t st) {
  if (g_prof_kind.load(std::memory_order_relaxed) != kind) return;
  cudaEvent_t b = nullptr, e = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (g_prof_kind.load(std::memory_order_relaxed) != kind) return;
    b = g_prof_begin;
    e = g_prof_end;
    g_prof_kind.store(0, std::memory_order_relaxed);
    g_prof_begin = g_prof_end = nullptr;
  }
  if (cudaEventRecord(b, st) != cudaSuccess) {
    (void)cudaGetLastError();  // a stale or foreign event: drop the request
    return;
  }
  t_prof_end = e;
  t_prof_kind = kind;
}
void prof_end(int kind, cudaStream_t st) {
  if (t_prof_kind != kind || t_prof_end == nullptr) return;
  if (cudaEventRecord(t_prof_end, st) != cudaSuccess) (void)cudaGetLastError();
  t_prof_end = nullptr;
  t_prof_kind = 0;
}

static int current_device(int* dev) {
  if (cudaGetDevice(dev) != cudaSuccess) return FA_ERR_CUDA;
  if (*dev < 0 || *dev >= 64) return FA_ERR_CUDA;
  return FA_OK;
}

// Driver entry points used to bind the caller's context to the calling thread.  Each
// is requested at an explicit version with its matching signature: the default
// version of cuStreamGetCtx in CUDA 12.5+ takes a third (green-context) output
// argument, and calling it through a two-argument pointer lets the driver write
// through an undefined pointer.
static PFN_cuStreamGetCtx_v9020 p_stream_get_ctx = nullptr;
static PFN_cuCtxGetCurrent_v4000 p_ctx_get_current = nullptr;
static PFN_cuCtxSetCurrent_v4000 p_ctx_set_current = nullptr;
static PFN_cuCtxGetId_v12000 p_ctx_get_id = nullptr;

static void* driver_fn(const char* name, unsigned int version) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion(name, &p, version, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return p;
}

// Makes the CUDA context of the caller's stream (or, for the default stream, the
// primary context of the runtime's current device) current on the calling thread.
// Needed because the library's driver calls (tensor-map encoding) need a current
// context, and a caller's worker thread -- e.g. torch's autograd thread -- may not
// have one bound yet even though its runtime "current device" is set.
static int bind_context(cudaStream_t st) {
  static std::once_flag once;
  std::call_once(once, [] {
    p_stream_get_ctx = reinterpret_cast<PFN_cuStreamGetCtx_v9020>(driver_fn("cuStreamGetCtx", 9020));
    p_ctx_get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(driver_fn("cuCtxGetCurrent", 4000));
    p_ctx_set_current = reinterpret_cast<PFN_cuCtxSetCurrent_v4000>(driver_fn("cuCtxSetCurrent", 4000));
    p_ctx_get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(driver_fn("cuCtxGetId", 12000));
  });
  const uintptr_t sv = reinterpret_cast<uintptr_t>(st);
  if (sv > 2 && p_stream_get_ctx && p_ctx_get_current && p_ctx_set_current) {
    CUcontext ctx = nullptr, cur = nullptr;
    if (p_stream_get_ctx(reinterpret_cast<CUstream>(st), &ctx) == CUDA_SUCCESS && ctx != nullptr) {
      p_ctx_get_current(&cur);
      if (cur != ctx && p_ctx_set_current(ctx) != CUDA_SUCCESS) {
        set_error_detail("cuCtxSetCurrent", __FILE__, __LINE__, "failed");
        return FA_ERR_CUDA;
      }
      return FA_OK;
    }
  }
  int dev = 0;
  FA_CUDA_TRY(cudaGetDevice(&dev));
  FA_CUDA_TRY(cudaSetDevice(dev));  // CUDA 12+: initialises and binds the primary context
  return FA_OK;
}

// Context slots.  A module global (the error word, the persistent scheduler's
// counters, the no-allocation decode scratch) has its own device address in every CUDA
// context, and kernel attributes are set per context, so whatever the library caches
// is keyed by the context a call runs in: by its id (cuCtxGetId), which is unique for
// the context's lifetime, whereas a destroyed context's handle may be reused.  Slots
// are never recycled; a process that creates more than kMaxContexts contexts gets
// FA_ERR_CUDA from the calls made in the extra ones.
static unsigned long long g_ctx_id[kMaxContexts] = {0};
static int g_ctx_count = 0;
static thread_local unsigned long long t_last_ctx_id = 0;
static thread_local int t_last_slot = -1;
static thread_local int t_call_slot = -1;

static int find_context_slot(int* slot) {
  CUcontext cur = nullptr;
  unsigned long long id = 0;
  if (p_ctx_get_current == nullptr || p_ctx_get_id == nullptr ||
      p_ctx_get_current(&cur) != CUDA_SUCCESS || cur == nullptr ||
      p_ctx_get_id(cur, &id) != CUDA_SUCCESS) {
    set_error_detail("cuCtxGetCurrent / cuCtxGetId", __FILE__, __LINE__, "no current context");
    return FA_ERR_CUDA;
  }
  if (id == t_last_ctx_id && t_last_slot >= 0) {
    *slot = t_last_slot;
    return FA_OK;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  int found = -1;
  for (int i = 0; i < g_ctx_count; ++i)
    if (g_ctx_id[i] == id) found = i;
  if (found < 0) {
    if (g_ctx_count == kMaxContexts) {
      set_error_detail("context slot", __FILE__, __LINE__, "more CUDA contexts than kMaxContexts");
      return FA_ERR_CUDA;
    }
    found = g_ctx_count++;
    g_ctx_id[found] = id;
  }
  t_last_ctx_id = id;
  t_last_slot = found;
  *slot = found;
  return FA_OK;
}

int call_context_slot() { return t_call_slot; }

// Per-call set-up: binds the caller's context and records its slot for the launchers
// (call_context_slot), checks the compute capability, caches the SM count (per
// device) and the device address of the error word (per context, looked up with that
// context current).
static int device_setup(int** err_out, cudaStream_t st = nullptr) {
  if (int s = bind_context(st)) return s;
  int dev;
  if (int s = current_device(&dev)) return s;
  int slot = -1;
  if (int s = find_context_slot(&slot)) return s;
  t_call_slot = slot;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_cc_ok[dev] == 0) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return FA_ERR_CUDA;
    g_cc_ok[dev] = (major == 10) ? 1 : -1;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = sms;
  }
  if (g_cc_ok[dev] < 0) return FA_ERR_NOT_SM100;
  if (g_err_ptr[slot] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_fa_device_error) != cudaSuccess) return FA_ERR_CUDA;
    g_err_ptr[slot] = static_cast<int*>(ptr);
  }
  *err_out = g_err_ptr[slot];
  return FA_OK;
}

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  return g_sm_count[dev] > 0 ? g_sm_count[dev] : 148;
}

CUresult encode_tmap(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                     const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                     CUtensorMapSwizzle swizzle) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(
        driver_fn("cuTensorMapEncodeTiled", 12000));
  });
  if (fn == nullptr) return CUDA_ERROR_NOT_FOUND;
  cuuint64_t gdim[5];
  cuuint64_t gstr[4];
  cuuint32_t bdim[5];
  cuuint32_t estr[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estr[i] = 1;
    if (i + 1 < rank) gstr[i] = strides_bytes[i];
  }
  return fn(map, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), gdim, gstr, bdim, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

static bool valid_dtype(int d) { return d == FA_DTYPE_F16 || d == FA_DTYPE_BF16; }
// Dense head dims: 64 / 128 / 256 natively, 32 / 96 on the 64 / 128 kernels.
static bool dense_head_dim(int d) { return d == 32 || d == 64 || d == 96 || d == 128 || d == 256; }

}  // namespace fa

using namespace fa;

extern "C" {

const char* fa_version(void) { return "fa_b200 1.0.0 (sm_100a)"; }

const char* fa_last_error_detail(void) { return g_err_detail; }



int64_t fa_launch_count(void) { return g_launches.load(); }

const char* fa_status_string(int status) {
  switch (status) {
    case FA_OK: return "ok";
    case FA_ERR_INVALID_ARG: return "invalid argument";
    case FA_ERR_UNSUPPORTED: return "unsupported head_dim / dtype / page_size / GQA ratio";
    case FA_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case FA_ERR_WORKSPACE: return "workspace missing or too small";
    case FA_ERR_CUDA: return "CUDA runtime/driver call failed";
    case FA_ERR_DEVICE_TIMEOUT: return "a kernel's bounded wait expired on the device";
    case FA_ERR_NOT_SM100: return "current device is not an sm_100 (B200-class) GPU";
    default: return "unknown status";
  }
}

int fa_read_device_error(int32_t* code, int32_t* site, int32_t* block, int32_t clear) {
  int* err = nullptr;
  if (int s = device_setup(&err)) return s;
  int host[4] = {0, 0, 0, 0};
  if (cudaDeviceSynchronize() != cudaSuccess) return FA_ERR_CUDA;
  if (cudaMemcpy(host, err, sizeof(host), cudaMemcpyDeviceToHost) != cudaSuccess)
    return FA_ERR_CUDA;
  if (code) *code = host[0];
  if (site) *site = host[1];
  if (block) *block = host[2];
  if (clear) {
    const int zero[4] = {0, 0, 0, 0};
    if (cudaMemcpy(err, zero, sizeof(zero), cudaMemcpyHostToDevice) != cudaSuccess)
      return FA_ERR_CUDA;
  }
  return FA_OK;
}

// softcap: 0 (off) or a finite positive cap with a positive softmax scale.
static bool valid_softcap(float cap, float scale) {
  if (cap == 0.f) return true;
  return std::isfinite(cap) && cap > 0.f && std::isfinite(scale) && scale > 0.f;
}

int fa_fwd(const fa_fwd_args_t* a, void* stream) {
  if (a == nullptr || a->q == nullptr || a->k == nullptr || a->v == nullptr ||
      a->out == nullptr || a->lse == nullptr)
    return FA_ERR_INVALID_ARG;
  if (a->batch < 0 || a->seqlen_q < 0 || a->seqlen_k < 0 || a->num_heads <= 0 ||
      a->num_heads_k <= 0 || a->num_heads % a->num_heads_k != 0)
    return FA_ERR_INVALID_ARG;
  if (!valid_dtype(a->dtype)) return FA_ERR_UNSUPPORTED;
  if (!dense_head_dim(a->head_dim)) return FA_ERR_UNSUPPORTED;
  if (!valid_softcap(a->softcap, a->softmax_scale)) return FA_ERR_INVALID_ARG;
  int* err = nullptr;
  if (int s = device_setup(&err, static_cast<cudaStream_t>(stream))) return s;
  return launch_fwd_dense(a, err, static_cast<cudaStream_t>(stream));
}

size_t fa_bwd_workspace_size(const fa_bwd_args_t* a) {
  if (a == nullptr) return 0;
  return bwd_workspace_bytes(a);
}

int fa_bwd(const fa_bwd_args_t* a, void* ws, size_t ws_bytes, void* stream) {
  if (a == nullptr || a->q == nullptr || a->k == nullptr || a->v == nullptr ||
      a->out == nullptr || a->dout == nullptr || a->lse == nullptr || a->dq == nullptr ||
      a->dk == nullptr || a->dv == nullptr)
    return FA_ERR_INVALID_ARG;
  if (a->batch < 0 || a->seqlen_q < 0 || a->seqlen_k < 0 || a->num_heads <= 0 ||
      a->num_heads_k <= 0 || a->num_heads % a->num_heads_k != 0)
    return FA_ERR_INVALID_ARG;
  if (!valid_dtype(a->dtype)) return FA_ERR_UNSUPPORTED;
  if (!dense_head_dim(a->head_dim)) return FA_ERR_UNSUPPORTED;
  if (!valid_softcap(a->softcap, a->softmax_scale)) return FA_ERR_INVALID_ARG;
  if (ws_bytes < bwd_workspace_bytes(a) || (bwd_workspace_bytes(a) > 0 && ws == nullptr))
    return FA_ERR_WORKSPACE;
  int* err = nullptr;
  if (int s = device_setup(&err, static_cast<cudaStream_t>(stream))) return s;
  return launch_bwd(a, ws, ws_bytes, err, static_cast<cudaStream_t>(stream));
}

// ---- dense varlen: the packed tensors as one batch entry of total rows + the offsets
static bool varlen_dims_ok(int batch, int total_q, int total_k, int max_q, int max_k, int h,
                           int hk) {
  return batch >= 0 && total_q >= 0 && total_k >= 0 && max_q >= 0 && max_k >= 0 && h > 0 &&
         hk > 0 && h % hk == 0;
}
static bool strides8(const int64_t* s) { return s[0] % 8 == 0 && s[1] % 8 == 0; }
// Batch stride of the one-entry view: past the last row (only its alignment is checked).
static void one_entry(int64_t dst[3], const int64_t src[2], int rows) {
  dst[0] = src[0] * (rows > 0 ? rows : 1);
  dst[1] = src[0];
  dst[2] = src[1];
}

int fa_varlen_fwd(const fa_varlen_fwd_args_t* a, void* stream) {
  if (a == nullptr || a->q == nullptr || a->k == nullptr || a->v == nullptr ||
      a->out == nullptr || a->lse == nullptr || a->cu_seqlens_q == nullptr ||
      a->cu_seqlens_k == nullptr)
    return FA_ERR_INVALID_ARG;
  if (!varlen_dims_ok(a->batch, a->total_q, a->total_k, a->max_seqlen_q, a->max_seqlen_k,
                      a->num_heads, a->num_heads_k))
    return FA_ERR_INVALID_ARG;
  if (!valid_dtype(a->dtype)) return FA_ERR_UNSUPPORTED;
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256) return FA_ERR_UNSUPPORTED;
  if (!valid_softcap(a->softcap, a->softmax_scale)) return FA_ERR_INVALID_ARG;
  if (!strides8(a->q_stride) || !strides8(a->k_stride) || !strides8(a->v_stride) ||
      !strides8(a->o_stride))
    return FA_ERR_ALIGNMENT;
  int* err = nullptr;
  if (int s = device_setup(&err, static_cast<cudaStream_t>(stream))) return s;
  return launch_varlen_fwd(a, err, static_cast<cudaStream_t>(stream));
}

// The dense backward's argument block for the packed tensors (one batch entry of total_q
// / total_k rows) and the varlen description that goes with it.
static void varlen_as_dense(const fa_varlen_bwd_args_t* a, fa_bwd_args_t* d, BwdVarlen* vl) {
  memset(d, 0, sizeof(*d));
  d->q = a->q;
  d->k = a->k;
  d->v = a->v;
  d->out = a->out;
  d->dout = a->dout;
  d->lse = a->lse;
  d->dq = a->dq;
  d->dk = a->dk;
  d->dv = a->dv;
  one_entry(d->q_stride, a->q_stride, a->total_q);
  one_entry(d->k_stride, a->k_stride, a->total_k);
  one_entry(d->v_stride, a->v_stride, a->total_k);
  one_entry(d->o_stride, a->o_stride, a->total_q);
  one_entry(d->do_stride, a->do_stride, a->total_q);
  one_entry(d->dq_stride, a->dq_stride, a->total_q);
  one_entry(d->dk_stride, a->dk_stride, a->total_k);
  one_entry(d->dv_stride, a->dv_stride, a->total_k);
  d->batch = 1;
  d->seqlen_q = a->total_q;
  d->seqlen_k = a->total_k;
  d->num_heads = a->num_heads;
  d->num_heads_k = a->num_heads_k;
  d->head_dim = a->head_dim;
  d->dtype = a->dtype;
  d->causal = a->causal;
  d->deterministic = a->deterministic;
  d->softmax_scale = a->softmax_scale;
  d->window_q = a->window_q;
  d->window_k = a->window_k;
  d->softcap = a->softcap;
  vl->cu_q = a->cu_seqlens_q;
  vl->cu_k = a->cu_seqlens_k;
  vl->batch = a->batch;
  vl->max_q = a->max_seqlen_q;
  vl->max_k = a->max_seqlen_k;
}

size_t fa_varlen_bwd_workspace_size(const fa_varlen_bwd_args_t* a) {
  if (a == nullptr) return 0;
  fa_bwd_args_t d;
  BwdVarlen vl;
  varlen_as_dense(a, &d, &vl);
  return bwd_workspace_bytes(&d, &vl);
}

int fa_varlen_bwd(const fa_varlen_bwd_args_t* a, void* ws, size_t ws_bytes, void* stream) {
  if (a == nullptr || a->q == nullptr || a->k == nullptr || a->v == nullptr ||
      a->out == nullptr || a->dout == nullptr || a->lse == nullptr || a->dq == nullptr ||
      a->dk == nullptr || a->dv == nullptr || a->cu_seqlens_q == nullptr ||
      a->cu_seqlens_k == nullptr)
    return FA_ERR_INVALID_ARG;
  if (!varlen_dims_ok(a->batch, a->total_q, a->total_k, a->max_seqlen_q, a->max_seqlen_k,
                      a->num_heads, a->num_heads_k))
    return FA_ERR_INVALID_ARG;
  if (!valid_dtype(a->dtype)) return FA_ERR_UNSUPPORTED;
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256) return FA_ERR_UNSUPPORTED;
  if (!valid_softcap(a->softcap, a->softmax_scale)) return FA_ERR_INVALID_ARG;
  const int64_t* strs[8] = {a->q_stride, a->k_stride, a->v_stride, a->o_stride,
                            a->do_stride, a->dq_stride, a->dk_stride, a->dv_stride};
  for (const int64_t* s : strs)
    if (!strides8(s)) return FA_ERR_ALIGNMENT;
  fa_bwd_args_t d;
  BwdVarlen vl;
  varlen_as_dense(a, &d, &vl);
  if (a->batch == 0) return FA_OK;
  if (ws_bytes < bwd_workspace_bytes(&d, &vl) || ws == nullptr) return FA_ERR_WORKSPACE;
  int* err = nullptr;
  if (int s = device_setup(&err, static_cast<cudaStream_t>(stream))) return s;
  return launch_bwd(&d, ws, ws_bytes, err, static_cast<cudaStream_t>(stream), &vl);
}

int fa_paged_prefill(const fa_paged_args_t* a, void* stream) {
  if (a == nullptr || a->q == nullptr || a->k_cache == nullptr || a->v_cache == nullptr ||
      a->block_table == nullptr || a->seq_lens == nullptr || a->query_start_loc == nullptr ||
      a->prefix_kv_lens == nullptr || a->out == nullptr)
    return FA_ERR_INVALID_ARG;
  if (a->num_tokens < 0 || a->num_seqs < 0 || a->num_heads <= 0 || a->num_kv_heads <= 0 ||
      a->num_heads % a->num_kv_heads != 0 || a->num_pages <= 0 || a->max_blocks <= 0)
    return FA_ERR_INVALID_ARG;
  if (!valid_dtype(a->dtype)) return FA_ERR_UNSUPPORTED;
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256 && a->head_dim != 512)
    return FA_ERR_UNSUPPORTED;
  int* err = nullptr;
  if (int s = device_setup(&err, static_cast<cudaStream_t>(stream))) return s;
  return launch_paged_prefill(a, err, static_cast<cudaStream_t>(stream));
}

size_t fa_decode_workspace_size(const fa_decode_args_t* a) {
  if (a == nullptr) return 0;
  return decode_workspace_bytes(a);
}

int fa_decode(const fa_decode_args_t* a, void* ws, size_t ws_bytes, void* stream) {
  if (a == nullptr || a->q == nullptr || a->k_cache == nullptr || a->v_cache == nullptr ||
      a->block_table == nullptr || a->seq_lens == nullptr || a->out == nullptr)
    return FA_ERR_INVALID_ARG;
  if (a->batch < 0 || a->num_heads <= 0 || a->num_kv_heads <= 0 ||
      a->num_heads % a->num_kv_heads != 0 || a->num_pages <= 0 || a->max_blocks <= 0 ||
      a->num_splits < 0)
    return FA_ERR_INVALID_ARG;
  if (!valid_dtype(a->dtype)) return FA_ERR_UNSUPPORTED;
  int* err = nullptr;
  if (int s = device_setup(&err, static_cast<cudaStream_t>(stream))) return s;
  return launch_decode(a, ws, ws_bytes, err, static_cast<cudaStream_t>(stream));
}

int fa_decode_noalloc(const fa_decode_args_t* a, void* stream) {
  if (a == nullptr || a->q == nullptr || a->k_cache == nullptr || a->v_cache == nullptr ||
      a->block_table == nullptr || a->seq_lens == nullptr || a->out == nullptr)
    return FA_ERR_INVALID_ARG;
  if (a->batch < 0 || a->num_heads <= 0 || a->num_kv_heads <= 0 ||
      a->num_heads % a->num_kv_heads != 0 || a->num_pages <= 0 || a->max_blocks <= 0 ||
      a->num_splits < 0)
    return FA_ERR_INVALID_ARG;
  if (!valid_dtype(a->dtype)) return FA_ERR_UNSUPPORTED;
  int* err = nullptr;
  if (int s = device_setup(&err, static_cast<cudaStream_t>(stream))) return s;
  return launch_decode_noalloc(a, err, static_cast<cudaStream_t>(stream));
}

size_t fa_decode_noalloc_scratch_bytes(void) { return decode_noalloc_scratch_bytes(); }

int fa_kv_cache_write(const fa_kv_write_args_t* a, void* stream) {
  if (a == nullptr) return FA_ERR_INVALID_ARG;
  if (a->num_tokens < 0 || a->num_kv_heads <= 0 || a->head_dim <= 0 || a->page_size <= 0 ||
      a->num_pages <= 0 || a->key_stride < 0 || a->value_stride < 0)
    return FA_ERR_INVALID_ARG;
  if (a->num_tokens > 0 && (a->key == nullptr || a->value == nullptr || a->k_cache == nullptr ||
                            a->v_cache == nullptr || a->slot_mapping == nullptr))
    return FA_ERR_INVALID_ARG;
  if (!valid_dtype(a->dtype)) return FA_ERR_UNSUPPORTED;
  int* err = nullptr;
  if (int s = device_setup(&err, static_cast<cudaStream_t>(stream))) return s;
  return launch_kv_cache_write(a, err, static_cast<cudaStream_t>(stream));
}

int fa_selftest_umma_rate(int32_t n, int32_t k, int32_t reps, int32_t a_tmem, int32_t a_mn,
                          int32_t b_mn, int32_t ctas, void* stream) {
  int* err = nullptr;
  if (int s = device_setup(&err, static_cast<cudaStream_t>(stream))) return s;
  return launch_umma_rate(n, k, reps, a_tmem, a_mn, b_mn, ctas, err,
                          static_cast<cudaStream_t>(stream));
}

int fa_profile_next_launch(int32_t kind, void* ev_begin, void* ev_end) {
  if (kind < 1 || kind > 4 || ev_begin == nullptr || ev_end == nullptr) return FA_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof_begin = static_cast<cudaEvent_t>(ev_begin);
  g_prof_end = static_cast<cudaEvent_t>(ev_end);
  g_prof_kind.store(kind, std::memory_order_relaxed);
  return FA_OK;
}

int fa_selftest_umma(const void* a, const void* b, float* c, int32_t n, int32_t k, int32_t dtype,
                     int32_t b_mn, int32_t a_tmem, void* stream) {
  if (a == nullptr || b == nullptr || c == nullptr) return FA_ERR_INVALID_ARG;
  if (!valid_dtype(dtype)) return FA_ERR_UNSUPPORTED;
  int* err = nullptr;
  if (int s = device_setup(&err, static_cast<cudaStream_t>(stream))) return s;
  return launch_selftest_umma(a, b, c, n, k, dtype, b_mn, a_tmem, err,
                              static_cast<cudaStream_t>(stream));
}

}  // extern "C"
