// Paged KV-cache write on sm_100a: the step before the paged prefill / decode path.
// A serving engine appends each new token's key and value rows to the vLLM cache
// layout [num_pages, page_size, Hkv, D] at the slot its scheduler assigned
// (slot = page * page_size + offset, as consumed through block_table by
// _kernels_paged.py:265-272 / :441-448 of the reference); a negative slot marks a
// padding token that is not written.  This is the operation vLLM performs with
// reshape_and_cache_flash (vllm/_custom_ops.py) for its flash-layout caches.
//
// A warp (or, for narrow rows, a group of lanes) moves one (token, K or V) row of
// Hkv * D 16-bit elements with 16-byte loads and stores; the token row of the source and
// the slot row of the cache are both contiguous.  The grid is a multiple of the SM count and loops over the rows.  The
// work is HBM-bound: 2 x num_tokens x Hkv x D x 2 bytes read and the same written.
#include "fa_ptx.cuh"
#include "fa_internal.h"

namespace fa {

constexpr int FA_DEVERR_BAD_SLOT = 3;
constexpr int FA_SITE_KV_WRITE = 41;

// `lpr` lanes (a power of two <= 32) copy one row; a warp covers 32 / lpr rows, so
// narrow rows (few kv heads) still keep every lane busy.
__global__ void __launch_bounds__(256)
    fa_kv_cache_write_kernel(const uint4* __restrict__ key, const uint4* __restrict__ value,
                             uint4* __restrict__ k_cache, uint4* __restrict__ v_cache,
                             const int64_t* __restrict__ slot_mapping, int64_t key_stride16,
                             int64_t value_stride16, int num_tokens, int row16, int lpr,
                             int64_t num_slots, int* err) {
  const int lane = threadIdx.x & 31;
  const int sub = lane / lpr, sl = lane % lpr;
  const int rpw = 32 / lpr;  // rows per warp
  const int64_t step = (int64_t)gridDim.x * (blockDim.x >> 5) * rpw;
  for (int64_t r = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * rpw + sub;
       r < 2 * (int64_t)num_tokens; r += step) {
    const bool is_v = r >= num_tokens;
    const int64_t t = is_v ? r - num_tokens : r;
    const int64_t slot = slot_mapping[t];
    if (slot < 0) continue;  // padding token
    if (slot >= num_slots) {  // out of the cache: never written, reported to the host
      if (sl == 0) record_device_error(err, FA_DEVERR_BAD_SLOT, FA_SITE_KV_WRITE);
      continue;
    }
    const uint4* src = is_v ? value + t * value_stride16 : key + t * key_stride16;
    uint4* dst = (is_v ? v_cache : k_cache) + slot * row16;
    // Four 16-byte loads per lane in flight before the stores.
    int i = sl;
    for (; i + 3 * lpr < row16; i += 4 * lpr) {
      const uint4 a0 = __ldcs(src + i), a1 = __ldcs(src + i + lpr);
      const uint4 a2 = __ldcs(src + i + 2 * lpr), a3 = __ldcs(src + i + 3 * lpr);
      dst[i] = a0;
      dst[i + lpr] = a1;
      dst[i + 2 * lpr] = a2;
      dst[i + 3 * lpr] = a3;
    }
    for (; i < row16; i += lpr) dst[i] = __ldcs(src + i);
  }
}

// fp8 caches (vLLM's fp8 KV cache with per-tensor scales): each 16-byte unit of eight
// 16-bit source elements becomes eight e4m3 bytes of x / scale, rounded to nearest and
// saturated to +-448 (cvt.rn.satfinite), written as one 8-byte store.
__device__ __forceinline__ uint32_t e4m3x2_of(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
template <typename T>
__device__ __forceinline__ uint2 quant8(uint4 v, float inv) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = Pack2<T>::unpack(w[i]);
    q[i] = e4m3x2_of(f.x * inv, f.y * inv);
  }
  return make_uint2(q[0] | (q[1] << 16), q[2] | (q[3] << 16));
}

template <typename T>
__global__ void __launch_bounds__(256)
    fa_kv_cache_write_fp8_kernel(const uint4* __restrict__ key, const uint4* __restrict__ value,
                                 uint2* __restrict__ k_cache, uint2* __restrict__ v_cache,
                                 const int64_t* __restrict__ slot_mapping, int64_t key_stride16,
                                 int64_t value_stride16, int num_tokens, int row16, int lpr,
                                 int64_t num_slots, float inv_k, float inv_v, int* err) {
  const int lane = threadIdx.x & 31;
  const int sub = lane / lpr, sl = lane % lpr;
  const int rpw = 32 / lpr;
  const int64_t step = (int64_t)gridDim.x * (blockDim.x >> 5) * rpw;
  for (int64_t r = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * rpw + sub;
       r < 2 * (int64_t)num_tokens; r += step) {
    const bool is_v = r >= num_tokens;
    const int64_t t = is_v ? r - num_tokens : r;
    const int64_t slot = slot_mapping[t];
    if (slot < 0) continue;
    if (slot >= num_slots) {
      if (sl == 0) record_device_error(err, FA_DEVERR_BAD_SLOT, FA_SITE_KV_WRITE);
      continue;
    }
    const uint4* src = is_v ? value + t * value_stride16 : key + t * key_stride16;
    uint2* dst = (is_v ? v_cache : k_cache) + slot * row16;
    const float inv = is_v ? inv_v : inv_k;
    for (int i = sl; i < row16; i += lpr) dst[i] = quant8<T>(__ldcs(src + i), inv);
  }
}

int launch_kv_cache_write(const fa_kv_write_args_t* a, int* err, cudaStream_t st) {
  if (a->num_tokens == 0) return FA_OK;
  if (a->cache_dtype != 0 && a->cache_dtype != FA_DTYPE_E4M3) return FA_ERR_UNSUPPORTED;
  const bool c8 = a->cache_dtype == FA_DTYPE_E4M3;
  if (c8 && !(a->k_scale > 0.f && a->v_scale > 0.f && isfinite(a->k_scale) &&
              isfinite(a->v_scale)))
    return FA_ERR_INVALID_ARG;
  const int64_t row = (int64_t)a->num_kv_heads * a->head_dim;  // 16-bit elements
  if (row % 8 || a->key_stride % 8 || a->value_stride % 8) return FA_ERR_ALIGNMENT;
  const void* p[4] = {a->key, a->value, a->k_cache, a->v_cache};
  for (const void* q : p)
    if (reinterpret_cast<uintptr_t>(q) & 7u) return FA_ERR_ALIGNMENT;
  for (int i = 0; i < 2; ++i)  // 16-bit tensors: 16-byte units
    if (reinterpret_cast<uintptr_t>(p[i]) & 15u) return FA_ERR_ALIGNMENT;
  if (a->cache_dtype == 0)
    for (int i = 2; i < 4; ++i)
      if (reinterpret_cast<uintptr_t>(p[i]) & 15u) return FA_ERR_ALIGNMENT;
  const int row16 = (int)(row / 8);
  int lpr = 32;
  while (lpr > 1 && lpr / 2 >= row16) lpr /= 2;  // smallest power of two >= row16, <= 32
  const int64_t rows = 2 * (int64_t)a->num_tokens;
  const int64_t want = (rows * lpr / 32 + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 16;
  const int grid = (int)(want < cap ? (want > 0 ? want : 1) : cap);
  if (c8) {
    const int64_t slots = (int64_t)a->num_pages * a->page_size;
    auto* kd = static_cast<uint2*>(a->k_cache);
    auto* vd = static_cast<uint2*>(a->v_cache);
    const auto* ks = static_cast<const uint4*>(a->key);
    const auto* vs = static_cast<const uint4*>(a->value);
    if (a->dtype == FA_DTYPE_BF16)
      fa_kv_cache_write_fp8_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
          ks, vs, kd, vd, a->slot_mapping, a->key_stride / 8, a->value_stride / 8, a->num_tokens,
          row16, lpr, slots, 1.f / a->k_scale, 1.f / a->v_scale, err);
    else
      fa_kv_cache_write_fp8_kernel<__half><<<grid, 256, 0, st>>>(
          ks, vs, kd, vd, a->slot_mapping, a->key_stride / 8, a->value_stride / 8, a->num_tokens,
          row16, lpr, slots, 1.f / a->k_scale, 1.f / a->v_scale, err);
    FA_CUDA_TRY(cudaGetLastError());
    count_launch();
    return FA_OK;
  }
  fa_kv_cache_write_kernel<<<grid, 256, 0, st>>>(
      static_cast<const uint4*>(a->key), static_cast<const uint4*>(a->value),
      static_cast<uint4*>(a->k_cache), static_cast<uint4*>(a->v_cache), a->slot_mapping,
      a->key_stride / 8, a->value_stride / 8, a->num_tokens, row16, lpr,
      (int64_t)a->num_pages * a->page_size, err);
  FA_CUDA_TRY(cudaGetLastError());
  count_launch();
  return FA_OK;
}

}  // namespace fa
