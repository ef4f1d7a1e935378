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

int launch_kv_cache_write(const fa_kv_write_args_t* a, int* err, cudaStream_t st) {
  if (a->num_tokens == 0) return FA_OK;
  const int64_t row = (int64_t)a->num_kv_heads * a->head_dim;  // 16-bit elements
  if (row % 8 || a->key_stride % 8 || a->value_stride % 8) return FA_ERR_ALIGNMENT;
  const void* p[4] = {a->key, a->value, a->k_cache, a->v_cache};
  for (const void* q : p)
    if (reinterpret_cast<uintptr_t>(q) & 15u) return FA_ERR_ALIGNMENT;
  const int row16 = (int)(row / 8);
  int lpr = 32;
  while (lpr > 1 && lpr / 2 >= row16) lpr /= 2;  // smallest power of two >= row16, <= 32
  const int64_t rows = 2 * (int64_t)a->num_tokens;
  const int64_t want = (rows * lpr / 32 + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 16;
  const int grid = (int)(want < cap ? (want > 0 ? want : 1) : cap);
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
