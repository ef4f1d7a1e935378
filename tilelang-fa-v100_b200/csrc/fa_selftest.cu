// Self-test of the tcgen05 building blocks the attention kernels rely on:
// TMA 128-byte-swizzled tiles, UMMA shared-memory descriptors (K-major and
// MN-major), the kind::f16 instruction descriptor, A from shared memory or from
// tensor memory (packed 16-bit pairs, lane = row), commit -> mbarrier, and the
// 32x32b tcgen05.ld accumulator read-back.  C[128, N] = A[128, K] * B^T.
#include "fa_ptx.cuh"
#include "fa_internal.h"

namespace fa {

struct SelftestCtl {
  uint64_t load_bar;
  uint64_t mma_bar;
  uint32_t tmem_base;
  int abort_flag;
};

template <typename T>
__global__ void __launch_bounds__(128, 1)
    fa_selftest_umma_kernel(const __grid_constant__ CUtensorMap tma,
                            const __grid_constant__ CUtensorMap tmb, float* c, int N, int K,
                            int b_mn, int a_tmem, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const uint32_t sA = base;
  const uint32_t a_bytes = 128 * K * 2;
  const uint32_t sB = base + a_bytes;
  const uint32_t b_bytes = N * K * 2;
  SelftestCtl* ctl = reinterpret_cast<SelftestCtl*>(base_ptr + a_bytes + b_bytes);
  const int warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    ctl->abort_flag = 0;
    mbar_init(smem_u32(&ctl->load_bar), 1);
    mbar_init(smem_u32(&ctl->mma_bar), 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t bar = smem_u32(&ctl->load_bar);
    mbar_arrive_expect_tx(bar, a_bytes + b_bytes);
    for (int kc = 0; kc < K / 64; ++kc) tma_load_2d(sA + kc * 128 * 128, &tma, bar, kc * 64, 0);
    if (!b_mn) {
      for (int kc = 0; kc < K / 64; ++kc) tma_load_2d(sB + kc * N * 128, &tmb, bar, kc * 64, 0);
    } else {
      for (int nc = 0; nc < N / 64; ++nc) tma_load_2d(sB + nc * K * 128, &tmb, bar, nc * 64, 0);
    }
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&ctl->tmem_base), 512);
    tmem_relinquish();
  }
  const bool loaded = mbar_wait(smem_u32(&ctl->load_bar), 0, &ctl->abort_flag, err, FA_SITE_SELFTEST);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const int r = threadIdx.x;

  if (a_tmem && loaded) {
    // Row r of A from the swizzled smem tile into TMEM columns [256, 256 + K/2).
    for (int k0 = 0; k0 < K; k0 += 32) {
      uint32_t v[16];
      for (int q = 0; q < 4; ++q) {
        const int k = k0 + q * 8;
        const int kc = k / 64, ch = (k % 64) / 8;
        const uint4 x = *reinterpret_cast<const uint4*>(
            base_ptr + kc * 128 * 128 + r * 128 + ((ch ^ (r & 7)) << 4));
        v[q * 4 + 0] = x.x;
        v[q * 4 + 1] = x.y;
        v[q * 4 + 2] = x.z;
        v[q * 4 + 3] = x.w;
      }
      tmem_st16(tmem + lane_off + 256 + k0 / 2, v);
    }
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (threadIdx.x == 0 && loaded) {
    const uint32_t idesc = idesc_f16(128, N, Pack2<T>::kBf16, false, b_mn != 0);
    for (int kk = 0; kk < K / 16; ++kk) {
      const uint32_t oa = (kk >> 2) * 128 * 128 + (kk & 3) * 32;
      uint64_t bdesc;
      if (!b_mn)
        bdesc = sdesc_sw128(sB + (kk >> 2) * N * 128 + (kk & 3) * 32, 16, 1024);
      else
        bdesc = sdesc_sw128(sB + kk * 2048, K * 128, 1024);
      if (a_tmem)
        mma_ts(tmem, tmem + 256 + kk * 8, bdesc, idesc, kk > 0);
      else
        mma_ss(tmem, sdesc_sw128(sA + oa, 16, 1024), bdesc, idesc, kk > 0);
    }
    mma_commit(smem_u32(&ctl->mma_bar));
  }
  bool done = loaded && mbar_wait(smem_u32(&ctl->mma_bar), 0, &ctl->abort_flag, err, FA_SITE_SELFTEST);
  done = __all_sync(0xffffffffu, done);
  if (done) {
    tc_fence_after();
    for (int n0 = 0; n0 < N; n0 += 32) {
      uint32_t v[32];
      tmem_ld32(tmem + lane_off + n0, v);
      tmem_wait_ld();
      for (int i = 0; i < 32; ++i) c[(int64_t)r * N + n0 + i] = __uint_as_float(v[i]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int launch_selftest_umma(const void* a, const void* b, float* c, int n, int k, int dtype, int b_mn,
                         int a_tmem, int* err, cudaStream_t st) {
  if (!(n == 64 || n == 128 || n == 256) || k < 64 || k > 256 || (k % 64) != 0)
    return FA_ERR_UNSUPPORTED;
  const CUtensorMapDataType dt = tmap_dtype(dtype);
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)k, 128};
    const uint64_t str[1] = {(uint64_t)k * 2};
    const uint32_t box[2] = {64, 128};
    FA_TMAP_TRY(encode_tmap(&ta, dt, 2, a, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  if (!b_mn) {
    const uint64_t dims[2] = {(uint64_t)k, (uint64_t)n};
    const uint64_t str[1] = {(uint64_t)k * 2};
    const uint32_t box[2] = {64, (uint32_t)n};
    FA_TMAP_TRY(encode_tmap(&tb, dt, 2, b, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
  } else {
    const uint64_t dims[2] = {(uint64_t)n, (uint64_t)k};
    const uint64_t str[1] = {(uint64_t)n * 2};
    const uint32_t box[2] = {64, (uint32_t)k};
    FA_TMAP_TRY(encode_tmap(&tb, dt, 2, b, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  const int smem = 1024 + 128 * k * 2 + n * k * 2 + 256;
  if (dtype == FA_DTYPE_BF16) {
    FA_CUDA_TRY(cudaFuncSetAttribute(fa_selftest_umma_kernel<__nv_bfloat16>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    fa_selftest_umma_kernel<__nv_bfloat16><<<1, 128, smem, st>>>(ta, tb, c, n, k, b_mn, a_tmem, err);
  } else {
    FA_CUDA_TRY(cudaFuncSetAttribute(fa_selftest_umma_kernel<__half>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    fa_selftest_umma_kernel<__half><<<1, 128, smem, st>>>(ta, tb, c, n, k, b_mn, a_tmem, err);
  }
  FA_CUDA_TRY(cudaGetLastError());
  count_launch();
  return FA_OK;
}


// Throughput probe: every CTA issues `reps` x (K/16) back-to-back UMMAs of 128 x N x 16
// on operands already in shared memory (contents irrelevant: zero-filled), then commits
// once.  Forms: A_TMEM (A from TMEM), A_MN / B_MN (MN-major smem operands).  All
// descriptors are computed before the timed loop, so the loop is issue-lean.
template <bool A_TMEM, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(128, 1)
    fa_umma_rate_kernel(int N, int K, int reps, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const uint32_t sA = base, sB = base + 128 * K * 2;
  SelftestCtl* ctl = reinterpret_cast<SelftestCtl*>(base_ptr + 128 * K * 2 + N * K * 2);
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (128 * K + N * K) / 8; i += blockDim.x)
    reinterpret_cast<uint4*>(base_ptr)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    ctl->abort_flag = 0;
    mbar_init(smem_u32(&ctl->mma_bar), 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&ctl->tmem_base), 512);
    tmem_relinquish();
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  if (threadIdx.x == 0) {
    const uint32_t idesc = idesc_f16(128, N, true, A_MN, B_MN);
    uint64_t ad[8], bd[8];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      bd[kk] = B_MN ? sdesc_sw128(sB + kk * 2048, K * 128, 1024)
                    : sdesc_sw128(sB + (kk >> 2) * N * 128 + (kk & 3) * 32, 16, 1024);
      ad[kk] = A_MN ? sdesc_sw128(sA + kk * 2048, K * 128, 1024)
                    : sdesc_sw128(sA + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
    }
    for (int r = 0; r < reps; ++r) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        if (A_TMEM)
          mma_ts(tmem, tmem + 256 + kk * 8, bd[kk], idesc, 1);
        else
          mma_ss(tmem, ad[kk], bd[kk], idesc, 1);
      }
    }
    mma_commit(smem_u32(&ctl->mma_bar));
  }
  bool done = mbar_wait(smem_u32(&ctl->mma_bar), 0, &ctl->abort_flag, err, FA_SITE_SELFTEST);
  (void)done;
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <bool AT, bool AM, bool BM>
static int launch_rate_t(int n, int k, int reps, int ctas, int* err, cudaStream_t st) {
  const int smem = 1024 + 128 * k * 2 + n * k * 2 + 256;
  FA_CUDA_TRY(cudaFuncSetAttribute(fa_umma_rate_kernel<AT, AM, BM>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  fa_umma_rate_kernel<AT, AM, BM><<<ctas, 128, smem, st>>>(n, k, reps, err);
  FA_CUDA_TRY(cudaGetLastError());
  count_launch();
  return FA_OK;
}

int launch_umma_rate(int n, int k, int reps, int a_tmem, int a_mn, int b_mn, int ctas, int* err,
                     cudaStream_t st) {
  if (!(n == 64 || n == 128 || n == 256) || k != 128 || reps < 1) return FA_ERR_UNSUPPORTED;
  if (a_tmem) return b_mn ? launch_rate_t<true, false, true>(n, k, reps, ctas, err, st)
                          : launch_rate_t<true, false, false>(n, k, reps, ctas, err, st);
  if (a_mn) return launch_rate_t<false, true, true>(n, k, reps, ctas, err, st);
  return b_mn ? launch_rate_t<false, false, true>(n, k, reps, ctas, err, st)
              : launch_rate_t<false, false, false>(n, k, reps, ctas, err, st);
}

}  // namespace fa
