// Attention backward at head_dim 256 on sm_100a (reference: tilelang_backward,
// _kernels_backward.py:200-208, whose dQ and dK/dV kernels :10-176 are generic in `dim`;
// its config space admits 256, _configs.py:28-51 / _utils.py:22-23).
//
// At D = 256 the D = 64/128 layout does not fit: a CTA owning 128 keys would need
// 2 x 256 TMEM columns for dK and dV alone next to S^T and dP^T, and K, V, Q and dO tiles
// of 64 KB each.  So the backward is split in two kernels after the shared prep kernel
// (row dot and LSE * log2 e, fa_bwd.cu):
//
//   fa_bwd_dkdv_d256  one CTA per (128-key tile, half of the head dimension, kv head,
//                     batch).  It recomputes the full S^T = K Q^T and dP^T = V dO^T (both
//                     contract over all 256 dims) for 64 queries per step and accumulates
//                     its half of dK and dV in TMEM:
//                       S^T  [0, 64)     dP^T [64, 128)   (fp32, M = 128 keys, N = 64)
//                       P^T, dS^T packed as 16-bit pairs over their own S^T / dP^T columns
//                       dV_h [128, 256)  dK_h [256, 384)  (TS MMAs, A from TMEM)
//                     Shared memory: K, V resident (64 KB each), Q in two 32 KB stages,
//                     dO in one (the row dot and LSE of each step ride with Q).
//   fa_bwd_dq_d256    one CTA per (128-query tile, head, batch) looping over 64-key steps:
//                     S = Q K^T [0, 64), dP = dO V^T [64, 128), dS packed over its own S
//                     columns, dQ += dS K into [128, 384) (TS MMA, B = K MN-major).
//                     Shared memory: Q and dO resident (64 KB each), K in two 32 KB
//                     stages, V in one.
// Both are deterministic (no atomics); dQ needs no fp32 accumulator, so both API modes
// run the same kernels at D = 256.
//
// Roles (384 threads): warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer, warps
// 2-3 idle, warps 4-11 two compute warpgroups (thread = TMEM lane = key row in dK/dV, query
// row in dQ; warpgroup c takes columns [32 c, 32 c + 32) of each 64-wide step).
#include "fa_ptx.cuh"
#include "fa_internal.h"
#include <cmath>

namespace fa {

constexpr int kB2Keys = 128;   // keys per dK/dV CTA (TMEM lanes)
constexpr int kB2QStep = 64;   // queries per dK/dV step
constexpr int kB2Rows = 128;   // query rows per dQ CTA
constexpr int kB2KStep = 64;   // keys per dQ step
constexpr int kB2Threads = 384;
constexpr int kB2Chunk128 = 128 * 128;  // 128 rows x 64 dims, 16-bit, 128-byte swizzled
constexpr int kB2Chunk64 = 64 * 128;    // 64 rows x 64 dims

struct B2Params {
  int B, Sq, Skv, H, Hk, G, Sq_pad, causal;
  int swq, swk;  // sliding window (dense_visible in fa_internal.h; <= 0: off)
  float scale, scale_log2;
  // softcap (0: off): as in the D = 64 / 128 backward's parameters
  float sc_a, sc_k, sc_ia, sc_t;
  // varlen (EXT kernels): packed-row offsets of the sequences, as in the D = 64 / 128
  // backward's parameters; null for dense
  const int32_t* cu_q;
  const int32_t* cu_k;
  const float* lse2;  // [B, H, Sq_pad] lse * log2(e), +inf for padded / empty rows
  const float* dsum;  // [B, H, Sq_pad] rowsum(O * dO)
  void* dq;
  void* dk;
  void* dv;
  int64_t dq_sb, dq_ss, dq_sh;
  int64_t dk_sb, dk_ss, dk_sh;
  int64_t dv_sb, dv_ss, dv_sh;
  int* err;
};

__device__ __forceinline__ void b2_bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                             uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void b2_drain_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > 200000000ull) return;
}
__device__ __forceinline__ void b2_ld_shared_v4f(uint32_t addr, float* v) {
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
               : "r"(addr));
}
// TMEM column of K-step kk (16 of the 64-wide step) of an operand that the two compute
// warpgroups packed over their own 32-column regions: steps 0-1 at columns 0-15, steps
// 2-3 at 32-47.
__device__ __forceinline__ uint32_t b2_packed_col(int kk) { return kk < 2 ? kk * 8 : 32 + (kk - 2) * 8; }

// Stores 64 fp32 TMEM columns of this thread's row (from `src`) as 16-bit values.
template <typename T>
__device__ __forceinline__ void b2_store_row64(uint32_t src, T* dst, bool ok, bool have) {
#pragma unroll
  for (int c0 = 0; c0 < 64; c0 += 32) {
    uint32_t v[32];
    if (have) {
      tmem_ld32(src + c0, v);
      tmem_wait_ld();
    }
    uint32_t pk[16];
#pragma unroll
    for (int x = 0; x < 16; ++x)
      pk[x] = have ? Pack2<T>::pack(__uint_as_float(v[2 * x]), __uint_as_float(v[2 * x + 1])) : 0u;
    if (ok) {
      uint4* d4 = reinterpret_cast<uint4*>(dst + c0);
      d4[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      d4[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      d4[2] = make_uint4(pk[8], pk[9], pk[10], pk[11]);
      d4[3] = make_uint4(pk[12], pk[13], pk[14], pk[15]);
    }
  }
}

// ---------------------------------------------------------------- dK / dV
struct B2KvCfg {
  static constexpr int OFF_K = 0;                          // 4 chunks x 16 KB
  static constexpr int OFF_V = 4 * kB2Chunk128;
  static constexpr int OFF_Q = 8 * kB2Chunk128;            // 2 stages x 4 chunks x 8 KB
  static constexpr int OFF_DO = OFF_Q + 2 * 4 * kB2Chunk64;  // 1 stage
  static constexpr int OFF_LSE = OFF_DO + 4 * kB2Chunk64;  // [2 stages][64] fp32
  static constexpr int OFF_DI = OFF_LSE + 2 * 64 * 4;
  static constexpr int OFF_CTL = OFF_DI + 2 * 64 * 4;
  static constexpr int USED = OFF_CTL + 256;
  static constexpr int SMEM_BYTES = USED + 1024;
  static_assert(SMEM_BYTES <= 232448, "dK/dV (D = 256) shared memory budget");
};
struct B2KvCtl {
  uint64_t kv_full;
  uint64_t q_full[2], q_empty[2];
  uint64_t do_full, do_empty;
  uint64_t s_full, dp_full, p_ready, ds_ready, final_done, drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(B2KvCtl) <= 256, "dK/dV (D = 256) control block");

template <typename T, bool EXT>
__global__ void __launch_bounds__(kB2Threads, 1)
    fa_bwd_dkdv_d256_kernel(const __grid_constant__ CUtensorMap tm_q,   // box 64 rows
                            const __grid_constant__ CUtensorMap tm_k,   // box 128 rows
                            const __grid_constant__ CUtensorMap tm_v,   // box 128 rows
                            const __grid_constant__ CUtensorMap tm_do,  // box 64 rows
                            const B2Params p) {
  using Cfg = B2KvCfg;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  if ((base - raw_addr) + Cfg::USED > (uint32_t)Cfg::SMEM_BYTES) {  // uniform
    if (threadIdx.x == 0) record_device_error(p.err, 2, FA_SITE_BWD_PRODUCER);
    return;
  }
  B2KvCtl* ctl = reinterpret_cast<B2KvCtl*>(base_ptr + Cfg::OFF_CTL);
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dh = blockIdx.x & 1;                 // half of the head dimension
  const int k0 = (blockIdx.x >> 1) * kB2Keys;    // first key (heaviest tiles first when causal)
  const int hk = blockIdx.y, b = blockIdx.z;
  const BwdSeq sq = bwd_seq<EXT>(p, b);
  if (EXT && k0 >= sq.Skv) return;  // varlen: past this sequence's keys (uniform, no setup yet)
  const int off = sq.Skv - sq.Sq;                // causal: key j visible to query i iff j <= i + off
  int s_start, s_end;  // query steps that see this CTA's keys (causal bound and window)
  dense_q_tiles(k0, kB2Keys, kB2QStep, sq.Sq, off, p.causal, EXT ? p.swq : 0, EXT ? p.swk : 0,
                s_start, s_end);
  const int nqs = s_end - s_start;
  const int n_iter = p.G * nqs;

  if (threadIdx.x == 0) {
    ctl->abort_flag = 0;
    mbar_init(smem_u32(&ctl->kv_full), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&ctl->q_full[s]), 1);
      mbar_init(smem_u32(&ctl->q_empty[s]), 1);
    }
    mbar_init(smem_u32(&ctl->do_full), 1);
    mbar_init(smem_u32(&ctl->do_empty), 1);
    mbar_init(smem_u32(&ctl->s_full), 1);
    mbar_init(smem_u32(&ctl->dp_full), 1);
    mbar_init(smem_u32(&ctl->p_ready), 256);
    mbar_init(smem_u32(&ctl->ds_ready), 256);
    mbar_init(smem_u32(&ctl->final_done), 1);
    mbar_init(smem_u32(&ctl->drain), 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t sK = base + Cfg::OFF_K, sV = base + Cfg::OFF_V;
  const uint32_t sQ = base + Cfg::OFF_Q, sdO = base + Cfg::OFF_DO;

  if (warp == 0) {
    // ============================================================ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      const uint32_t kvb = smem_u32(&ctl->kv_full);
      mbar_arrive_expect_tx(kvb, 8 * kB2Chunk128);
      for (int c = 0; c < 4; ++c) {
        tma_load_4d(sK + c * kB2Chunk128, &tm_k, kvb, c * 64, hk, sq.kr + k0, sq.tb);
        tma_load_4d(sV + c * kB2Chunk128, &tm_v, kvb, c * 64, hk, sq.kr + k0, sq.tb);
      }
      int i = 0, n_do = 0;
      for (; i < n_iter; ++i) {
        const int s = i & 1;
        if (!mbar_wait(smem_u32(&ctl->q_empty[s]), ((i >> 1) & 1) ^ 1, abort_flag, p.err,
                       FA_SITE_BWD_PRODUCER))
          break;
        const int g = i / nqs, q0 = (s_start + i % nqs) * kB2QStep, h = hk * p.G + g;
        const uint32_t fb = smem_u32(&ctl->q_full[s]);
        mbar_arrive_expect_tx(fb, 4 * kB2Chunk64 + 2 * 256);
        for (int c = 0; c < 4; ++c)
          tma_load_4d(sQ + (s * 4 + c) * kB2Chunk64, &tm_q, fb, c * 64, h, sq.qr + q0, sq.tb);
        const int64_t row0 = ((int64_t)b * p.H + h) * p.Sq_pad + q0;
        b2_bulk_load(base + Cfg::OFF_LSE + s * 256, p.lse2 + row0, 256, fb);
        b2_bulk_load(base + Cfg::OFF_DI + s * 256, p.dsum + row0, 256, fb);
        // dO(i) into its single slot once dV(i - 1), its last reader, completed.
        if (!mbar_wait(smem_u32(&ctl->do_empty), (i & 1) ^ 1, abort_flag, p.err,
                       FA_SITE_BWD_PRODUCER)) {
          ++i;  // Q(i) is in flight: drain it below
          break;
        }
        const uint32_t db = smem_u32(&ctl->do_full);
        mbar_arrive_expect_tx(db, 4 * kB2Chunk64);
        for (int c = 0; c < 4; ++c)
          tma_load_4d(sdO + c * kB2Chunk64, &tm_do, db, c * 64, h, sq.qr + q0, sq.tb);
        n_do = i + 1;
      }
      b2_drain_wait(kvb, 0);
      for (int k = max(0, i - 2); k < i; ++k) b2_drain_wait(smem_u32(&ctl->q_full[k & 1]), (k >> 1) & 1);
      if (n_do > 0) b2_drain_wait(smem_u32(&ctl->do_full), (n_do - 1) & 1);
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      constexpr bool kBf16 = Pack2<T>::kBf16;
      constexpr uint32_t idS = idesc_f16(128, kB2QStep, kBf16, false, false);  // S^T, dP^T
      constexpr uint32_t idKV = idesc_f16(128, 128, kBf16, false, true);       // dV_h, dK_h
      const uint32_t tS = tmem, tdP = tmem + 64, tdV = tmem + 128, tdK = tmem + 256;
      // K-major forms (S^T, dP^T: A = K / V rows of 128 keys, B = Q / dO rows of 64
      // queries; K-step kk = 16 dims: +32 B inside a 64-dim chunk, chunks 16 / 8 KB apart)
      const uint64_t dK_k = sdesc_sw128(sK, 16, 1024), dV_k = sdesc_sw128(sV, 16, 1024);
      const uint64_t dQ_k = sdesc_sw128(sQ, 16, 1024), ddO_k = sdesc_sw128(sdO, 16, 1024);
      // MN-major forms of this CTA's half of Q / dO (B of dK_h / dV_h: K-step = 16 query
      // rows = 2 KB, the half's two 64-dim chunks 8 KB apart)
      const uint64_t dQ_m = sdesc_sw128(sQ + 2 * dh * kB2Chunk64, kB2Chunk64, 1024);
      const uint64_t ddO_m = sdesc_sw128(sdO + 2 * dh * kB2Chunk64, kB2Chunk64, 1024);
      auto issue_S = [&](int s) {
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)
          mma_ss(tS, desc_add(dK_k, (kk >> 2) * kB2Chunk128 + (kk & 3) * 32),
                 desc_add(dQ_k, (s * 4 + (kk >> 2)) * kB2Chunk64 + (kk & 3) * 32), idS, kk > 0);
        mma_commit(smem_u32(&ctl->s_full));
      };
      auto issue_dP = [&]() {
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)
          mma_ss(tdP, desc_add(dV_k, (kk >> 2) * kB2Chunk128 + (kk & 3) * 32),
                 desc_add(ddO_k, (kk >> 2) * kB2Chunk64 + (kk & 3) * 32), idS, kk > 0);
        mma_commit(smem_u32(&ctl->dp_full));
      };
      bool ok = mbar_wait(smem_u32(&ctl->kv_full), 0, abort_flag, p.err, FA_SITE_BWD_MMA);
      if (ok && n_iter > 0) {
        ok = mbar_wait(smem_u32(&ctl->q_full[0]), 0, abort_flag, p.err, FA_SITE_BWD_MMA);
        if (ok) {
          tc_fence_after();
          issue_S(0);
          ok = mbar_wait(smem_u32(&ctl->do_full), 0, abort_flag, p.err, FA_SITE_BWD_MMA);
          if (ok) {
            tc_fence_after();
            issue_dP();
          }
        }
      }
      // Step i: dV(i) once P^T(i) is in TMEM, then S^T(i + 1) (the MMAs run in issue
      // order, so dV(i) has read P^T(i) before S^T(i + 1) overwrites those columns), then
      // dK(i) once dS^T(i) is in TMEM, then dP^T(i + 1) (after dK(i) read dS^T(i)).
      for (int i = 0; i < n_iter && ok; ++i) {
        const int s = i & 1;
        const uint32_t par = i & 1;
        const bool has_next = i + 1 < n_iter;
        ok = mbar_wait(smem_u32(&ctl->p_ready), par, abort_flag, p.err, FA_SITE_BWD_MMA);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ts(tdV, tS + b2_packed_col(kk), desc_add(ddO_m, kk * 2048), idKV,
                 (i > 0 || kk > 0) ? 1u : 0u);
        mma_commit(smem_u32(&ctl->do_empty));  // dO(i): read by dP^T(i) and dV(i)
        if (has_next) {
          ok = mbar_wait(smem_u32(&ctl->q_full[s ^ 1]), ((i + 1) >> 1) & 1, abort_flag, p.err,
                         FA_SITE_BWD_MMA);
          if (!ok) break;
          tc_fence_after();
          issue_S(s ^ 1);
        }
        ok = mbar_wait(smem_u32(&ctl->ds_ready), par, abort_flag, p.err, FA_SITE_BWD_MMA);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ts(tdK, tdP + b2_packed_col(kk), desc_add(dQ_m, s * 4 * kB2Chunk64 + kk * 2048),
                 idKV, (i > 0 || kk > 0) ? 1u : 0u);
        mma_commit(smem_u32(&ctl->q_empty[s]));  // Q(i): read by S^T(i) and dK(i)
        if (has_next) {
          ok = mbar_wait(smem_u32(&ctl->do_full), (i + 1) & 1, abort_flag, p.err, FA_SITE_BWD_MMA);
          if (!ok) break;
          tc_fence_after();
          issue_dP();
        }
      }
      mma_commit(smem_u32(&ctl->final_done));
      mma_commit(smem_u32(&ctl->drain));
      b2_drain_wait(smem_u32(&ctl->drain), 0);
    }
  } else if (warp >= 4) {
    // ============================================================ compute warpgroups
    const int c = (warp - 4) >> 2;              // query columns [32 c, 32 c + 32) of a step
    const int j = ((warp & 3) << 5) | lane;     // key row = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off, tdP = tmem + lane_off + 64;
    const int key = k0 + j;
    const bool key_ok = key < sq.Skv;
    const float c2 = p.scale_log2;
    bool ok = true;
    for (int i = 0; i < n_iter; ++i) {
      const int s = i & 1;
      const uint32_t par = i & 1;
      const int qbase = (s_start + i % nqs) * kB2QStep + 32 * c;
      bool w = mbar_wait(smem_u32(&ctl->q_full[s]), (i >> 1) & 1, abort_flag, p.err,
                         FA_SITE_BWD_COMPUTE);
      w = w && mbar_wait(smem_u32(&ctl->s_full), par, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      tc_fence_after();
      // ---- pass A: P^T = exp2(S^T * scale * log2e - lse * log2e), masked
      float pv[32];
      {
        uint32_t sv[32];
        tmem_ld32(tS + 32 * c, sv);
        float lv[32];
#pragma unroll
        for (int m = 0; m < 8; ++m)
          b2_ld_shared_v4f(base + Cfg::OFF_LSE + s * 256 + (32 * c + 4 * m) * 4, lv + 4 * m);
        tmem_wait_ld();
        if constexpr (EXT) {
          if (p.sc_a != 0.f) {
#pragma unroll
            for (int x = 0; x < 32; ++x)
              sv[x] = __float_as_uint(softcap_score(__uint_as_float(sv[x]), p.sc_a, p.sc_k));
          }
          const bool full = key_ok && dense_visible(key, qbase, off, p.causal, 0, p.swk) &&
                            dense_visible(key, qbase + 31, off, 0, p.swq, 0);
#pragma unroll
          for (int x = 0; x < 32; ++x) {
            const bool vis =
                full || (key_ok && dense_visible(key, qbase + x, off, p.causal, p.swq, p.swk));
            pv[x] = vis ? ex2_approx(fmaf(__uint_as_float(sv[x]), c2, -lv[x])) : 0.f;
          }
        } else {
          const bool full = key_ok && (!p.causal || key <= qbase + off);
#pragma unroll
          for (int x = 0; x < 32; ++x) {
            const bool vis = full || (key_ok && key <= qbase + x + off);
            pv[x] = vis ? ex2_approx(fmaf(__uint_as_float(sv[x]), c2, -lv[x])) : 0.f;
          }
        }
        uint32_t pk[16];
#pragma unroll
        for (int x = 0; x < 16; ++x) pk[x] = Pack2<T>::pack(pv[2 * x], pv[2 * x + 1]);
        tmem_st16(tS + 32 * c, pk);
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl->p_ready));
      if constexpr (EXT) {
        // softcap: pv takes P (1 - tanh^2) (tanh from P and the LSE) now that P^T is in TMEM
        if (p.sc_a != 0.f) {
          float lv[32];
#pragma unroll
          for (int m = 0; m < 8; ++m)
            b2_ld_shared_v4f(base + Cfg::OFF_LSE + s * 256 + (32 * c + 4 * m) * 4, lv + 4 * m);
#pragma unroll
          for (int x = 0; x < 32; ++x) pv[x] = softcap_grad_p(pv[x], lv[x], p.sc_t);
        }
      }
      // ---- pass B: dS^T = P^T (dP^T - D) * scale, packed over its own dP^T columns
      w = mbar_wait(smem_u32(&ctl->dp_full), par, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      tc_fence_after();
      {
        uint32_t dv[32];
        tmem_ld32(tdP + 32 * c, dv);
        float di[32];
#pragma unroll
        for (int m = 0; m < 8; ++m)
          b2_ld_shared_v4f(base + Cfg::OFF_DI + s * 256 + (32 * c + 4 * m) * 4, di + 4 * m);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int x = 0; x < 16; ++x) {
          const float d0 = pv[2 * x] * (__uint_as_float(dv[2 * x]) - di[2 * x]) * p.scale;
          const float d1 = pv[2 * x + 1] * (__uint_as_float(dv[2 * x + 1]) - di[2 * x + 1]) * p.scale;
          pk[x] = Pack2<T>::pack(d0, d1);
        }
        tmem_st16(tdP + 32 * c, pk);
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl->ds_ready));
    }
    if (ok) {
      const bool w = mbar_wait(smem_u32(&ctl->final_done), 0, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
    }
    if (ok) {
      tc_fence_after();
      const int d0 = 128 * dh + 64 * c;  // this warpgroup's 64 dims of the CTA's half
      T* dvr = reinterpret_cast<T*>(p.dv) + (int64_t)b * p.dv_sb + (int64_t)(sq.kr + key) * p.dv_ss +
               (int64_t)hk * p.dv_sh + d0;
      T* dkr = reinterpret_cast<T*>(p.dk) + (int64_t)b * p.dk_sb + (int64_t)(sq.kr + key) * p.dk_ss +
               (int64_t)hk * p.dk_sh + d0;
      b2_store_row64<T>(tmem + lane_off + 128 + 64 * c, dvr, key_ok, n_iter > 0);
      b2_store_row64<T>(tmem + lane_off + 256 + 64 * c, dkr, key_ok, n_iter > 0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------- dQ
struct B2DqCfg {
  static constexpr int OFF_Q = 0;                          // 4 chunks x 16 KB
  static constexpr int OFF_DO = 4 * kB2Chunk128;
  static constexpr int OFF_K = 8 * kB2Chunk128;            // 2 stages x 4 chunks x 8 KB
  static constexpr int OFF_V = OFF_K + 2 * 4 * kB2Chunk64; // 1 stage
  static constexpr int OFF_CTL = OFF_V + 4 * kB2Chunk64;
  static constexpr int USED = OFF_CTL + 256;
  static constexpr int SMEM_BYTES = USED + 1024;
  static_assert(SMEM_BYTES <= 232448, "dQ (D = 256) shared memory budget");
};
struct B2DqCtl {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full, v_empty;
  uint64_t s_full, dp_full, ds_ready, final_done, drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(B2DqCtl) <= 256, "dQ (D = 256) control block");

template <typename T, bool EXT>
__global__ void __launch_bounds__(kB2Threads, 1)
    fa_bwd_dq_d256_kernel(const __grid_constant__ CUtensorMap tm_q,   // box 128 rows
                          const __grid_constant__ CUtensorMap tm_k,   // box 64 rows
                          const __grid_constant__ CUtensorMap tm_v,   // box 64 rows
                          const __grid_constant__ CUtensorMap tm_do,  // box 128 rows
                          const B2Params p) {
  using Cfg = B2DqCfg;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  if ((base - raw_addr) + Cfg::USED > (uint32_t)Cfg::SMEM_BYTES) {
    if (threadIdx.x == 0) record_device_error(p.err, 2, FA_SITE_BWD_PRODUCER);
    return;
  }
  B2DqCtl* ctl = reinterpret_cast<B2DqCtl*>(base_ptr + Cfg::OFF_CTL);
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z, hk = h / p.G;
  const int qt = p.causal ? (gridDim.x - 1 - blockIdx.x) : blockIdx.x;  // heaviest first
  const int q0 = qt * kB2Rows;
  const BwdSeq sq = bwd_seq<EXT>(p, b);
  if (EXT && q0 >= sq.Sq) return;  // varlen: past this sequence's rows (uniform, no setup yet)
  const int off = sq.Skv - sq.Sq;
  // Key steps j0 .. j0 + nks - 1 hold the keys this Q tile sees (causal bound and window);
  // the loops below count j from 0 (pipeline index) and read step j0 + j.
  int j0, j1;
  dense_k_tiles(q0, kB2Rows, kB2KStep, sq.Sq, sq.Skv, off, p.causal, EXT ? p.swq : 0,
                EXT ? p.swk : 0, j0, j1);
  const int nks = j1 - j0;

  if (threadIdx.x == 0) {
    ctl->abort_flag = 0;
    mbar_init(smem_u32(&ctl->q_full), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&ctl->k_full[s]), 1);
      mbar_init(smem_u32(&ctl->k_empty[s]), 1);
    }
    mbar_init(smem_u32(&ctl->v_full), 1);
    mbar_init(smem_u32(&ctl->v_empty), 1);
    mbar_init(smem_u32(&ctl->s_full), 1);
    mbar_init(smem_u32(&ctl->dp_full), 1);
    mbar_init(smem_u32(&ctl->ds_ready), 256);
    mbar_init(smem_u32(&ctl->final_done), 1);
    mbar_init(smem_u32(&ctl->drain), 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t sQ = base + Cfg::OFF_Q, sdO = base + Cfg::OFF_DO;
  const uint32_t sK = base + Cfg::OFF_K, sV = base + Cfg::OFF_V;

  if (warp == 0) {
    // ============================================================ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      const uint32_t qb = smem_u32(&ctl->q_full);
      mbar_arrive_expect_tx(qb, 8 * kB2Chunk128);
      for (int c = 0; c < 4; ++c) {
        tma_load_4d(sQ + c * kB2Chunk128, &tm_q, qb, c * 64, h, sq.qr + q0, sq.tb);
        tma_load_4d(sdO + c * kB2Chunk128, &tm_do, qb, c * 64, h, sq.qr + q0, sq.tb);
      }
      int jk = 0, jv = 0;
      bool ok = true;
      for (int j = 0; j < nks && ok; ++j) {
        const int s = j & 1;
        ok = mbar_wait(smem_u32(&ctl->k_empty[s]), ((j >> 1) & 1) ^ 1, abort_flag, p.err,
                       FA_SITE_BWD_PRODUCER);
        if (!ok) break;
        const uint32_t kb = smem_u32(&ctl->k_full[s]);
        mbar_arrive_expect_tx(kb, 4 * kB2Chunk64);
        for (int c = 0; c < 4; ++c)
          tma_load_4d(sK + (s * 4 + c) * kB2Chunk64, &tm_k, kb, c * 64, hk,
                      sq.kr + (j0 + j) * kB2KStep, sq.tb);
        jk = j + 1;
        ok = mbar_wait(smem_u32(&ctl->v_empty), (j & 1) ^ 1, abort_flag, p.err, FA_SITE_BWD_PRODUCER);
        if (!ok) break;
        const uint32_t vb = smem_u32(&ctl->v_full);
        mbar_arrive_expect_tx(vb, 4 * kB2Chunk64);
        for (int c = 0; c < 4; ++c)
          tma_load_4d(sV + c * kB2Chunk64, &tm_v, vb, c * 64, hk, sq.kr + (j0 + j) * kB2KStep,
                      sq.tb);
        jv = j + 1;
      }
      b2_drain_wait(qb, 0);
      for (int k = max(0, jk - 2); k < jk; ++k) b2_drain_wait(smem_u32(&ctl->k_full[k & 1]), (k >> 1) & 1);
      if (jv > 0) b2_drain_wait(smem_u32(&ctl->v_full), (jv - 1) & 1);
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      constexpr bool kBf16 = Pack2<T>::kBf16;
      constexpr uint32_t idS = idesc_f16(128, kB2KStep, kBf16, false, false);  // S, dP
      constexpr uint32_t idQ = idesc_f16(128, 256, kBf16, false, true);        // dQ
      const uint32_t tS = tmem, tdP = tmem + 64, tdQ = tmem + 128;
      const uint64_t dQ_k = sdesc_sw128(sQ, 16, 1024), ddO_k = sdesc_sw128(sdO, 16, 1024);
      const uint64_t dK_k = sdesc_sw128(sK, 16, 1024), dV_k = sdesc_sw128(sV, 16, 1024);
      // K as the MN-major B of dQ += dS K: K-step = 16 key rows = 2 KB, 64-dim chunks 8 KB apart
      const uint64_t dK_m = sdesc_sw128(sK, kB2Chunk64, 1024);
      bool ok = mbar_wait(smem_u32(&ctl->q_full), 0, abort_flag, p.err, FA_SITE_BWD_MMA);
      // Step j: S(j) = Q K(j)^T, dP(j) = dO V(j)^T, then (dS(j) in TMEM) dQ += dS(j) K(j);
      // S(j + 1) is issued after dQ(j), which reads dS(j) from the same columns.
      for (int j = 0; j < nks && ok; ++j) {
        const int s = j & 1;
        ok = mbar_wait(smem_u32(&ctl->k_full[s]), (j >> 1) & 1, abort_flag, p.err, FA_SITE_BWD_MMA);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)
          mma_ss(tS, desc_add(dQ_k, (kk >> 2) * kB2Chunk128 + (kk & 3) * 32),
                 desc_add(dK_k, (s * 4 + (kk >> 2)) * kB2Chunk64 + (kk & 3) * 32), idS, kk > 0);
        mma_commit(smem_u32(&ctl->s_full));
        ok = mbar_wait(smem_u32(&ctl->v_full), j & 1, abort_flag, p.err, FA_SITE_BWD_MMA);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)
          mma_ss(tdP, desc_add(ddO_k, (kk >> 2) * kB2Chunk128 + (kk & 3) * 32),
                 desc_add(dV_k, (kk >> 2) * kB2Chunk64 + (kk & 3) * 32), idS, kk > 0);
        mma_commit(smem_u32(&ctl->dp_full));
        mma_commit(smem_u32(&ctl->v_empty));
        ok = mbar_wait(smem_u32(&ctl->ds_ready), j & 1, abort_flag, p.err, FA_SITE_BWD_MMA);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ts(tdQ, tS + b2_packed_col(kk), desc_add(dK_m, s * 4 * kB2Chunk64 + kk * 2048), idQ,
                 (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(smem_u32(&ctl->k_empty[s]));
      }
      mma_commit(smem_u32(&ctl->final_done));
      mma_commit(smem_u32(&ctl->drain));
      b2_drain_wait(smem_u32(&ctl->drain), 0);
    }
  } else if (warp >= 4) {
    // ============================================================ compute warpgroups
    const int c = (warp - 4) >> 2;           // key columns [32 c, 32 c + 32) of a step
    const int r = ((warp & 3) << 5) | lane;  // query row = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off, tdP = tmem + lane_off + 64;
    const int qi = q0 + r;
    const bool q_ok = qi < sq.Sq;
    const int64_t row = ((int64_t)b * p.H + h) * p.Sq_pad + qi;
    const float lse2 = p.lse2[row];  // padded / empty rows hold +inf -> P = 0
    const float di = p.dsum[row];
    const float c2 = p.scale_log2;
    bool ok = true;
    for (int j = 0; j < nks; ++j) {
      bool w = mbar_wait(smem_u32(&ctl->s_full), j & 1, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      tc_fence_after();
      float pv[32];
      {
        uint32_t sv[32];
        tmem_ld32(tS + 32 * c, sv);
        tmem_wait_ld();
        const int kb = (j0 + j) * kB2KStep + 32 * c;
        if constexpr (EXT) {
          // softcap: pv takes P (1 - tanh^2), the factor dS picks up from the cap
          const bool capped = p.sc_a != 0.f;
#pragma unroll
          for (int x = 0; x < 32; ++x) {
            const int key = kb + x;
            const bool vis =
                q_ok && key < sq.Skv && dense_visible(key, qi, off, p.causal, p.swq, p.swk);
            float sx = __uint_as_float(sv[x]), g = 1.f;
            if (capped) {
              sx = softcap_score(sx, p.sc_a, p.sc_k);
              const float t = sx * p.sc_ia;
              g = fmaf(-t, t, 1.f);
            }
            pv[x] = vis ? ex2_approx(fmaf(sx, c2, -lse2)) * g : 0.f;
          }
        } else {
#pragma unroll
          for (int x = 0; x < 32; ++x) {
            const int key = kb + x;
            const bool vis = q_ok && key < sq.Skv && (!p.causal || key <= qi + off);
            pv[x] = vis ? ex2_approx(fmaf(__uint_as_float(sv[x]), c2, -lse2)) : 0.f;
          }
        }
      }
      w = mbar_wait(smem_u32(&ctl->dp_full), j & 1, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      tc_fence_after();
      {
        uint32_t dv[32];
        tmem_ld32(tdP + 32 * c, dv);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int x = 0; x < 16; ++x)
          pk[x] = Pack2<T>::pack(pv[2 * x] * (__uint_as_float(dv[2 * x]) - di) * p.scale,
                                 pv[2 * x + 1] * (__uint_as_float(dv[2 * x + 1]) - di) * p.scale);
        // dS row r, keys 32 c .. 32 c + 31 of the step, over its own S columns
        tmem_st16(tS + 32 * c, pk);
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl->ds_ready));
    }
    if (ok) {
      const bool w = mbar_wait(smem_u32(&ctl->final_done), 0, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
    }
    if (ok) {
      tc_fence_after();
      T* dst = reinterpret_cast<T*>(p.dq) + (int64_t)b * p.dq_sb + (int64_t)(sq.qr + qi) * p.dq_ss +
               (int64_t)h * p.dq_sh + 128 * c;
      b2_store_row64<T>(tmem + lane_off + 128 + 128 * c, dst, q_ok, nks > 0);
      b2_store_row64<T>(tmem + lane_off + 128 + 128 * c + 64, dst + 64, q_ok, nks > 0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------- host side
template <typename T, bool EXT>
static int launch_bwd_d256_impl(const fa_bwd_args_t* a, const B2Params& p, cudaStream_t st) {
  const CUtensorMapDataType dt = tmap_dtype(a->dtype);
  auto enc = [&](CUtensorMap* m, const void* ptr, const int64_t* s, int heads, int seq, int rows) {
    const uint64_t dims[4] = {256, (uint64_t)heads, (uint64_t)seq, (uint64_t)a->batch};
    const uint64_t str[3] = {(uint64_t)s[2] * 2, (uint64_t)s[1] * 2, (uint64_t)s[0] * 2};
    const uint32_t box[4] = {64, 1, (uint32_t)rows, 1};
    return encode_tmap(m, dt, 4, ptr, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
  };
  CUtensorMap tq64, tdo64, tk128, tv128, tq128, tdo128, tk64, tv64;
  FA_TMAP_TRY(enc(&tq64, a->q, a->q_stride, a->num_heads, a->seqlen_q, 64));
  FA_TMAP_TRY(enc(&tdo64, a->dout, a->do_stride, a->num_heads, a->seqlen_q, 64));
  FA_TMAP_TRY(enc(&tk128, a->k, a->k_stride, a->num_heads_k, a->seqlen_k, 128));
  FA_TMAP_TRY(enc(&tv128, a->v, a->v_stride, a->num_heads_k, a->seqlen_k, 128));
  FA_TMAP_TRY(enc(&tq128, a->q, a->q_stride, a->num_heads, a->seqlen_q, 128));
  FA_TMAP_TRY(enc(&tdo128, a->dout, a->do_stride, a->num_heads, a->seqlen_q, 128));
  FA_TMAP_TRY(enc(&tk64, a->k, a->k_stride, a->num_heads_k, a->seqlen_k, 64));
  FA_TMAP_TRY(enc(&tv64, a->v, a->v_stride, a->num_heads_k, a->seqlen_k, 64));
  auto kkv = fa_bwd_dkdv_d256_kernel<T, EXT>;
  auto kq = fa_bwd_dq_d256_kernel<T, EXT>;
  static std::atomic<bool> attr_kv[kMaxContexts], attr_q[kMaxContexts];
  if (int s = smem_attr_once(kkv, B2KvCfg::SMEM_BYTES, attr_kv)) return s;
  if (int s = smem_attr_once(kq, B2DqCfg::SMEM_BYTES, attr_q)) return s;
  const dim3 gkv(2 * ((p.Skv + kB2Keys - 1) / kB2Keys), a->num_heads_k, p.B);
  prof_begin(FA_PROF_BWD_DKDV, st);
  kkv<<<gkv, kB2Threads, B2KvCfg::SMEM_BYTES, st>>>(tq64, tk128, tv128, tdo64, p);
  prof_end(FA_PROF_BWD_DKDV, st);
  FA_CUDA_TRY(cudaGetLastError());
  count_launch();
  const dim3 gq((p.Sq + kB2Rows - 1) / kB2Rows, a->num_heads, p.B);
  kq<<<gq, kB2Threads, B2DqCfg::SMEM_BYTES, st>>>(tq128, tk64, tv64, tdo128, p);
  FA_CUDA_TRY(cudaGetLastError());
  count_launch();
  return FA_OK;
}

int launch_bwd_d256(const fa_bwd_args_t* a, const float* lse2, const float* dsum, int sq_pad,
                    int* err, cudaStream_t st, const BwdVarlen* vl) {
  B2Params p{};
  p.B = vl ? vl->batch : a->batch;
  p.Sq = vl ? vl->max_q : a->seqlen_q;
  p.Skv = vl ? vl->max_k : a->seqlen_k;
  if (vl) {
    p.cu_q = vl->cu_q;
    p.cu_k = vl->cu_k;
  }
  p.H = a->num_heads;
  p.Hk = a->num_heads_k;
  p.G = a->num_heads / a->num_heads_k;
  p.Sq_pad = sq_pad;
  p.causal = a->causal;
  p.swq = a->window_q > 0 ? a->window_q : 0;
  p.swk = a->window_k > 0 ? a->window_k : 0;
  p.scale = a->softmax_scale;
  p.scale_log2 = a->softmax_scale * 1.4426950408889634f;
  if (a->softcap > 0.f) {
    p.sc_a = a->softcap / a->softmax_scale;
    p.sc_k = 2.f * 1.4426950408889634f / p.sc_a;
    p.sc_ia = a->softmax_scale / a->softcap;
    p.sc_t = 1.f / (1.4426950408889634f * a->softcap);
  }
  p.lse2 = lse2;
  p.dsum = dsum;
  p.dq = a->dq;
  p.dk = a->dk;
  p.dv = a->dv;
  p.dq_sb = vl ? 0 : a->dq_stride[0];  // varlen: rows through the packed offsets
  p.dq_ss = a->dq_stride[1];
  p.dq_sh = a->dq_stride[2];
  p.dk_sb = vl ? 0 : a->dk_stride[0];
  p.dk_ss = a->dk_stride[1];
  p.dk_sh = a->dk_stride[2];
  p.dv_sb = vl ? 0 : a->dv_stride[0];
  p.dv_ss = a->dv_stride[1];
  p.dv_sh = a->dv_stride[2];
  p.err = err;
  const bool bf16 = a->dtype == FA_DTYPE_BF16;
  if (p.swq > 0 || p.swk > 0 || p.sc_a != 0.f || vl != nullptr)
    return bf16 ? launch_bwd_d256_impl<__nv_bfloat16, true>(a, p, st)
                : launch_bwd_d256_impl<__half, true>(a, p, st);
  return bf16 ? launch_bwd_d256_impl<__nv_bfloat16, false>(a, p, st)
              : launch_bwd_d256_impl<__half, false>(a, p, st);
}

}  // namespace fa
