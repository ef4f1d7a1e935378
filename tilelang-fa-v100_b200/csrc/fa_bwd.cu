// Attention backward on sm_100a (reference: tilelang_backward,
// _kernels_backward.py:200-208, with the dQ kernel :10-85 and the dK/dV kernel
// :88-176).  P is recomputed from the saved LSE; dS = P * (dP - D) * scale with the
// row-dot D = rowsum(O * dO) (:203).
//
// Kernels (all on the caller's stream):
//   1. fa_bwd_prep     D = rowsum(O * dO) in fp32 and LSE * log2(e), per query row, padded
//                      to a multiple of 128 rows (+inf / 0 in the padding so padded rows
//                      contribute P = 0); in atomic mode it also clears the dQ accumulator.
//   2. fa_bwd_dkdv     one CTA per (128-key KV tile, kv head, batch) owns dK and dV in
//                      TMEM and loops over the G query heads of its kv head x the query
//                      tiles that can see its keys (causal skips the rest).  Per 128-row
//                      query tile, five tcgen05 GEMMs:
//                        S^T  = K Q^T            (SS)      -> TMEM [0,128)
//                        dP^T = V dO^T           (SS)      -> TMEM [128,256)
//                        dV  += P^T dO           (TS, A = P^T from TMEM)
//                        dK  += dS^T Q           (SS, A = dS^T K-major in smem)
//                        dQ^T = K^T dS^T         (SS, both MN-major) -> the dP^T columns
//                      and dQ is added to an fp32 accumulator (atomic mode): at D = 128
//                      each 64-query half is staged in shared memory and added by one
//                      bulk reduce-add, at D = 64 by per-thread fp32 atomics.  In
//                      deterministic mode the last GEMM is skipped.  All five are
//                      M = 128, N = 128 (N = D for dV / dK).
//                      Issue order per step i: dV(i), S(i+1), dQ(i), dK(i), dP(i+1), so
//                      S(i+1) overlaps the dS pass of step i and the dQ drain overlaps dK(i).
//   2b. fa_bwd_dkdv_persist  the same pipeline as 2, one CTA per SM looping over the
//                      work items, for atomic mode at D = 128 with one query head per kv
//                      head and short items (bwd_persistent on the host).
//   3. fa_bwd_dq       deterministic mode only: one CTA per (128-row Q tile, head,
//                      batch) loops over KV tiles and accumulates dQ in TMEM
//                      (S = Q K^T, dP = dO V^T, dQ += dS K), no atomics.
//   4. fa_bwd_dq_conv  atomic mode: fp32 accumulator -> dq in the input dtype (BSHD).
//
// Roles in fa_bwd_dkdv (512 threads): warp 0 TMA producer (K, V once; Q, LSE, D per
// query tile in a 2-stage ring; dO in its own 1- or 2-slot ring), warp 1 TMEM allocator
// + MMA issuer, warps 4-11 two compute warpgroups: thread = key row (TMEM lane);
// warpgroup c handles query columns [64c, 64c+64) of S^T / dP^T, writes P^T to TMEM
// columns [64c, 64c+32) (over S^T columns it has already read) and dS^T to the
// shared-memory dS tile; warps 12-15 (atomic mode) move dQ out of TMEM and add it to
// the fp32 accumulator.
#include "fa_ptx.cuh"
#include "fa_internal.h"
#include <cmath>

namespace fa {

constexpr int kBwdBN = 128;  // keys per CTA
constexpr int kBwdBM = 128;  // query rows per iteration
constexpr int kBwdOrderGroup = 8;  // (batch, kv head) units ordered together, heaviest tile first

template <int D>
struct BwdCfg {
  static constexpr int DH = D / 64;
  static constexpr int TILE = 128 * D * 2;
  static constexpr int CHUNK = 128 * 128;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = TILE;
  // D = 128: dQ halves are staged in shared memory ([64 q][D] fp32 = TILE bytes) and
  // added by bulk reduce; the staging tile is the room a second dO buffer would take,
  // so dO has one buffer (loaded after dV(i), its last reader, in time for dP(i+1)).
  // D = 64: per-thread fp32 atomics (measured equal or faster there) and two dO buffers.
  static constexpr bool BULK_DQ = D == 128;
  static constexpr int DO_ST = BULK_DQ ? 1 : 2;
  static constexpr int STG_N = BULK_DQ ? 1 : 0;
  static constexpr int OFF_Q = 2 * TILE;           // 2 stages
  static constexpr int OFF_DO = 4 * TILE;
  static constexpr int OFF_STG = OFF_DO + DO_ST * TILE;
  static constexpr int OFF_DS = OFF_STG + STG_N * TILE;  // [2 q chunks][128 keys][64 q] 16-bit
  static constexpr int OFF_LSE = OFF_DS + 128 * 128 * 2;  // [2][128] fp32
  static constexpr int OFF_DI = OFF_LSE + 2 * 128 * 4;    // [2][128] fp32
  static constexpr int OFF_CTL = OFF_DI + 2 * 128 * 4;
  static constexpr int USED = OFF_CTL + 256;
  static constexpr int SMEM_BYTES = (USED + 1024 <= 232448) ? USED + 1024 : 232448;
  static_assert(USED <= 232448, "backward shared memory budget");
  static constexpr int TMEM_COLS = 512;
  static_assert(256 + 2 * D <= TMEM_COLS, "TMEM: S^T, dP^T, dV, dK");
};

struct BwdParams {
  int B, Sq, Skv, H, Hk, G, Sq_pad;
  int d_real;  // the caller's head_dim (32 / 96 run the 64 / 128 kernels)
  int causal;
  int swq, swk;  // sliding window (dense_visible in fa_internal.h; <= 0: off)
  // softcap (0: off): sc_a = softcap / scale, sc_k = 2 log2(e) / sc_a (softcap_score),
  // sc_ia = 1 / sc_a, sc_t = 1 / (log2(e) softcap) (tanh of a score from its P)
  float sc_a, sc_k, sc_ia, sc_t;
  // varlen (packed sequences, EXT kernels only): sequence b's query rows are [cu_q[b],
  // cu_q[b + 1]) and key rows [cu_k[b], cu_k[b + 1]) of [total, heads, D] tensors; B, Sq
  // and Skv are then the batch and the longest lengths (grids, padded lse2 / dsum / dQ
  // accumulator rows).  Null for dense launches.
  const int32_t* cu_q;
  const int32_t* cu_k;
  int n_t, n_u, n_items;  // KV tiles per (batch, kv head), B * Hk units, n_t * n_u items
  float scale, scale_log2;
  const float* lse2;  // [B, H, Sq_pad] lse * log2(e); +inf for padded / empty rows
  const float* dsum;  // [B, H, Sq_pad] rowsum(O * dO)
  float* dq_acc;      // [B, H, Sq_pad, D] fp32 (atomic mode)
  void* dq;           // deterministic mode writes here directly
  void* dk;
  void* dv;
  int64_t dq_sb, dq_ss, dq_sh;
  int64_t dk_sb, dk_ss, dk_sh;
  int64_t dv_sb, dv_ss, dv_sh;
  int* err;
};

struct BwdCtl {
  uint64_t kv_full, kv_empty;  // kv_empty: persistent kernel only
  uint64_t st_full[2];
  uint64_t st_empty[2];
  uint64_t s_full, p_ready, ds_ready, final_done, drain;
  uint64_t dp_full, dq_full, dq_free;
  uint64_t do_full[2], do_empty[2];
  uint32_t tmem_base;
  int abort_flag;
  int smem_ok;
};
static_assert(sizeof(BwdCtl) <= 256, "backward control block");

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > 200000000ull) return;
}

// Stores up to 32 16-bit values (four 16-byte units) of a gradient row; units at or past
// `cols` (the head dims left in the row) are skipped: head_dim 32 / 96 run the 64 / 128
// kernels, whose extra columns hold zeros that belong to no tensor.
template <typename T>
__device__ __forceinline__ void store_units(T* dst, const uint32_t* pk, int cols) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int u = 0; u < 4; ++u)
    if (8 * u < cols) d4[u] = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
}

// ---------------------------------------------------------------- 1. preprocess
// D / 8 lanes per row (16-byte loads), 32 / (D / 8) rows per warp and pass, kPrepPasses
// passes per warp with every load issued before the arithmetic.  With a dQ accumulator
// (atomic mode) the same kernel clears its rows, so no separate memset is needed.
constexpr int kPrepPasses = 4;

template <typename T, int D, bool VARLEN>
__global__ void __launch_bounds__(256) fa_bwd_prep_kernel(const T* __restrict__ o,
                                                          const T* __restrict__ dout,
                                                          const float* __restrict__ lse,
                                                          float* lse2, float* dsum, float* dq_acc,
                                                          int B, int Sq, int H, int Sq_pad,
                                                          int64_t o_sb, int64_t o_ss, int64_t o_sh,
                                                          int64_t do_sb, int64_t do_ss,
                                                          int64_t do_sh, int d_real,
                                                          const int32_t* __restrict__ cu_q,
                                                          int total_q) {
  constexpr int TPR = D / 8;
  constexpr int RPW = 32 / TPR;
  const int lane = threadIdx.x & 31;
  const int sub = lane / TPR, cl = lane % TPR;
  const int64_t warp = ((int64_t)blockIdx.x * 256 + threadIdx.x) >> 5;
  const int64_t rows = (int64_t)B * H * Sq_pad;
  const int64_t row0 = warp * RPW * kPrepPasses;
  uint4 av[kPrepPasses], dv[kPrepPasses];
  bool live[kPrepPasses];
#pragma unroll
  for (int ps = 0; ps < kPrepPasses; ++ps) {
    const int64_t row = row0 + ps * RPW + sub;
    const int i = (int)(row % Sq_pad);
    const int64_t bh = row / Sq_pad;
    live[ps] = row < rows && i < Sq;
    int64_t tok = i;
    if constexpr (VARLEN) {
      // row i of sequence b is packed row cu_q[b] + i (the batch strides are 0)
      if (row < rows) {
        const int b = (int)(bh / H);
        live[ps] = i < min(cu_q[b + 1] - cu_q[b], Sq);
        tok = (int64_t)cu_q[b] + i;
      }
    }
    av[ps] = dv[ps] = make_uint4(0u, 0u, 0u, 0u);
    if (live[ps] && cl * 8 < d_real) {
      const int h = (int)(bh % H), b = (int)(bh / H);
      av[ps] = __ldcs(reinterpret_cast<const uint4*>(o + b * o_sb + tok * o_ss +
                                                     (int64_t)h * o_sh) + cl);
      dv[ps] = __ldcs(reinterpret_cast<const uint4*>(dout + b * do_sb + tok * do_ss +
                                                     (int64_t)h * do_sh) + cl);
    }
  }
#pragma unroll
  for (int ps = 0; ps < kPrepPasses; ++ps) {
    const int64_t row = row0 + ps * RPW + sub;
    const uint32_t* a = reinterpret_cast<const uint32_t*>(&av[ps]);
    const uint32_t* c = reinterpret_cast<const uint32_t*>(&dv[ps]);
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = Pack2<T>::unpack(a[e]);
      const float2 y = Pack2<T>::unpack(c[e]);
      acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
    }
#pragma unroll
    for (int sh = TPR / 2; sh > 0; sh >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, sh);
    if (row < rows) {
      if (cl == 0) {
        float l2 = INFINITY;  // padded rows: P = exp2(S - inf) = 0
        if (live[ps]) {
          const int i = (int)(row % Sq_pad);
          const int64_t bh = row / Sq_pad;
          // lse: dense [B, H, Sq]; varlen [H, total_q] (FA2's varlen layout)
          const float L = VARLEN ? lse[(bh % H) * (int64_t)total_q + cu_q[bh / H] + i]
                                 : lse[bh * Sq + i];
          l2 = (L == -INFINITY) ? INFINITY : L * 1.4426950408889634f;
        }
        lse2[row] = l2;
        dsum[row] = live[ps] ? acc : 0.f;
      }
      if (dq_acc != nullptr) {
        float4* z = reinterpret_cast<float4*>(dq_acc + row * D);
#pragma unroll
        for (int q = cl; q < D / 4; q += TPR) z[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  }
}

// ---------------------------------------------------------------- 4. dQ convert
template <typename T, int D, bool VARLEN>
__global__ void __launch_bounds__(256) fa_bwd_dq_convert_kernel(const float* __restrict__ acc,
                                                                T* dq, int B, int Sq, int H,
                                                                int Sq_pad, int64_t sb,
                                                                int64_t ss, int64_t sh,
                                                                int d_real,
                                                                const int32_t* __restrict__ cu_q) {
  const int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x;  // one thread per 4 elements
  const int64_t total = (int64_t)B * H * Sq * (d_real / 4);
  if (idx >= total) return;
  const int c4 = idx % (d_real / 4);
  const int64_t row = idx / (d_real / 4);
  const int h = row % H;
  const int64_t bi = row / H;
  const int i = bi % Sq;
  const int b = bi / Sq;
  // varlen: Sq is the longest sequence; rows past this one's end hold nothing
  int64_t tok = i;
  if constexpr (VARLEN) {
    if (i >= cu_q[b + 1] - cu_q[b]) return;
    tok = (int64_t)cu_q[b] + i;
  }
  const float4 v =
      *reinterpret_cast<const float4*>(acc + (((int64_t)b * H + h) * Sq_pad + i) * D + c4 * 4);
  uint2 pk;
  pk.x = Pack2<T>::pack(v.x, v.y);
  pk.y = Pack2<T>::pack(v.z, v.w);
  *reinterpret_cast<uint2*>(dq + b * sb + tok * ss + (int64_t)h * sh + c4 * 4) = pk;
}

// ---------------------------------------------------------------- 2. dK / dV (+ dQ atomics)
__device__ __forceinline__ void ld_shared_v4f(uint32_t addr, float* v) {
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
               : "r"(addr));
}

// cp.async.bulk.wait_group.read 1: at most one committed bulk operation of this thread may
// still be reading shared memory.
__device__ __forceinline__ void bulk_wait_group_read_1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

// One step of the dQ warpgroup (atomic mode): thread = head-dim column dl (TMEM lane of
// dQ^T, whose 128 columns are the step's queries) moves dQ^T out of TMEM and adds it to
// the fp32 accumulator rows acc[0, 128).
// D = 128: all 128 columns go to registers and the TMEM columns are released (dq_free)
// at once, so dP^T(i+1) never waits for the adds.  The adds are bulk reduce-adds from
// shared memory (they run in the TMA unit and L2, not as per-thread atomics), in four
// 32-query pieces of 16 KB through two staging buffers: a piece is written while the
// previous one is read by its reduce, which keeps the SM's reduce path (~40 GB/s per SM,
// measured; 64 KB per step) busy.  A warp stores 32 consecutive d of a row: 128
// contiguous bytes.  The issuer (thread 384) checks that the reduce that last used a
// buffer has read it before the buffer is written again; named barrier 1 (these 128
// threads) orders both, and its AND ends the loop for all four warps together when a wait
// failed in any of them, so none is left at the barrier.
// D = 64: per-thread atomics, one warp instruction per 128-byte row, the columns released
// after the second half is in registers.  Returns false after a failed wait.
template <int D, bool BULK>
__device__ __forceinline__ bool dq_drain_step(BwdCtl* ctl, uint32_t tq, uint32_t stg, float* acc,
                                              int dl, bool issuer, uint32_t par,
                                              volatile int* abort_flag, int* err, int step) {
  bool w = mbar_wait(smem_u32(&ctl->dq_full), par, abort_flag, err, FA_SITE_BWD_COMPUTE);
  w = __all_sync(0xffffffffu, w);
  if constexpr (BULK) {
    if (!bar_red_and(1, 128, w)) return false;
    if (issuer) FA_TRACE_EVENT(10, step);
    tc_fence_after();
    uint32_t v[128];
#pragma unroll
    for (int c = 0; c < 4; ++c) tmem_ld32(tq + 32 * c, v + 32 * c);
    tmem_wait_ld();
    tc_fence_before();
    mbar_arrive(smem_u32(&ctl->dq_free));
#pragma unroll
    for (int pc = 0; pc < 4; ++pc) {
      const uint32_t buf = stg + (pc & 1) * (32 * D * 4);
      if (issuer) bulk_wait_group_read_1();  // the reduce two pieces back has read `buf`
      bar_sync_n(1, 128);
#pragma unroll
      for (int x = 0; x < 32; ++x)
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(buf + (x * D + dl) * 4), "r"(v[32 * pc + x])
                     : "memory");
      fence_async_shared();
      bar_sync_n(1, 128);
      if (issuer) {
        bulk_reduce_add_f32(acc + 32 * pc * D, buf, 32 * D * 4);
        bulk_commit_group();
        FA_TRACE_EVENT(16 + pc, step);
      }
    }
    if (issuer) FA_TRACE_EVENT(11, step);
    return true;
  } else {
    if (!w) return false;
    tc_fence_after();
    uint32_t v[64];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      tmem_ld32(tq + 64 * hh, v);
      tmem_ld32(tq + 64 * hh + 32, v + 32);
      tmem_wait_ld();
      if (hh == 1) {
        tc_fence_before();
        mbar_arrive(smem_u32(&ctl->dq_free));
      }
      if (dl < D) {
        float* a = acc + (int64_t)(64 * hh) * D + dl;
#pragma unroll
        for (int x = 0; x < 64; ++x) atomicAdd(a + (int64_t)x * D, __uint_as_float(v[x]));
      }
    }
    return true;
  }
}

// 512 threads = 4 warpgroups.  Launch: 128 registers per thread (65,536).  Warpgroup 0
// (producer, MMA issuer, 2 idle warps) drops to 56, the two compute warpgroups rise to
// 144 and the dQ warpgroup to 168 (it holds a step's 128 dQ^T columns); the split is
// sized by ptxas spill reports (none at these values) and uses all 65,536.
constexpr int kBwdThreads = 512;
constexpr int kBwdRegLow = 56;
constexpr int kBwdRegDq = 168;
constexpr int kBwdRegHigh = 144;
static_assert(128 * kBwdRegLow + 256 * kBwdRegHigh + 128 * kBwdRegDq <= 65536,
              "register split exceeds the launch");
// The persistent kernel's compute warpgroups carry the item loop's state as well: they
// get 152 registers (ptxas reports spills at 144), the dQ warpgroup 152.
constexpr int kBwdPRegLow = 56;
constexpr int kBwdPRegDq = 152;
constexpr int kBwdPRegHigh = 152;
static_assert(128 * kBwdPRegLow + 256 * kBwdPRegHigh + 128 * kBwdPRegDq <= 65536,
              "register split exceeds the launch");

template <typename T, int D, bool ATOMIC_DQ, bool EXT>
__global__ void __launch_bounds__(kBwdThreads, 1)
    fa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_do, const BwdParams p) {
  using Cfg = BwdCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const bool smem_ok = (base - raw_addr) + Cfg::USED <= (uint32_t)Cfg::SMEM_BYTES;
  if (!smem_ok) {  // uniform across the CTA: the layout would not fit
    if (threadIdx.x == 0) record_device_error(p.err, 2, FA_SITE_BWD_PRODUCER);
    return;
  }
  BwdCtl* ctl = reinterpret_cast<BwdCtl*>(base_ptr + Cfg::OFF_CTL);
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Work order: the grid's linear index walks groups of kBwdOrderGroup (batch, kv head)
  // units, and inside a group the kv tiles heaviest first (causal: tile 0 sees every query
  // tile) across all its units, so the last CTAs to start are light ones; a group's units
  // run together and share their Q / dO in L2.  (Per-unit heaviest-first left long CTAs
  // for the end when CTAs are long, e.g. GQA looping over several query heads.)
  const int n_t = gridDim.x, n_u = gridDim.y * gridDim.z;
  const int L = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int gsz = min(kBwdOrderGroup, n_u);
  const int grp = L / (gsz * n_t), within = L % (gsz * n_t);
  const int gbase = grp * gsz, gcount = min(gsz, n_u - gbase);
  const int nblk = within / gcount;
  const int unit = gbase + within % gcount;
  const int hk = unit % gridDim.y, b = unit / gridDim.y;
  const int k0 = nblk * kBwdBN;
  const BwdSeq sq = bwd_seq<EXT>(p, b);
  // varlen: the grid spans the longest sequence; tiles past this one's keys have no work
  // (uniform, before any barrier or TMEM is set up)
  if (EXT && k0 >= sq.Skv) return;
  const int off = sq.Skv - sq.Sq;
  int t_start, t_end;  // query tiles that see this CTA's keys (causal bound and window)
  dense_q_tiles(k0, kBwdBN, kBwdBM, sq.Sq, off, p.causal, EXT ? p.swq : 0, EXT ? p.swk : 0,
                t_start, t_end);
  const int nqt = t_end - t_start;
  const int n_iter = p.G * nqt;

  if (threadIdx.x == 0) {
    ctl->abort_flag = 0;
    mbar_init(smem_u32(&ctl->kv_full), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&ctl->st_full[s]), 1);
      mbar_init(smem_u32(&ctl->st_empty[s]), 1);
    }
    mbar_init(smem_u32(&ctl->s_full), 1);
    mbar_init(smem_u32(&ctl->p_ready), 256);
    mbar_init(smem_u32(&ctl->ds_ready), 256);
    mbar_init(smem_u32(&ctl->dp_full), 1);
    mbar_init(smem_u32(&ctl->dq_full), 1);
    mbar_init(smem_u32(&ctl->dq_free), 128);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&ctl->do_full[s]), 1);
      mbar_init(smem_u32(&ctl->do_empty[s]), 1);
    }
    mbar_init(smem_u32(&ctl->final_done), 1);
    mbar_init(smem_u32(&ctl->drain), 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t sK = base + Cfg::OFF_K, sV = base + Cfg::OFF_V;
  const uint32_t sDS = base + Cfg::OFF_DS;
  if (warp < 4) {
    setmaxnreg_dec<kBwdRegLow>();
  if (warp == 0) {
    // ============================================================ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      const uint32_t kvb = smem_u32(&ctl->kv_full);
      mbar_arrive_expect_tx(kvb, 2 * Cfg::TILE);
      for (int dh = 0; dh < Cfg::DH; ++dh) {
        tma_load_4d(sK + dh * Cfg::CHUNK, &tm_k, kvb, dh * 64, hk, sq.kr + k0, sq.tb);
        tma_load_4d(sV + dh * Cfg::CHUNK, &tm_v, kvb, dh * 64, hk, sq.kr + k0, sq.tb);
      }
      int i = 0, n_do = 0;
      for (; i < n_iter; ++i) {
        const int s = i & 1;
        if (!mbar_wait(smem_u32(&ctl->st_empty[s]), ((i >> 1) & 1) ^ 1, abort_flag, p.err,
                       FA_SITE_BWD_PRODUCER))
          break;
        FA_TRACE_EVENT(12, i);
        const int g = i / nqt, qt = t_start + i % nqt, h = hk * p.G + g;
        const uint32_t fb = smem_u32(&ctl->st_full[s]);
        mbar_arrive_expect_tx(fb, Cfg::TILE + 1024);
        const uint32_t sQ = base + Cfg::OFF_Q + s * Cfg::TILE;
        for (int dh = 0; dh < Cfg::DH; ++dh)
          tma_load_4d(sQ + dh * Cfg::CHUNK, &tm_q, fb, dh * 64, h, sq.qr + qt * kBwdBM, sq.tb);
        const int64_t row0 = ((int64_t)b * p.H + h) * p.Sq_pad + qt * kBwdBM;
        bulk_load(base + Cfg::OFF_LSE + s * 512, p.lse2 + row0, 512, fb);
        bulk_load(base + Cfg::OFF_DI + s * 512, p.dsum + row0, 512, fb);
        // dO(i) goes into its slot once dV(i - DO_ST), the slot's last reader, completed.
        const int ds = i % Cfg::DO_ST, du = i / Cfg::DO_ST;
        if (!mbar_wait(smem_u32(&ctl->do_empty[ds]), (du & 1) ^ 1, abort_flag, p.err,
                       FA_SITE_BWD_PRODUCER)) {
          ++i;  // Q(i) is in flight: drain it below
          break;
        }
        const uint32_t db = smem_u32(&ctl->do_full[ds]);
        mbar_arrive_expect_tx(db, Cfg::TILE);
        for (int dh = 0; dh < Cfg::DH; ++dh)
          tma_load_4d(base + Cfg::OFF_DO + ds * Cfg::TILE + dh * Cfg::CHUNK, &tm_do, db, dh * 64,
                      h, sq.qr + qt * kBwdBM, sq.tb);
        n_do = i + 1;
      }
      drain_wait(kvb, 0);
      for (int k = max(0, i - 2); k < i; ++k) drain_wait(smem_u32(&ctl->st_full[k & 1]), (k >> 1) & 1);
      for (int k = max(0, n_do - Cfg::DO_ST); k < n_do; ++k)
        drain_wait(smem_u32(&ctl->do_full[k % Cfg::DO_ST]), (k / Cfg::DO_ST) & 1);
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      constexpr bool kBf16 = Pack2<T>::kBf16;
      constexpr uint32_t idS = idesc_f16(128, 128, kBf16, false, false);
      constexpr uint32_t idKV = idesc_f16(128, D, kBf16, false, true);
      // dQ^T = K^T dS^T (M = 128 head-dim rows; at D = 64 rows 64..127 read the next
      // 16 KB of shared memory and are ignored), N = 128 queries, both operands MN-major.
      constexpr uint32_t idQT = idesc_f16(128, 128, kBf16, true, true);
      const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 256 + D;
      // Descriptors built once (K-major forms for S^T / dP^T, MN-major for the rest).
      const uint64_t dK_k = sdesc_sw128(sK, 16, 1024), dV_k = sdesc_sw128(sV, 16, 1024);
      const uint64_t dQ_k0 = sdesc_sw128(base + Cfg::OFF_Q, 16, 1024);
      const uint64_t ddO_k0 = sdesc_sw128(base + Cfg::OFF_DO, 16, 1024);
      const uint64_t dQ_m0 = sdesc_sw128(base + Cfg::OFF_Q, Cfg::CHUNK, 1024);
      const uint64_t ddO_m0 = sdesc_sw128(base + Cfg::OFF_DO, Cfg::CHUNK, 1024);
      const uint64_t dDS_m = sdesc_sw128(sDS, Cfg::CHUNK, 1024);
      const uint64_t dK_m = sdesc_sw128(sK, Cfg::CHUNK, 1024);
      const uint64_t dDS_k = sdesc_sw128(sDS, 16, 1024);
      // S^T(i) = K Q(i)^T into [0, 128).
      auto issue_S = [&](int st) {
        const uint64_t dQk = desc_add(opaque(dQ_k0), st * Cfg::TILE), dKk = opaque(dK_k);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t o = (kk >> 2) * Cfg::CHUNK + (kk & 3) * 32;
          mma_ss(tS, desc_add(dKk, o), desc_add(dQk, o), idS, kk > 0);
        }
      };
      // dP^T(i) = V dO(i)^T into [128, 256).
      auto issue_dP = [&](int ds) {
        const uint64_t ddOk = desc_add(opaque(ddO_k0), ds * Cfg::TILE), dVk = opaque(dV_k);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t o = (kk >> 2) * Cfg::CHUNK + (kk & 3) * 32;
          mma_ss(tdP, desc_add(dVk, o), desc_add(ddOk, o), idS, kk > 0);
        }
        mma_commit(smem_u32(&ctl->dp_full));
      };
      // dQ^T(i) = K^T dS^T(i) into the dP^T columns, which the dS pass has read.
      auto issue_dQ = [&]() {
        const uint64_t dKm = opaque(dK_m), dDSm = opaque(dDS_m);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ss(tdP, desc_add(dKm, kk * 2048), desc_add(dDSm, kk * 2048), idQT, kk > 0);
        mma_commit(smem_u32(&ctl->dq_full));
      };
      bool ok = mbar_wait(smem_u32(&ctl->kv_full), 0, abort_flag, p.err, FA_SITE_BWD_MMA);
      if (ok && n_iter > 0) {
        ok = mbar_wait(smem_u32(&ctl->st_full[0]), 0, abort_flag, p.err, FA_SITE_BWD_MMA);
        if (ok) {
          tc_fence_after();
          issue_S(0);
          mma_commit(smem_u32(&ctl->s_full));
          ok = mbar_wait(smem_u32(&ctl->do_full[0]), 0, abort_flag, p.err, FA_SITE_BWD_MMA);
          if (ok) {
            tc_fence_after();
            issue_dP(0);
          }
        }
      }
      // Step i: dV(i) as soon as P^T(i) is in TMEM, then S(i+1) (its columns are free:
      // the tensor pipe runs MMAs in issue order, so dV(i) has read P^T first), then
      // dQ^T(i) and dK(i) from the dS tile in shared memory, then dP(i+1) once dQ^T(i)
      // has left TMEM (the dQ warpgroup moves it out while dK(i) runs).  The compute
      // warpgroups find S(i+1) ready when they finish step i.  Every GEMM is N = 128:
      // a tcgen05.mma costs about as long at N = 64 as at N = 128 (measured), so halves
      // would double the tensor time of dP^T and dQ^T.
      for (int i = 0; i < n_iter && ok; ++i) {
        const int s = i & 1;
        const uint32_t par = i & 1;
        const bool has_next = i + 1 < n_iter;
        const int ds = i % Cfg::DO_ST, ds1 = (i + 1) % Cfg::DO_ST;
        const uint64_t dQm = desc_add(opaque(dQ_m0), s * Cfg::TILE);
        const uint64_t ddOm = desc_add(opaque(ddO_m0), ds * Cfg::TILE);
        // dV += P^T dO   (P^T for q 0..63 in columns 0..31, q 64..127 in 64..95)
        ok = mbar_wait(smem_u32(&ctl->p_ready), par, abort_flag, p.err, FA_SITE_BWD_MMA);
        if (!ok) break;
        FA_TRACE_EVENT(3, i);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t acol = (kk < 4) ? kk * 8 : 64 + (kk - 4) * 8;
          mma_ts(tdV, tS + acol, desc_add(ddOm, kk * 2048), idKV, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(smem_u32(&ctl->do_empty[ds]));  // dO(i) read by dP(i) and dV(i)
        if (has_next) {
          ok = mbar_wait(smem_u32(&ctl->st_full[s ^ 1]), ((i + 1) >> 1) & 1, abort_flag, p.err,
                         FA_SITE_BWD_MMA);
          if (!ok) break;
          FA_TRACE_EVENT(2, i);
          tc_fence_after();
          issue_S(s ^ 1);
          mma_commit(smem_u32(&ctl->s_full));
        }
        ok = mbar_wait(smem_u32(&ctl->ds_ready), par, abort_flag, p.err, FA_SITE_BWD_MMA);
        if (!ok) break;
        FA_TRACE_EVENT(4, i);
        tc_fence_after();
        if (ATOMIC_DQ) issue_dQ();
        const uint64_t dDSk = opaque(dDS_k);
        // dK += dS^T Q   (A = dS^T, K-major in shared memory; B = Q MN-major)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t o = (kk >> 2) * Cfg::CHUNK + (kk & 3) * 32;
          mma_ss(tdK, desc_add(dDSk, o), desc_add(dQm, kk * 2048), idKV, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(smem_u32(&ctl->st_empty[s]));
        FA_TRACE_EVENT(5, i);
        if (has_next) {
          ok = mbar_wait(smem_u32(&ctl->do_full[ds1]), ((i + 1) / Cfg::DO_ST) & 1, abort_flag, p.err,
                         FA_SITE_BWD_MMA);
          FA_TRACE_EVENT(0, i);
          if (ok && ATOMIC_DQ)
            ok = mbar_wait(smem_u32(&ctl->dq_free), par, abort_flag, p.err, FA_SITE_BWD_MMA);
          if (ok) {
            FA_TRACE_EVENT(1, i);
            tc_fence_after();
            issue_dP(ds1);
          }
        }
      }
      mma_commit(smem_u32(&ctl->final_done));
      mma_commit(smem_u32(&ctl->drain));
      drain_wait(smem_u32(&ctl->drain), 0);
    }
  }
  } else if (warp < 12) {
    // ============================================================ compute warpgroups
    setmaxnreg_inc<kBwdRegHigh>();
    const int c = (warp - 4) >> 2;              // query-column half
    const int j = ((warp & 3) << 5) | lane;     // key row = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off, tdP = tmem + lane_off + 128;
    const int key = k0 + j;
    const bool key_ok = key < sq.Skv;
    const float c2 = p.scale_log2;
    bool ok = true;
    for (int i = 0; i < n_iter; ++i) {
      const int s = i & 1;
      const uint32_t par = i & 1;
      const int qt = t_start + i % nqt;
      const int q0 = qt * kBwdBM;
      const uint32_t lse_a = base + Cfg::OFF_LSE + s * 512 + 64 * c * 4;
      const uint32_t di_a = base + Cfg::OFF_DI + s * 512 + 64 * c * 4;
      bool w = mbar_wait(smem_u32(&ctl->st_full[s]), (i >> 1) & 1, abort_flag, p.err,
                         FA_SITE_BWD_COMPUTE);
      w = w && mbar_wait(smem_u32(&ctl->s_full), par, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      if (threadIdx.x == 128) FA_TRACE_EVENT(6, i);
      if (threadIdx.x == 128) FA_TRACE_CYCLES(20, i);
      tc_fence_after();
      // ---- pass A: P^T = exp2(S^T * scale*log2e - lse*log2e), masked; 32 columns at a time
      const int qbase = q0 + 64 * c;
      // Every one of the 64 query columns sees this key (row): the first and last
      // columns bound the causal and window conditions.  EXT (a sliding window or a
      // softcap) is a kernel variant, so launches without either run the causal-only
      // masks and raw scores.
      const bool full = EXT ? key_ok && dense_visible(key, qbase, off, p.causal, 0, p.swk) &&
                                  dense_visible(key, qbase + 63, off, 0, p.swq, 0)
                            : key_ok && (!p.causal || key <= qbase + off);
      // Both 32-column halves of S^T are requested before the one wait, so a single TMEM
      // load latency is exposed per pass.
      float pv[64];
      {
        uint32_t sv[64];
        tmem_ld32(tS + 64 * c, sv);
        tmem_ld32(tS + 64 * c + 32, sv + 32);
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          float lv[32];
#pragma unroll
          for (int m = 0; m < 8; ++m) ld_shared_v4f(lse_a + (32 * ch + 4 * m) * 4, lv + 4 * m);
          if (ch == 0) {
            tmem_wait_ld();
            if (threadIdx.x == 128) FA_TRACE_CYCLES(22, i);
          }
          if constexpr (EXT) {
            if (p.sc_a != 0.f) {
#pragma unroll
              for (int x = 0; x < 32; ++x)
                sv[32 * ch + x] = __float_as_uint(
                    softcap_score(__uint_as_float(sv[32 * ch + x]), p.sc_a, p.sc_k));
            }
          }
          if (full) {
#pragma unroll
            for (int x = 0; x < 32; ++x)
              pv[32 * ch + x] = ex2_approx(fmaf(__uint_as_float(sv[32 * ch + x]), c2, -lv[x]));
          } else if constexpr (EXT) {
#pragma unroll
            for (int x = 0; x < 32; ++x) {
              const bool vis =
                  key_ok && dense_visible(key, qbase + 32 * ch + x, off, p.causal, p.swq, p.swk);
              pv[32 * ch + x] =
                  vis ? ex2_approx(fmaf(__uint_as_float(sv[32 * ch + x]), c2, -lv[x])) : 0.f;
            }
          } else {
#pragma unroll
            for (int x = 0; x < 32; ++x) {
              const bool vis = key_ok && key <= qbase + 32 * ch + x + off;
              pv[32 * ch + x] =
                  vis ? ex2_approx(fmaf(__uint_as_float(sv[32 * ch + x]), c2, -lv[x])) : 0.f;
            }
          }
        }
      }
      if (threadIdx.x == 128) FA_TRACE_EVENT(14, i);
      if (threadIdx.x == 128) FA_TRACE_CYCLES(21, i);
      {
        uint32_t pk[32];
#pragma unroll
        for (int x = 0; x < 32; ++x) pk[x] = Pack2<T>::pack(pv[2 * x], pv[2 * x + 1]);
        tmem_st32(tS + 64 * c, pk);
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl->p_ready));
      if (threadIdx.x == 128) FA_TRACE_EVENT(7, i);
      if constexpr (EXT) {
        // softcap: dS picks up d(capped)/d(scaled) = 1 - tanh^2.  P^T is in TMEM for dV
        // already, so pv now takes P (1 - tanh^2), tanh recovered from P and the LSE while
        // dP^T is computed.
        if (p.sc_a != 0.f) {
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            float lv[32];
#pragma unroll
            for (int m = 0; m < 8; ++m) ld_shared_v4f(lse_a + (32 * ch + 4 * m) * 4, lv + 4 * m);
#pragma unroll
            for (int x = 0; x < 32; ++x)
              pv[32 * ch + x] = softcap_grad_p(pv[32 * ch + x], lv[x], p.sc_t);
          }
        }
      }
      // ---- pass B: dS^T = P^T (dP^T - D) * scale, to shared memory (K-major A of dK,
      // MN-major B of dQ^T).  dP^T(i) was committed after dQ^T(i-1) and dK(i-1), so once
      // dp_full(i) has fired those MMAs have finished reading the previous dS tile.
      w = mbar_wait(smem_u32(&ctl->dp_full), par, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      if (threadIdx.x == 128) FA_TRACE_EVENT(8, i);
      if (threadIdx.x == 256) FA_TRACE_EVENT(13, i);
      tc_fence_after();
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t dv[32];
        tmem_ld32(tdP + 64 * c + 32 * hf, dv);
        float di[32];
#pragma unroll
        for (int m = 0; m < 8; ++m) ld_shared_v4f(di_a + (32 * hf + 4 * m) * 4, di + 4 * m);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int x = 0; x < 16; ++x) {
          const int xx = 32 * hf + 2 * x;
          const float d0 = pv[xx] * (__uint_as_float(dv[2 * x]) - di[2 * x]) * p.scale;
          const float d1 = pv[xx + 1] * (__uint_as_float(dv[2 * x + 1]) - di[2 * x + 1]) * p.scale;
          pk[x] = Pack2<T>::pack(d0, d1);
        }
        // dS^T row j, query columns 64c + 32hf .. +31 (128-byte swizzled rows)
        const uint32_t row = sDS + c * Cfg::CHUNK + j * 128;
#pragma unroll
        for (int m = 0; m < 4; ++m)
          st_shared_v4(row + ((((hf << 2) + m) ^ (j & 7)) << 4), pk[4 * m], pk[4 * m + 1],
                       pk[4 * m + 2], pk[4 * m + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl->ds_ready));
      if (threadIdx.x == 128) FA_TRACE_EVENT(9, i);
      if (threadIdx.x == 256) FA_TRACE_EVENT(15, i);
    }
    // ---- dK, dV rows (lane = key row)
    if (ok) {
      bool w = mbar_wait(smem_u32(&ctl->final_done), 0, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
    }
    if (ok) {
      tc_fence_after();
      T* dkr = reinterpret_cast<T*>(p.dk) + (int64_t)b * p.dk_sb + (int64_t)(sq.kr + key) * p.dk_ss +
               (int64_t)hk * p.dk_sh + c * (D / 2);
      T* dvr = reinterpret_cast<T*>(p.dv) + (int64_t)b * p.dv_sb + (int64_t)(sq.kr + key) * p.dv_ss +
               (int64_t)hk * p.dv_sh + c * (D / 2);
#pragma unroll
      for (int w2 = 0; w2 < 2; ++w2) {
        const uint32_t src = tmem + lane_off + 256 + (w2 ? D : 0) + c * (D / 2);
        T* dst = w2 ? dkr : dvr;
#pragma unroll
        for (int c0 = 0; c0 < D / 2; c0 += 32) {
          uint32_t v[32];
          if (n_iter > 0) {
            tmem_ld32(src + c0, v);
            tmem_wait_ld();
          }
          uint32_t pk[16];
#pragma unroll
          for (int x = 0; x < 16; ++x)
            pk[x] = n_iter > 0 ? Pack2<T>::pack(__uint_as_float(v[2 * x]), __uint_as_float(v[2 * x + 1]))
                               : 0u;
          if (key_ok) store_units<T>(dst + c0, pk, p.d_real - (c * (D / 2) + c0));
        }
      }
    }
  } else {
    setmaxnreg_inc<kBwdRegDq>();
    if (ATOMIC_DQ) {
    // ============================================================ dQ warpgroup
    const int dl = ((warp & 3) << 5) | lane;
    const bool issuer = threadIdx.x == 384;
    const uint32_t tq = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + 128;
    const uint32_t stg = base + Cfg::OFF_STG;
    for (int i = 0; i < n_iter; ++i) {
      const int g = i / nqt, qt = t_start + i % nqt, h = hk * p.G + g;
      float* acc = p.dq_acc + (((int64_t)b * p.H + h) * p.Sq_pad + qt * kBwdBM) * D;
      if (!dq_drain_step<D, Cfg::BULK_DQ>(ctl, tq, stg, acc, dl, issuer, i & 1, abort_flag, p.err, i))
        break;
    }
    if (issuer) bulk_wait_group_all();  // the adds complete before the CTA's memory goes
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- 2b. dK / dV, persistent
// fa_bwd_dkdv_persist_kernel runs the per-step pipeline of fa_bwd_dkdv_kernel (same roles,
// shared-memory layout and TMEM map) in a loop over work items; the host launches it for
// <T, 128, atomic dQ> only.
//
// Work item L -> (KV tile, kv head, batch) and its query-tile loop.  Order: groups of
// kBwdOrderGroup (batch, kv head) units, and inside a group the kv tiles heaviest first
// (causal: tile 0 sees every query tile) across all its units, so the last items to start
// are light and a group's units run together and share their Q / dO in L2.  (Per-unit
// heaviest-first left long items for the end when items are long, e.g. GQA looping over
// several query heads.)
struct BwdItem {
  int b, hk, k0, t_start, nqt, n_iter;
};
__device__ __forceinline__ BwdItem bwd_item(const BwdParams& p, int L) {
  const int gsz = min(kBwdOrderGroup, p.n_u);
  const int grp = L / (gsz * p.n_t), within = L % (gsz * p.n_t);
  const int gbase = grp * gsz, gcount = min(gsz, p.n_u - gbase);
  const int unit = gbase + within % gcount;
  BwdItem it;
  it.hk = unit % p.Hk;
  it.b = unit / p.Hk;
  it.k0 = (within / gcount) * kBwdBN;
  // The persistent kernel serves launches without a sliding window or softcap only
  // (bwd_persistent):
  // query tiles from the first one the causal bound lets see these keys.
  const int nqt_all = (p.Sq + kBwdBM - 1) / kBwdBM;
  it.t_start = p.causal ? min(nqt_all, max(0, it.k0 - (p.Skv - p.Sq)) / kBwdBM) : 0;
  it.nqt = nqt_all - it.t_start;
  it.n_iter = p.G * it.nqt;
  return it;
}

template <typename T, int D, bool ATOMIC_DQ>
__global__ void __launch_bounds__(kBwdThreads, 1)
    fa_bwd_dkdv_persist_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_do, const BwdParams p) {
  using Cfg = BwdCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const bool smem_ok = (base - raw_addr) + Cfg::USED <= (uint32_t)Cfg::SMEM_BYTES;
  if (!smem_ok) {  // uniform across the CTA: the layout would not fit
    if (threadIdx.x == 0) record_device_error(p.err, 2, FA_SITE_BWD_PRODUCER);
    return;
  }
  BwdCtl* ctl = reinterpret_cast<BwdCtl*>(base_ptr + Cfg::OFF_CTL);
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // CTA x takes work items x, x + gridDim.x, ...: with gridDim.x = n_items one item per
  // CTA; with one CTA per SM the CTA keeps its barriers and TMEM, and the next item's
  // K / V, Q and dO loads and its first S and dP^T run while this item's dK / dV leave
  // TMEM.  Pipeline parities run over the CTA's query-tile steps (gi) and its items with
  // at least one step (kc); items with none only write dK = dV = 0.
  const int off = p.Skv - p.Sq;

  if (threadIdx.x == 0) {
    ctl->abort_flag = 0;
    mbar_init(smem_u32(&ctl->kv_full), 1);
    mbar_init(smem_u32(&ctl->kv_empty), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&ctl->st_full[s]), 1);
      mbar_init(smem_u32(&ctl->st_empty[s]), 1);
    }
    mbar_init(smem_u32(&ctl->s_full), 1);
    mbar_init(smem_u32(&ctl->p_ready), 256);
    mbar_init(smem_u32(&ctl->ds_ready), 256);
    mbar_init(smem_u32(&ctl->dp_full), 1);
    mbar_init(smem_u32(&ctl->dq_full), 1);
    mbar_init(smem_u32(&ctl->dq_free), 128);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&ctl->do_full[s]), 1);
      mbar_init(smem_u32(&ctl->do_empty[s]), 1);
    }
    mbar_init(smem_u32(&ctl->final_done), 1);
    mbar_init(smem_u32(&ctl->drain), 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t sK = base + Cfg::OFF_K, sV = base + Cfg::OFF_V;
  const uint32_t sDS = base + Cfg::OFF_DS;
  if (warp < 4) {
    setmaxnreg_dec<kBwdPRegLow>();
  if (warp == 0) {
    // ============================================================ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      const uint32_t kvb = smem_u32(&ctl->kv_full);
      int gi = 0, kc = 0, n_do = 0;
      bool ok = true;
      for (int L = blockIdx.x; L < p.n_items && ok; L += gridDim.x) {
        const BwdItem it = bwd_item(p, L);
        if (it.n_iter == 0) continue;
        // K / V replace the last item's once its MMAs have completed (kv_empty).
        if (!mbar_wait(smem_u32(&ctl->kv_empty), (kc & 1) ^ 1, abort_flag, p.err,
                       FA_SITE_BWD_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(kvb, 2 * Cfg::TILE);
        for (int dh = 0; dh < Cfg::DH; ++dh) {
          tma_load_4d(sK + dh * Cfg::CHUNK, &tm_k, kvb, dh * 64, it.hk, it.k0, it.b);
          tma_load_4d(sV + dh * Cfg::CHUNK, &tm_v, kvb, dh * 64, it.hk, it.k0, it.b);
        }
        ++kc;
        for (int i = 0; i < it.n_iter; ++i, ++gi) {
          const int s = gi & 1;
          if (!mbar_wait(smem_u32(&ctl->st_empty[s]), ((gi >> 1) & 1) ^ 1, abort_flag, p.err,
                         FA_SITE_BWD_PRODUCER)) {
            ok = false;
            break;
          }
          FA_TRACE_EVENT(12, gi);
          const int g = i / it.nqt, qt = it.t_start + i % it.nqt, h = it.hk * p.G + g;
          const uint32_t fb = smem_u32(&ctl->st_full[s]);
          mbar_arrive_expect_tx(fb, Cfg::TILE + 1024);
          const uint32_t sQ = base + Cfg::OFF_Q + s * Cfg::TILE;
          for (int dh = 0; dh < Cfg::DH; ++dh)
            tma_load_4d(sQ + dh * Cfg::CHUNK, &tm_q, fb, dh * 64, h, qt * kBwdBM, it.b);
          const int64_t row0 = ((int64_t)it.b * p.H + h) * p.Sq_pad + qt * kBwdBM;
          bulk_load(base + Cfg::OFF_LSE + s * 512, p.lse2 + row0, 512, fb);
          bulk_load(base + Cfg::OFF_DI + s * 512, p.dsum + row0, 512, fb);
          // dO goes into its slot once dV of the step DO_ST before, the slot's last
          // reader, has completed.
          const int ds = gi % Cfg::DO_ST, du = gi / Cfg::DO_ST;
          if (!mbar_wait(smem_u32(&ctl->do_empty[ds]), (du & 1) ^ 1, abort_flag, p.err,
                         FA_SITE_BWD_PRODUCER)) {
            ++gi;  // Q of this step is in flight: drain it below
            ok = false;
            break;
          }
          const uint32_t db = smem_u32(&ctl->do_full[ds]);
          mbar_arrive_expect_tx(db, Cfg::TILE);
          for (int dh = 0; dh < Cfg::DH; ++dh)
            tma_load_4d(base + Cfg::OFF_DO + ds * Cfg::TILE + dh * Cfg::CHUNK, &tm_do, db,
                        dh * 64, h, qt * kBwdBM, it.b);
          n_do = gi + 1;
        }
      }
      // Loads still in flight complete before the CTA exits.
      if (kc > 0) drain_wait(kvb, (kc - 1) & 1);
      for (int k = max(0, gi - 2); k < gi; ++k) drain_wait(smem_u32(&ctl->st_full[k & 1]), (k >> 1) & 1);
      for (int k = max(0, n_do - Cfg::DO_ST); k < n_do; ++k)
        drain_wait(smem_u32(&ctl->do_full[k % Cfg::DO_ST]), (k / Cfg::DO_ST) & 1);
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      constexpr bool kBf16 = Pack2<T>::kBf16;
      constexpr uint32_t idS = idesc_f16(128, 128, kBf16, false, false);
      constexpr uint32_t idKV = idesc_f16(128, D, kBf16, false, true);
      // dQ^T = K^T dS^T (M = 128 head-dim rows; at D = 64 rows 64..127 read the next
      // 16 KB of shared memory and are ignored), N = 128 queries, both operands MN-major.
      constexpr uint32_t idQT = idesc_f16(128, 128, kBf16, true, true);
      const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 256 + D;
      // Descriptors built once (K-major forms for S^T / dP^T, MN-major for the rest).
      const uint64_t dK_k = sdesc_sw128(sK, 16, 1024), dV_k = sdesc_sw128(sV, 16, 1024);
      const uint64_t dQ_k0 = sdesc_sw128(base + Cfg::OFF_Q, 16, 1024);
      const uint64_t ddO_k0 = sdesc_sw128(base + Cfg::OFF_DO, 16, 1024);
      const uint64_t dQ_m0 = sdesc_sw128(base + Cfg::OFF_Q, Cfg::CHUNK, 1024);
      const uint64_t ddO_m0 = sdesc_sw128(base + Cfg::OFF_DO, Cfg::CHUNK, 1024);
      const uint64_t dDS_m = sdesc_sw128(sDS, Cfg::CHUNK, 1024);
      const uint64_t dK_m = sdesc_sw128(sK, Cfg::CHUNK, 1024);
      const uint64_t dDS_k = sdesc_sw128(sDS, 16, 1024);
      // S^T(i) = K Q(i)^T into [0, 128).
      auto issue_S = [&](int st) {
        const uint64_t dQk = desc_add(opaque(dQ_k0), st * Cfg::TILE), dKk = opaque(dK_k);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t o = (kk >> 2) * Cfg::CHUNK + (kk & 3) * 32;
          mma_ss(tS, desc_add(dKk, o), desc_add(dQk, o), idS, kk > 0);
        }
      };
      // dP^T(i) = V dO(i)^T into [128, 256).
      auto issue_dP = [&](int ds) {
        const uint64_t ddOk = desc_add(opaque(ddO_k0), ds * Cfg::TILE), dVk = opaque(dV_k);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t o = (kk >> 2) * Cfg::CHUNK + (kk & 3) * 32;
          mma_ss(tdP, desc_add(dVk, o), desc_add(ddOk, o), idS, kk > 0);
        }
        mma_commit(smem_u32(&ctl->dp_full));
      };
      // dQ^T(i) = K^T dS^T(i) into the dP^T columns, which the dS pass has read.
      auto issue_dQ = [&]() {
        const uint64_t dKm = opaque(dK_m), dDSm = opaque(dDS_m);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ss(tdP, desc_add(dKm, kk * 2048), desc_add(dDSm, kk * 2048), idQT, kk > 0);
        mma_commit(smem_u32(&ctl->dq_full));
      };
      // Per item: wait for its K / V, issue S and dP^T of its first step (dP^T waits
      // until the dQ warpgroup has moved the last step's dQ^T out of those columns), then
      // the steps.  Step g: dV(g) as soon as P^T(g) is in TMEM, then S(g+1) (its columns
      // are free: the tensor pipe runs MMAs in issue order, so dV(g) has read P^T first),
      // then dQ^T(g) and dK(g) from the dS tile in shared memory, then dP(g+1) once
      // dQ^T(g) has left TMEM.  The compute warpgroups find S(g+1) ready when they finish
      // step g.  After the item's last step:
      // final_done (its dK / dV are complete in TMEM) and kv_empty (K / V are free).  The
      // next item's first dV / dK overwrite the accumulators only after its p_ready /
      // ds_ready, which the compute warpgroups give after they have read dK / dV out.
      bool ok = true;
      int gi = 0, kc = 0;
      for (int L = blockIdx.x; L < p.n_items && ok; L += gridDim.x) {
        const int n_iter = bwd_item(p, L).n_iter;
        if (n_iter == 0) continue;
        ok = mbar_wait(smem_u32(&ctl->kv_full), kc & 1, abort_flag, p.err, FA_SITE_BWD_MMA);
        ok = ok && mbar_wait(smem_u32(&ctl->st_full[gi & 1]), (gi >> 1) & 1, abort_flag, p.err,
                             FA_SITE_BWD_MMA);
        if (!ok) break;
        tc_fence_after();
        issue_S(gi & 1);
        mma_commit(smem_u32(&ctl->s_full));
        ok = mbar_wait(smem_u32(&ctl->do_full[gi % Cfg::DO_ST]), (gi / Cfg::DO_ST) & 1, abort_flag,
                       p.err, FA_SITE_BWD_MMA);
        if (ok && ATOMIC_DQ && gi > 0)
          ok = mbar_wait(smem_u32(&ctl->dq_free), (gi - 1) & 1, abort_flag, p.err, FA_SITE_BWD_MMA);
        if (ok) {
          tc_fence_after();
          issue_dP(gi % Cfg::DO_ST);
        }
        for (int i = 0; i < n_iter && ok; ++i) {
          const int g = gi + i;
          const int s = g & 1;
          const uint32_t par = g & 1;
          const bool has_next = i + 1 < n_iter;
          const int ds = g % Cfg::DO_ST, ds1 = (g + 1) % Cfg::DO_ST;
          const uint64_t dQm = desc_add(opaque(dQ_m0), s * Cfg::TILE);
          const uint64_t ddOm = desc_add(opaque(ddO_m0), ds * Cfg::TILE);
          // dV += P^T dO   (P^T for q 0..63 in columns 0..31, q 64..127 in 64..95)
          ok = mbar_wait(smem_u32(&ctl->p_ready), par, abort_flag, p.err, FA_SITE_BWD_MMA);
          if (!ok) break;
          FA_TRACE_EVENT(3, g);
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t acol = (kk < 4) ? kk * 8 : 64 + (kk - 4) * 8;
            mma_ts(tdV, tS + acol, desc_add(ddOm, kk * 2048), idKV, (i > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(smem_u32(&ctl->do_empty[ds]));  // dO(g) read by dP(g) and dV(g)
          if (has_next) {
            ok = mbar_wait(smem_u32(&ctl->st_full[s ^ 1]), ((g + 1) >> 1) & 1, abort_flag, p.err,
                           FA_SITE_BWD_MMA);
            if (!ok) break;
            tc_fence_after();
            issue_S(s ^ 1);
            mma_commit(smem_u32(&ctl->s_full));
          }
          ok = mbar_wait(smem_u32(&ctl->ds_ready), par, abort_flag, p.err, FA_SITE_BWD_MMA);
          if (!ok) break;
          FA_TRACE_EVENT(4, g);
          tc_fence_after();
          if (ATOMIC_DQ) issue_dQ();
          const uint64_t dDSk = opaque(dDS_k);
          // dK += dS^T Q   (A = dS^T, K-major in shared memory; B = Q MN-major)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t o = (kk >> 2) * Cfg::CHUNK + (kk & 3) * 32;
            mma_ss(tdK, desc_add(dDSk, o), desc_add(dQm, kk * 2048), idKV, (i > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(smem_u32(&ctl->st_empty[s]));
          FA_TRACE_EVENT(5, g);
          if (has_next) {
            ok = mbar_wait(smem_u32(&ctl->do_full[ds1]), ((g + 1) / Cfg::DO_ST) & 1, abort_flag,
                           p.err, FA_SITE_BWD_MMA);
            if (ok && ATOMIC_DQ)
              ok = mbar_wait(smem_u32(&ctl->dq_free), par, abort_flag, p.err, FA_SITE_BWD_MMA);
            if (ok) {
              tc_fence_after();
              issue_dP(ds1);
            }
          }
        }
        if (!ok) break;
        gi += n_iter;
        ++kc;
        mma_commit(smem_u32(&ctl->final_done));
        mma_commit(smem_u32(&ctl->kv_empty));
      }
      mma_commit(smem_u32(&ctl->drain));
      drain_wait(smem_u32(&ctl->drain), 0);
    }
  }
  } else if (warp < 12) {
    // ============================================================ compute warpgroups
    setmaxnreg_inc<kBwdPRegHigh>();
    const int c = (warp - 4) >> 2;              // query-column half
    const int j = ((warp & 3) << 5) | lane;     // key row = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off, tdP = tmem + lane_off + 128;
    const float c2 = p.scale_log2;
    bool ok = true;
    int gi = 0, kc = 0;
    for (int L = blockIdx.x; L < p.n_items && ok; L += gridDim.x) {
    const BwdItem it = bwd_item(p, L);
    const int key = it.k0 + j;
    const bool key_ok = key < p.Skv;
    for (int i = 0; i < it.n_iter; ++i) {
      const int g = gi + i;
      const int s = g & 1;
      const uint32_t par = g & 1;
      const int qt = it.t_start + i % it.nqt;
      const int q0 = qt * kBwdBM;
      const uint32_t lse_a = base + Cfg::OFF_LSE + s * 512 + 64 * c * 4;
      const uint32_t di_a = base + Cfg::OFF_DI + s * 512 + 64 * c * 4;
      bool w = mbar_wait(smem_u32(&ctl->st_full[s]), (g >> 1) & 1, abort_flag, p.err,
                         FA_SITE_BWD_COMPUTE);
      w = w && mbar_wait(smem_u32(&ctl->s_full), par, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      if (threadIdx.x == 128) FA_TRACE_EVENT(6, g);
      tc_fence_after();
      // ---- pass A: P^T = exp2(S^T * scale*log2e - lse*log2e), masked; 32 columns at a time
      const int qbase = q0 + 64 * c;
      // Every one of the 64 query columns sees this key (row).  Windowed launches run the
      // one-CTA-per-item kernel (bwd_persistent), so only the causal bound applies here.
      const bool full = key_ok && (!p.causal || key <= qbase + off);
      // Both 32-column halves of S^T are requested before the one wait, so a single TMEM
      // load latency is exposed per pass.
      float pv[64];
      {
        uint32_t sv[64];
        tmem_ld32(tS + 64 * c, sv);
        tmem_ld32(tS + 64 * c + 32, sv + 32);
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          float lv[32];
#pragma unroll
          for (int m = 0; m < 8; ++m) ld_shared_v4f(lse_a + (32 * ch + 4 * m) * 4, lv + 4 * m);
          if (ch == 0) tmem_wait_ld();
          if (full) {
#pragma unroll
            for (int x = 0; x < 32; ++x)
              pv[32 * ch + x] = ex2_approx(fmaf(__uint_as_float(sv[32 * ch + x]), c2, -lv[x]));
          } else {
#pragma unroll
            for (int x = 0; x < 32; ++x) {
              const bool vis = key_ok && key <= qbase + 32 * ch + x + off;
              pv[32 * ch + x] =
                  vis ? ex2_approx(fmaf(__uint_as_float(sv[32 * ch + x]), c2, -lv[x])) : 0.f;
            }
          }
        }
      }
      if (threadIdx.x == 128) FA_TRACE_EVENT(14, g);
      {
        uint32_t pk[32];
#pragma unroll
        for (int x = 0; x < 32; ++x) pk[x] = Pack2<T>::pack(pv[2 * x], pv[2 * x + 1]);
        tmem_st32(tS + 64 * c, pk);
        tmem_wait_st();
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl->p_ready));
      if (threadIdx.x == 128) FA_TRACE_EVENT(7, g);
      // ---- pass B: dS^T = P^T (dP^T - D) * scale, to shared memory (K-major A of dK,
      // MN-major B of dQ^T).  dP^T(i) was committed after dQ^T(i-1) and dK(i-1), so once
      // dp_full(i) has fired those MMAs have finished reading the previous dS tile.
      w = mbar_wait(smem_u32(&ctl->dp_full), par, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      if (threadIdx.x == 128) FA_TRACE_EVENT(8, g);
      tc_fence_after();
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t dv[32];
        tmem_ld32(tdP + 64 * c + 32 * hf, dv);
        float di[32];
#pragma unroll
        for (int m = 0; m < 8; ++m) ld_shared_v4f(di_a + (32 * hf + 4 * m) * 4, di + 4 * m);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int x = 0; x < 16; ++x) {
          const int xx = 32 * hf + 2 * x;
          const float d0 = pv[xx] * (__uint_as_float(dv[2 * x]) - di[2 * x]) * p.scale;
          const float d1 = pv[xx + 1] * (__uint_as_float(dv[2 * x + 1]) - di[2 * x + 1]) * p.scale;
          pk[x] = Pack2<T>::pack(d0, d1);
        }
        // dS^T row j, query columns 64c + 32hf .. +31 (128-byte swizzled rows)
        const uint32_t row = sDS + c * Cfg::CHUNK + j * 128;
#pragma unroll
        for (int m = 0; m < 4; ++m)
          st_shared_v4(row + ((((hf << 2) + m) ^ (j & 7)) << 4), pk[4 * m], pk[4 * m + 1],
                       pk[4 * m + 2], pk[4 * m + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl->ds_ready));
      if (threadIdx.x == 128) FA_TRACE_EVENT(9, g);
    }
    if (!ok) break;
    // ---- dK, dV rows (lane = key row); an item with no step writes zeros
    const int n_iter = it.n_iter;
    if (n_iter > 0) {
      bool w = mbar_wait(smem_u32(&ctl->final_done), kc & 1, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      tc_fence_after();
    }
    {
      const BwdItem ie = bwd_item(p, L);  // recomputed: b, hk need no register in the steps
      T* dkr = reinterpret_cast<T*>(p.dk) + (int64_t)ie.b * p.dk_sb + (int64_t)key * p.dk_ss +
               (int64_t)ie.hk * p.dk_sh + c * (D / 2);
      T* dvr = reinterpret_cast<T*>(p.dv) + (int64_t)ie.b * p.dv_sb + (int64_t)key * p.dv_ss +
               (int64_t)ie.hk * p.dv_sh + c * (D / 2);
#pragma unroll
      for (int w2 = 0; w2 < 2; ++w2) {
        const uint32_t src = tmem + lane_off + 256 + (w2 ? D : 0) + c * (D / 2);
        T* dst = w2 ? dkr : dvr;
#pragma unroll
        for (int c0 = 0; c0 < D / 2; c0 += 32) {
          uint32_t v[32];
          if (n_iter > 0) {
            tmem_ld32(src + c0, v);
            tmem_wait_ld();
          }
          uint32_t pk[16];
#pragma unroll
          for (int x = 0; x < 16; ++x)
            pk[x] = n_iter > 0 ? Pack2<T>::pack(__uint_as_float(v[2 * x]), __uint_as_float(v[2 * x + 1]))
                               : 0u;
          if (key_ok) store_units<T>(dst + c0, pk, p.d_real - (c * (D / 2) + c0));
        }
      }
    }
    if (n_iter > 0) {
      tc_fence_before();  // dK / dV reads ordered before this item's next p_ready
      gi += n_iter;
      ++kc;
    }
    }
  } else {
    setmaxnreg_inc<kBwdPRegDq>();
    if (ATOMIC_DQ) {
    // ============================================================ dQ warpgroup
    const int dl = ((warp & 3) << 5) | lane;
    const bool issuer = threadIdx.x == 384;
    const uint32_t tq = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + 128;
    const uint32_t stg = base + Cfg::OFF_STG;
    bool ok = true;
    int gi = 0;
    for (int L = blockIdx.x; L < p.n_items && ok; L += gridDim.x) {
      const BwdItem it = bwd_item(p, L);
      for (int i = 0; i < it.n_iter && ok; ++i) {
        const int gs = gi + i;
        const int g = i / it.nqt, qt = it.t_start + i % it.nqt, h = it.hk * p.G + g;
        float* acc = p.dq_acc + (((int64_t)it.b * p.H + h) * p.Sq_pad + qt * kBwdBM) * D;
        ok = dq_drain_step<D, Cfg::BULK_DQ>(ctl, tq, stg, acc, dl, issuer, gs & 1, abort_flag,
                                            p.err, gs);
      }
      gi += it.n_iter;
    }
    if (issuer) bulk_wait_group_all();  // the adds complete before the CTA's memory goes
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- 3. deterministic dQ
template <int D>
struct DqCfg {
  static constexpr int DH = D / 64;
  static constexpr int TILE = 128 * D * 2;
  static constexpr int CHUNK = 128 * 128;
  static constexpr int STAGES = (D == 64) ? 4 : 2;  // K/V pairs
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = TILE;
  static constexpr int OFF_KV = 2 * TILE;          // STAGES x (K, V)
  static constexpr int OFF_DS = OFF_KV + STAGES * 2 * TILE;  // [2 key chunks][128 q][64 keys]
  static constexpr int OFF_CTL = OFF_DS + 128 * 128 * 2;
  static constexpr int USED = OFF_CTL + 256;
  static constexpr int SMEM_BYTES = (USED + 1024 <= 232448) ? USED + 1024 : 232448;
  static_assert(USED <= 232448, "dQ kernel shared memory budget");
};

struct DqCtl {
  uint64_t q_full;
  uint64_t kv_full[4];
  uint64_t kv_empty[4];
  uint64_t s_full, dp_full, ds_ready, final_done, drain;
  uint32_t tmem_base;
  int abort_flag;
};

template <typename T, int D, bool EXT>
__global__ void __launch_bounds__(384, 1)
    fa_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_do, const BwdParams p) {
  using Cfg = DqCfg<D>;
  constexpr int ST = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  if ((base - raw_addr) + Cfg::USED > (uint32_t)Cfg::SMEM_BYTES) {
    if (threadIdx.x == 0) record_device_error(p.err, 2, FA_SITE_BWD_PRODUCER);
    return;
  }
  DqCtl* ctl = reinterpret_cast<DqCtl*>(base_ptr + Cfg::OFF_CTL);
  volatile int* abort_flag = &ctl->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z, hk = h / p.G;
  const int qt = p.causal ? (gridDim.x - 1 - blockIdx.x) : blockIdx.x;
  const int q0 = qt * kBwdBM;
  const BwdSeq sq = bwd_seq<EXT>(p, b);
  // varlen: the grid spans the longest sequence; tiles past this one's rows have no work
  // (uniform, before any barrier or TMEM is set up)
  if (EXT && q0 >= sq.Sq) return;
  const int off = sq.Skv - sq.Sq;
  // KV tiles j0 .. j0 + nkv - 1 hold the keys this Q tile sees (causal bound and window);
  // the loops below count j from 0 (pipeline index) and read tile j0 + j.
  int j0, j1;
  dense_k_tiles(q0, kBwdBM, kBwdBN, sq.Sq, sq.Skv, off, p.causal, EXT ? p.swq : 0,
                EXT ? p.swk : 0, j0, j1);
  const int nkv = j1 - j0;

  if (threadIdx.x == 0) {
    ctl->abort_flag = 0;
    mbar_init(smem_u32(&ctl->q_full), 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(smem_u32(&ctl->kv_full[s]), 1);
      mbar_init(smem_u32(&ctl->kv_empty[s]), 1);
    }
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
  const uint32_t sQ = base + Cfg::OFF_Q, sdO = base + Cfg::OFF_DO, sDS = base + Cfg::OFF_DS;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t qb = smem_u32(&ctl->q_full);
      mbar_arrive_expect_tx(qb, 2 * Cfg::TILE);
      for (int dh = 0; dh < Cfg::DH; ++dh) {
        tma_load_4d(sQ + dh * Cfg::CHUNK, &tm_q, qb, dh * 64, h, sq.qr + q0, sq.tb);
        tma_load_4d(sdO + dh * Cfg::CHUNK, &tm_do, qb, dh * 64, h, sq.qr + q0, sq.tb);
      }
      int j = 0;
      for (; j < nkv; ++j) {
        const int s = j % ST;
        if (!mbar_wait(smem_u32(&ctl->kv_empty[s]), ((j / ST) & 1) ^ 1, abort_flag, p.err,
                       FA_SITE_BWD_PRODUCER))
          break;
        const uint32_t fb = smem_u32(&ctl->kv_full[s]);
        mbar_arrive_expect_tx(fb, 2 * Cfg::TILE);
        const uint32_t dk = base + Cfg::OFF_KV + s * 2 * Cfg::TILE;
        for (int dh = 0; dh < Cfg::DH; ++dh) {
          tma_load_4d(dk + dh * Cfg::CHUNK, &tm_k, fb, dh * 64, hk, sq.kr + (j0 + j) * kBwdBN,
                      sq.tb);
          tma_load_4d(dk + Cfg::TILE + dh * Cfg::CHUNK, &tm_v, fb, dh * 64, hk,
                      sq.kr + (j0 + j) * kBwdBN, sq.tb);
        }
      }
      drain_wait(qb, 0);
      for (int k = max(0, j - ST); k < j; ++k) drain_wait(smem_u32(&ctl->kv_full[k % ST]), (k / ST) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr bool kBf16 = Pack2<T>::kBf16;
      constexpr uint32_t idS = idesc_f16(128, 128, kBf16, false, false);
      constexpr uint32_t idQ = idesc_f16(128, D, kBf16, false, true);
      const uint32_t tS = tmem, tdP = tmem + 128, tdQ = tmem + 256;
      const uint64_t dQd = sdesc_sw128(sQ, 16, 1024), ddOd = sdesc_sw128(sdO, 16, 1024);
      const uint64_t dKV_k0 = sdesc_sw128(base + Cfg::OFF_KV, 16, 1024);
      const uint64_t dKV_m0 = sdesc_sw128(base + Cfg::OFF_KV, Cfg::CHUNK, 1024);
      const uint64_t dDS_k = sdesc_sw128(sDS, 16, 1024);
      bool ok = mbar_wait(smem_u32(&ctl->q_full), 0, abort_flag, p.err, FA_SITE_BWD_MMA);
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j % ST;
        ok = mbar_wait(smem_u32(&ctl->kv_full[s]), (j / ST) & 1, abort_flag, p.err, FA_SITE_BWD_MMA);
        if (!ok) break;
        tc_fence_after();
        const uint64_t dKk = desc_add(dKV_k0, s * 2 * Cfg::TILE);
        const uint64_t dVk = desc_add(dKV_k0, s * 2 * Cfg::TILE + Cfg::TILE);
        const uint64_t dKm = desc_add(dKV_m0, s * 2 * Cfg::TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t o = (kk >> 2) * Cfg::CHUNK + (kk & 3) * 32;
          mma_ss(tS, desc_add(dQd, o), desc_add(dKk, o), idS, kk > 0);
        }
        mma_commit(smem_u32(&ctl->s_full));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t o = (kk >> 2) * Cfg::CHUNK + (kk & 3) * 32;
          mma_ss(tdP, desc_add(ddOd, o), desc_add(dVk, o), idS, kk > 0);
        }
        mma_commit(smem_u32(&ctl->dp_full));
        ok = mbar_wait(smem_u32(&ctl->ds_ready), j & 1, abort_flag, p.err, FA_SITE_BWD_MMA);
        if (!ok) break;
        tc_fence_after();
        // dQ += dS K: A = dS K-major from smem ([2 key chunks][128 q][64 keys]), B = K MN-major
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ss(tdQ, desc_add(dDS_k, (kk >> 2) * Cfg::CHUNK + (kk & 3) * 32),
                 desc_add(dKm, kk * 2048), idQ, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(smem_u32(&ctl->kv_empty[s]));
      }
      mma_commit(smem_u32(&ctl->final_done));
      mma_commit(smem_u32(&ctl->drain));
      drain_wait(smem_u32(&ctl->drain), 0);
    }
  } else if (warp >= 4) {
    const int c = (warp - 4) >> 2;           // key-column half
    const int r = ((warp & 3) << 5) | lane;  // query row
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int qi = q0 + r;
    const bool q_ok = qi < sq.Sq;
    const int64_t row = ((int64_t)b * p.H + h) * p.Sq_pad + qi;
    const float lse2 = p.lse2[row];  // padded rows hold +inf -> P = 0
    const float di = p.dsum[row];
    const float c2 = p.scale_log2;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      bool w = mbar_wait(smem_u32(&ctl->s_full), j & 1, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      tc_fence_after();
      float pv[64];
      {
        uint32_t sv[64];
        tmem_ld32(tmem + lane_off + 64 * c, sv);
        tmem_ld32(tmem + lane_off + 64 * c + 32, sv + 32);
        tmem_wait_ld();
        const int kb = (j0 + j) * kBwdBN + 64 * c;
        if constexpr (EXT) {
          // softcap: pv takes P (1 - tanh^2), the factor dS picks up from the cap
          const bool capped = p.sc_a != 0.f;
#pragma unroll
          for (int x = 0; x < 64; ++x) {
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
          for (int x = 0; x < 64; ++x) {
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
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t dv[32];
        tmem_ld32(tmem + lane_off + 128 + 64 * c + 32 * hf, dv);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int x = 0; x < 16; ++x) {
          const int xx = 32 * hf + 2 * x;
          pk[x] = Pack2<T>::pack(pv[xx] * (__uint_as_float(dv[2 * x]) - di) * p.scale,
                                 pv[xx + 1] * (__uint_as_float(dv[2 * x + 1]) - di) * p.scale);
        }
        // dS row r, keys 64c + 32hf .. +31 -> K-major smem tile (key chunk c)
        const uint32_t rowa = sDS + c * Cfg::CHUNK + r * 128;
#pragma unroll
        for (int m = 0; m < 4; ++m)
          st_shared_v4(rowa + ((((hf << 2) + m) ^ (r & 7)) << 4), pk[4 * m], pk[4 * m + 1],
                       pk[4 * m + 2], pk[4 * m + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl->ds_ready));
    }
    if (ok) {
      bool w = mbar_wait(smem_u32(&ctl->final_done), 0, abort_flag, p.err, FA_SITE_BWD_COMPUTE);
      ok = __all_sync(0xffffffffu, w);
    }
    if (ok) {
      tc_fence_after();
      T* dst = reinterpret_cast<T*>(p.dq) + (int64_t)b * p.dq_sb + (int64_t)(sq.qr + qi) * p.dq_ss +
               (int64_t)h * p.dq_sh + c * (D / 2);
#pragma unroll
      for (int c0 = 0; c0 < D / 2; c0 += 32) {
        uint32_t v[32];
        if (nkv > 0) {
          tmem_ld32(tmem + lane_off + 256 + c * (D / 2) + c0, v);
          tmem_wait_ld();
        }
        uint32_t pk[16];
#pragma unroll
        for (int x = 0; x < 16; ++x)
          pk[x] = nkv > 0 ? Pack2<T>::pack(__uint_as_float(v[2 * x]), __uint_as_float(v[2 * x + 1])) : 0u;
        if (q_ok) store_units<T>(dst + c0, pk, p.d_real - (c * (D / 2) + c0));
      }
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
static int pad128(int x) { return (x + 127) / 128 * 128; }

// head_dim 32 / 96 run the 64 / 128 kernels (TMA zero-fills the missing columns on
// load; the prep kernel and the gradient stores stop at the real head_dim).
static int bwd_kernel_dim(int d) { return d == 32 ? 64 : (d == 96 ? 128 : d); }

size_t bwd_workspace_bytes(const fa_bwd_args_t* a, const BwdVarlen* vl) {
  const size_t rows = (size_t)(vl ? vl->batch : a->batch) * a->num_heads *
                      pad128(vl ? vl->max_q : a->seqlen_q);
  size_t n = 2 * (rows * 4 + 256);                         // lse2, dsum
  // dQ accumulator (atomic mode at D = 64 / 128; the D = 256 kernels write dQ directly)
  if (!a->deterministic && a->head_dim != 256) n += rows * bwd_kernel_dim(a->head_dim) * 4 + 256;
  return n + 256;
}

template <typename K>
static int set_smem(K kern, int bytes) {
  FA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  return FA_OK;
}

constexpr int kBwdRegTotal = 128 * kBwdRegLow + 256 * kBwdRegHigh + 128 * kBwdRegDq;
constexpr int kBwdPRegTotal = 128 * kBwdPRegLow + 256 * kBwdPRegHigh + 128 * kBwdPRegDq;

// Atomic-mode dK / dV at D = 128 with one query head per kv head runs on the persistent
// kernel (one CTA per SM looping over the work items) when an item averages at most
// kBwdPersistMaxSteps query-tile steps: its fixed costs (K / V load, first MMAs, dK / dV
// epilogue) then weigh more and the loop overlaps them.  Measured (bf16 causal backward,
// B x S = 64 x 512: 1.38-1.43 -> 1.19 ms; 32 x 1024: 1.67 -> 1.46; 16 x 2048: 2.25 ->
// 2.12; 128 x 256: 1.13 -> 0.99).  Longer items gain nothing (S = 4096: 3.39 -> 3.37), and
// GQA (G query heads per item) and D = 64 lost 10-20 % to the static item assignment.
constexpr int kBwdPersistMaxSteps = 8;
template <int D>
static bool bwd_persistent(const BwdParams& p) {
  if (D != 128 || p.G != 1 || p.swq > 0 || p.swk > 0 || p.sc_a != 0.f) return false;
  const int nqt_all = (p.Sq + kBwdBM - 1) / kBwdBM;
  const int avg_steps = p.causal ? (nqt_all + 1) / 2 : nqt_all;
  return avg_steps <= kBwdPersistMaxSteps;
}

// Row dot D = rowsum(O * dO), lse * log2 e and (atomic mode) the cleared dQ accumulator.
template <typename T, int D>
static int launch_bwd_prep(const fa_bwd_args_t* a, const BwdParams& p, cudaStream_t st) {
  const int64_t rows = (int64_t)p.B * a->num_heads * p.Sq_pad;
  const int64_t rows_per_block = 8 * (32 / (D / 8)) * kPrepPasses;
  const int blocks = (int)((rows + rows_per_block - 1) / rows_per_block);
  // varlen: `a` describes the packed tensors as one batch entry of total_q rows (its
  // seqlen_q); rows are found through cu_q, so the batch strides drop out
  const bool vl = p.cu_q != nullptr;
  auto kern = vl ? fa_bwd_prep_kernel<T, D, true> : fa_bwd_prep_kernel<T, D, false>;
  kern<<<blocks, 256, 0, st>>>(
      reinterpret_cast<const T*>(a->out), reinterpret_cast<const T*>(a->dout), a->lse,
      const_cast<float*>(p.lse2), const_cast<float*>(p.dsum), p.dq_acc, p.B, p.Sq,
      a->num_heads, p.Sq_pad, vl ? 0 : a->o_stride[0], a->o_stride[1], a->o_stride[2],
      vl ? 0 : a->do_stride[0], a->do_stride[1], a->do_stride[2], p.d_real, p.cu_q,
      a->seqlen_q);
  FA_CUDA_TRY(cudaGetLastError());
  count_launch();
  return FA_OK;
}

// EXT: the launch has a sliding window or a softcap (kernel variants with the window
// masks and the softcap transforms; the persistent kernel has neither and serves the
// launches without them).
template <typename T, int D, bool EXT>
static int launch_bwd_impl(const fa_bwd_args_t* a, const CUtensorMap& tq, const CUtensorMap& tk,
                           const CUtensorMap& tv, const CUtensorMap& tdo, BwdParams& p,
                           cudaStream_t st) {
  if (int s = launch_bwd_prep<T, D>(a, p, st)) return s;
  if (!EXT && !a->deterministic && bwd_persistent<D>(p)) {
    auto kern = fa_bwd_dkdv_persist_kernel<T, 128, true>;
    static std::atomic<bool> attr[kMaxContexts];
    const int slot = call_context_slot();
    if (slot < 0 || slot >= kMaxContexts) return FA_ERR_CUDA;
    if (!attr[slot].load(std::memory_order_acquire)) {
      if (int s = check_reg_split(kern, kBwdThreads, kBwdPRegTotal)) return s;
      if (int s = set_smem(kern, BwdCfg<128>::SMEM_BYTES)) return s;
      attr[slot].store(true, std::memory_order_release);
    }
    const unsigned grid = (unsigned)min(p.n_items, num_sms());
    prof_begin(FA_PROF_BWD_DKDV, st);
    kern<<<grid, kBwdThreads, BwdCfg<128>::SMEM_BYTES, st>>>(tq, tk, tv, tdo, p);
    prof_end(FA_PROF_BWD_DKDV, st);
    FA_CUDA_TRY(cudaGetLastError());
    count_launch();
    const int64_t n4 = (int64_t)p.B * a->num_heads * p.Sq * (p.d_real / 4);
    auto conv = p.cu_q != nullptr ? fa_bwd_dq_convert_kernel<T, D, true>
                                  : fa_bwd_dq_convert_kernel<T, D, false>;
    conv<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(
        p.dq_acc, reinterpret_cast<T*>(a->dq), p.B, p.Sq, a->num_heads, p.Sq_pad, p.dq_sb,
        p.dq_ss, p.dq_sh, p.d_real, p.cu_q);
    FA_CUDA_TRY(cudaGetLastError());
    count_launch();
  } else if (!a->deterministic) {
    auto kern = fa_bwd_dkdv_kernel<T, D, true, EXT>;
    static std::atomic<bool> attr[kMaxContexts];
    const int slot = call_context_slot();
    if (slot < 0 || slot >= kMaxContexts) return FA_ERR_CUDA;
    if (!attr[slot].load(std::memory_order_acquire)) {
      if (int s = check_reg_split(kern, kBwdThreads, kBwdRegTotal)) return s;
      if (int s = set_smem(kern, BwdCfg<D>::SMEM_BYTES)) return s;
      attr[slot].store(true, std::memory_order_release);
    }
    dim3 grid((p.Skv + kBwdBN - 1) / kBwdBN, a->num_heads_k, p.B);
    prof_begin(FA_PROF_BWD_DKDV, st);
    kern<<<grid, kBwdThreads, BwdCfg<D>::SMEM_BYTES, st>>>(tq, tk, tv, tdo, p);
    prof_end(FA_PROF_BWD_DKDV, st);
    FA_CUDA_TRY(cudaGetLastError());
    count_launch();
    const int64_t n4 = (int64_t)p.B * a->num_heads * p.Sq * (p.d_real / 4);
    auto conv = p.cu_q != nullptr ? fa_bwd_dq_convert_kernel<T, D, true>
                                  : fa_bwd_dq_convert_kernel<T, D, false>;
    conv<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(
        p.dq_acc, reinterpret_cast<T*>(a->dq), p.B, p.Sq, a->num_heads, p.Sq_pad, p.dq_sb,
        p.dq_ss, p.dq_sh, p.d_real, p.cu_q);
    FA_CUDA_TRY(cudaGetLastError());
    count_launch();
  } else {
    auto kern = fa_bwd_dkdv_kernel<T, D, false, EXT>;
    auto kq = fa_bwd_dq_kernel<T, D, EXT>;
    static std::atomic<bool> attr[kMaxContexts];
    const int slot = call_context_slot();
    if (slot < 0 || slot >= kMaxContexts) return FA_ERR_CUDA;
    if (!attr[slot].load(std::memory_order_acquire)) {
      if (int s = check_reg_split(kern, kBwdThreads, kBwdRegTotal)) return s;
      if (int s = set_smem(kern, BwdCfg<D>::SMEM_BYTES)) return s;
      if (int s = set_smem(kq, DqCfg<D>::SMEM_BYTES)) return s;
      attr[slot].store(true, std::memory_order_release);
    }
    dim3 grid((p.Skv + kBwdBN - 1) / kBwdBN, a->num_heads_k, p.B);
    prof_begin(FA_PROF_BWD_DKDV, st);
    kern<<<grid, kBwdThreads, BwdCfg<D>::SMEM_BYTES, st>>>(tq, tk, tv, tdo, p);
    prof_end(FA_PROF_BWD_DKDV, st);
    FA_CUDA_TRY(cudaGetLastError());
    count_launch();
    dim3 gq((p.Sq + kBwdBM - 1) / kBwdBM, a->num_heads, p.B);
    kq<<<gq, 384, DqCfg<D>::SMEM_BYTES, st>>>(tq, tk, tv, tdo, p);
    FA_CUDA_TRY(cudaGetLastError());
    count_launch();
  }
  return FA_OK;
}

static uintptr_t align256(uintptr_t x) { return (x + 255) & ~uintptr_t(255); }

int launch_bwd(const fa_bwd_args_t* a, void* ws, size_t ws_bytes, int* err, cudaStream_t st,
               const BwdVarlen* vl) {
  const int D = bwd_kernel_dim(a->head_dim);
  if (D != 64 && D != 128 && D != 256) return FA_ERR_UNSUPPORTED;
  if (a->batch == 0) return FA_OK;
  if (a->seqlen_q == 0 || a->seqlen_k == 0) {
    // Nothing attends: every gradient is zero (outputs are dense BSHD allocations).
    if (a->seqlen_q > 0)
      FA_CUDA_TRY(cudaMemsetAsync(a->dq, 0, (size_t)a->dq_stride[0] * a->batch * 2, st));
    if (a->seqlen_k > 0) {
      FA_CUDA_TRY(cudaMemsetAsync(a->dk, 0, (size_t)a->dk_stride[0] * a->batch * 2, st));
      FA_CUDA_TRY(cudaMemsetAsync(a->dv, 0, (size_t)a->dv_stride[0] * a->batch * 2, st));
    }
    return FA_OK;
  }
  const void* ptrs[9] = {a->q, a->k, a->v, a->out, a->dout, a->dq, a->dk, a->dv, a->lse};
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) & 15u) return FA_ERR_ALIGNMENT;
  const int64_t* strs[8] = {a->q_stride, a->k_stride, a->v_stride, a->o_stride,
                            a->do_stride, a->dq_stride, a->dk_stride, a->dv_stride};
  for (const int64_t* s : strs)
    for (int i = 0; i < 3; ++i)
      if (s[i] % 8) return FA_ERR_ALIGNMENT;
  const int G = a->num_heads / a->num_heads_k;
  const CUtensorMapDataType dt = tmap_dtype(a->dtype);
  CUtensorMap tq, tk, tv, tdo;
  auto enc = [&](CUtensorMap* m, const void* ptr, const int64_t* s, int heads, int seq) {
    const uint64_t dims[4] = {(uint64_t)a->head_dim, (uint64_t)heads, (uint64_t)(seq > 0 ? seq : 1),
                              (uint64_t)a->batch};
    const uint64_t str[3] = {(uint64_t)s[2] * 2, (uint64_t)s[1] * 2, (uint64_t)s[0] * 2};
    const uint32_t box[4] = {64, 1, 128, 1};
    return encode_tmap(m, dt, 4, ptr, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
  };
  FA_TMAP_TRY(enc(&tq, a->q, a->q_stride, a->num_heads, a->seqlen_q));
  FA_TMAP_TRY(enc(&tdo, a->dout, a->do_stride, a->num_heads, a->seqlen_q));
  FA_TMAP_TRY(enc(&tk, a->k, a->k_stride, a->num_heads_k, a->seqlen_k));
  FA_TMAP_TRY(enc(&tv, a->v, a->v_stride, a->num_heads_k, a->seqlen_k));

  BwdParams p{};
  p.B = vl ? vl->batch : a->batch;
  p.Sq = vl ? vl->max_q : a->seqlen_q;
  p.Skv = vl ? vl->max_k : a->seqlen_k;
  if (vl) {
    p.cu_q = vl->cu_q;
    p.cu_k = vl->cu_k;
  }
  p.H = a->num_heads;
  p.Hk = a->num_heads_k;
  p.G = G;
  p.Sq_pad = pad128(p.Sq);
  p.d_real = a->head_dim;
  p.causal = a->causal;
  p.swq = a->window_q > 0 ? a->window_q : 0;
  p.swk = a->window_k > 0 ? a->window_k : 0;
  p.n_t = (p.Skv + kBwdBN - 1) / kBwdBN;
  p.n_u = a->num_heads_k * p.B;
  p.n_items = p.n_t * p.n_u;
  p.scale = a->softmax_scale;
  p.scale_log2 = a->softmax_scale * 1.4426950408889634f;
  if (a->softcap > 0.f) {
    p.sc_a = a->softcap / a->softmax_scale;
    p.sc_k = 2.f * 1.4426950408889634f / p.sc_a;
    p.sc_ia = a->softmax_scale / a->softcap;
    p.sc_t = 1.f / (1.4426950408889634f * a->softcap);
  }
  const size_t rows = (size_t)p.B * a->num_heads * p.Sq_pad;
  uintptr_t w = align256(reinterpret_cast<uintptr_t>(ws));
  p.lse2 = reinterpret_cast<const float*>(w);
  w = align256(w + rows * 4);
  p.dsum = reinterpret_cast<const float*>(w);
  w = align256(w + rows * 4);
  p.dq_acc = (a->deterministic || D == 256) ? nullptr : reinterpret_cast<float*>(w);
  p.dq = a->dq;
  p.dk = a->dk;
  p.dv = a->dv;
  // varlen: rows are addressed through the packed offsets, so the batch strides drop out
  p.dq_sb = vl ? 0 : a->dq_stride[0];
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
  const bool ext = p.swq > 0 || p.swk > 0 || p.sc_a != 0.f || vl != nullptr;
  if (D == 256) {
    // prep (row dot, LSE * log2 e) here, then the two D = 256 kernels of fa_bwd256.cu
    const int s = bf16 ? launch_bwd_prep<__nv_bfloat16, 256>(a, p, st)
                       : launch_bwd_prep<__half, 256>(a, p, st);
    if (s != FA_OK) return s;
    return launch_bwd_d256(a, p.lse2, p.dsum, p.Sq_pad, err, st, vl);
  }
  if (D == 64)
    return ext ? (bf16 ? launch_bwd_impl<__nv_bfloat16, 64, true>(a, tq, tk, tv, tdo, p, st)
                       : launch_bwd_impl<__half, 64, true>(a, tq, tk, tv, tdo, p, st))
               : (bf16 ? launch_bwd_impl<__nv_bfloat16, 64, false>(a, tq, tk, tv, tdo, p, st)
                       : launch_bwd_impl<__half, 64, false>(a, tq, tk, tv, tdo, p, st));
  return ext ? (bf16 ? launch_bwd_impl<__nv_bfloat16, 128, true>(a, tq, tk, tv, tdo, p, st)
                     : launch_bwd_impl<__half, 128, true>(a, tq, tk, tv, tdo, p, st))
             : (bf16 ? launch_bwd_impl<__nv_bfloat16, 128, false>(a, tq, tk, tv, tdo, p, st)
                     : launch_bwd_impl<__half, 128, false>(a, tq, tk, tv, tdo, p, st));
}

}  // namespace fa

#ifdef FA_TRACE
// Diagnostic build only: copies (and clears) the backward kernel's phase trace.
extern "C" int fa_debug_trace_read(unsigned long long* dst, size_t n) {
  using namespace fa;
  const size_t total = sizeof(g_fa_trace) / sizeof(unsigned long long);
  if (n > total) n = total;
  if (cudaDeviceSynchronize() != cudaSuccess) return FA_ERR_CUDA;
  if (cudaMemcpyFromSymbol(dst, g_fa_trace, n * sizeof(unsigned long long)) != cudaSuccess)
    return FA_ERR_CUDA;
  static unsigned long long zeros[FA_TRACE_CTAS * FA_TRACE_EVENTS * FA_TRACE_ITERS];
  if (cudaMemcpyToSymbol(g_fa_trace, zeros, sizeof(zeros)) != cudaSuccess) return FA_ERR_CUDA;
  return FA_OK;
}
#endif
