// Paged prefill at head_dim 512 on sm_100a: tilelang_paged_forward with D = 512, the
// reference's tuned entry _BEST_CONFIGS[512] (_kernels_paged.py:357-363) over its generic
// paged kernel (_kernels_paged.py:193-344).  Same masks, LSE and output layout as the
// D <= 256 paged kernels in fa_fwd.cu.
//
// At D = 512 one Q tile's fp32 output (128 rows x 512 columns) fills all of tensor
// memory and leaves no column for S.  A work item therefore produces HALF of the output
// columns: CTA = (q block of one sequence, kv head, output half h).  Both halves compute
// the same S = Q K^T over all 512 dims and the same softmax, and each accumulates
// O_h = P V[:, 256 h .. 256 h + 255].  That repeats S once per q block (1.5x the
// attention's MMA work) and in exchange S is double buffered next to O_h:
//   TMEM (512 columns): S_0 [0, 128) | S_1 [128, 256) | O_h [256, 512), fp32; P_j is
//   packed as 16-bit pairs onto the first 64 columns of its S buffer.
// The MMA issuer runs S_{j+1} into the other buffer while the softmax works on S_j, so
// the tensor pipe alternates PV_{j-1} and S_{j+1} without waiting for the softmax.
//
// Shared memory: Q (rows x 512 dims as eight 128-byte-swizzled 64-dim chunks, 128 KB,
// resident) and a ring of 3 slots of 32 KB; a slot holds 128 keys x 128 dims (two 64-dim
// chunks).  A KV tile is 4 K slots (dims 0..511) and 2 V slots (this half's 256 dims),
// loaded in the order the MMAs read them: K_0, K_1, V_0, K_2, V_1, ..., V_{n-1}.
//
// Roles (192 threads):
//   warp 0     TMA producer (lane r issues page box r of every slot, as in fa_fwd.cu)
//   warp 1     TMEM allocator + single-thread MMA issuer
//   warps 2-5  softmax and epilogue, thread = row; warp w reads TMEM lanes 32 (w % 4)..
// Rows pack the G = H / Hkv query heads of the kv head (row = token_local * G + head), so
// each K/V byte loaded serves the whole group.
#include "fa_ptx.cuh"
#include "fa_internal.h"
#include <atomic>
#include <cmath>

namespace fa {

namespace {

constexpr int kP5D = 512;            // head dim
constexpr int kP5DH = 256;           // output columns per work item
constexpr int kP5BN = 128;           // keys per KV tile
constexpr int kP5Chunk = 128 * 128;  // 128 rows x 64 dims, 16-bit, 128-byte swizzled
constexpr int kP5Slot = 2 * kP5Chunk;  // 128 keys x 128 dims
constexpr int kP5Stages = 3;
constexpr int kP5Threads = 192;
constexpr int kP5SmemQ = 8 * kP5Chunk;
constexpr int kP5SmemBytes = 1024 + kP5SmemQ + kP5Stages * kP5Slot + 1024;
static_assert(kP5SmemBytes <= 232448, "D = 512 paged prefill: shared memory budget");
static_assert(2 * 128 + kP5DH <= 512, "D = 512 paged prefill: TMEM budget");

struct P5Ctl {
  uint64_t q_full;
  uint64_t kv_full[kP5Stages];
  uint64_t kv_empty[kP5Stages];
  uint64_t s_full[2];
  uint64_t p_ready[2];
  uint64_t pv_done;   // one phase per PV_j
  uint64_t o_staged;  // output half staged in the Q buffer (TMA store may start)
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int b, tok0, q_len, kv_len, off, tok_base, j0, nkv, valid;
};

// Final, abort-insensitive bounded wait used while draining in-flight copies.
__device__ __forceinline__ void p5_wait_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > 200000000ull) return;
  }
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kP5Threads, 1)
    fa_paged512_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_o, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const uint32_t sQ = base;
  const uint32_t sRing = base + kP5SmemQ;
  P5Ctl* ctl = reinterpret_cast<P5Ctl*>(base_ptr + kP5SmemQ + kP5Stages * kP5Slot);
  volatile int* abort_flag = &ctl->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.G;
  const int TPT = 128 / G;  // tokens per Q tile (rows TPT * G .. 127 unused when G does not divide 128)
  const int hk = blockIdx.y;
  // The two output halves of a q block are adjacent in launch order (blockIdx.x & 1), so
  // the second one reads Q and the K/V pages from L2.
  const int half = blockIdx.x & 1;  // output columns [256 half, 256 half + 256)
  const int qblk = blockIdx.x >> 1;

  // ---------------------------------------------------------------- work item
  if (threadIdx.x == 0) {
    // blockIdx.x -> (sequence, q block) by a running count of q blocks per sequence
    int b = 0, tile = 0, valid = 0;
    for (int s = 0, cum = 0; s < p.num_seqs; ++s) {
      const int ql = p.qsl[s + 1] - p.qsl[s];
      const int nb = ql > 0 ? (ql + TPT - 1) / TPT : 0;
      if (qblk < cum + nb) {
        b = s;
        tile = qblk - cum;
        valid = 1;
        break;
      }
      cum += nb;
    }
    const int tok0 = tile * TPT;
    int q_len = 0, kv_len = 0, off = 0, tok_base = 0, j0 = 0, j1 = 0;
    if (valid) {
      q_len = p.qsl[b + 1] - p.qsl[b];
      kv_len = clamp_seq_len(p.seq_lens[b], p.max_blocks, p.page_size, p.err,
                             FA_SITE_PAGED_SEQLEN, true);
      off = p.pkl[b];
      tok_base = p.qsl[b];
      fwd_kv_range<true>(p, tok0, TPT, q_len, kv_len, off, j0, j1);
    }
    ctl->b = b;
    ctl->tok0 = tok0;
    ctl->q_len = q_len;
    ctl->kv_len = kv_len;
    ctl->off = off;
    ctl->tok_base = tok_base;
    ctl->j0 = j0;
    ctl->nkv = valid ? max(0, j1 - j0) : 0;
    ctl->valid = valid;
    ctl->abort_flag = 0;
    mbar_init(smem_u32(&ctl->q_full), 1);
    for (int s = 0; s < kP5Stages; ++s) {
      mbar_init(smem_u32(&ctl->kv_full[s]), 1);
      mbar_init(smem_u32(&ctl->kv_empty[s]), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&ctl->s_full[t]), 1);
      mbar_init(smem_u32(&ctl->p_ready[t]), 128);
    }
    mbar_init(smem_u32(&ctl->pv_done), 1);
    mbar_init(smem_u32(&ctl->o_staged), 128);
    mbar_init(smem_u32(&ctl->drain), 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (!ctl->valid) return;  // uniform: no TMEM held, no copies issued

  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const int b = ctl->b, tok0 = ctl->tok0, q_len = ctl->q_len, kv_len = ctl->kv_len;
  const int off = ctl->off, tok_base = ctl->tok_base, j0 = ctl->j0, nkv = ctl->nkv;

  if (warp == 0) {
    // ============================================================ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const uint32_t qbar = smem_u32(&ctl->q_full);
      mbar_arrive_expect_tx(qbar, 8 * TPT * G * 128);
      for (int dh = 0; dh < 8; ++dh)
        tma_load_4d(sQ + dh * kP5Chunk, &tm_q, qbar, dh * 64, hk * G, tok_base + tok0, 0);
    }
    const int box_rows = min(p.page_size, kP5BN);
    const int boxes = kP5BN / box_rows;  // page boxes per slot (<= 16: page_size >= 8)
    const int n_valid_pages = min((kv_len + p.page_size - 1) / p.page_size, p.max_blocks);
    // Page id of box `lane` of KV tile j; pages past the sequence are fetched out of range
    // (page id num_pages), which TMA fills with zeros.
    auto page_of = [&](int j) -> int {
      int pg = p.num_pages;
      if (lane < boxes) {
        const int lp = (j * kP5BN + lane * box_rows) / p.page_size;
        if (lp < n_valid_pages) pg = p.block_table[(int64_t)b * p.max_blocks + lp];
      }
      return pg;
    };
    int it = 0;
    // One slot: 128 keys of tile j x dims [dim0, dim0 + 128) of the tensor map.
    auto load_slot = [&](int j, int pg, const CUtensorMap* tm, int dim0) -> bool {
      const int s = it % kP5Stages;
      int okl = 1;
      if (lane == 0)
        okl = mbar_wait(smem_u32(&ctl->kv_empty[s]), ((it / kP5Stages) & 1) ^ 1, abort_flag,
                        p.err, FA_SITE_FWD_PRODUCER);
      if (__shfl_sync(0xffffffffu, okl, 0) == 0) return false;
      const uint32_t fb = smem_u32(&ctl->kv_full[s]);
      if (lane == 0) mbar_arrive_expect_tx(fb, kP5Slot);
      __syncwarp();
      if (lane < boxes) {
        const int in_page = (j * kP5BN + lane * box_rows) % p.page_size;
        const uint32_t dst = sRing + s * kP5Slot + lane * box_rows * 128;
        tma_load_4d(dst, tm, fb, dim0, hk, in_page, pg);
        tma_load_4d(dst + kP5Chunk, tm, fb, dim0 + 64, hk, in_page, pg);
      }
      ++it;
      return true;
    };
    bool ok = true;
    if (nkv > 0) {
      // MMA order: K_0; then per tile j: K_{j+1} (S_{j+1} runs ahead), V_j (this half)
      int pg_cur = page_of(j0);
      for (int c = 0; c < 4 && ok; ++c) ok = load_slot(j0, pg_cur, &tm_k, 128 * c);
      for (int jj = 0; jj < nkv && ok; ++jj) {
        const int j = j0 + jj;
        int pg_nxt = pg_cur;
        if (jj + 1 < nkv) {
          pg_nxt = page_of(j + 1);
          for (int c = 0; c < 4 && ok; ++c) ok = load_slot(j + 1, pg_nxt, &tm_k, 128 * c);
        }
        for (int c = 0; c < 2 && ok; ++c) ok = load_slot(j, pg_cur, &tm_v, kP5DH * half + 128 * c);
        pg_cur = pg_nxt;
      }
    }
    // Drain: every copy issued must have landed before the CTA may exit.
    if (lane == 0) {
      for (int k = max(0, it - kP5Stages); k < it; ++k)
        p5_wait_drain(smem_u32(&ctl->kv_full[k % kP5Stages]), (k / kP5Stages) & 1);
      p5_wait_drain(smem_u32(&ctl->q_full), 0);
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      constexpr bool kBf16 = Pack2<T>::kBf16;
      constexpr uint32_t idS = idesc_f16(128, kP5BN, kBf16, false, false);
      constexpr uint32_t idPV = idesc_f16(128, 128, kBf16, false, true);
      bool ok = mbar_wait(smem_u32(&ctl->q_full), 0, abort_flag, p.err, FA_SITE_FWD_MMA);
      tc_fence_after();
      const uint64_t q_desc0 = sdesc_sw128(sQ, 16, 1024);             // K-major Q chunks
      const uint64_t k_desc0 = sdesc_sw128(sRing, 16, 1024);          // K-major K, slot 0
      const uint64_t v_desc0 = sdesc_sw128(sRing, kP5Chunk, 1024);    // MN-major V, slot 0
      int it = 0;
      auto wait_slot = [&](int& s) -> bool {
        s = it % kP5Stages;
        const bool w = mbar_wait(smem_u32(&ctl->kv_full[s]), (it / kP5Stages) & 1, abort_flag,
                                 p.err, FA_SITE_FWD_MMA);
        tc_fence_after();
        return w;
      };
      // S_buf = Q K_j^T: four slots of 128 dims, 8 steps of 16 each (K-major, 128-byte
      // swizzle: step = +32 B inside a 64-dim chunk, next chunk at +16 KB).
      auto issue_S = [&](int buf) -> bool {
        for (int c = 0; c < 4; ++c) {
          int s;
          if (!wait_slot(s)) return false;
          const uint64_t qa = desc_add(opaque(q_desc0), 2 * c * kP5Chunk);
          const uint64_t ka = desc_add(opaque(k_desc0), s * kP5Slot);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t o = (kk >> 2) * kP5Chunk + (kk & 3) * 32;
            mma_ss(tmem + buf * 128, desc_add(qa, o), desc_add(ka, o), idS, (c | kk) ? 1u : 0u);
          }
          mma_commit(smem_u32(&ctl->kv_empty[s]));
          ++it;
        }
        mma_commit(smem_u32(&ctl->s_full[buf]));
        return true;
      };
      // O_h[:, 128 c ..] += P_buf V_j: two slots of 128 output columns, 8 steps of 16 keys
      // (V MN-major: step = 16 rows = +2 KB; P's 16-bit pairs: 16 keys = 8 TMEM columns).
      auto issue_PV = [&](int buf, bool acc) -> bool {
        for (int c = 0; c < 2; ++c) {
          int s;
          if (!wait_slot(s)) return false;
          const uint64_t va = desc_add(opaque(v_desc0), s * kP5Slot);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ts(tmem + 256 + 128 * c, tmem + buf * 128 + kk * 8, desc_add(va, kk * 2048), idPV,
                   (acc || kk > 0) ? 1u : 0u);
          mma_commit(smem_u32(&ctl->kv_empty[s]));
          ++it;
        }
        mma_commit(smem_u32(&ctl->pv_done));
        return true;
      };
      // S_{j+1} goes into the other buffer ahead of PV_j; the buffer it overwrites held
      // P_{j-1}, whose PV was issued before it (tcgen05 MMAs of one thread run in order).
      if (ok && nkv > 0) ok = issue_S(0);
      for (int jj = 0; jj < nkv && ok; ++jj) {
        if (jj + 1 < nkv && !(ok = issue_S((jj + 1) & 1))) break;
        ok = mbar_wait(smem_u32(&ctl->p_ready[jj & 1]), (jj >> 1) & 1, abort_flag, p.err,
                       FA_SITE_FWD_MMA);
        if (!ok) break;
        tc_fence_after();
        ok = issue_PV(jj & 1, jj > 0);
      }
      mma_commit(smem_u32(&ctl->drain));
      p5_wait_drain(smem_u32(&ctl->drain), 0);
    }
  } else {
    // ============================================================ softmax / epilogue
    const int q4 = warp & 3;  // TMEM lane quarter of this warp
    const int r = (q4 << 5) | lane;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    const uint32_t tO = tmem + lane_off + 256;
    const int tr = r / G;                 // token of this row inside the tile
    const int lt = tok0 + tr;             // token index within the sequence's query chunk
    const int h = hk * G + (r - tr * G);  // query head
    const bool row_valid = tr < TPT && lt < q_len;
    const int limit = lt + off;           // causal: key <= limit
    const bool window = fwd_window_on<true>(p);
    const float c2 = p.scale_log2;
    const float NEG_INF = -INFINITY;
    float m_run = NEG_INF, m_ref = NEG_INF, l = 0.f;
    bool ok = true;
    for (int jj = 0; jj < nkv; ++jj) {
      const int buf = jj & 1;
      const uint32_t tS = tmem + lane_off + buf * 128;
      bool w = mbar_wait(smem_u32(&ctl->s_full[buf]), (jj >> 1) & 1, abort_flag, p.err,
                         FA_SITE_FWD_SOFTMAX);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      tc_fence_after();
      uint32_t s[128];
      tmem_ld32(tS + 0, s);
      tmem_ld32(tS + 32, s + 32);
      tmem_ld32(tS + 64, s + 64);
      tmem_ld32(tS + 96, s + 96);
      tmem_wait_ld();
      // Paged visibility (_kernels_paged.py:275-303): key < seq_len; causal key <= prefix +
      // token; sliding window anchored on the token (only with causal).
      const int key0 = (j0 + jj) * kP5BN;
      const bool need_mask =
          (key0 + kP5BN > kv_len) || (p.causal && (key0 + kP5BN - 1 > limit)) || window;
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const int key = key0 + c;
          bool vis = key < kv_len;
          if (p.causal) vis = vis && key <= limit;
          if (window) {
            if (p.swq > 0) vis = vis && (lt < key + p.swq);
            if (p.swk > 0) vis = vis && (key < lt + p.swk);
          }
          if (!vis) s[c] = __float_as_uint(NEG_INF);
        }
      }
      float mx4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        mx4[u] = fmax3(__uint_as_float(s[u]), __uint_as_float(s[u + 4]), __uint_as_float(s[u + 8]));
#pragma unroll
      for (int c = 12; c < 124; c += 8)
#pragma unroll
        for (int u = 0; u < 4; ++u)
          mx4[u] = fmax3(mx4[u], __uint_as_float(s[c + u]), __uint_as_float(s[c + 4 + u]));
#pragma unroll
      for (int u = 0; u < 4; ++u) mx4[u] = fmaxf(mx4[u], __uint_as_float(s[124 + u]));
      const float m_new = fmaxf(m_run, fmaxf(fmax3(mx4[0], mx4[1], mx4[2]), mx4[3]));
      m_run = m_new;
      // Lazy rescale: the reference max moves only when the running max exceeds it by
      // more than 8 (log2 units), as in fa_fwd.cu.
      bool rescale_o = false;
      float factor = 1.f;
      if (jj == 0) {
        m_ref = m_new;
      } else {
        const bool need = (m_new - m_ref) * c2 > 8.0f;
        if (__any_sync(0xffffffffu, need)) {
          if (m_new != NEG_INF) {
            factor = ex2_approx((m_ref - m_new) * c2);
            m_ref = m_new;
          }
          l *= factor;
          rescale_o = true;
        }
      }
      const float mref_s = (m_ref == NEG_INF) ? 0.f : m_ref * c2;
      float rs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      // P_j onto the first 64 columns of its S buffer (S_j is in registers; PV_{j-2}, the
      // last reader of these columns, finished before S_j was written).
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t pk[32];
#pragma unroll
        for (int cc = 0; cc < 32; ++cc) {
          const int c = 32 * hf + cc;
          const float p0 = ex2_approx(fmaf(__uint_as_float(s[2 * c]), c2, -mref_s));
          const float p1 = ex2_approx(fmaf(__uint_as_float(s[2 * c + 1]), c2, -mref_s));
          rs[c & 7] += p0 + p1;
          pk[cc] = Pack2<T>::pack(p0, p1);
        }
        tmem_st32(tS + 32 * hf, pk);
      }
      l += ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
      if (jj > 0) {
        // PV_{j-1} (one pv_done phase per tile, consumed in order) has accumulated into O:
        // only then may O be rescaled for tile j.
        w = mbar_wait(smem_u32(&ctl->pv_done), (jj - 1) & 1, abort_flag, p.err,
                      FA_SITE_FWD_SOFTMAX);
        ok = __all_sync(0xffffffffu, w);
        if (!ok) break;
        if (rescale_o) {
          tc_fence_after();
#pragma unroll 1
          for (int c0 = 0; c0 < kP5DH; c0 += 32) {
            uint32_t o[32];
            tmem_ld32(tO + c0, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * factor);
            tmem_st32(tO + c0, o);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl->p_ready[buf]));
    }

    // ---------------------------------------------------------- epilogue
    if (ok && nkv > 0) {
      const bool w = mbar_wait(smem_u32(&ctl->pv_done), (nkv - 1) & 1, abort_flag, p.err,
                               FA_SITE_FWD_SOFTMAX);
      ok = __all_sync(0xffffffffu, w);
    }
    if (ok) {
      tc_fence_after();
      const bool have = l > 0.f;
      const float inv = have ? 1.f / l : 0.f;
      // The output half goes through the Q buffer (every S MMA that read it finished before
      // the last PV) and four TMA stores of 64 columns when all the tile's tokens belong to
      // this sequence; otherwise per-row stores (the next rows are another sequence's).
      const bool tma_out = tok0 + TPT <= q_len;
      T* orow = reinterpret_cast<T*>(p.out) + (int64_t)(tok_base + lt) * p.o_st +
                (int64_t)h * p.o_sh + kP5DH * half;
#pragma unroll 1
      for (int c0 = 0; c0 < kP5DH; c0 += 32) {
        uint32_t o[32];
        if (nkv > 0) {
          tmem_ld32(tO + c0, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = 0u;
        }
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c)
          pk[c] = Pack2<T>::pack(have ? __uint_as_float(o[2 * c]) * inv : 0.f,
                                 have ? __uint_as_float(o[2 * c + 1]) * inv : 0.f);
        if (tma_out) {
          // row r of the 128-byte-swizzled 64-column chunk c0 / 64, 16-byte units
          // (c0 % 64) / 8 .. + 3
          const uint32_t rowa = sQ + (c0 >> 6) * kP5Chunk + r * 128;
          const int u0 = (c0 & 63) >> 3;
#pragma unroll
          for (int m = 0; m < 4; ++m)
            st_shared_v4(rowa + (((u0 + m) ^ (r & 7)) << 4), pk[4 * m], pk[4 * m + 1],
                         pk[4 * m + 2], pk[4 * m + 3]);
        } else if (row_valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c0);
          dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          dst[2] = make_uint4(pk[8], pk[9], pk[10], pk[11]);
          dst[3] = make_uint4(pk[12], pk[13], pk[14], pk[15]);
        }
      }
      if (row_valid && half == 0 && p.lse != nullptr)
        p.lse[(int64_t)h * p.lse_sh + tok_base + lt] = have ? m_ref * p.scale + logf(l) : NEG_INF;
      if (tma_out) {
        fence_async_shared();
        mbar_arrive(smem_u32(&ctl->o_staged));
        if ((threadIdx.x & 127) == 0 &&
            mbar_wait(smem_u32(&ctl->o_staged), 0, abort_flag, p.err, FA_SITE_FWD_SOFTMAX)) {
#pragma unroll
          for (int dh = 0; dh < kP5DH / 64; ++dh)
            tma_store_4d(&tm_o, sQ + dh * kP5Chunk, kP5DH * half + 64 * dh, hk * G,
                         tok_base + tok0, 0);
          bulk_commit_group();
          bulk_wait_group_read();
        }
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
template <typename T>
static int launch_p5(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                     const CUtensorMap& to, const FwdParams& p, int grid_x, cudaStream_t st) {
  auto kern = fa_paged512_kernel<T>;
  static std::atomic<bool> attr[kMaxContexts];
  if (int s = smem_attr_once(kern, kP5SmemBytes, attr)) return s;
  const dim3 grid(2 * grid_x, p.Hk);
  prof_begin(FA_PROF_PAGED, st);
  kern<<<grid, kP5Threads, kP5SmemBytes, st>>>(tq, tk, tv, to, p);
  prof_end(FA_PROF_PAGED, st);
  FA_CUDA_TRY(cudaGetLastError());
  count_launch();
  return FA_OK;
}

// Called by launch_paged_prefill after its checks (G <= 128, page size a power of two
// >= 8, 16-byte aligned pointers, tokens and sequences present).
int launch_paged512(const fa_paged_args_t* a, int* err, cudaStream_t st) {
  const int G = a->num_heads / a->num_kv_heads;
  const int ps = a->page_size;
  const CUtensorMapDataType dt = tmap_dtype(a->dtype);
  CUtensorMap tq, tk, tv, to;
  {
    const uint64_t dims[4] = {(uint64_t)kP5D, (uint64_t)a->num_heads, (uint64_t)a->num_tokens, 1};
    const uint64_t str[3] = {(uint64_t)kP5D * 2, (uint64_t)a->num_heads * kP5D * 2,
                             (uint64_t)a->num_tokens * a->num_heads * kP5D * 2};
    const uint32_t box[4] = {64, (uint32_t)G, (uint32_t)(128 / G), 1};  // TPT tokens x G heads
    FA_TMAP_TRY(encode_tmap(&tq, dt, 4, a->q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
    FA_TMAP_TRY(encode_tmap(&to, dt, 4, a->out, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  const void* kv_ptr[2] = {a->k_cache, a->v_cache};
  CUtensorMap* kv_map[2] = {&tk, &tv};
  for (int w = 0; w < 2; ++w) {
    const uint64_t dims[4] = {(uint64_t)kP5D, (uint64_t)a->num_kv_heads, (uint64_t)ps,
                              (uint64_t)a->num_pages};
    const uint64_t str[3] = {(uint64_t)kP5D * 2, (uint64_t)a->num_kv_heads * kP5D * 2,
                             (uint64_t)ps * a->num_kv_heads * kP5D * 2};
    const uint32_t box[4] = {64, 1, (uint32_t)(ps < kP5BN ? ps : kP5BN), 1};
    FA_TMAP_TRY(encode_tmap(kv_map[w], dt, 4, kv_ptr[w], dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  FwdParams p{};
  p.H = a->num_heads;
  p.Hk = a->num_kv_heads;
  p.G = G;
  p.causal = a->causal;
  p.scale = a->softmax_scale;
  p.scale_log2 = a->softmax_scale * 1.4426950408889634f;
  p.out = a->out;
  p.lse = a->lse;
  p.o_st = (int64_t)a->num_heads * kP5D;
  p.o_sh = kP5D;
  p.lse_sh = a->num_tokens;
  p.block_table = a->block_table;
  p.seq_lens = a->seq_lens;
  p.qsl = a->query_start_loc;
  p.pkl = a->prefix_kv_lens;
  p.num_seqs = a->num_seqs;
  p.max_blocks = a->max_blocks;
  p.page_size = ps;
  p.num_pages = a->num_pages;
  p.swq = a->causal ? a->sliding_window_q : 0;
  p.swk = a->causal ? a->sliding_window_k : 0;
  p.err = err;
  // Sum over sequences of ceil(q_len / TPT) <= num_tokens / TPT + num_seqs.
  const int grid_x = a->num_tokens / (128 / G) + a->num_seqs;
  return a->dtype == FA_DTYPE_BF16 ? launch_p5<__nv_bfloat16>(tq, tk, tv, to, p, grid_x, st)
                                   : launch_p5<__half>(tq, tk, tv, to, p, grid_x, st);
}

}  // namespace fa
