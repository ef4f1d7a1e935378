// Attention forward on sm_100a: tcgen05 MMAs with S, P and O in tensor memory,
// TMA-fed K/V ring, warp-specialised roles, for the dense BSHD path
// (tilelang_flash_attn_func, reference kernel _kernels_forward.py:94-172) and the paged
// vLLM-cache path (tilelang_paged_forward, reference kernel _kernels_paged.py:193-344).
// Two schedules of the same per-item pipeline, chosen per launch (fwd_persistent):
//   fa_fwd_kernel          one CTA per work item (dense D = 256 non-causal with long items)
//   fa_fwd_persist_kernel  one CTA per SM claiming work items in the same order, the
//                          next item's Q load and first S overlapping the current
//                          item's tail (paged prefill, dense D = 64 and 128, short dense
//                          items, dense D = 256 causal)
//
// CTA work item: NQ Q tiles of 128 rows for one kv head.  A row is a (token, head)
// pair: the G = H / Hk query heads that share a kv head are packed into the rows
// of a tile (row = token_local * G + head_in_group), so every K/V tile that is
// loaded serves all of them (GQA/MQA; G = 1 for plain MHA).
//
// Roles (128 + 128 * NQ threads):
//   warp 0      TMA producer: Q tiles once, then K_j, V_j into a STAGES-slot ring
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warps 2-3   idle
//   warpgroup t softmax + O correction + epilogue of Q tile t (thread = row)
// TMEM (512 columns): S_t at [t*128, t*128+128) fp32, P_t aliased onto the first
// 64 columns of S_t as packed 16-bit pairs, O_t at [NQ*128 + t*D, ... + D) fp32.
// Per KV tile j and Q tile t:  S_t = Q_t K_j^T (SS, K-major both), softmax writes
// P_t, O_t += P_t V_j (TS: A = P from TMEM, B = V MN-major).  tcgen05 MMAs issued
// by one thread execute in issue order, so S_{j+1} may be issued right behind the
// PV_j that reads P from the same columns.
//
// Online softmax (reference: _kernels_forward.py:147-165): running max m, row sum
// l, p = 2^((s - m_ref) * scale * log2 e) computed with ex2; the O rescale is lazy:
// the reference max m_ref only moves when the running max exceeds it by more than
// 8 (log2 units), so O and l are rescaled rarely and p <= 256.  Final
// O = acc / l, LSE = m_ref * scale + ln(l) (natural log, as _kernels_forward.py:170).
#include "fa_ptx.cuh"
#include "fa_internal.h"
#include <atomic>
#include <cmath>

namespace fa {

constexpr int kFwdBM = 128;  // rows per Q tile = TMEM lanes
constexpr int kFwdOrderGroup = 8;  // (batch, kv head) units ordered together (dense)
// Two-tile CTAs (384 threads, 168 registers a thread at launch): the producer / MMA
// warpgroup drops to 56 registers and the two softmax warpgroups rise to 224, enough for
// a row's 128 S values at once.  The issuer's descriptors are laundered per use (opaque)
// so the MMA warp fits 56; ptxas reports no spills at these values.
constexpr int kFwdRegLow = 56;
constexpr int kFwdRegHigh = 224;
static_assert(128 * kFwdRegLow + 256 * kFwdRegHigh <= 384 * 168,
              "forward register split exceeds the launch");

// Dense work order over n_t q blocks x n_u (batch, kv head) units: linear index L walks
// groups of kFwdOrderGroup units and, inside a group, the q block ranks across all its
// units (causal: rank 0 = the heaviest block), so the last work to start is light; a
// group's units run together and share their K/V in L2.  Returns the q block rank x and
// the unit.
__device__ __forceinline__ void fwd_dense_order(int L, int n_t, int n_u, int& x, int& unit) {
  const int gsz = min(kFwdOrderGroup, n_u);
  const int grp = L / (gsz * n_t), within = L % (gsz * n_t);
  const int gbase = grp * gsz, gcount = min(gsz, n_u - gbase);
  x = within / gcount;
  unit = gbase + within % gcount;
}

// FA2 softcap (dense launches only; the paged API has none): each score becomes
// softcap_score(s) before the mask, the row max and the exponentials, so the running max,
// the rescale test and LSE = m * scale + ln l all work on the capped scores.  Only the
// persistent kernel has it, as its CAP variant: launches without a softcap run kernels
// without the code (as a runtime branch it cost those launches 4-12 %).
// Caps n consecutive scores held as raw bits in v.
template <int N>
__device__ __forceinline__ void fwd_softcap(uint32_t* v, const FwdParams& p) {
  const float a = p.sc_a, k = p.sc_k;
#pragma unroll
  for (int c = 0; c < N; ++c) v[c] = __float_as_uint(softcap_score(__uint_as_float(v[c]), a, k));
}
template <int D, int NQ>
struct FwdCfg {
  static constexpr int DH = D / 64;                       // 128-byte column chunks
  static constexpr int TILE_BYTES = 128 * D * 2;          // one Q, K or V tile
  static constexpr int CHUNK_BYTES = 128 * 128;           // one 64-column chunk of a tile
  static constexpr int STAGES = (D == 64) ? 6 : (D == 128 ? 5 : 2);
  static constexpr int NTHREADS = 128 + 128 * NQ;
  static constexpr int TMEM_COLS = 512;
  static_assert(NQ * (128 + D) <= TMEM_COLS, "TMEM budget: S + O per Q tile");
  static constexpr int SMEM_Q = NQ * TILE_BYTES;
  static constexpr int SMEM_KV = STAGES * TILE_BYTES;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + SMEM_Q + SMEM_KV + 1024 /*barriers*/;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget (227 KB per CTA)");
};

struct FwdSmemCtl {
  uint64_t q_full;
  uint64_t kv_full[8];
  uint64_t kv_empty[8];
  uint64_t s_full[2];
  uint64_t p_half[2];   // first 64 keys of P_t in TMEM (PV over them may start)
  uint64_t p_ready[2];  // all of P_t in TMEM
  uint64_t o_final[2];
  uint64_t exp_turn[2];  // softmax ping-pong: warpgroup t may run its exp phase
  uint64_t o_staged[2];  // output tile t written to shared memory (TMA store may start)
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  // work item
  int b, tok0, q_len, kv_len, off, tok_base, j0, nkv, valid;
};

// Final, abort-insensitive bounded wait used while draining in-flight copies.
__device__ __forceinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > 200000000ull) return;
  }
}

template <typename T, int D, int NQ, bool PAGED>
__global__ void __launch_bounds__(FwdCfg<D, NQ>::NTHREADS, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                  const FwdParams p) {
  using Cfg = FwdCfg<D, NQ>;
  constexpr int ST = Cfg::STAGES;
  // Release P_t in two halves (PV over the first 64 keys overlaps the second half's
  // exponentials).  Measured faster for dense D >= 128; for D = 64 (cheap PV) and the
  // paged path the extra barrier costs more than the overlap gains.
  constexpr bool kSplitP = (D >= 128) && !PAGED;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const uint32_t sQ = base;
  const uint32_t sKV = base + Cfg::SMEM_Q;
  FwdSmemCtl* ctl = reinterpret_cast<FwdSmemCtl*>(base_ptr + Cfg::SMEM_Q + Cfg::SMEM_KV);
  volatile int* abort_flag = &ctl->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.G;
  const int TPT = kFwdBM / G;       // tokens per Q tile (rows TPT*G .. 127 unused when G does not divide 128)
  const int TPB = NQ * TPT;         // tokens per CTA block
  // Dense: grouped order (fwd_dense_order); paged: blockIdx.x is the sequence block.
  int hk = blockIdx.y, dense_b = blockIdx.z, dense_x = blockIdx.x;
  if constexpr (!PAGED) {
    int unit;
    fwd_dense_order(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z), gridDim.x,
                     gridDim.y * gridDim.z, dense_x, unit);
    hk = unit % gridDim.y;
    dense_b = unit / gridDim.y;
  }

  // ---------------------------------------------------------------- work item
  if (threadIdx.x == 0) {
    int b = 0, tile = 0, valid = 1, q_len, kv_len, off, tok_base;
    if constexpr (PAGED) {
      // Map blockIdx.x onto (sequence, q block) by a running count of blocks per sequence.
      int t = blockIdx.x, cum = 0;
      valid = 0;
      for (int s = 0; s < p.num_seqs; ++s) {
        const int ql = p.qsl[s + 1] - p.qsl[s];
        const int nb = ql > 0 ? (ql + TPB - 1) / TPB : 0;
        if (t < cum + nb) {
          b = s;
          tile = t - cum;
          valid = 1;
          break;
        }
        cum += nb;
      }
      if (valid) {
        q_len = p.qsl[b + 1] - p.qsl[b];
        kv_len = clamp_seq_len(p.seq_lens[b], p.max_blocks, p.page_size, p.err,
                               FA_SITE_PAGED_SEQLEN, true);
        off = p.pkl[b];
        tok_base = p.qsl[b];
      } else {
        q_len = kv_len = off = tok_base = 0;
      }
    } else {
      b = dense_b;
      tile = p.causal ? (gridDim.x - 1 - dense_x) : dense_x;  // heaviest blocks first
      q_len = p.Sq;
      kv_len = p.Skv;
      off = p.Skv - p.Sq;
      tok_base = 0;
    }
    const int tok0 = tile * TPB;
    int j0 = 0, j1 = 0;
    if (valid) fwd_kv_range<PAGED>(p, tok0, TPB, q_len, kv_len, off, j0, j1);
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
    for (int s = 0; s < ST; ++s) {
      mbar_init(smem_u32(&ctl->kv_full[s]), 1);
      mbar_init(smem_u32(&ctl->kv_empty[s]), 1);
    }
    for (int t = 0; t < NQ; ++t) {
      mbar_init(smem_u32(&ctl->s_full[t]), 1);
      mbar_init(smem_u32(&ctl->p_half[t]), 128);
      mbar_init(smem_u32(&ctl->p_ready[t]), 128);
      mbar_init(smem_u32(&ctl->o_final[t]), 1);
      mbar_init(smem_u32(&ctl->exp_turn[t]), 128);
      mbar_init(smem_u32(&ctl->o_staged[t]), 128);
    }
    mbar_init(smem_u32(&ctl->drain), 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (!ctl->valid) return;  // uniform: no TMEM held, no copies issued

  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl->tmem_base), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  const int b = ctl->b, tok0 = ctl->tok0, q_len = ctl->q_len, kv_len = ctl->kv_len;
  const int off = ctl->off, tok_base = ctl->tok_base, j0 = ctl->j0, nkv = ctl->nkv;

  if (warp < 4) {
    if (NQ == 2) setmaxnreg_dec<kFwdRegLow>();
  if (warp == 0) {
    // ============================================================ TMA producer
    // Dense: lane 0 issues every copy.  Paged: lane r fetches the page id of box r of the
    // next KV tile while the current tile's copies go out, and issues box r's copies
    // itself, so block-table reads never sit between two copies.
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const uint32_t qbar = smem_u32(&ctl->q_full);
      mbar_arrive_expect_tx(qbar, NQ * Cfg::DH * TPT * G * 128);
      for (int t = 0; t < NQ; ++t) {
        const int tok = tok_base + tok0 + t * TPT;
        for (int dh = 0; dh < Cfg::DH; ++dh)
          tma_load_4d(sQ + t * Cfg::TILE_BYTES + dh * Cfg::CHUNK_BYTES, &tm_q, qbar, dh * 64,
                      hk * G, tok, PAGED ? 0 : b);
      }
    }
    const int box_rows = PAGED ? min(p.page_size, kFwdBN) : kFwdBN;
    const int boxes = kFwdBN / box_rows;  // page boxes per KV tile (<= 16: page_size >= 8)
    const int n_valid_pages =
        PAGED ? min((kv_len + p.page_size - 1) / p.page_size, p.max_blocks) : 0;
    // Page id of box `lane` of KV tile j; pages past the sequence are fetched out of
    // range (page id num_pages), which TMA fills with zeros.
    auto page_of = [&](int j) -> int {
      int pg = p.num_pages;
      if (PAGED && lane < boxes) {
        const int lp = (j * kFwdBN + lane * box_rows) / p.page_size;
        if (lp < n_valid_pages) pg = p.block_table[(int64_t)b * p.max_blocks + lp];
      }
      return pg;
    };
    int pg_next = (PAGED && nkv > 0) ? page_of(j0) : 0;
    int it = 0;
    bool ok = true;
    for (int jj = 0; jj < nkv && ok; ++jj) {
      const int j = j0 + jj;
      const int pg_cur = pg_next;
      if (PAGED && jj + 1 < nkv) pg_next = page_of(j + 1);
      for (int w = 0; w < 2 && ok; ++w, ++it) {
        const int s = it % ST;
        const uint32_t ph = (it / ST) & 1;
        int okl = 1;
        if (lane == 0)
          okl = mbar_wait(smem_u32(&ctl->kv_empty[s]), ph ^ 1, abort_flag, p.err,
                          FA_SITE_FWD_PRODUCER);
        ok = __shfl_sync(0xffffffffu, okl, 0) != 0;
        if (!ok) break;
        const uint32_t fb = smem_u32(&ctl->kv_full[s]);
        const CUtensorMap* tm = (w == 0) ? &tm_k : &tm_v;
        const uint32_t dst = sKV + s * Cfg::TILE_BYTES;
        if (lane == 0) mbar_arrive_expect_tx(fb, Cfg::TILE_BYTES);
        if constexpr (PAGED) {
          // Lane r issues the copies of page box r, so the (up to 16) page copies of a
          // tile go out in parallel instead of one after another from lane 0.
          __syncwarp();
          if (lane < boxes) {
            const int in_page = (j * kFwdBN + lane * box_rows) % p.page_size;
            for (int dh = 0; dh < Cfg::DH; ++dh)
              tma_load_4d(dst + dh * Cfg::CHUNK_BYTES + lane * box_rows * 128, tm, fb, dh * 64, hk,
                          in_page, pg_cur);
          }
        } else {
          if (lane == 0)
            for (int dh = 0; dh < Cfg::DH; ++dh)
              tma_load_4d(dst + dh * Cfg::CHUNK_BYTES, tm, fb, dh * 64, hk, j * kFwdBN, b);
        }
      }
    }
    // Drain: every copy issued must have landed before the CTA may exit.
    if (lane == 0) {
      for (int k = max(0, it - ST); k < it; ++k)
        mbar_wait_drain(smem_u32(&ctl->kv_full[k % ST]), (k / ST) & 1);
      mbar_wait_drain(smem_u32(&ctl->q_full), 0);
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      constexpr bool kBf16 = Pack2<T>::kBf16;
      constexpr uint32_t idS = idesc_f16(128, kFwdBN, kBf16, false, false);
      constexpr uint32_t idPV = idesc_f16(128, D, kBf16, false, true);
      bool ok = mbar_wait(smem_u32(&ctl->q_full), 0, abort_flag, p.err, FA_SITE_FWD_MMA);
      tc_fence_after();
      // Descriptors: built once; per slot / per K step they are base + constant.
      const uint64_t q_desc0 = sdesc_sw128(sQ, 16, 1024);            // K-major Q tiles
      const uint64_t k_desc0 = sdesc_sw128(sKV, 16, 1024);           // K-major K in slot 0
      const uint64_t v_desc0 = sdesc_sw128(sKV, Cfg::CHUNK_BYTES, 1024);  // MN-major V, slot 0
      // S_t = Q_t K^T over D in steps of 16 (K-major, 128-byte swizzle: step = +32 B
      // inside a 64-column chunk, next chunk at +16 KB).
      auto issue_S = [&](int t, int slot) {
        const uint64_t qa = desc_add(opaque(q_desc0), t * Cfg::TILE_BYTES);
        const uint64_t ka = desc_add(opaque(k_desc0), slot * Cfg::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t o = (kk >> 2) * Cfg::CHUNK_BYTES + (kk & 3) * 32;
          mma_ss(tmem + t * 128, desc_add(qa, o), desc_add(ka, o), idS, kk > 0 ? 1u : 0u);
        }
      };
      // O_t += P_t V over keys [64 hf, 64 hf + 64) in steps of 16 (V MN-major: step = 16
      // rows = +2 KB, 64-column chunks of D at +16 KB = LBO).  P's 16-bit pairs: 16 keys
      // = 8 TMEM columns.
      auto issue_PV = [&](int t, int slot, bool acc, int hf) {
        const uint64_t va = desc_add(opaque(v_desc0), slot * Cfg::TILE_BYTES);
#pragma unroll
        for (int k4 = 0; k4 < kFwdBN / 32; ++k4) {
          const int kk = hf * (kFwdBN / 32) + k4;
          mma_ts(tmem + NQ * 128 + t * D, tmem + t * 128 + kk * 8, desc_add(va, kk * 2048), idPV,
                 (acc || kk > 0) ? 1u : 0u);
        }
      };
      int it = 0;
      if (ok && nkv > 0) {
        const int s = it % ST;
        ok = mbar_wait(smem_u32(&ctl->kv_full[s]), (it / ST) & 1, abort_flag, p.err,
                       FA_SITE_FWD_MMA);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < NQ; ++t) {
            issue_S(t, s);
            mma_commit(smem_u32(&ctl->s_full[t]));
          }
          mma_commit(smem_u32(&ctl->kv_empty[s]));
        }
        ++it;
      }
      for (int jj = 0; jj < nkv && ok; ++jj) {
        const int sv = it % ST;
        const uint32_t phv = (it / ST) & 1;
        ++it;
        const bool has_next = jj + 1 < nkv;
        const int sk = it % ST;
        const uint32_t phk = (it / ST) & 1;
        if (has_next) ++it;
        ok = mbar_wait(smem_u32(&ctl->kv_full[sv]), phv, abort_flag, p.err, FA_SITE_FWD_MMA);
        if (!ok) break;
        for (int t = 0; t < NQ && ok; ++t) {
          if (kSplitP) {
            // PV over the first 64 keys runs while the softmax computes the second half.
            ok = mbar_wait(smem_u32(&ctl->p_half[t]), jj & 1, abort_flag, p.err, FA_SITE_FWD_MMA);
            if (!ok) break;
            FA_TRACE_EVENT(8 * t + 6, jj);
            tc_fence_after();
            issue_PV(t, sv, jj > 0, 0);
          }
          ok = mbar_wait(smem_u32(&ctl->p_ready[t]), jj & 1, abort_flag, p.err, FA_SITE_FWD_MMA);
          if (!ok) break;
          tc_fence_after();
          if (!kSplitP) issue_PV(t, sv, jj > 0, 0);
          issue_PV(t, sv, true, 1);
          // V_j's slot is free once the last PV reading it completes, ahead of S_{j+1}.
          if (t == NQ - 1) mma_commit(smem_u32(&ctl->kv_empty[sv]));
          if (has_next) {
            if (t == 0) {
              ok = mbar_wait(smem_u32(&ctl->kv_full[sk]), phk, abort_flag, p.err,
                             FA_SITE_FWD_MMA);
              if (!ok) break;
              tc_fence_after();
            }
            issue_S(t, sk);
            mma_commit(smem_u32(&ctl->s_full[t]));
          }
          FA_TRACE_EVENT(8 * t + 7, jj);
        }
        if (!ok) break;
        if (has_next) mma_commit(smem_u32(&ctl->kv_empty[sk]));
      }
      for (int t = 0; t < NQ; ++t) mma_commit(smem_u32(&ctl->o_final[t]));
      mma_commit(smem_u32(&ctl->drain));
      mbar_wait_drain(smem_u32(&ctl->drain), 0);
    }
  }
  } else {
    if (NQ == 2) setmaxnreg_inc<kFwdRegHigh>();
    // ============================================================ softmax / epilogue
    const int t = (warp - 4) >> 2;
    const int r = ((warp & 3) << 5) | lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * 128;
    const uint32_t tO = tmem + lane_off + NQ * 128 + t * D;
    const int tr = r / G;                    // token of this row inside the tile
    const int lt = tok0 + t * TPT + tr;      // token index within the sequence / query chunk
    const int h = hk * G + (r - tr * G);     // query head
    const bool row_valid = tr < TPT && lt < q_len;
    const int limit = lt + off;              // causal: key <= limit
    const bool window = fwd_window_on<PAGED>(p);
    const float c2 = p.scale_log2;
    const float NEG_INF = -INFINITY;
    float m_run = NEG_INF, m_ref = NEG_INF, l = 0.f;
    bool ok = true;
    if (NQ == 2 && t == 1) mbar_arrive(smem_u32(&ctl->exp_turn[0]));  // tile 0 goes first

    for (int jj = 0; jj < nkv; ++jj) {
      const int j = j0 + jj;
      const bool tr = (threadIdx.x & 127) == 0;  // first thread of each softmax warpgroup
      if (tr) FA_TRACE_EVENT(8 * t + 0, jj);
      bool w_ok = mbar_wait(smem_u32(&ctl->s_full[t]), jj & 1, abort_flag, p.err,
                            FA_SITE_FWD_SOFTMAX);
      ok = __all_sync(0xffffffffu, w_ok);
      if (!ok) break;
      if (tr) FA_TRACE_EVENT(8 * t + 1, jj);
      tc_fence_after();
      uint32_t s[128];
      tmem_ld32(tS + 0, s);
      tmem_ld32(tS + 32, s + 32);
      tmem_ld32(tS + 64, s + 64);
      tmem_ld32(tS + 96, s + 96);
      tmem_wait_ld();
      if (tr) FA_TRACE_EVENT(8 * t + 2, jj);
      const int key0 = j * kFwdBN;
      const bool need_mask =
          (key0 + kFwdBN > kv_len) || (p.causal && (key0 + kFwdBN - 1 > limit)) || window;
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const int key = key0 + c;
          bool vis = key < kv_len;
          if (p.causal) vis = vis && key <= limit;
          if (window) {
            const int wa = PAGED ? lt : lt + off;  // window anchor
            if (p.swq > 0) vis = vis && (wa < key + p.swq);
            if (p.swk > 0) vis = vis && (key < wa + p.swk);
          }
          if (!vis) s[c] = __float_as_uint(NEG_INF);
        }
      }
      // Row max with three-input max: four chains over columns (u, u+4, ...).
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
      const float mx = fmaxf(fmax3(mx4[0], mx4[1], mx4[2]), mx4[3]);
      const float m_new = fmaxf(m_run, mx);
      m_run = m_new;
      if (tr) FA_TRACE_EVENT(8 * t + 3, jj);
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
      // With two Q tiles the warpgroups take turns on the exponential unit: tile 0's
      // exp phase of KV tile j, then tile 1's, then tile 0's of j + 1, ... so one
      // tile's exponentials run while the other tile's MMAs do.
      if (NQ == 2) {
        const bool turn = mbar_wait(smem_u32(&ctl->exp_turn[t]), jj & 1, abort_flag, p.err,
                                    FA_SITE_FWD_SOFTMAX);
        if (!__all_sync(0xffffffffu, turn)) {
          ok = false;
          break;
        }
      }
      float rs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      // P in two halves of 64 keys, each stored to TMEM as soon as it is packed.  With
      // kSplitP the first half is released to the MMA issuer (p_half) before the second is
      // computed, except by a warp that must rescale O first (PV_j accumulates onto the
      // rescaled O): it arrives on p_half after its rescale.
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t pk[32];
        {
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) {
            const int c = 32 * hf + cc;
            const float p0 = ex2_approx(fmaf(__uint_as_float(s[2 * c]), c2, -mref_s));
            const float p1 = ex2_approx(fmaf(__uint_as_float(s[2 * c + 1]), c2, -mref_s));
            rs[c & 7] += p0 + p1;
            pk[cc] = Pack2<T>::pack(p0, p1);
          }
        }
        tmem_st32(tS + 32 * hf, pk);
        if (kSplitP && hf == 0 && !rescale_o) {
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(smem_u32(&ctl->p_half[t]));
        }
      }
      if (NQ == 2) mbar_arrive(smem_u32(&ctl->exp_turn[t ^ 1]));
      l += ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
      if (tr) FA_TRACE_EVENT(8 * t + 4, jj);
      if (rescale_o) {
        // PV_{j-1} is complete: the commit that signalled S_j covered every earlier MMA.
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(tO + c0, o);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * factor);
          tmem_st32(tO + c0, o);
        }
        if (kSplitP) {
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(smem_u32(&ctl->p_half[t]));
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl->p_ready[t]));
      if (tr) FA_TRACE_EVENT(8 * t + 5, jj);
    }

    // ---------------------------------------------------------- epilogue
    if (ok) {
      bool w_ok = mbar_wait(smem_u32(&ctl->o_final[t]), 0, abort_flag, p.err, FA_SITE_FWD_SOFTMAX);
      ok = __all_sync(0xffffffffu, w_ok);
    }
    if (ok) {
      tc_fence_after();
      const bool have = l > 0.f;
      const float inv = have ? 1.f / l : 0.f;
      // Output tile through shared memory and one TMA store per 64-column chunk (the Q
      // tile's buffer: every MMA that read it finished before o_final).  Dense tiles
      // always (the tensor map clips rows past Sq); paged tiles when all their tokens
      // belong to this sequence, else per-row stores (the next rows are another
      // sequence's).
      const bool tma_out = PAGED ? (tok0 + t * TPT + TPT <= q_len) : true;
      const uint32_t stage = sQ + t * Cfg::TILE_BYTES;
      T* orow = reinterpret_cast<T*>(p.out) + (PAGED ? 0 : (int64_t)b * p.o_sb) +
                (int64_t)(tok_base + lt) * p.o_st + (int64_t)h * p.o_sh;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t o[32];
        if (nkv > 0) {
          tmem_ld32(tO + c0, o);
          tmem_wait_ld();
        }
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float a0 = have ? __uint_as_float(o[2 * c]) * inv : 0.f;
          const float a1 = have ? __uint_as_float(o[2 * c + 1]) * inv : 0.f;
          pk[c] = Pack2<T>::pack(a0, a1);
        }
        if (tma_out) {
          // row r of the 128-byte-swizzled tile, 16-byte units (c0 % 64) / 8 .. + 3
          const uint32_t rowa = stage + (c0 >> 6) * Cfg::CHUNK_BYTES + r * 128;
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
      if (row_valid && p.lse != nullptr) {
        const float lse = have ? m_ref * p.scale + logf(l) : NEG_INF;
        p.lse[(PAGED ? 0 : (int64_t)b * p.lse_sb) + (int64_t)h * p.lse_sh + tok_base + lt] = lse;
      }
      if (tma_out) {
        fence_async_shared();
        mbar_arrive(smem_u32(&ctl->o_staged[t]));
        if ((threadIdx.x & 127) == 0 &&
            mbar_wait(smem_u32(&ctl->o_staged[t]), 0, abort_flag, p.err, FA_SITE_FWD_SOFTMAX)) {
          const int tok = tok_base + tok0 + t * TPT;
#pragma unroll
          for (int dh = 0; dh < Cfg::DH; ++dh)
            tma_store_4d(&tm_o, stage + dh * Cfg::CHUNK_BYTES, dh * 64, hk * G, tok, PAGED ? 0 : b);
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
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

template <int D, int NQ>
struct FwdPersistCfg {
  static constexpr int DH = D / 64;                       // 128-byte column chunks
  static constexpr int TILE_BYTES = 128 * D * 2;          // one Q, K or V tile
  static constexpr int CHUNK_BYTES = 128 * 128;           // one 64-column chunk of a tile
  // Two sets of Q buffers where they fit next to the K/V ring: the next work item's Q
  // tiles load while the current item finishes (its epilogue stages O in its own set).
  static constexpr int QB = (D <= 128) ? 2 : 1;
  static constexpr int STAGES = (D == 64) ? 6 : (D == 128 ? 3 : 2);
  static constexpr int NTHREADS = 128 + 128 * NQ;
  static constexpr int TMEM_COLS = 512;
  static_assert(NQ * (128 + D) <= TMEM_COLS, "TMEM budget: S + O per Q tile");
  static constexpr int SMEM_Q = QB * NQ * TILE_BYTES;
  static constexpr int SMEM_KV = STAGES * TILE_BYTES;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + SMEM_Q + SMEM_KV + 1024 /*barriers*/;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget (227 KB per CTA)");
};


// One work item: NQ Q tiles (TPB tokens x the G heads of kv head hk) of one sequence.
struct FwdItem {
  int live;  // 0: the work list is exhausted
  int b, hk, tok0, q_len, kv_len, off, tok_base, j0, nkv;
  int kv_row0;  // varlen: the sequence's first row of the packed K / V
};

struct FwdPersistCtl {
  uint64_t q_full[2];
  uint64_t q_empty[2];   // Q buffer set free: its item's S MMAs done and its O stored
  uint64_t kv_full[8];
  uint64_t kv_empty[8];
  uint64_t s_full[2];
  uint64_t p_half[2];    // first 64 keys of P_t in TMEM (PV over them may start)
  uint64_t p_ready[2];   // all of P_t in TMEM
  uint64_t o_final[2];
  uint64_t o_empty[2];   // O_t read out by the epilogue (the next item's PV may overwrite it)
  uint64_t exp_turn[2];  // softmax ping-pong: warpgroup t may run its exp phase
  uint64_t o_staged[2];  // output tile t written to shared memory (TMA store may start)
  uint64_t item_full[2];
  uint64_t item_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  FwdItem item[2];       // work items published by the producer, double-buffered
};

// Work list entry L -> item, in the order of the one-CTA-per-item launch: dense in the
// grouped order of fwd_dense_order (q block ranks, kv heads, batches).  Paged: the q block index runs over all sequences' blocks (p.nbx
// slots per kv head, the tail empty).  Returns false for an empty slot.  Called by all 32
// lanes of a warp (the paged scan over sequences takes 32 of them per step); the result is
// the same in every lane.
template <int NQ, bool PAGED, bool VARLEN>
__device__ bool fwd_decode_item(int L, const FwdParams& p, FwdItem& it, int lane) {
  const int TPB = NQ * (kFwdBM / p.G);
  int x = L % p.nbx;
  it.hk = (L / p.nbx) % p.Hk;
  int tile, unit = L / p.nbx;
  if constexpr (!PAGED) {
    fwd_dense_order(L, p.nbx, p.n_items / p.nbx, x, unit);
    it.hk = unit % p.Hk;
  }
  if constexpr (PAGED) {
    // Sequence s owns q block slots [cum_s, cum_s + nb_s); find the first whose end > x.
    int s = -1, cum = 0, base = 0;
    for (int s0 = 0; s0 < p.num_seqs; s0 += 32) {
      const int sl = s0 + lane;
      int nb = 0;
      if (sl < p.num_seqs) {
        const int ql = p.qsl[sl + 1] - p.qsl[sl];
        nb = ql > 0 ? (ql + TPB - 1) / TPB : 0;
      }
      int incl = nb;  // inclusive prefix sum of block counts across the warp
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += v;
      }
      const int end = base + incl;
      const unsigned hit = __ballot_sync(0xffffffffu, sl < p.num_seqs && x < end);
      if (hit != 0u) {
        const int l = __ffs(hit) - 1;
        s = s0 + l;
        cum = __shfl_sync(0xffffffffu, end - nb, l);
        break;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (s < 0) return false;
    it.b = s;
    tile = x - cum;
    it.q_len = p.qsl[s + 1] - p.qsl[s];
    if constexpr (VARLEN) {
      // varlen: packed K / V rows, bottom-right alignment of the sequence's own lengths
      it.kv_row0 = p.cu_k[s];
      it.kv_len = p.cu_k[s + 1] - it.kv_row0;
      it.off = it.kv_len - it.q_len;
    } else {
      it.kv_row0 = 0;
      it.kv_len = clamp_seq_len(p.seq_lens[s], p.max_blocks, p.page_size, p.err,
                                FA_SITE_PAGED_SEQLEN, lane == 0);
      it.off = p.pkl[s];
    }
    it.tok_base = p.qsl[s];
  } else {
    it.b = unit / p.Hk;
    tile = p.causal ? (p.nbx - 1 - x) : x;
    it.q_len = p.Sq;
    it.kv_len = p.Skv;
    it.off = p.Skv - p.Sq;
    it.tok_base = 0;
    it.kv_row0 = 0;
  }
  it.tok0 = tile * TPB;
  int j0 = 0, j1 = 0;
  fwd_kv_range<PAGED, VARLEN>(p, it.tok0, TPB, it.q_len, it.kv_len, it.off, j0, j1);
  it.j0 = j0;
  it.nkv = max(0, j1 - j0);
  it.live = 1;
  return true;
}

// Persistent: one CTA per SM claims work items from a device counter (p.sched) in list
// order, so the claim order matches a one-CTA-per-item launch while the next item's
// loads and first S overlap the current item's tail.
template <typename T, int D, int NQ, bool PAGED, bool CAP, bool VARLEN>
__global__ void __launch_bounds__(FwdPersistCfg<D, NQ>::NTHREADS, 1)
    fa_fwd_persist_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                  const FwdParams p) {
  using Cfg = FwdPersistCfg<D, NQ>;
  constexpr int ST = Cfg::STAGES;
  constexpr int QB = Cfg::QB;
  constexpr bool kReloadS = false;  // true: S values re-read from TMEM (for a tighter register budget)
  // Release P_t in two halves (PV over the first 64 keys overlaps the second half's
  // exponentials).  Measured faster for dense D >= 128; for D = 64 (cheap PV) and the
  // paged path the extra barrier costs more than the overlap gains.
  constexpr bool kSplitP = (D >= 128) && !PAGED;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const uint32_t sQ = base;  // Q buffer set q: sQ + q * NQ * TILE_BYTES
  const uint32_t sKV = base + Cfg::SMEM_Q;
  FwdPersistCtl* ctl = reinterpret_cast<FwdPersistCtl*>(base_ptr + Cfg::SMEM_Q + Cfg::SMEM_KV);
  volatile int* abort_flag = &ctl->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = p.G;
  const int TPT = kFwdBM / G;       // tokens per Q tile (rows TPT*G .. 127 unused when G does not divide 128)

  if (threadIdx.x == 0) {
    ctl->abort_flag = 0;
    for (int q = 0; q < 2; ++q) {
      mbar_init(smem_u32(&ctl->q_full[q]), 1);
      mbar_init(smem_u32(&ctl->q_empty[q]), 1 + NQ);
      mbar_init(smem_u32(&ctl->item_full[q]), 1);
      mbar_init(smem_u32(&ctl->item_empty[q]), 1 + 128 * NQ);
    }
    for (int s = 0; s < ST; ++s) {
      mbar_init(smem_u32(&ctl->kv_full[s]), 1);
      mbar_init(smem_u32(&ctl->kv_empty[s]), 1);
    }
    for (int t = 0; t < NQ; ++t) {
      mbar_init(smem_u32(&ctl->s_full[t]), 1);
      mbar_init(smem_u32(&ctl->p_half[t]), 128);
      mbar_init(smem_u32(&ctl->p_ready[t]), 128);
      mbar_init(smem_u32(&ctl->o_final[t]), 1);
      mbar_init(smem_u32(&ctl->o_empty[t]), 128);
      mbar_init(smem_u32(&ctl->exp_turn[t]), 128);
      mbar_init(smem_u32(&ctl->o_staged[t]), 128);
    }
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

  if (warp < 4) {
    if (NQ == 2) setmaxnreg_dec<kFwdRegLow>();
  if (warp == 0) {
    // ============================================================ scheduler + TMA producer
    // Lane 0 claims and publishes each work item.  Dense: lane 0 issues every copy.
    // Paged: lane r fetches the page id of box r of the next KV tile while the current
    // tile's copies go out, and issues box r's copies itself, so block-table reads never
    // sit between two copies.
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
    }
    const int box_rows = PAGED ? min(p.page_size, kFwdBN) : kFwdBN;
    const int boxes = kFwdBN / box_rows;  // page boxes per KV tile (<= 16: page_size >= 8)
    int it = 0, k = 0, q_loaded = 0;
    bool ok = true;
    for (;; ++k) {
      int okl = 1;
      if (lane == 0 && k >= 2)
        okl = mbar_wait(smem_u32(&ctl->item_empty[k & 1]), ((k >> 1) - 1) & 1, abort_flag,
                        p.err, FA_SITE_FWD_PRODUCER);
      okl = __shfl_sync(0xffffffffu, okl, 0);
      // The whole warp claims (lane 0's ticket) and decodes the next item with work.
      FwdItem item;
      item.live = 0;
      if (okl) {
        for (;;) {
          int L = 0;
          if (lane == 0) L = atomicAdd(p.sched, 1);
          L = __shfl_sync(0xffffffffu, L, 0);
          if (L >= p.n_items) break;
          if (fwd_decode_item<NQ, PAGED, VARLEN>(L, p, item, lane)) break;
        }
      }
      if (lane == 0) {
        ctl->item[k & 1] = item;
        mbar_arrive(smem_u32(&ctl->item_full[k & 1]));
      }
      ok = okl != 0;
      if (!ok || !item.live) break;
      const int b = item.b, hk = item.hk, j0 = item.j0, nkv = item.nkv;
      // Q tiles of item k into buffer set k % QB, once item k - QB has released it.
      const int qb = k % QB;
      if (lane == 0) {
        if (k >= QB)
          okl = mbar_wait(smem_u32(&ctl->q_empty[qb]), ((k / QB) - 1) & 1, abort_flag, p.err,
                          FA_SITE_FWD_PRODUCER);
        if (okl) {
          const uint32_t qbar = smem_u32(&ctl->q_full[qb]);
          mbar_arrive_expect_tx(qbar, NQ * Cfg::DH * TPT * G * 128);
          for (int t = 0; t < NQ; ++t) {
            const int tok = item.tok_base + item.tok0 + t * TPT;
            for (int dh = 0; dh < Cfg::DH; ++dh)
              tma_load_4d(sQ + (qb * NQ + t) * Cfg::TILE_BYTES + dh * Cfg::CHUNK_BYTES, &tm_q,
                          qbar, dh * 64, hk * G, tok, PAGED ? 0 : b);
          }
          ++q_loaded;
        }
      }
      ok = __shfl_sync(0xffffffffu, okl, 0) != 0;
      if (!ok) break;
      constexpr bool linear = !PAGED || VARLEN;  // dense / varlen: 128-row K/V boxes
      const int n_valid_pages =
          linear ? 0 : min((item.kv_len + p.page_size - 1) / p.page_size, p.max_blocks);
      // Page id of box `lane` of KV tile j; pages past the sequence are fetched out of
      // range (page id num_pages), which TMA fills with zeros.
      auto page_of = [&](int j) -> int {
        int pg = p.num_pages;
        if (!linear && lane < boxes) {
          const int lp = (j * kFwdBN + lane * box_rows) / p.page_size;
          if (lp < n_valid_pages) pg = p.block_table[(int64_t)b * p.max_blocks + lp];
        }
        return pg;
      };
      int pg_next = (!linear && nkv > 0) ? page_of(j0) : 0;
      for (int jj = 0; jj < nkv && ok; ++jj) {
        const int j = j0 + jj;
        const int pg_cur = pg_next;
        if (!linear && jj + 1 < nkv) pg_next = page_of(j + 1);
        for (int w = 0; w < 2 && ok; ++w, ++it) {
          const int s = it % ST;
          const uint32_t ph = (it / ST) & 1;
          okl = 1;
          if (lane == 0)
            okl = mbar_wait(smem_u32(&ctl->kv_empty[s]), ph ^ 1, abort_flag, p.err,
                            FA_SITE_FWD_PRODUCER);
          ok = __shfl_sync(0xffffffffu, okl, 0) != 0;
          if (!ok) break;
          const uint32_t fb = smem_u32(&ctl->kv_full[s]);
          const CUtensorMap* tm = (w == 0) ? &tm_k : &tm_v;
          const uint32_t dst = sKV + s * Cfg::TILE_BYTES;
          if (lane == 0) mbar_arrive_expect_tx(fb, Cfg::TILE_BYTES);
          if constexpr (!linear) {
            __syncwarp();
            if (lane < boxes) {
              const int in_page = (j * kFwdBN + lane * box_rows) % p.page_size;
              for (int dh = 0; dh < Cfg::DH; ++dh)
                tma_load_4d(dst + dh * Cfg::CHUNK_BYTES + lane * box_rows * 128, tm, fb, dh * 64, hk,
                            in_page, pg_cur);
            }
          } else {
            // dense: batch b's rows; varlen: rows from the sequence's first packed row
            // (rows past it belong to the next sequence or lie past the tensor: masked)
            if (lane == 0)
              for (int dh = 0; dh < Cfg::DH; ++dh)
                tma_load_4d(dst + dh * Cfg::CHUNK_BYTES, tm, fb, dh * 64, hk,
                            item.kv_row0 + j * kFwdBN, PAGED ? 0 : b);
          }
        }
      }
      if (!ok) break;
    }
    // Drain: every copy issued must have landed before the CTA may exit.
    if (lane == 0) {
      for (int kk = max(0, it - ST); kk < it; ++kk)
        mbar_wait_drain(smem_u32(&ctl->kv_full[kk % ST]), (kk / ST) & 1);
      for (int kk = max(0, q_loaded - QB); kk < q_loaded; ++kk)
        mbar_wait_drain(smem_u32(&ctl->q_full[kk % QB]), (kk / QB) & 1);
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      constexpr bool kBf16 = Pack2<T>::kBf16;
      constexpr uint32_t idS = idesc_f16(128, kFwdBN, kBf16, false, false);
      constexpr uint32_t idPV = idesc_f16(128, D, kBf16, false, true);
      // Descriptors: built once; per slot / per K step they are base + constant.
      const uint64_t q_desc0 = sdesc_sw128(sQ, 16, 1024);            // K-major Q tiles
      const uint64_t k_desc0 = sdesc_sw128(sKV, 16, 1024);           // K-major K in slot 0
      const uint64_t v_desc0 = sdesc_sw128(sKV, Cfg::CHUNK_BYTES, 1024);  // MN-major V, slot 0
      int qoff = 0;  // byte offset of the current item's Q buffer set
      // S_t = Q_t K^T over D in steps of 16 (K-major, 128-byte swizzle: step = +32 B
      // inside a 64-column chunk, next chunk at +16 KB).
      auto issue_S = [&](int t, int slot) {
        const uint64_t qa = desc_add(opaque(q_desc0), qoff + t * Cfg::TILE_BYTES);
        const uint64_t ka = desc_add(opaque(k_desc0), slot * Cfg::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t o = (kk >> 2) * Cfg::CHUNK_BYTES + (kk & 3) * 32;
          mma_ss(tmem + t * 128, desc_add(qa, o), desc_add(ka, o), idS, kk > 0 ? 1u : 0u);
        }
      };
      // O_t += P_t V over keys [64 hf, 64 hf + 64) in steps of 16 (V MN-major: step = 16
      // rows = +2 KB, 64-column chunks of D at +16 KB = LBO).  P's 16-bit pairs: 16 keys
      // = 8 TMEM columns.
      auto issue_PV = [&](int t, int slot, bool acc, int hf) {
        const uint64_t va = desc_add(opaque(v_desc0), slot * Cfg::TILE_BYTES);
#pragma unroll
        for (int k4 = 0; k4 < kFwdBN / 32; ++k4) {
          const int kk = hf * (kFwdBN / 32) + k4;
          mma_ts(tmem + NQ * 128 + t * D, tmem + t * 128 + kk * 8, desc_add(va, kk * 2048), idPV,
                 (acc || kk > 0) ? 1u : 0u);
        }
      };
      int it = 0, gj = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        ok = mbar_wait(smem_u32(&ctl->item_full[k & 1]), (k >> 1) & 1, abort_flag, p.err,
                       FA_SITE_FWD_MMA);
        if (!ok) break;
        if (!ctl->item[k & 1].live) break;
        const int nkv = ctl->item[k & 1].nkv;
        const int qb = k % QB;
        qoff = qb * NQ * Cfg::TILE_BYTES;
        ok = mbar_wait(smem_u32(&ctl->q_full[qb]), (k / QB) & 1, abort_flag, p.err, FA_SITE_FWD_MMA);
        if (!ok) break;
        tc_fence_after();
        if (nkv > 0) {
          // First S of the item: its columns were last read by the previous item's final
          // PV, issued earlier (MMAs run in issue order).
          const int s = it % ST;
          ok = mbar_wait(smem_u32(&ctl->kv_full[s]), (it / ST) & 1, abort_flag, p.err,
                         FA_SITE_FWD_MMA);
          if (!ok) break;
          tc_fence_after();
          for (int t = 0; t < NQ; ++t) {
            issue_S(t, s);
            mma_commit(smem_u32(&ctl->s_full[t]));
          }
          mma_commit(smem_u32(&ctl->kv_empty[s]));
          ++it;
        }
        for (int jj = 0; jj < nkv && ok; ++jj, ++gj) {
          const int sv = it % ST;
          const uint32_t phv = (it / ST) & 1;
          ++it;
          const bool has_next = jj + 1 < nkv;
          const int sk = it % ST;
          const uint32_t phk = (it / ST) & 1;
          if (has_next) ++it;
          ok = mbar_wait(smem_u32(&ctl->kv_full[sv]), phv, abort_flag, p.err, FA_SITE_FWD_MMA);
          if (!ok) break;
          for (int t = 0; t < NQ && ok; ++t) {
            if (jj == 0 && k > 0) {
              // The item's first PV overwrites O_t: the previous item's epilogue must have
              // read it out.
              ok = mbar_wait(smem_u32(&ctl->o_empty[t]), (k - 1) & 1, abort_flag, p.err,
                             FA_SITE_FWD_MMA);
              if (!ok) break;
            }
            if (kSplitP) {
              // PV over the first 64 keys runs while the softmax computes the second half.
              ok = mbar_wait(smem_u32(&ctl->p_half[t]), gj & 1, abort_flag, p.err, FA_SITE_FWD_MMA);
              if (!ok) break;
              tc_fence_after();
              issue_PV(t, sv, jj > 0, 0);
            }
            ok = mbar_wait(smem_u32(&ctl->p_ready[t]), gj & 1, abort_flag, p.err, FA_SITE_FWD_MMA);
            if (!ok) break;
            tc_fence_after();
            if (!kSplitP) issue_PV(t, sv, jj > 0, 0);
            issue_PV(t, sv, true, 1);
            // V_j's slot is free once the last PV reading it completes, ahead of S_{j+1}.
            if (t == NQ - 1) mma_commit(smem_u32(&ctl->kv_empty[sv]));
            if (has_next) {
              if (t == 0) {
                ok = mbar_wait(smem_u32(&ctl->kv_full[sk]), phk, abort_flag, p.err,
                               FA_SITE_FWD_MMA);
                if (!ok) break;
                tc_fence_after();
              }
              issue_S(t, sk);
              mma_commit(smem_u32(&ctl->s_full[t]));
            }
          }
          if (!ok) break;
          if (has_next) mma_commit(smem_u32(&ctl->kv_empty[sk]));
        }
        if (!ok) break;
        if (nkv == 0 && k > 0) {
          // No PV for this item: consume the previous item's O release all the same, so
          // the o_empty phases stay in step with the items.
          for (int t = 0; t < NQ && ok; ++t)
            ok = mbar_wait(smem_u32(&ctl->o_empty[t]), (k - 1) & 1, abort_flag, p.err,
                           FA_SITE_FWD_MMA);
          if (!ok) break;
        }
        for (int t = 0; t < NQ; ++t) mma_commit(smem_u32(&ctl->o_final[t]));
        mma_commit(smem_u32(&ctl->q_empty[qb]));  // every S of this item has read its Q
        mbar_arrive(smem_u32(&ctl->item_empty[k & 1]));
      }
      mma_commit(smem_u32(&ctl->drain));
      mbar_wait_drain(smem_u32(&ctl->drain), 0);
    }
  }
  } else {
    if (NQ == 2) setmaxnreg_inc<kFwdRegHigh>();
    // ============================================================ softmax / epilogue
    const int t = (warp - 4) >> 2;
    const int r = ((warp & 3) << 5) | lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * 128;
    const uint32_t tO = tmem + lane_off + NQ * 128 + t * D;
    const int tr = r / G;                    // token of this row inside the tile
    const float c2 = p.scale_log2;
    const float NEG_INF = -INFINITY;
    const bool window = fwd_window_on<PAGED, VARLEN>(p);
    constexpr bool capped = CAP;  // softcap variant (dense and varlen)
    bool ok = true;
    int gj = 0, n_staged = 0;
    if (NQ == 2 && t == 1) mbar_arrive(smem_u32(&ctl->exp_turn[0]));  // tile 0 goes first

    for (int k = 0; ok; ++k) {
      bool w_ok = mbar_wait(smem_u32(&ctl->item_full[k & 1]), (k >> 1) & 1, abort_flag, p.err,
                            FA_SITE_FWD_SOFTMAX);
      ok = __all_sync(0xffffffffu, w_ok);
      if (!ok) break;
      // The item stays in its slot until this item's end (item_empty is arrived after the
      // epilogue), so its fields are read from shared memory where they are used.
      const FwdItem* itp = &ctl->item[k & 1];
      if (!itp->live) break;
      const int nkv = itp->nkv;
      float m_run = NEG_INF, m_ref = NEG_INF, l = 0.f;

      for (int jj = 0; jj < nkv; ++jj, ++gj) {
        const int j = itp->j0 + jj;
        w_ok = mbar_wait(smem_u32(&ctl->s_full[t]), gj & 1, abort_flag, p.err, FA_SITE_FWD_SOFTMAX);
        ok = __all_sync(0xffffffffu, w_ok);
        if (!ok) break;
        tc_fence_after();
        // Visible keys of this row form one range [lo, hi): key < kv_len; causal: key <=
        // lt + off; sliding window: anchor - swq < key and key < anchor + swk, anchor = lt
        // (paged, with causal) or lt + off (dense).
        const int key0 = j * kFwdBN;
        const int lt = itp->tok0 + t * TPT + tr;  // token index within the sequence / chunk
        int lo = 0, hi = itp->kv_len;
        if (p.causal) hi = min(hi, lt + itp->off + 1);
        if (window) {
          const int wa = fwd_paged_window<PAGED, VARLEN>() ? lt : lt + itp->off;
          if (p.swq > 0) lo = max(lo, wa - p.swq + 1);
          if (p.swk > 0) hi = min(hi, wa + p.swk);
        }
        const int clo = lo - key0, chi = hi - key0;  // visible columns [clo, chi)
        const bool masked = clo > 0 || chi < kFwdBN;
        // Keys 64..127 are read first (their max), then keys 0..63 (kept for the first half
        // of P).  Two-tile CTAs (168 registers a thread) keep 64 S values at a time and load
        // keys 64..127 again during the first half's exponentials; one-tile CTAs keep all
        // 128.  P overwrites only S columns already read.
        auto mask64 = [&](uint32_t* v, int c0) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c0 + c < clo || c0 + c >= chi) v[c] = __float_as_uint(NEG_INF);
        };
        // Row max with three-input max over 64 values: four chains (u, u+4, ...).
        auto max64 = [&](const uint32_t* v) -> float {
          float mx4[4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            mx4[u] = fmax3(__uint_as_float(v[u]), __uint_as_float(v[u + 4]), __uint_as_float(v[u + 8]));
#pragma unroll
          for (int c = 12; c < 60; c += 8)
#pragma unroll
            for (int u = 0; u < 4; ++u)
              mx4[u] = fmax3(mx4[u], __uint_as_float(v[c + u]), __uint_as_float(v[c + 4 + u]));
#pragma unroll
          for (int u = 0; u < 4; ++u) mx4[u] = fmaxf(mx4[u], __uint_as_float(v[60 + u]));
          return fmaxf(fmax3(mx4[0], mx4[1], mx4[2]), mx4[3]);
        };
        uint32_t s[64], s_hi[64];
        tmem_ld32(tS + 64, s_hi);
        tmem_ld32(tS + 96, s_hi + 32);
        tmem_wait_ld();
        if constexpr (capped) fwd_softcap<64>(s_hi, p);
        if (masked) mask64(s_hi, 64);
        const float mx_hi = max64(s_hi);
        tmem_ld32(tS + 0, s);
        tmem_ld32(tS + 32, s + 32);
        tmem_wait_ld();
        if constexpr (capped) fwd_softcap<64>(s, p);
        if (masked) mask64(s, 0);
        const float mx = fmaxf(mx_hi, max64(s));
        const float m_new = fmaxf(m_run, mx);
        m_run = m_new;
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
        // With two Q tiles the warpgroups take turns on the exponential unit: tile 0's
        // exp phase of KV tile j, then tile 1's, then tile 0's of j + 1, ... so one
        // tile's exponentials run while the other tile's MMAs do.
        if (NQ == 2) {
          const bool turn = mbar_wait(smem_u32(&ctl->exp_turn[t]), gj & 1, abort_flag, p.err,
                                      FA_SITE_FWD_SOFTMAX);
          if (!__all_sync(0xffffffffu, turn)) {
            ok = false;
            break;
          }
        }
        float rs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        // P in two halves of 64 keys, each stored to TMEM as soon as it is packed.  With
        // kSplitP the first half is released to the MMA issuer (p_half) before the second is
        // computed, except by a warp that must rescale O first (PV_j accumulates onto the
        // rescaled O): it arrives on p_half after its rescale.
        {
          uint32_t pk[32];
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) {
            const float p0 = ex2_approx(fmaf(__uint_as_float(s[2 * cc]), c2, -mref_s));
            const float p1 = ex2_approx(fmaf(__uint_as_float(s[2 * cc + 1]), c2, -mref_s));
            rs[cc & 7] += p0 + p1;
            pk[cc] = Pack2<T>::pack(p0, p1);
            if (kReloadS && cc == 15) {
              // keys 0..31 are consumed: bring keys 64..127 back while 32..63 are computed
              tmem_ld32(tS + 64, s_hi);
              tmem_ld32(tS + 96, s_hi + 32);
            }
          }
          tmem_st32(tS, pk);
        }
        if (kSplitP && !rescale_o) {
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(smem_u32(&ctl->p_half[t]));
        }
        if (kReloadS) {
          tmem_wait_ld();
          if constexpr (capped) fwd_softcap<64>(s_hi, p);
          if (masked) mask64(s_hi, 64);
        }
        {
          uint32_t pk[32];
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) {
            const float p0 = ex2_approx(fmaf(__uint_as_float(s_hi[2 * cc]), c2, -mref_s));
            const float p1 = ex2_approx(fmaf(__uint_as_float(s_hi[2 * cc + 1]), c2, -mref_s));
            rs[cc & 7] += p0 + p1;
            pk[cc] = Pack2<T>::pack(p0, p1);
          }
          tmem_st32(tS + 32, pk);
        }
        if (NQ == 2) mbar_arrive(smem_u32(&ctl->exp_turn[t ^ 1]));
        l += ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
        if (rescale_o) {
          // PV_{j-1} is complete: the commit that signalled S_j covered every earlier MMA.
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 32) {
            uint32_t o[32];
            tmem_ld32(tO + c0, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * factor);
            tmem_st32(tO + c0, o);
          }
          if (kSplitP) {
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(smem_u32(&ctl->p_half[t]));
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(smem_u32(&ctl->p_ready[t]));
      }
      if (!ok) break;

      // -------------------------------------------------------- epilogue of item k
      w_ok = mbar_wait(smem_u32(&ctl->o_final[t]), k & 1, abort_flag, p.err, FA_SITE_FWD_SOFTMAX);
      ok = __all_sync(0xffffffffu, w_ok);
      if (!ok) break;
      tc_fence_after();
      const bool have = l > 0.f;
      const float inv = have ? 1.f / l : 0.f;
      const int b = itp->b, tok0 = itp->tok0, q_len = itp->q_len, tok_base = itp->tok_base;
      const int qb = k % QB;
      const int lt = tok0 + t * TPT + tr;
      const int h = itp->hk * G + (r - tr * G);  // query head
      const bool row_valid = tr < TPT && lt < q_len;
      // Output tile through shared memory (this item's Q tile buffer: every MMA that read
      // it finished before o_final) and one TMA store per 64-column chunk.  Dense tiles
      // always (the tensor map clips rows past Sq); paged tiles when all their tokens
      // belong to this sequence, else per-row stores (the next rows are another
      // sequence's).
      const bool tma_out = PAGED ? (tok0 + t * TPT + TPT <= q_len) : true;
      const uint32_t stage = sQ + (qb * NQ + t) * Cfg::TILE_BYTES;
      T* orow = reinterpret_cast<T*>(p.out) + (PAGED ? 0 : (int64_t)b * p.o_sb) +
                (int64_t)(tok_base + lt) * p.o_st + (int64_t)h * p.o_sh;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t o[32];
        if (nkv > 0) {
          tmem_ld32(tO + c0, o);
          tmem_wait_ld();
        }
        if (c0 + 32 == D) {
          // All of O_t is in registers: the next item's first PV may overwrite it.
          tc_fence_before();
          mbar_arrive(smem_u32(&ctl->o_empty[t]));
        }
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float a0 = have ? __uint_as_float(o[2 * c]) * inv : 0.f;
          const float a1 = have ? __uint_as_float(o[2 * c + 1]) * inv : 0.f;
          pk[c] = Pack2<T>::pack(a0, a1);
        }
        if (tma_out) {
          // row r of the 128-byte-swizzled tile, 16-byte units (c0 % 64) / 8 .. + 3
          const uint32_t rowa = stage + (c0 >> 6) * Cfg::CHUNK_BYTES + r * 128;
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
      if (row_valid && p.lse != nullptr) {
        const float lse = have ? m_ref * p.scale + logf(l) : NEG_INF;
        p.lse[(PAGED ? 0 : (int64_t)b * p.lse_sb) + (int64_t)h * p.lse_sh + tok_base + lt] = lse;
      }
      const bool leader = (threadIdx.x & 127) == 0;
      if (tma_out) {
        fence_async_shared();
        mbar_arrive(smem_u32(&ctl->o_staged[t]));
        if (leader) {
          if (mbar_wait(smem_u32(&ctl->o_staged[t]), n_staged & 1, abort_flag, p.err,
                        FA_SITE_FWD_SOFTMAX)) {
            const int tok = tok_base + tok0 + t * TPT;
#pragma unroll
            for (int dh = 0; dh < Cfg::DH; ++dh)
              tma_store_4d(&tm_o, stage + dh * Cfg::CHUNK_BYTES, dh * 64, itp->hk * G, tok,
                           PAGED ? 0 : b);
            bulk_commit_group();
            bulk_wait_group_read();
          }
        }
        ++n_staged;
      }
      // The Q buffer set is free for item k + QB once the staged tile has been read.
      if (leader) mbar_arrive(smem_u32(&ctl->q_empty[qb]));
      mbar_arrive(smem_u32(&ctl->item_empty[k & 1]));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// ------------------------------------------------------------------- host side
// Work-item counters of the persistent kernel: each launch takes the next of
// kFwdSchedSlots device words and zeroes it on its stream first, so launches in flight
// on other streams use other words (kFwdSchedSlots launches would have to overlap on
// the GPU for two to share one).
constexpr int kFwdSchedSlots = 64;
__device__ int g_fwd_sched[kFwdSchedSlots];

static int* fwd_sched_counter(cudaStream_t st) {
  static std::atomic<unsigned> next{0};
  static std::atomic<int*> base_of[kMaxContexts];  // the counters' address per context
  const int slot = call_context_slot();
  if (slot < 0 || slot >= kMaxContexts) return nullptr;
  int* base = base_of[slot].load(std::memory_order_acquire);
  if (base == nullptr) {
    // Every thread that gets here stores the same address.
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&base), g_fwd_sched) != cudaSuccess)
      return nullptr;
    base_of[slot].store(base, std::memory_order_release);
  }
  int* c = base + (next.fetch_add(1) % kFwdSchedSlots);
  if (cudaMemsetAsync(c, 0, sizeof(int), st) != cudaSuccess) return nullptr;
  return c;
}
// Which schedule serves a launch.  The persistent kernel hides each work item's set-up
// (Q load, first S, epilogue) behind the previous item.  With the register split
// (softmax warpgroups at 224 registers, a row's 128 S values loaded once) its KV steps
// are as fast as the one-CTA-per-item kernel's, so it serves every D = 128 launch.
// Measured (bf16, TFLOP/s, one-CTA-per-item -> persistent, same process): D = 128 causal
// S = 4096 849 -> 940-978, S = 2048 (B 16) 750-789 -> 747-765, GQA 32/8 883-896 ->
// 997-1017, fp16 causal 758-815 -> 883-937, non-causal S = 4096 1047-1168 -> 1040-1166;
// D = 256 non-causal S = 4096 1006-1056 -> 975-1040 (earlier, without the split: causal
// 860 -> 945).  Hence: paged, D = 64 and D = 128 always persistent; D = 256 causal always,
// non-causal when a work item averages at most 12 KV tiles.
constexpr int kFwdPersistMaxTiles = 12;
template <int D, bool PAGED>
constexpr bool fwd_may_persist() { return true; }
template <int D, bool PAGED>
constexpr bool fwd_may_direct() { return !PAGED && D != 64; }
template <int D, bool PAGED>
static bool fwd_persistent(bool causal, int kv_len) {
  if (!fwd_may_direct<D, PAGED>() || D == 128) return true;
  const int tiles = (kv_len + kFwdBN - 1) / kFwdBN;
  const int avg_tiles = causal ? (tiles + 1) / 2 : tiles;  // per work item
  if (D == 256 && causal) return true;
  return avg_tiles <= kFwdPersistMaxTiles;
}

template <typename T, int D, int NQ, bool PAGED, bool CAP, bool VARLEN = false>
static int launch_fwd_persist(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                              const CUtensorMap& to, const FwdParams& p, int kind, cudaStream_t st) {
  using Cfg = FwdPersistCfg<D, NQ>;
  auto kern = fa_fwd_persist_kernel<T, D, NQ, PAGED, CAP, VARLEN>;
  static std::atomic<bool> attr_set[kMaxContexts];
  if (int s = smem_attr_once(kern, Cfg::SMEM_BYTES, attr_set)) return s;
  FwdParams q = p;
  q.sched = fwd_sched_counter(st);
  if (q.sched == nullptr) return FA_ERR_CUDA;
  const dim3 grid(p.n_items < num_sms() ? p.n_items : num_sms());
  prof_begin(kind, st);
  kern<<<grid, Cfg::NTHREADS, Cfg::SMEM_BYTES, st>>>(tq, tk, tv, to, q);
  prof_end(kind, st);
  return FA_OK;
}

template <typename T, int D, int NQ, bool PAGED>
static int launch_fwd_direct(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                             const CUtensorMap& to, const FwdParams& p, int kind, cudaStream_t st) {
  using Cfg = FwdCfg<D, NQ>;
  auto kern = fa_fwd_kernel<T, D, NQ, PAGED>;
  static std::atomic<bool> attr_set[kMaxContexts];
  if (int s = smem_attr_once(kern, Cfg::SMEM_BYTES, attr_set)) return s;
  // one CTA per work item: q blocks x kv heads x batch
  const dim3 grid(p.nbx, p.Hk, p.n_items / (p.nbx * p.Hk));
  prof_begin(kind, st);
  kern<<<grid, Cfg::NTHREADS, Cfg::SMEM_BYTES, st>>>(tq, tk, tv, to, p);
  prof_end(kind, st);
  return FA_OK;
}

template <typename T, int D, int NQ, bool PAGED>
static int launch_fwd_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                           const CUtensorMap& to, const FwdParams& p, cudaStream_t st) {
  const int kind = PAGED ? FA_PROF_PAGED : FA_PROF_FWD;
  int s = FA_OK;
  if (!PAGED && p.sc_a != 0.f) {
    // dense softcap: the persistent kernel's CAP variant serves every shape
    if constexpr (!PAGED) s = launch_fwd_persist<T, D, NQ, false, true>(tq, tk, tv, to, p, kind, st);
  } else if (fwd_persistent<D, PAGED>(p.causal != 0, p.Skv)) {
    if constexpr (fwd_may_persist<D, PAGED>())
      s = launch_fwd_persist<T, D, NQ, PAGED, false>(tq, tk, tv, to, p, kind, st);
  } else {
    if constexpr (fwd_may_direct<D, PAGED>())
      s = launch_fwd_direct<T, D, NQ, PAGED>(tq, tk, tv, to, p, kind, st);
  }
  if (s != FA_OK) return s;
  FA_CUDA_TRY(cudaGetLastError());
  count_launch();
  return FA_OK;
}

template <int D, int NQ, bool PAGED>
static int dispatch_dtype(int dtype, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& to,
                          const CUtensorMap& tv, const FwdParams& p, cudaStream_t st) {
  if (dtype == FA_DTYPE_BF16)
    return launch_fwd_impl<__nv_bfloat16, D, NQ, PAGED>(tq, tk, tv, to, p, st);
  return launch_fwd_impl<__half, D, NQ, PAGED>(tq, tk, tv, to, p, st);
}

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// Varlen launches: the persistent kernel's VARLEN variant (with CAP for a softcap).
template <int D, int NQ>
static int dispatch_varlen(int dtype, const CUtensorMap& tq, const CUtensorMap& tk,
                           const CUtensorMap& to, const CUtensorMap& tv, const FwdParams& p,
                           cudaStream_t st) {
  const bool bf16 = dtype == FA_DTYPE_BF16, cap = p.sc_a != 0.f;
  int s;
  if (bf16)
    s = cap ? launch_fwd_persist<__nv_bfloat16, D, NQ, true, true, true>(tq, tk, tv, to, p, FA_PROF_FWD, st)
            : launch_fwd_persist<__nv_bfloat16, D, NQ, true, false, true>(tq, tk, tv, to, p, FA_PROF_FWD, st);
  else
    s = cap ? launch_fwd_persist<__half, D, NQ, true, true, true>(tq, tk, tv, to, p, FA_PROF_FWD, st)
            : launch_fwd_persist<__half, D, NQ, true, false, true>(tq, tk, tv, to, p, FA_PROF_FWD, st);
  if (s != FA_OK) return s;
  FA_CUDA_TRY(cudaGetLastError());
  count_launch();
  return FA_OK;
}

int launch_fwd_dense(const fa_fwd_args_t* a, int* err, cudaStream_t st) {
  // head_dim 32 and 96 run the 64 / 128 kernels: the tensor maps keep the real head dim
  // as their inner extent, so TMA loads fill the missing columns with zeros (they add
  // nothing to Q K^T, and P V writes zeros there) and TMA stores clip them.
  const int D = (a->head_dim == 32) ? 64 : (a->head_dim == 96 ? 128 : a->head_dim);
  const int G = a->num_heads / a->num_heads_k;
  const int NQ = (D == 256) ? 1 : 2;
  if (G > 128) return FA_ERR_UNSUPPORTED;
  if (a->seqlen_q == 0 || a->batch == 0) return FA_OK;
  for (int i = 0; i < 3; ++i) {
    if ((a->q_stride[i] % 8) || (a->k_stride[i] % 8) || (a->v_stride[i] % 8) ||
        (a->o_stride[i] % 8))
      return FA_ERR_ALIGNMENT;
  }
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out))
    return FA_ERR_ALIGNMENT;
  const CUtensorMapDataType dt = tmap_dtype(a->dtype);
  CUtensorMap tq, tk, tv, to;
  {
    const uint64_t dims[4] = {(uint64_t)a->head_dim, (uint64_t)a->num_heads,
                              (uint64_t)a->seqlen_q, (uint64_t)a->batch};
    const uint64_t str[3] = {(uint64_t)a->q_stride[2] * 2, (uint64_t)a->q_stride[1] * 2,
                             (uint64_t)a->q_stride[0] * 2};
    const uint32_t box[4] = {64, (uint32_t)G, (uint32_t)(128 / G), 1};  // TPT tokens x G heads
    FA_TMAP_TRY(encode_tmap(&tq, dt, 4, a->q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
    const uint64_t ostr[3] = {(uint64_t)a->o_stride[2] * 2, (uint64_t)a->o_stride[1] * 2,
                              (uint64_t)a->o_stride[0] * 2};
    FA_TMAP_TRY(encode_tmap(&to, dt, 4, a->out, dims, ostr, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  const void* kv_ptr[2] = {a->k, a->v};
  const int64_t* kv_str[2] = {a->k_stride, a->v_stride};
  CUtensorMap* kv_map[2] = {&tk, &tv};
  for (int w = 0; w < 2; ++w) {
    const uint64_t dims[4] = {(uint64_t)a->head_dim, (uint64_t)a->num_heads_k,
                              (uint64_t)(a->seqlen_k > 0 ? a->seqlen_k : 1), (uint64_t)a->batch};
    const uint64_t str[3] = {(uint64_t)kv_str[w][2] * 2, (uint64_t)kv_str[w][1] * 2,
                             (uint64_t)kv_str[w][0] * 2};
    const uint32_t box[4] = {64, 1, 128, 1};
    FA_TMAP_TRY(encode_tmap(kv_map[w], dt, 4, kv_ptr[w], dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  FwdParams p{};
  p.Sq = a->seqlen_q;
  p.Skv = a->seqlen_k;
  p.H = a->num_heads;
  p.Hk = a->num_heads_k;
  p.G = G;
  p.causal = a->causal;
  p.swq = a->window_q > 0 ? a->window_q : 0;
  p.swk = a->window_k > 0 ? a->window_k : 0;
  p.scale = a->softmax_scale;
  p.scale_log2 = a->softmax_scale * 1.4426950408889634f;
  if (a->softcap > 0.f) {
    p.sc_a = a->softcap / a->softmax_scale;
    p.sc_k = 2.f * 1.4426950408889634f / p.sc_a;
  }
  p.out = a->out;
  p.lse = a->lse;
  p.o_sb = a->o_stride[0];
  p.o_st = a->o_stride[1];
  p.o_sh = a->o_stride[2];
  p.lse_sb = (int64_t)a->num_heads * a->seqlen_q;
  p.lse_sh = a->seqlen_q;
  p.err = err;
  const int TPB = NQ * (128 / G);
  p.nbx = (a->seqlen_q + TPB - 1) / TPB;
  p.n_items = p.nbx * a->num_heads_k * a->batch;
  switch (D) {
    case 64: return dispatch_dtype<64, 2, false>(a->dtype, tq, tk, to, tv, p, st);
    case 128: return dispatch_dtype<128, 2, false>(a->dtype, tq, tk, to, tv, p, st);
    case 256: return dispatch_dtype<256, 1, false>(a->dtype, tq, tk, to, tv, p, st);
    default: return FA_ERR_UNSUPPORTED;
  }
}

int launch_paged_prefill(const fa_paged_args_t* a, int* err, cudaStream_t st) {
  const int D = a->head_dim;
  const int G = a->num_heads / a->num_kv_heads;
  const int NQ = (D == 256) ? 1 : 2;
  if (G > 128) return FA_ERR_UNSUPPORTED;
  const int ps = a->page_size;
  if (ps < 8 || (ps & (ps - 1)) != 0) return FA_ERR_UNSUPPORTED;
  if (a->num_tokens == 0 || a->num_seqs == 0) return FA_OK;
  if (!aligned16(a->q) || !aligned16(a->k_cache) || !aligned16(a->v_cache) || !aligned16(a->out))
    return FA_ERR_ALIGNMENT;
  if (D == 512) return launch_paged512(a, err, st);  // half-width work items (fa_paged512.cu)
  const CUtensorMapDataType dt = tmap_dtype(a->dtype);
  CUtensorMap tq, tk, tv, to;
  {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)a->num_heads, (uint64_t)a->num_tokens, 1};
    const uint64_t str[3] = {(uint64_t)D * 2, (uint64_t)a->num_heads * D * 2,
                             (uint64_t)a->num_tokens * a->num_heads * D * 2};
    const uint32_t box[4] = {64, (uint32_t)G, (uint32_t)(128 / G), 1};  // TPT tokens x G heads
    FA_TMAP_TRY(encode_tmap(&tq, dt, 4, a->q, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
    FA_TMAP_TRY(encode_tmap(&to, dt, 4, a->out, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  const void* kv_ptr[2] = {a->k_cache, a->v_cache};
  CUtensorMap* kv_map[2] = {&tk, &tv};
  for (int w = 0; w < 2; ++w) {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)a->num_kv_heads, (uint64_t)ps,
                              (uint64_t)a->num_pages};
    const uint64_t str[3] = {(uint64_t)D * 2, (uint64_t)a->num_kv_heads * D * 2,
                             (uint64_t)ps * a->num_kv_heads * D * 2};
    const uint32_t box[4] = {64, 1, (uint32_t)(ps < 128 ? ps : 128), 1};
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
  p.o_sb = 0;
  p.o_st = (int64_t)a->num_heads * D;
  p.o_sh = D;
  p.lse_sb = 0;
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
  const int TPB = NQ * (128 / G);
  // Sum over sequences of ceil(q_len / TPB) <= num_tokens / TPB + num_seqs.
  p.nbx = a->num_tokens / TPB + a->num_seqs;
  p.n_items = p.nbx * a->num_kv_heads;
  switch (D) {
    case 64: return dispatch_dtype<64, 2, true>(a->dtype, tq, tk, to, tv, p, st);
    case 128: return dispatch_dtype<128, 2, true>(a->dtype, tq, tk, to, tv, p, st);
    case 256: return dispatch_dtype<256, 1, true>(a->dtype, tq, tk, to, tv, p, st);
    default: return FA_ERR_UNSUPPORTED;
  }
}

// Dense varlen: packed sequences run through the paged pipeline (one work list over the
// sequences' q blocks, GQA rows packed per kv head, LSE [H, total_q]) with K / V read as
// 128-row boxes from each sequence's first packed row instead of through a block table,
// and FA2's window anchor.
int launch_varlen_fwd(const fa_varlen_fwd_args_t* a, int* err, cudaStream_t st) {
  const int D = a->head_dim;
  const int G = a->num_heads / a->num_heads_k;
  const int NQ = (D == 256) ? 1 : 2;
  if (G > 128) return FA_ERR_UNSUPPORTED;
  if (a->total_q == 0 || a->batch == 0) return FA_OK;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out))
    return FA_ERR_ALIGNMENT;
  const CUtensorMapDataType dt = tmap_dtype(a->dtype);
  CUtensorMap tq, tk, tv, to;
  auto rows_map = [&](CUtensorMap* m, const void* ptr, const int64_t* str2, int heads, int rows,
                      uint32_t box_h, uint32_t box_r) {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)heads, (uint64_t)(rows > 0 ? rows : 1), 1};
    const uint64_t str[3] = {(uint64_t)str2[1] * 2, (uint64_t)str2[0] * 2,
                             (uint64_t)str2[0] * 2 * (uint64_t)(rows > 0 ? rows : 1)};
    const uint32_t box[4] = {64, box_h, box_r, 1};
    return encode_tmap(m, dt, 4, ptr, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
  };
  FA_TMAP_TRY(rows_map(&tq, a->q, a->q_stride, a->num_heads, a->total_q, G, 128 / G));
  FA_TMAP_TRY(rows_map(&to, a->out, a->o_stride, a->num_heads, a->total_q, G, 128 / G));
  FA_TMAP_TRY(rows_map(&tk, a->k, a->k_stride, a->num_heads_k, a->total_k, 1, kFwdBN));
  FA_TMAP_TRY(rows_map(&tv, a->v, a->v_stride, a->num_heads_k, a->total_k, 1, kFwdBN));
  FwdParams p{};
  p.H = a->num_heads;
  p.Hk = a->num_heads_k;
  p.G = G;
  p.causal = a->causal;
  p.scale = a->softmax_scale;
  p.scale_log2 = a->softmax_scale * 1.4426950408889634f;
  if (a->softcap > 0.f) {
    p.sc_a = a->softcap / a->softmax_scale;
    p.sc_k = 2.f * 1.4426950408889634f / p.sc_a;
  }
  p.out = a->out;
  p.lse = a->lse;
  p.o_st = a->o_stride[0];
  p.o_sh = a->o_stride[1];
  p.lse_sh = a->total_q;
  p.qsl = a->cu_seqlens_q;
  p.cu_k = a->cu_seqlens_k;
  p.num_seqs = a->batch;
  p.page_size = kFwdBN;  // unused by varlen loads; keeps the page-box arithmetic defined
  p.swq = a->window_q > 0 ? a->window_q : 0;
  p.swk = a->window_k > 0 ? a->window_k : 0;
  p.err = err;
  const int TPB = NQ * (128 / G);
  // Sum over sequences of ceil(q_len / TPB) <= total_q / TPB + batch.
  p.nbx = a->total_q / TPB + a->batch;
  p.n_items = p.nbx * a->num_heads_k;
  switch (D) {
    case 64: return dispatch_varlen<64, 2>(a->dtype, tq, tk, to, tv, p, st);
    case 128: return dispatch_varlen<128, 2>(a->dtype, tq, tk, to, tv, p, st);
    case 256: return dispatch_varlen<256, 1>(a->dtype, tq, tk, to, tv, p, st);
    default: return FA_ERR_UNSUPPORTED;
  }
}

}  // namespace fa

#ifdef FA_TRACE
// Diagnostic build only: copies (and clears) the forward kernel's phase trace.
extern "C" int fa_debug_trace_read_fwd(unsigned long long* dst, size_t n) {
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
