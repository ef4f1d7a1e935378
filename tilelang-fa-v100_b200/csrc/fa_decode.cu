// Paged decode on sm_100a: split-KV + LSE-weighted combine.
// Reference: tilelang_decode_forward -> _decode_adapter.py:15-47 -> _decode_kernel_func
// (_kernels_paged.py:393-489), which runs one CTA per (q head, sequence) over the whole
// sequence and re-reads every KV page once per q head of a GQA group.
//
// Here the work is HBM-bound (one query token per sequence), so the kernel is built to
// read each K/V byte exactly once:
//   * CTA = (split, kv-head group, sequence).  A split is a contiguous range of
//     16-token chunks of one sequence; splits run in parallel across SMs.
//   * warp 0 lane 0 streams chunks with TMA (one 16-row x 128-byte box per kv head
//     and 64-column half) into a STAGES-deep ring of 128-byte-swizzled slots.
//   * one compute warp per kv head (D / 128 above D = 128, each accumulating 128 of the
//     output columns): the G = H/Hkv query heads of the group are the rows of an
//     m16n8k16 MMA, so one read of K/V serves the whole group.
//   * per split: partial O (normalised) and LSE in an fp32 workspace; a second
//     kernel merges the splits with LSE weights.  With one split the first kernel
//     writes the final output directly.
#include "fa_ptx.cuh"
#include "fa_internal.h"
#include <cmath>
#include <cstdio>
#include <mutex>
#include <type_traits>

namespace fa {

constexpr int kDecChunk = 16;  // tokens per pipeline chunk

// Kv heads per CTA and ring stages, per head dim (64 / 128 / 256 / 512) and cache type.
// A CTA streams its split of the caches through its ring once, so each CTA ramps its
// pipeline up and down.  HBM stays busy when several CTAs share an SM and overlap those
// ramps.  So the 16-bit tables use small CTAs (one or two kv heads, 48 KB rings) and the
// kernel promises the compiler several blocks per SM (DecCfg::MINB), which caps
// registers.  Measured against one CTA per SM with 192 KB rings, same process, same
// outputs:
//   configs[4] (32 / 8 heads, D = 128)   0.938 -> 0.720 ms (5.05 -> 6.58 TB/s);
//   D = 64, 16 / 16 heads                 1.185 -> 0.714 ms;
//   D = 256, 32 / 8 heads                 0.927 -> 0.711 ms; D = 256, 8 / 1 heads even.
// fp8 caches at D = 128 gain the same way once their MMAs run in f16 (8 -> 2 kv heads
// per CTA: 0.732 -> 0.505 ms at configs[4]); at D = 256 two heads per CTA lose (0.69 ->
// 0.83 ms: its 160-register warps cap the CTAs per SM), and D = 512 is bound by its
// compute chains (MMAs, conversions), not the stream: it keeps larger CTAs.
constexpr int kDecMaxG16[4] = {2, 2, 1, 1};
constexpr int kDecStages16[4] = {6, 3, 3, 6};
constexpr int kDecMaxG8[4] = {2, 2, 4, 1};  // fp8 caches (head_dim 128 and up)
constexpr int kDecStages8[4] = {6, 6, 6, 8};
constexpr int dec_dim_index(int D) { return D == 64 ? 0 : D == 128 ? 1 : D == 256 ? 2 : 3; }
constexpr int dec_maxg(int D, bool kv8) {
  return kv8 ? kDecMaxG8[dec_dim_index(D)] : kDecMaxG16[dec_dim_index(D)];
}

// KV8: the caches hold fp8 e4m3 (one byte per element, 128 elements per 128-byte box
// row) instead of the query's 16-bit type (64 per box row).
template <int D, bool KV8 = false>
struct DecCfg {
  static constexpr int ELEM = KV8 ? 1 : 2;                // cache bytes per element
  static constexpr int BOX_ELEMS = 128 / ELEM;            // elements per 128-byte box row
  static constexpr int DH = D / BOX_ELEMS;                // boxes per head row
  // compute warps per kv head: one up to D = 128, then one per 128 output columns
  static constexpr int WPH = D > 128 ? D / 128 : 1;
  static constexpr int DW = D / WPH;                      // output columns per compute warp
  static constexpr int MAXG = dec_maxg(D, KV8);        // kv heads per CTA
  static constexpr int NTHREADS = 32 + 32 * MAXG * WPH;   // producer warp + compute warps
  // Blocks per SM promised to the compiler: a register cap of 224 per thread whatever the
  // CTA size, so small CTAs (one or two kv heads) still fit several to an SM.
  static constexpr int MINB = 65536 / (224 * NTHREADS) > 1 ? 65536 / (224 * NTHREADS) : 1;
  static constexpr int HEAD_BYTES = kDecChunk * D * ELEM; // one kv head, one chunk, K or V
  static constexpr int STAGE_BYTES_MAX = 2 * MAXG * HEAD_BYTES;
  static constexpr int STAGES =
      KV8 ? kDecStages8[dec_dim_index(D)] : kDecStages16[dec_dim_index(D)];
  static_assert(STAGES <= 8, "decode ring: DecSmemCtl holds 8 stages");
  // Above D = 128 the WPH warps of a kv head each form the partial S over their own
  // D / WPH dims and exchange it through shared memory (double buffered per chunk):
  // 16 rows x 16 tokens fp32 per warp.
  static constexpr int KS = (WPH > 1 ? DW : D) / 16;      // S k-steps per compute warp
  static constexpr int XCH_BYTES_PER_HEAD = WPH > 1 ? 2 * WPH * 32 * 8 * 4 : 0;
  static constexpr int SMEM_BYTES =
      1024 + STAGES * STAGE_BYTES_MAX + 256 + MAXG * XCH_BYTES_PER_HEAD;
  static_assert(SMEM_BYTES <= 232448, "decode smem budget");
};

struct DecParams {
  const void* q;       // [B, H, D]
  void* out;           // [B, H, D]
  float* lse;          // [B, H] or null
  float* o_part;       // [B, S, H, D]
  float* lse_part;     // [B, S, H]
  const int32_t* block_table;
  const int32_t* seq_lens;
  int B, H, Hkv, G, HG;  // HG = kv heads per CTA
  int page_size, num_pages, max_blocks;
  int num_splits, chunks_per_split;
  float scale_log2, scale;  // (fp8 caches: times k_scale)
  float v_scale;            // 1, or the fp8 value cache's scale
  int* err;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
template <bool BF16>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Byte offset of (row, 16-byte chunk) inside a 128-byte-swizzled [rows][64] block.
__device__ __forceinline__ uint32_t swz(int row, int chunk16) {
  return static_cast<uint32_t>(row * 128 + ((chunk16 ^ (row & 7)) << 4));
}

// fp8 caches: byte address of element d of row `row` in a chunk of 128-byte-swizzled
// boxes (128 elements per box row, boxes kDecChunk x 128 bytes apart).
__device__ __forceinline__ uint32_t swz8(uint32_t base, int row, int d) {
  return base + (d >> 7) * (kDecChunk * 128) + swz(row, (d & 127) >> 4) + (d & 15);
}
// Bytes (lo, hi) of a 32-bit word picked by a prmt selector, as a 16-bit value.
__device__ __forceinline__ uint32_t prmt(uint32_t x, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(x), "r"(sel));
  return r;
}
// Two e4m3 values (the first in the low byte) as an f16x2 pair: one cvt, exact (every
// e4m3 value is an f16 normal or zero).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t v) {
  uint32_t h;
  const uint16_t v16 = static_cast<uint16_t>(v);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(v16));
  return h;
}

struct DecSmemCtl {
  uint64_t full[8];
  uint64_t empty[8];
  int abort_flag;
};

template <typename T, int D, bool KV8>
__global__ void __launch_bounds__(DecCfg<D, KV8>::NTHREADS, DecCfg<D, KV8>::MINB)
    fa_decode_split_kernel(const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const DecParams p) {
  using Cfg = DecCfg<D, KV8>;
  constexpr int ST = Cfg::STAGES;
  // fp8 caches run the MMAs in f16 whatever the query type: the cache bytes convert
  // with one exact cvt, and P keeps 11 bits.  (A bf16 query converts once, below.)
  using MT = std::conditional_t<KV8, __half, T>;
  constexpr bool kBf16 = Pack2<MT>::kBf16;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const int HG = p.HG;
  const int stage_bytes = 2 * HG * Cfg::HEAD_BYTES;  // K heads then V heads
  DecSmemCtl* ctl = reinterpret_cast<DecSmemCtl*>(base_ptr + ST * stage_bytes);
  volatile int* abort_flag = &ctl->abort_flag;

  const int split = blockIdx.x;
  const int hk0 = blockIdx.y * HG;
  const int b = blockIdx.z;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int L = clamp_seq_len(p.seq_lens[b], p.max_blocks, p.page_size, p.err,
                              FA_SITE_DEC_SEQLEN, threadIdx.x == 0);
  const int c_begin = split * p.chunks_per_split;
  const int c_end = min((L + kDecChunk - 1) / kDecChunk, c_begin + p.chunks_per_split);
  const int nchunks = c_end - c_begin;
  if (nchunks <= 0) {
    // Empty split: the combine ignores it.  With a single split this CTA owns the
    // output, so an empty sequence gets zeros and LSE = -inf.
    if (p.num_splits == 1 && split == 0) {
      for (int i = threadIdx.x; i < HG * p.G * D; i += blockDim.x) {
        const int h = hk0 * p.G + i / D;
        reinterpret_cast<T*>(p.out)[((int64_t)b * p.H + h) * D + i % D] = T(0.f);
        if (p.lse != nullptr && i % D == 0) p.lse[(int64_t)b * p.H + h] = -INFINITY;
      }
    }
    return;
  }
  const int ncompute = HG * Cfg::WPH;

  if (threadIdx.x == 0) {
    ctl->abort_flag = 0;
    for (int s = 0; s < ST; ++s) {
      mbar_init(smem_u32(&ctl->full[s]), 1);
      mbar_init(smem_u32(&ctl->empty[s]), ncompute);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const int n_valid_pages = min((L + p.page_size - 1) / p.page_size, p.max_blocks);
      int it = 0;
      for (; it < nchunks; ++it) {
        const int s = it % ST;
        if (!mbar_wait(smem_u32(&ctl->empty[s]), ((it / ST) & 1) ^ 1, abort_flag, p.err,
                       FA_SITE_DEC_PRODUCER))
          break;
        const uint32_t fb = smem_u32(&ctl->full[s]);
        mbar_arrive_expect_tx(fb, stage_bytes);
        const int tok = (c_begin + it) * kDecChunk;
        const int lp = tok / p.page_size;
        const int in_page = tok - lp * p.page_size;
        const int page =
            lp < n_valid_pages ? p.block_table[(int64_t)b * p.max_blocks + lp] : p.num_pages;
        const uint32_t dst = base + s * stage_bytes;
        for (int w = 0; w < 2; ++w) {
          const CUtensorMap* tm = w == 0 ? &tm_k : &tm_v;
          for (int hh = 0; hh < HG; ++hh)
            for (int dh = 0; dh < Cfg::DH; ++dh)
              tma_load_4d(dst + (w * HG + hh) * Cfg::HEAD_BYTES + dh * (kDecChunk * 128), tm, fb,
                          dh * Cfg::BOX_ELEMS, hk0 + hh, in_page, page);
        }
      }
      for (int k = max(0, it - ST); k < it; ++k) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(smem_u32(&ctl->full[k % ST]), (k / ST) & 1))
          if (globaltimer_ns() - t0 > 200000000ull) break;
      }
    }
    return;
  }
  const int hh = (warp - 1) / Cfg::WPH;    // kv head of this compute warp
  const int part = (warp - 1) % Cfg::WPH;  // 128-column part of the output (D > 128)
  if (hh >= HG) return;
  const int hk = hk0 + hh;
  const int G = p.G;
  const int g = lane >> 2;       // MMA row group (row g and g + 8)
  const int qd = (lane & 3) * 2;  // column pair inside an 8-wide n tile

  // Q fragment (A operand, rows = query heads of the group, zero beyond G) of this warp's
  // S k-steps: all of D up to D = 128, else its own D / WPH dims.
  constexpr int KS = Cfg::KS;
  const int ks0 = Cfg::WPH > 1 ? part * KS : 0;
  uint32_t qa[KS][4];
  // A bf16 query over fp8 caches enters the f16 MMAs scaled by 2^qk, qk chosen so that
  // the largest |q| of the kv head's group lies in [2^14, 2^15): every element down to
  // 2^-28 of that maximum is an f16 normal and converts exactly (bf16 has 8 significant
  // bits, f16 11), smaller ones round as f16 subnormals, and S carries the factor 2^qk,
  // which the softmax scales divide out (power-of-two scalings are exact).  The warps of
  // a kv head read the same group, so they agree on qk.  qk is clamped to [-100, 100] to
  // keep the softmax scales times 2^-qk normal floats; only a group whose largest |q| is
  // below 2^-86 stays under 2^14 after scaling (its elements are exact down to 2^-14).
  float q_up = 1.f, q_down = 1.f;
  if constexpr (KV8 && Pack2<T>::kBf16) {
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(
        reinterpret_cast<const T*>(p.q) + ((int64_t)b * p.H + hk * G) * D);
    float amax = 0.f;
    for (int i = lane; i < G * D / 2; i += 32) {
      const float2 f = Pack2<T>::unpack(qw[i]);
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const int eb = (__float_as_int(amax) >> 23) & 0xFF;  // biased exponent of the maximum
    const int qk = max(-100, min(100, 141 - eb));        // 14 - (eb - 127)
    q_up = __int_as_float((127 + qk) << 23);
    q_down = __int_as_float((127 - qk) << 23);
  }
  {
    const T* qb = reinterpret_cast<const T*>(p.q) + ((int64_t)b * p.H + hk * G) * D;
#pragma unroll
    for (int i = 0; i < KS; ++i) {
      const int ks = ks0 + i;
      // fp8 caches: the K fragments come from ldmatrix over the byte rows, which gives
      // lane (g, j = lane & 3) dims 4 j .. 4 j + 3 of its 16-dim step; the MMA's k index
      // 2 j + e then stands for dim 4 j + e and 8 + 2 j + e for dim 4 j + 2 + e, and the
      // Q fragment takes the same permutation (the sum over k is unchanged).
      const int k0 = KV8 ? ks * 16 + 2 * qd : ks * 16 + qd;
      const int k8 = KV8 ? k0 + 2 : k0 + 8;
      auto ld2 = [&](int row, int col) -> uint32_t {
        if (row >= G) return 0u;
        const uint32_t w = *reinterpret_cast<const uint32_t*>(qb + (int64_t)row * D + col);
        if constexpr (KV8 && Pack2<T>::kBf16) {
          const float2 f = Pack2<T>::unpack(w);
          return Pack2<__half>::pack(f.x * q_up, f.y * q_up);
        } else {
          return w;
        }
      };
      qa[i][0] = ld2(g, k0);
      qa[i][1] = ld2(g + 8, k0);
      qa[i][2] = ld2(g, k8);
      qa[i][3] = ld2(g + 8, k8);
    }
  }
  constexpr int DW = Cfg::DW;
  float o[DW / 8][4];
#pragma unroll
  for (int i = 0; i < DW / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float c2 = p.scale_log2 * q_down;  // S carries the query's 2^qk

  // Partial-S exchange slots of this kv head: [2 chunk parities][WPH warps][32 lanes][8].
  float* const xch = reinterpret_cast<float*>(base_ptr + ST * stage_bytes + 256) +
                     hh * (Cfg::XCH_BYTES_PER_HEAD / 4);
  for (int it = 0; it < nchunks; ++it) {
    const int s = it % ST;
    const bool w_ok =
        mbar_wait(smem_u32(&ctl->full[s]), (it / ST) & 1, abort_flag, p.err, FA_SITE_DEC_COMPUTE);
    // One warp per kv head decides alone; the warps of a head that share S decide together
    // at the exchange barrier below (a barrier some of them skipped would never open).
    if constexpr (Cfg::WPH == 1) {
      if (!__all_sync(0xffffffffu, w_ok)) break;
    }
    const uint32_t kbase = base + s * stage_bytes + hh * Cfg::HEAD_BYTES;
    const uint32_t vbase = base + s * stage_bytes + (HG + hh) * Cfg::HEAD_BYTES;
    // S[16 rows x 16 tokens] = Q K^T over this warp's k-steps
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int i = 0; i < KS; ++i) {
      const int ks = ks0 + i;
      if constexpr (KV8) {
        // Two k steps per ldmatrix x4 over the byte rows (each 8x8 b16 matrix = 8 tokens
        // x 16 dims): matrices (tokens 0-7, dims 32 kp ..), (8-15, same), (0-7, +16),
        // (8-15, +16); each lane's word holds 4 consecutive dims of one token.
        if (i & 1) continue;  // handled with i - 1 (ks0 is even)
        const int mi = lane >> 3;
        const int tok = ((mi & 1) << 3) + (lane & 7);
        uint32_t r0, r1, r2, r3;
        ldsm_x4(swz8(kbase, tok, ks * 16 + (mi >> 1) * 16), r0, r1, r2, r3);
        const uint32_t w[4] = {r0, r1, r2, r3};
        uint32_t c[8];
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          c[2 * x] = e4m3x2_to_f16x2(w[x] & 0xFFFFu);
          c[2 * x + 1] = e4m3x2_to_f16x2(w[x] >> 16);
        }
        mma16816<kBf16>(sc[0], qa[i], c[0], c[1]);
        mma16816<kBf16>(sc[1], qa[i], c[2], c[3]);
        mma16816<kBf16>(sc[0], qa[i + 1], c[4], c[5]);
        mma16816<kBf16>(sc[1], qa[i + 1], c[6], c[7]);
      } else {
        // matrices: (tokens 0-7, d lo), (tokens 0-7, d hi), (tokens 8-15, d lo), (tokens 8-15, d hi)
        const int mi = lane >> 3;
        const int row = ((mi >> 1) << 3) + (lane & 7);
        const int dchunk = (ks & 3) * 2 + (mi & 1);
        const uint32_t addr = kbase + (ks >> 2) * (kDecChunk * 128) + swz(row, dchunk);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(addr, b0, b1, b2, b3);
        mma16816<kBf16>(sc[0], qa[i], b0, b1);
        mma16816<kBf16>(sc[1], qa[i], b2, b3);
      }
    }
    if constexpr (Cfg::WPH > 1) {
      // S = the sum of the WPH partials, added in warp order by every warp of the head
      // so all of them hold the same S (and the same P).  Double buffered by chunk
      // parity: a slot is rewritten two chunks later, after every warp has passed the
      // next chunk's barrier and so finished reading it.
      float* slot = xch + (it & 1) * (Cfg::WPH * 256);
      float4* mine = reinterpret_cast<float4*>(slot + (part * 32 + lane) * 8);
      mine[0] = make_float4(sc[0][0], sc[0][1], sc[0][2], sc[0][3]);
      mine[1] = make_float4(sc[1][0], sc[1][1], sc[1][2], sc[1][3]);
      if (!bar_red_and(1 + hh, 32 * Cfg::WPH, w_ok)) break;
#pragma unroll
      for (int w = 0; w < Cfg::WPH; ++w) {
        const float4* x = reinterpret_cast<const float4*>(slot + (w * 32 + lane) * 8);
        const float4 a = x[0], c = x[1];
        if (w == 0) {
          sc[0][0] = a.x; sc[0][1] = a.y; sc[0][2] = a.z; sc[0][3] = a.w;
          sc[1][0] = c.x; sc[1][1] = c.y; sc[1][2] = c.z; sc[1][3] = c.w;
        } else {
          sc[0][0] += a.x; sc[0][1] += a.y; sc[0][2] += a.z; sc[0][3] += a.w;
          sc[1][0] += c.x; sc[1][1] += c.y; sc[1][2] += c.z; sc[1][3] += c.w;
        }
      }
    }
    const int tok0 = (c_begin + it) * kDecChunk;
    if (tok0 + kDecChunk > L) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (tok0 + nt * 8 + qd + (e & 1) >= L) sc[nt][e] = -INFINITY;
    }
    float mx0 = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
    float mx1 = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float f0 = (mn0 == -INFINITY) ? 1.f : ex2_approx((m0 - mn0) * c2);
    const float f1 = (mn1 == -INFINITY) ? 1.f : ex2_approx((m1 - mn1) * c2);
    m0 = mn0;
    m1 = mn1;
    const float ms0 = (mn0 == -INFINITY) ? 0.f : mn0 * c2;
    const float ms1 = (mn1 == -INFINITY) ? 0.f : mn1 * c2;
    float pr[2][4];
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      pr[nt][0] = ex2_approx(fmaf(sc[nt][0], c2, -ms0));
      pr[nt][1] = ex2_approx(fmaf(sc[nt][1], c2, -ms0));
      pr[nt][2] = ex2_approx(fmaf(sc[nt][2], c2, -ms1));
      pr[nt][3] = ex2_approx(fmaf(sc[nt][3], c2, -ms1));
      rs0 += pr[nt][0] + pr[nt][1];
      rs1 += pr[nt][2] + pr[nt][3];
    }
    l0 = l0 * f0 + rs0;  // partial (per-thread) row sums, reduced across the quad at the end
    l1 = l1 * f1 + rs1;
    uint32_t pa[4];
    pa[0] = Pack2<MT>::pack(pr[0][0], pr[0][1]);
    pa[1] = Pack2<MT>::pack(pr[0][2], pr[0][3]);
    pa[2] = Pack2<MT>::pack(pr[1][0], pr[1][1]);
    pa[3] = Pack2<MT>::pack(pr[1][2], pr[1][3]);
#pragma unroll
    for (int dn = 0; dn < DW / 8; ++dn) {
      o[dn][0] *= f0;
      o[dn][1] *= f0;
      o[dn][2] *= f1;
      o[dn][3] *= f1;
    }
    // O[16 x DW] += P[16 x 16 tokens] V[16 tokens x this warp's DW columns]
#pragma unroll
    for (int dpl = 0; dpl < DW / 16; ++dpl) {
      const int dp = part * (DW / 16) + dpl;
      if constexpr (KV8) {
        // ldmatrix.trans over the byte rows, two 16-dim groups per x4: matrices (tokens
        // 0-7, dims 16 dp ..), (8-15, same), (0-7, dims 16 dp + 16 ..), (8-15, same); lane
        // (g, j) gets tokens 2 j, 2 j + 1 x dims 2 g, 2 g + 1 of each group.  prmt splits
        // them into an even-dim and an odd-dim column tile: o[2 dpl] / o[2 dpl + 1] hold,
        // at n = g, dims 16 dp + 2 g and 16 dp + 2 g + 1.
        if (dpl & 1) continue;  // handled with dpl - 1
        const int mi = lane >> 3;
        const int tok = ((mi & 1) << 3) + (lane & 7);
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(swz8(vbase, tok, dp * 16 + (mi >> 1) * 16), r0, r1, r2, r3);
        const uint32_t w[4] = {r0, r1, r2, r3};
#pragma unroll
        for (int gp = 0; gp < 2; ++gp) {
          const uint32_t lo = w[2 * gp], hi = w[2 * gp + 1];  // tokens 0-7 / 8-15
          mma16816<kBf16>(o[2 * (dpl + gp)], pa, e4m3x2_to_f16x2(prmt(lo, 0x0020)),
                          e4m3x2_to_f16x2(prmt(hi, 0x0020)));
          mma16816<kBf16>(o[2 * (dpl + gp) + 1], pa, e4m3x2_to_f16x2(prmt(lo, 0x0031)),
                          e4m3x2_to_f16x2(prmt(hi, 0x0031)));
        }
      } else {
        // matrices: (tok 0-7, d 16dp..+7), (tok 8-15, same), (tok 0-7, d +8..+15), (tok 8-15, +8..)
        const int mi = lane >> 3;
        const int row = ((mi & 1) << 3) + (lane & 7);
        const int dchunk = ((dp * 2) & 7) + (mi >> 1);
        const uint32_t addr = vbase + ((dp * 16) >> 6) * (kDecChunk * 128) + swz(row, dchunk);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(addr, b0, b1, b2, b3);
        mma16816<kBf16>(o[2 * dpl], pa, b0, b1);
        mma16816<kBf16>(o[2 * dpl + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&ctl->empty[s]));
  }

  // Row sums across the quad, then write.
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? p.v_scale / l0 : 0.f;
  const float inv1 = l1 > 0.f ? p.v_scale / l1 : 0.f;
  const float lse0 = l0 > 0.f ? m0 * (p.scale * q_down) + logf(l0) : -INFINITY;
  const float lse1 = l1 > 0.f ? m1 * (p.scale * q_down) + logf(l1) : -INFINITY;
  const bool direct = p.num_splits == 1;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int row = g + half * 8;
    if (row >= G) continue;
    const int h = hk * G + row;
    const float inv = half ? inv1 : inv0;
    const float lse = half ? lse1 : lse0;
    if (direct && KV8) {
      // even / odd column tiles: this lane's dims 16 dpl + 2 qd .. + 3
      T* dst = reinterpret_cast<T*>(p.out) + ((int64_t)b * p.H + h) * D + part * DW;
#pragma unroll
      for (int dpl = 0; dpl < DW / 16; ++dpl) {
        const float* e = o[2 * dpl];
        const float* od = o[2 * dpl + 1];
        *reinterpret_cast<uint2*>(dst + dpl * 16 + 2 * qd) =
            make_uint2(Pack2<T>::pack(e[half * 2] * inv, od[half * 2] * inv),
                       Pack2<T>::pack(e[half * 2 + 1] * inv, od[half * 2 + 1] * inv));
      }
      if (p.lse != nullptr && (lane & 3) == 0 && part == 0) p.lse[(int64_t)b * p.H + h] = lse;
    } else if (direct) {
      T* dst = reinterpret_cast<T*>(p.out) + ((int64_t)b * p.H + h) * D + part * DW;
#pragma unroll
      for (int dn = 0; dn < DW / 8; ++dn) {
        const uint32_t v = Pack2<T>::pack(o[dn][half * 2] * inv, o[dn][half * 2 + 1] * inv);
        *reinterpret_cast<uint32_t*>(dst + dn * 8 + qd) = v;
      }
      if (p.lse != nullptr && (lane & 3) == 0 && part == 0) p.lse[(int64_t)b * p.H + h] = lse;
    } else {
      float* dst = p.o_part + (((int64_t)b * p.num_splits + split) * p.H + h) * D + part * DW;
      if constexpr (KV8) {
#pragma unroll
        for (int dpl = 0; dpl < DW / 16; ++dpl) {
          const float* e = o[2 * dpl];
          const float* od = o[2 * dpl + 1];
          *reinterpret_cast<float4*>(dst + dpl * 16 + 2 * qd) =
              make_float4(e[half * 2] * inv, od[half * 2] * inv, e[half * 2 + 1] * inv,
                          od[half * 2 + 1] * inv);
        }
      } else {
#pragma unroll
        for (int dn = 0; dn < DW / 8; ++dn)
          *reinterpret_cast<float2*>(dst + dn * 8 + qd) =
              make_float2(o[dn][half * 2] * inv, o[dn][half * 2 + 1] * inv);
      }
      if ((lane & 3) == 0 && part == 0)
        p.lse_part[((int64_t)b * p.num_splits + split) * p.H + h] = lse;
    }
  }
}

// Merge the splits of each (sequence, head): out = sum_s exp(lse_s - lse) * o_s.
template <typename T, int D>
__global__ void __launch_bounds__(256) fa_decode_combine_kernel(const DecParams p) {
  const int b = blockIdx.y;
  const int L = clamp_seq_len(p.seq_lens[b], p.max_blocks, p.page_size, p.err,
                              FA_SITE_DEC_SEQLEN, false);
  const int used =
      min(p.num_splits, (((L + kDecChunk - 1) / kDecChunk) + p.chunks_per_split - 1) /
                            p.chunks_per_split);
  constexpr int TPH = D / 4;  // threads per head (float4 each)
  const int h = blockIdx.x * (256 / TPH) + threadIdx.x / TPH;
  const int d4 = (threadIdx.x % TPH) * 4;
  if (h >= p.H) return;
  const float* lp = p.lse_part + (int64_t)b * p.num_splits * p.H + h;
  float mx = -INFINITY;
  for (int s = 0; s < used; ++s) mx = fmaxf(mx, lp[(int64_t)s * p.H]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float wsum = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < used; ++s) {
      const float w = __expf(lp[(int64_t)s * p.H] - mx);
      if (w == 0.f) continue;
      const float4 v = *reinterpret_cast<const float4*>(
          p.o_part + (((int64_t)b * p.num_splits + s) * p.H + h) * D + d4);
      acc.x += w * v.x;
      acc.y += w * v.y;
      acc.z += w * v.z;
      acc.w += w * v.w;
      wsum += w;
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  T* dst = reinterpret_cast<T*>(p.out) + ((int64_t)b * p.H + h) * D + d4;
  uint2 pk;
  pk.x = Pack2<T>::pack(acc.x * inv, acc.y * inv);
  pk.y = Pack2<T>::pack(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(dst) = pk;
  if (p.lse != nullptr && d4 == 0)
    p.lse[(int64_t)b * p.H + h] = wsum > 0.f ? mx + logf(wsum) : -INFINITY;
}

// ------------------------------------------------------------------- host side
static int dec_group(int hkv, int max_group) {
  for (int g = max_group; g >= 1; --g)
    if (hkv % g == 0) return g;
  return 1;
}

int decode_num_splits(const fa_decode_args_t* a) {
  if (a->num_splits > 0) return a->num_splits;
  const int max_tokens = a->max_blocks * a->page_size;
  // ~512 tokens per split: enough CTAs to fill 148 SMs several times over with a
  // short tail, while the partial-output traffic stays a few % of the KV bytes.
  int s = (max_tokens + 511) / 512;
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  return s;
}

static int chunks_per_split(const fa_decode_args_t* a, int splits) {
  const int max_chunks = (a->max_blocks * a->page_size + kDecChunk - 1) / kDecChunk;
  return (max_chunks + splits - 1) / splits;
}

size_t decode_workspace_bytes(const fa_decode_args_t* a) {
  const int s = decode_num_splits(a);
  if (s <= 1) return 0;
  const size_t n = (size_t)a->batch * s * a->num_heads;
  return (n * a->head_dim + n) * sizeof(float) + 256;
}

template <typename T, int D, bool KV8>
static int launch_decode_impl(const CUtensorMap& tk, const CUtensorMap& tv, const DecParams& p,
                              cudaStream_t st) {
  using Cfg = DecCfg<D, KV8>;
  auto kern = fa_decode_split_kernel<T, D, KV8>;
  static std::atomic<bool> attr_set[kMaxContexts];
  if (int s = smem_attr_once(kern, Cfg::SMEM_BYTES, attr_set)) return s;
  dim3 grid(p.num_splits, p.Hkv / p.HG, p.B);
  // Shared memory for the actual group: small groups (few kv heads) fit several CTAs
  // per SM, which keeps enough K/V bytes in flight.
  const int smem =
      1024 + Cfg::STAGES * 2 * p.HG * Cfg::HEAD_BYTES + 256 + p.HG * Cfg::XCH_BYTES_PER_HEAD;
  prof_begin(FA_PROF_DECODE, st);
  kern<<<grid, 32 + 32 * p.HG * Cfg::WPH, smem, st>>>(tk, tv, p);
  prof_end(FA_PROF_DECODE, st);
  FA_CUDA_TRY(cudaGetLastError());
  count_launch();
  if (p.num_splits > 1) {
    constexpr int HPB = 256 / (D / 4);
    dim3 g2((p.H + HPB - 1) / HPB, p.B);
    fa_decode_combine_kernel<T, D><<<g2, 256, 0, st>>>(p);
    FA_CUDA_TRY(cudaGetLastError());
    count_launch();
  }
  return FA_OK;
}

int launch_decode(const fa_decode_args_t* a, void* ws, size_t ws_bytes, int* err,
                  cudaStream_t st) {
  const int D = a->head_dim;
  if (D != 64 && D != 128 && D != 256 && D != 512) return FA_ERR_UNSUPPORTED;
  const int G = a->num_heads / a->num_kv_heads;
  if (G > 16) return FA_ERR_UNSUPPORTED;
  const int ps = a->page_size;
  if (ps < kDecChunk || (ps & (ps - 1)) != 0) return FA_ERR_UNSUPPORTED;
  if (a->kv_dtype != 0 && a->kv_dtype != FA_DTYPE_E4M3) return FA_ERR_UNSUPPORTED;
  const bool kv8 = a->kv_dtype == FA_DTYPE_E4M3;
  if (kv8 && D == 64) return FA_ERR_UNSUPPORTED;  // fp8 rows of 64 bytes: not built
  if (kv8 && !(a->k_scale > 0.f && a->v_scale > 0.f && std::isfinite(a->k_scale) &&
               std::isfinite(a->v_scale)))
    return FA_ERR_INVALID_ARG;
  if (a->batch == 0) return FA_OK;
  const int splits = decode_num_splits(a);
  if (decode_workspace_bytes(a) > ws_bytes || (splits > 1 && ws == nullptr))
    return FA_ERR_WORKSPACE;
  const CUtensorMapDataType dt = kv8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : tmap_dtype(a->dtype);
  const uint64_t eb = kv8 ? 1 : 2;  // cache bytes per element
  CUtensorMap tk, tv;
  const void* kv_ptr[2] = {a->k_cache, a->v_cache};
  CUtensorMap* kv_map[2] = {&tk, &tv};
  for (int w = 0; w < 2; ++w) {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)a->num_kv_heads, (uint64_t)ps,
                              (uint64_t)a->num_pages};
    const uint64_t str[3] = {(uint64_t)D * eb, (uint64_t)a->num_kv_heads * D * eb,
                             (uint64_t)ps * a->num_kv_heads * D * eb};
    const uint32_t box[4] = {(uint32_t)(128 / eb), 1, (uint32_t)kDecChunk, 1};
    FA_TMAP_TRY(encode_tmap(kv_map[w], dt, 4, kv_ptr[w], dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  DecParams p{};
  p.q = a->q;
  p.out = a->out;
  p.lse = a->lse;
  p.block_table = a->block_table;
  p.seq_lens = a->seq_lens;
  p.B = a->batch;
  p.H = a->num_heads;
  p.Hkv = a->num_kv_heads;
  p.G = G;
  p.HG = dec_group(a->num_kv_heads, dec_maxg(D, kv8));
  p.page_size = ps;
  p.num_pages = a->num_pages;
  p.max_blocks = a->max_blocks;
  p.num_splits = splits;
  p.chunks_per_split = chunks_per_split(a, splits);
  // fp8 caches hold key / k_scale: the true scores are k_scale x (q . k8)
  const float ks = kv8 ? a->k_scale : 1.f;
  p.scale = a->softmax_scale * ks;
  p.scale_log2 = a->softmax_scale * ks * 1.4426950408889634f;
  p.v_scale = kv8 ? a->v_scale : 1.f;
  p.err = err;
  if (splits > 1) {
    const size_t n = (size_t)a->batch * splits * a->num_heads;
    uintptr_t w = (reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255);
    p.o_part = reinterpret_cast<float*>(w);
    p.lse_part = p.o_part + n * D;
  }
  const bool bf16 = a->dtype == FA_DTYPE_BF16;
  if (kv8) {
    if (D == 512)
      return bf16 ? launch_decode_impl<__nv_bfloat16, 512, true>(tk, tv, p, st)
                  : launch_decode_impl<__half, 512, true>(tk, tv, p, st);
    if (D == 256)
      return bf16 ? launch_decode_impl<__nv_bfloat16, 256, true>(tk, tv, p, st)
                  : launch_decode_impl<__half, 256, true>(tk, tv, p, st);
    return bf16 ? launch_decode_impl<__nv_bfloat16, 128, true>(tk, tv, p, st)
                : launch_decode_impl<__half, 128, true>(tk, tv, p, st);
  }
  if (D == 64)
    return bf16 ? launch_decode_impl<__nv_bfloat16, 64, false>(tk, tv, p, st)
                : launch_decode_impl<__half, 64, false>(tk, tv, p, st);
  if (D == 512)
    return bf16 ? launch_decode_impl<__nv_bfloat16, 512, false>(tk, tv, p, st)
                : launch_decode_impl<__half, 512, false>(tk, tv, p, st);
  if (D == 256)
    return bf16 ? launch_decode_impl<__nv_bfloat16, 256, false>(tk, tv, p, st)
                : launch_decode_impl<__half, 256, false>(tk, tv, p, st);
  return bf16 ? launch_decode_impl<__nv_bfloat16, 128, false>(tk, tv, p, st)
              : launch_decode_impl<__half, 128, false>(tk, tv, p, st);
}

// ------------------------------------------------------------------- no-allocation decode
// Scratch for fa_decode_noalloc: the per-split partial outputs and LSEs live in this
// fixed device array instead of a caller-provided workspace.  Every GPU that loads the
// library holds it until the process exits.  In host code the name is only a
// stand-in for the symbol; its device address comes from cudaGetSymbolAddress.
constexpr size_t kDecodeStaticScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_decode_scratch[kDecodeStaticScratchBytes];

static std::mutex g_scratch_mu;
static void* g_scratch_addr[kMaxContexts] = {nullptr};  // per context slot

size_t decode_noalloc_scratch_bytes() { return kDecodeStaticScratchBytes; }

int launch_decode_noalloc(const fa_decode_args_t* a, int* err, cudaStream_t st) {
  const int slot = call_context_slot();
  if (slot < 0 || slot >= kMaxContexts) return FA_ERR_CUDA;
  void* scratch = nullptr;
  {
    // First call in a context (each GPU's primary context, or any other context the
    // caller's stream belongs to): look up the array's device address with that
    // context current -- the entry point bound it.
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (g_scratch_addr[slot] == nullptr) {
      void* ptr = nullptr;
      FA_CUDA_TRY(cudaGetSymbolAddress(&ptr, g_decode_scratch));
      g_scratch_addr[slot] = ptr;
    }
    scratch = g_scratch_addr[slot];
  }
  fa_decode_args_t b = *a;
  if (b.num_splits == 0) {
    // Heuristic split count, reduced until the partials fit in the static scratch.
    b.num_splits = decode_num_splits(a);
    while (b.num_splits > 1 && decode_workspace_bytes(&b) > kDecodeStaticScratchBytes)
      --b.num_splits;
  }
  const size_t need = decode_workspace_bytes(&b);
  if (need > kDecodeStaticScratchBytes) {
    char msg[160];
    snprintf(msg, sizeof(msg), "needs %zu bytes of split scratch, the static scratch holds %zu",
             need, kDecodeStaticScratchBytes);
    set_error_detail("fa_decode_noalloc", __FILE__, __LINE__, msg);
    return FA_ERR_WORKSPACE;
  }
  // The partials need no clearing: the combine reads only the splits that the split
  // kernel wrote for the current call (derived from seq_lens).
  return launch_decode(&b, scratch, kDecodeStaticScratchBytes, err, st);
}

}  // namespace fa
