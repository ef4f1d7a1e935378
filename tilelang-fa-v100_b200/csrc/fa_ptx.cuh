// Thin inline-PTX wrappers for sm_100a: mbarriers, TMA (cp.async.bulk.tensor),
// tcgen05 (TMEM alloc / MMA / ld / st / commit / fences) and the UMMA shared-memory
// and instruction descriptors.  Every wait on an mbarrier is bounded: a wait that
// runs past FA_WAIT_LIMIT_NS sets the CTA's abort flag and the library's device
// error word and returns false, so a pipeline bug ends the kernel with an error
// status instead of hanging a shared GPU.
//
// Every TMA load is issued by the CTA that consumes it and reads this GPU's own memory;
// no load is shared across the CTAs of a cluster.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#ifndef FA_WAIT_LIMIT_NS
#define FA_WAIT_LIMIT_NS 2000000000ull  // 2 s: far beyond any legitimate wait
#endif

namespace fa {

// Error sites written into the device error word (second slot) on a timeout.
enum : int {
  FA_SITE_FWD_PRODUCER = 1,
  FA_SITE_FWD_MMA = 2,
  FA_SITE_FWD_SOFTMAX = 3,
  FA_SITE_BWD_PRODUCER = 11,
  FA_SITE_BWD_MMA = 12,
  FA_SITE_BWD_COMPUTE = 13,
  FA_SITE_DEC_PRODUCER = 21,
  FA_SITE_DEC_COMPUTE = 22,
  FA_SITE_SELFTEST = 31,
  FA_SITE_PAGED_SEQLEN = 4,
  FA_SITE_DEC_SEQLEN = 23,
};
constexpr int FA_DEVERR_TIMEOUT = 1;
// seq_lens[b] asks for more keys than the sequence's block-table row maps
// (max_blocks * page_size): the keys are clamped to the mapped ones and this is recorded.
constexpr int FA_DEVERR_SEQLEN = 4;



__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Records the first device-side error: err[0] = code, err[1] = site, err[2] = block.
__device__ __forceinline__ void record_device_error(int* err, int code, int site) {
  if (err != nullptr) {
    if (atomicCAS(err, 0, code) == 0) {
      err[1] = site;
      err[2] = static_cast<int>(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
    }
  }
}

// Keys of sequence b that the kernels may read: seq_lens[b] clamped to the pages its
// block-table row maps.  A longer seq_len would otherwise make the zero-filled
// out-of-range loads count as real keys.  `report` selects the thread that records it.
__device__ __forceinline__ int clamp_seq_len(int len, int max_blocks, int page_size, int* err,
                                             int site, bool report) {
  const int cap = max_blocks * page_size;
  if (len > cap) {
    if (report) record_device_error(err, FA_DEVERR_SEQLEN, site);
    return cap;
  }
  return len;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  `abort_flag` is a CTA-shared word: once any role of the CTA has
// timed out, every other wait gives up quickly as well.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* err, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (*abort_flag) return false;
      // Another CTA already timed out: this wait is very likely stuck for the same
      // reason, so give up without waiting out the full limit.
      if (err != nullptr && *reinterpret_cast<volatile int*>(err) != 0 &&
          globaltimer_ns() - t0 > 1000000ull) {
        *abort_flag = 1;
        return false;
      }
      if (globaltimer_ns() - t0 > FA_WAIT_LIMIT_NS) {
        *abort_flag = 1;
        record_device_error(err, FA_DEVERR_TIMEOUT, site);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- named barriers
// Barrier `id` (1..15; 0 is __syncthreads) over `count` threads, whole warps, every warp
// converged.  The reduction form returns the AND of `pred` over all of them, so a
// decision taken after it is uniform across the participating warps.
__device__ __forceinline__ bool bar_red_and(int id, int count, bool pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\tselp.s32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<int>(pred)), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void bar_sync_n(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, uint32_t bar, int c0,
                                            int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
// Tiled TMA store smem -> global (bulk-group completion).  Coordinates must be
// non-negative; the innermost one times the element size a multiple of 16 bytes.
__device__ __forceinline__ void tma_store_4d(const void* tmap, uint32_t src, int c0, int c1, int c2,
                                             int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tmap)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until the committed bulk stores have read their shared-memory source (the
// global writes then complete on their own before the grid completes).
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Waits until every committed bulk operation of this thread has completed.
__device__ __forceinline__ void bulk_wait_group_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Element-wise fp32 add of `bytes` (a multiple of 16; both addresses 16-byte aligned)
// from shared memory into global memory, performed at L2 (bulk-group completion).
__device__ __forceinline__ void bulk_reduce_add_f32(float* dst, uint32_t src, uint32_t bytes) {
  asm volatile(
      "cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(
          reinterpret_cast<uint64_t>(dst)),
      "r"(src), "r"(bytes)
      : "memory");
}
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, uint32_t bar, int c0,
                                            int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
// TMEM address: bits [31:16] lane, bits [15:0] column.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc].  The issuing thread is on the critical
// path of every attention kernel, so descriptors are built once per tile and the
// per-K-step ones are base + constant (desc_add); no compiler memory clobber here --
// ordering against other async tcgen05 work comes from volatile issue order and the
// mbarrier / commit protocol.
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// The value of x, opaque to the compiler at this point: a descriptor laundered inside a
// loop is not hoisted (with everything derived from it) out of the loop, which keeps the
// MMA issuer's unrolled descriptor sets from occupying registers across the whole loop.
__device__ __forceinline__ uint64_t opaque(uint64_t x) {
  asm volatile("" : "+l"(x));
  return x;
}
// Descriptor of a sub-tile `byte_off` bytes past the one `d` describes (the start
// address field holds addr >> 4 in its low 14 bits; shared addresses stay < 256 KB).
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t byte_off) {
  return d + static_cast<uint64_t>(byte_off >> 4);
}
// Arrive (once) on `bar` when every tcgen05 async op issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32-bit: thread i of the warp receives 32 consecutive columns of lane i.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// ---------------------------------------------------------------- descriptors
// UMMA shared-memory descriptor for a 128-byte-swizzled tile whose swizzle atoms
// (8 rows x 128 B) start on 1024-byte boundaries.
//   K-major operand : rows are M/N, 128 B of K per row; SBO = stride between
//                     8-row groups (1024 B when packed), LBO unused (16 B).
//   MN-major operand: rows are K, 128 B (64 x 16-bit) of M/N per row; LBO =
//                     stride between 64-wide M/N chunks, SBO = stride between
//                     8-row K groups.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // 128-byte swizzle
  return d;
}
// Instruction descriptor for kind::f16 with fp32 accumulation.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool bf16, bool a_mn_major,
                                                 bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------- tracing
// Compiled in only with -DFA_TRACE (a separate diagnostic build): records
// %globaltimer at named phases of the first FA_TRACE_CTAS CTAs so the pipeline's
// per-phase latencies can be read back with fa_debug_trace_read().
#ifdef FA_TRACE
constexpr int FA_TRACE_CTAS = 2, FA_TRACE_EVENTS = 24, FA_TRACE_ITERS = 64;
// One copy per translation unit (no relocatable device code); the unit that traces
// also exports the reader.
static __device__ unsigned long long g_fa_trace[FA_TRACE_CTAS][FA_TRACE_EVENTS][FA_TRACE_ITERS];
#define FA_TRACE_EVENT(ev, it)                                                              \
  do {                                                                                      \
    const unsigned cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);   \
    if (cta_ < (unsigned)FA_TRACE_CTAS && (it) < FA_TRACE_ITERS)                            \
      g_fa_trace[cta_][(ev)][(it)] = ::fa::globaltimer_ns();                                \
  } while (0)
// Same slots, SM clock cycles instead of nanoseconds (for the achieved clock rate).
#define FA_TRACE_CYCLES(ev, it)                                                             \
  do {                                                                                      \
    const unsigned cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);   \
    if (cta_ < (unsigned)FA_TRACE_CTAS && (it) < FA_TRACE_ITERS)                            \
      g_fa_trace[cta_][(ev)][(it)] = clock64();                                             \
  } while (0)
#else
#define FA_TRACE_CYCLES(ev, it) \
  do {                          \
  } while (0)
#define FA_TRACE_EVENT(ev, it) \
  do {                         \
  } while (0)
#endif

// ---------------------------------------------------------------- register split
// setmaxnreg: executed by every warp of a warpgroup; the raised counts of all
// warpgroups together must fit the block's launch allocation (checked on the host).
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------- misc math
// max(a, b, c) in one instruction (three-input max.f32, sm_100+).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float y;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
  return y;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Softcapped score in raw-score units (FA2 softcap c, softmax scale sc):
// a * tanh(s / a) with a = c / sc, so that scale * result = c * tanh(scale * s / c) and the
// softmax around it is unchanged.  From tanh(u) = 1 - 2 / (1 + e^(2u)) with e^(2u) =
// 2^(k s), k = 2 log2(e) / a: one exponential, one reciprocal.  Saturates to +-a (e^(2u)
// overflowing to +inf gives a reciprocal of 0).  The absolute error is a few units of
// 2^-23 * a (ex2 and rcp are both within about 2 ulp); for small |u| the result is a
// difference near 0 with the same absolute error, which is what the softmax sees.
__device__ __forceinline__ float softcap_score(float s, float a, float k) {
  return fmaf(-2.f * a, rcp_approx(1.f + ex2_approx(s * k)), a);
}
// P * (1 - tanh^2) for a softcapped score, from P alone: the capped score times
// scale * log2(e) is lg2(P) + lse2, so tanh = (lg2(P) + lse2) * t_k with
// t_k = 1 / (log2(e) * softcap).  P = 0 (masked or underflowed) gives 0.
__device__ __forceinline__ float softcap_grad_p(float pv, float lse2, float t_k) {
  const float t = (lg2_approx(pv) + lse2) * t_k;
  return pv > 0.f ? pv * fmaf(-t, t, 1.f) : 0.f;
}
template <typename T>
struct Pack2;
template <>
struct Pack2<__half> {
  __device__ __forceinline__ static uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static float2 unpack(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
  }
  static constexpr bool kBf16 = false;
};
template <>
struct Pack2<__nv_bfloat16> {
  __device__ __forceinline__ static uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static float2 unpack(uint32_t u) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&u);
    return __bfloat1622float2(h);
  }
  static constexpr bool kBf16 = true;
};

}  // namespace fa
