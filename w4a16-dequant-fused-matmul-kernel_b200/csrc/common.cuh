// common.cuh -- shared helpers for the sm_100a W4A16 kernels: status plumbing,
// the sticky device error word, bounded mbarrier waits, and the inline PTX for
// TMA, mbarriers and tcgen05 (5th-generation tensor cores with TMEM).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "w4a16_b200.h"

namespace w4a16 {

// ---------------------------------------------------------------------------
// Sticky device error word (one per device, lives in this library's module;
// the library is one translation unit, so this is its only definition).
// Bit 0: a bounded pipeline wait expired and a CTA abandoned its tile.
// ---------------------------------------------------------------------------
constexpr uint32_t kErrWaitTimeout = 1u;
__device__ uint32_t g_device_error = 0;

// Default time budget of one bounded wait, in nanoseconds of %globaltimer. Every
// legitimate wait in these kernels is bounded by one CTA's own pipeline (at
// most milliseconds even for very long K) or by the peers' matching launches, so
// 4 s only expires on a lost wait, while still allowing for time-slicing with
// other contexts. The host passes the budget to every launch (kernel parameter),
// so a caller can shorten it (w4a16_set_wait_budget_ns).
constexpr uint64_t kWaitBudgetNs = 4ull * 1000ull * 1000ull * 1000ull;

__device__ __forceinline__ void flag_error(uint32_t bits) {
  atomicOr(&g_device_error, bits);
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// Small PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  // (a & mask) | orv in one LOP3 (immLut 0xEA = (A & B) | C).
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Dequantise one packed word (8 consecutive K of one column) into 8 fp16 in
// natural K order: pairs (k0,k1) (k2,k3) (k4,k5) (k6,k7). Byte b of the word
// holds nibbles (2b, 2b+1); PRMT copies it into bytes 0 and 2, then one LOP3
// keeps the low nibble in the low half (as fp16 1024 + n, magic 0x6400) and
// the high nibble of the copy in the high half (as fp16 64 + n, magic 0x5400,
// nibble at mantissa bits 4-7). zc = (1024+z, 64+z) makes the subtraction
// exact; one fp16 multiply by ss = (s, s) is the reference's (q - z) * s.
__device__ __forceinline__ uint32_t dequant_byte_pair(uint32_t w, uint32_t sel, uint32_t zc,
                                                      uint32_t ss) {
  const uint32_t t = lop3_and_or(prmt(w, 0u, sel), 0x00F0000Fu, 0x54006400u);
  return hmul2_u32(hsub2_u32(t, zc), ss);
}

__device__ __forceinline__ uint4 dequant_word_nat(uint32_t w, uint32_t zc, uint32_t ss) {
  uint4 r;
  r.x = dequant_byte_pair(w, 0x4040u, zc, ss);
  r.y = dequant_byte_pair(w, 0x4141u, zc, ss);
  r.z = dequant_byte_pair(w, 0x4242u, zc, ss);
  r.w = dequant_byte_pair(w, 0x4343u, zc, ss);
  return r;
}

// (1024 + z, 64 + z) as one half2, from the fp16 bits of z: the subtrahend of
// dequant_word_nat.
__device__ __forceinline__ uint32_t zero_pair_nat(uint32_t zbits) {
  const __half zv = __ushort_as_half(static_cast<unsigned short>(zbits));
  return static_cast<uint32_t>(__half_as_ushort(__hadd(zv, __float2half_rn(1024.0f)))) |
         (static_cast<uint32_t>(__half_as_ushort(__hadd(zv, __float2half_rn(64.0f)))) << 16);
}

__device__ __forceinline__ uint32_t hadd2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Dequantise one packed word into 4 half2 pairs with one shift and four LOP3s:
// p[j] = (nibble j, nibble j + 4) for j = 0..3 (the low half from bits 4j..4j+3, the
// high half from bits 4j+16..4j+19). In the reference's nibble order (row 8i+j at
// nibble j) that is (k0,k4) (k1,k5) (k2,k6) (k3,k7); in the kernel order w4a16_repack
// writes (nibbles k0,k2,k4,k6,k1,k3,k5,k7) it is (k0,k1) (k2,k3) (k4,k5) (k6,k7).
// za = half2(1024+z), zb = half2(64+z), ss = half2(s): (q - z) exact, one rounding at * s.
__device__ __forceinline__ void dequant_word_perm(uint32_t w, uint32_t za, uint32_t zb, uint32_t ss,
                                                  uint32_t (&p)[4]) {
  const uint32_t w8 = w >> 8;
  p[0] = hmul2_u32(hsub2_u32(lop3_and_or(w, 0x000F000Fu, 0x64006400u), za), ss);
  p[1] = hmul2_u32(hsub2_u32(lop3_and_or(w, 0x00F000F0u, 0x54005400u), zb), ss);
  p[2] = hmul2_u32(hsub2_u32(lop3_and_or(w8, 0x000F000Fu, 0x64006400u), za), ss);
  p[3] = hmul2_u32(hsub2_u32(lop3_and_or(w8, 0x00F000F0u, 0x54005400u), zb), ss);
}

// The output rounding of every GEMM epilogue: fp32 v to fp16 (or bf16 when `bf16`),
// then, with a bias of the same type, y + bias[n] rounded again (W4A16Linear's
// separate add). Returns the 16 bits.
__device__ __forceinline__ uint32_t out_bits(float v, const void* bias, long long n, bool bf16) {
  if (bf16) {
    __nv_bfloat16 h = __float2bfloat16_rn(v);
    if (bias != nullptr)
      h = __float2bfloat16_rn(__bfloat162float(h) + __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[n]));
    return __bfloat16_as_ushort(h);
  }
  __half h = __float2half_rn(v);
  if (bias != nullptr) h = __float2half_rn(__half2float(h) + __half2float(static_cast<const __half*>(bias)[n]));
  return __half_as_ushort(h);
}

// SwiGLU of one output element: h = fp16(silu(g) * u) of the fp16-rounded gate and
// up values, in fp32 with one final rounding. Every path (the separate kernel on an
// fp16 gate/up output, and the GEMM epilogues that fuse it) uses this function.
__device__ __forceinline__ __half swiglu_h(float g, float u) {
  const float gh = __half2float(__float2half_rn(g));
  const float uh = __half2float(__float2half_rn(u));
  return __float2half_rn(gh / (1.0f + expf(-gh)) * uh);
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  // Streamed once: keep it out of L1.
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Streamed once per CTA and tile: keep it out of L1.
__device__ __forceinline__ uint32_t ldg_nc_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg_nc_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// try_wait suspends the thread until the phase completes or the hinted time
// (ns) passes, so a waiting warp issues almost nothing while it waits. (Measured
// on B200: the hint length does not change the hand-off latency of any kernel here;
// the form without a hint, and 20 us, gave the same times.)
constexpr uint32_t kSuspendHintNs = 1000000u;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity has completed. Returns false (and
// raises the sticky error bit) when `budget_ns` of %globaltimer runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t budget_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 7u) == 0u && global_timer_ns() - t0 > budget_ns) break;
  }
  flag_error(kErrWaitTimeout);
  return false;
}

// mbar_wait that sleeps `sleep_ns` between polls: for roles whose waits are long or
// off the critical path (an epilogue waiting for a tile's accumulators, dequantisers
// running ahead of the MMAs), so that their polling leaves the issue slots to the
// warps doing work -- on a busy SM a spinning poller slows the MMA issuer's own waits.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, uint64_t budget_ns,
                                                  uint32_t sleep_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(sleep_ns);
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 7u) == 0u && global_timer_ns() - t0 > budget_ns) break;
  }
  flag_error(kErrWaitTimeout);
  return false;
}

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* m, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// TMA tensor store from shared memory (bulk-group completion). Rows/columns of
// the box outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* smem_src, int32_t x,
                                             int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
// The same store with an L2 cache policy (e.g. l2_evict_first() for output that no
// later CTA of the launch reads, so it does not push the inputs out of L2).
__device__ __forceinline__ void tma_store_2d_hint(const CUtensorMap* m, const void* smem_src, int32_t x,
                                                  int32_t y, uint64_t policy) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y), "l"(policy)
               : "memory");
}
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until every committed bulk store has finished reading its shared-memory source.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until at most one committed bulk store still reads its shared-memory source.
__device__ __forceinline__ void bulk_wait_group_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// Wait until every committed bulk store has completed.
__device__ __forceinline__ void bulk_wait_group0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 / TMEM
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
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

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem desc)^T, fp16 inputs, fp32 accumulate. A (M=128 rows)
// lives in tensor memory: row i in lane i, K elements packed two per 32-bit column,
// so one K=16 step reads 8 columns from a_tmem.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Each thread of the warp writes 16 consecutive columns of its TMEM lane (warp's
// 32-lane quarter); tmem_st_wait() returns once the warp's stores have completed.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrive once on the mbarrier when every tcgen05 op this thread issued so far completes.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Each thread of the warp reads its TMEM lane (warp's 32-lane quarter) x 32 columns.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major tile stored in the 128-byte
// swizzle layout: rows of 64 fp16 (128 B), 8-row atoms of 1024 B; SBO = 1024 B
// between atoms along M/N; LBO unused for this layout; version field = 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;            // LBO (ignored for SW128 K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;    // SBO
  d |= static_cast<uint64_t>(1u) << 46;            // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;            // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: A = B = fp16, D = fp32, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(uint32_t M, uint32_t N) {
  return (1u << 4)                // D format: f32
         | (0u << 7)              // A format: f16
         | (0u << 10)             // B format: f16
         | ((N >> 3) << 17)       // N / 8
         | ((M >> 4) << 24);      // M / 16
}

}  // namespace w4a16

// Host-side launch status helper.
#define W4A16_RETURN_IF_LAUNCH_FAILED()                  \
  do {                                                   \
    cudaError_t e_ = cudaGetLastError();                 \
    if (e_ != cudaSuccess) return W4A16_ERR_LAUNCH;      \
  } while (0)
