// prefill_tcgen05.cuh -- compute-bound W4A16 GEMM for M > 32 tokens (prefill)
// on the 5th-generation tensor cores (tcgen05, accumulators in TMEM).
//
// Replaces the reference's Triton kernel (w4a16-kernel/src/w4a16/triton_kernel.py:62-128)
// for large M. One CTA computes a 128 x 256 tile of y; the K loop runs in
// 64-wide steps through a 3-deep shared-memory ring:
//
//   warp 0      TMA producer: x tile [128 x 64] fp16 (128-byte swizzle),
//               packed qweight tile [8 x 256] int32, and the step's scale and
//               zero rows [256] fp16, all on one transaction-counted mbarrier.
//   warps 2..9  dequantisers: thread t owns column t of the tile, unpacks its 8
//               words (magic-number nibble extraction, exact (q - z), one fp16
//               multiply by s: the reference's rounding) and writes the fp16
//               weights K-major into the 128-byte-swizzled B tile, then
//               fence.proxy.async + arrive so the tensor core may read them.
//   warp 1      TMEM allocator + single-thread MMA issuer:
//               tcgen05.mma.cta_group::1.kind::f16, M=128 N=256 K=16, four per
//               step, fp32 accumulator in 256 TMEM columns; tcgen05.commit
//               frees the ring slot.
//   epilogue    warps 2..9 read the accumulator with tcgen05.ld (each warp its
//               32-lane TMEM quarter, 128 columns), round to fp16, add the
//               optional bias (rounded again, as W4A16Linear does) and store.
//
// Every mbarrier wait is bounded; on expiry the CTA raises the sticky device
// error bit, drains its in-flight copies, frees its TMEM and exits.
#pragma once

#include "common.cuh"

namespace w4a16 {
namespace prefill {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 3;
constexpr int A_BYTES = BM * BK * 2;        // 16384
constexpr int B_BYTES = BN * BK * 2;        // 32768
constexpr int P_BYTES = (BK / 8) * BN * 4;  // 8192
constexpr int SZ_BYTES = BN * 2;            // 512
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + P_BYTES + 2 * SZ_BYTES;  // 58368 = 57 KiB
constexpr int TX_BYTES = A_BYTES + P_BYTES + 2 * SZ_BYTES;               // via TMA
constexpr int NUM_WARPS = 10;
constexpr int THREADS = NUM_WARPS * 32;
constexpr int DQ_THREADS = 256;
constexpr uint32_t TMEM_COLS = 256;
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
constexpr uint32_t IDESC = umma_idesc_f16_f32(BM, BN);

static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment");

struct Params {
  const __half* bias;
  __half* y;
  int M, N, K, G;
  long long ldy;
  int vec_store;   // y and ldy allow 16-byte stores
};

// Dequantise one packed word (8 consecutive K of one column) into 8 fp16 in
// natural K order: pairs (k0,k1) (k2,k3) (k4,k5) (k6,k7). Byte b of the word
// holds nibbles (2b, 2b+1); PRMT copies it into bytes 0 and 2, then one LOP3
// keeps the low nibble in the low half (as fp16 1024 + n, magic 0x6400) and
// the high nibble of the copy in the high half (as fp16 64 + n, magic 0x5400,
// nibble at mantissa bits 4-7). zc = (1024+z, 64+z) makes the subtraction exact.
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

__global__ void __launch_bounds__(THREADS, 1)
    w4a16_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_x,
                         const __grid_constant__ CUtensorMap tm_p,
                         const __grid_constant__ CUtensorMap tm_s,
                         const __grid_constant__ CUtensorMap tm_z, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* bfull = full + STAGES;
  uint64_t* empty = bfull + STAGES;
  uint64_t* accfull = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accfull + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM;
  const int n0 = blockIdx.y * BN;
  const int KT = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bfull[s], DQ_THREADS);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accfull, 1);
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer --------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_p);
      int issued = 0;
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % STAGES;
        if (kt >= STAGES) {
          if (!mbar_wait(&empty[s], ((kt / STAGES) - 1) & 1)) break;
        }
        uint8_t* st = smem + s * STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], TX_BYTES);
        tma_load_2d(st, &tm_x, &full[s], kt * BK, m0);
        tma_load_2d(st + A_BYTES + B_BYTES, &tm_p, &full[s], n0, kt * (BK / 8));
        const int grow = (kt * BK) / p.G;
        tma_load_2d(st + A_BYTES + B_BYTES + P_BYTES, &tm_s, &full[s], n0, grow);
        tma_load_2d(st + A_BYTES + B_BYTES + P_BYTES + SZ_BYTES, &tm_z, &full[s], n0, grow);
        ++issued;
      }
      for (int kt = max(0, issued - STAGES); kt < issued; ++kt) {
        mbar_wait(&full[kt % STAGES], (kt / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0) {
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (kt / STAGES) & 1;
        if (!mbar_wait(&full[s], ph)) break;
        if (!mbar_wait(&bfull[s], ph)) break;
        tc_fence_after();
        uint8_t* st = smem + s * STAGE_BYTES;
        const uint64_t adesc = umma_desc_sw128(smem_u32(st));
        const uint64_t bdesc = umma_desc_sw128(smem_u32(st + A_BYTES));
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // advance 16 fp16 = 32 bytes along K inside the swizzled rows
          tc_mma_f16(tmem_base, adesc + static_cast<uint64_t>(kk * 2),
                     bdesc + static_cast<uint64_t>(kk * 2), IDESC, (kt | kk) != 0 ? 1u : 0u);
        }
        tc_commit(&empty[s]);
      }
      tc_commit(accfull);   // also issued on the abort path: tracks whatever is in flight
    }
  } else {
    // ------------------------------ dequantisers --------------------------
    const int t = threadIdx.x - 64;   // column of the tile owned by this thread
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % STAGES;
      if (!mbar_wait(&full[s], (kt / STAGES) & 1)) break;
      uint8_t* st = smem + s * STAGE_BYTES;
      const __half sv = reinterpret_cast<const __half*>(st + A_BYTES + B_BYTES + P_BYTES)[t];
      const __half zv =
          reinterpret_cast<const __half*>(st + A_BYTES + B_BYTES + P_BYTES + SZ_BYTES)[t];
      const uint32_t ss = static_cast<uint32_t>(__half_as_ushort(sv)) * 0x10001u;
      const uint32_t zc =
          static_cast<uint32_t>(__half_as_ushort(__hadd(zv, __float2half_rn(1024.0f)))) |
          (static_cast<uint32_t>(__half_as_ushort(__hadd(zv, __float2half_rn(64.0f)))) << 16);
      const uint32_t* pk = reinterpret_cast<const uint32_t*>(st + A_BYTES + B_BYTES);
      uint8_t* brow = st + A_BYTES + t * 128;
#pragma unroll
      for (int c = 0; c < BK / 8; ++c) {
        const uint32_t w = pk[c * BN + t];
        const uint4 v = dequant_word_nat(w, zc, ss);
        *reinterpret_cast<uint4*>(brow + ((c ^ (t & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(&bfull[s]);
    }

    // ------------------------------ epilogue -------------------------------
    const bool acc_ok = mbar_wait(accfull, 0);
    __syncwarp();   // tcgen05.ld is .sync.aligned: reconverge after the wait loop
    tc_fence_after();
    if (acc_ok) {
      const int quarter = warp & 3;
      const int chalf = (warp - 2) >> 2;
      const int row = quarter * 32 + lane;
      const int m = m0 + row;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        const int col = chalf * 128 + cc * 32;
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + col, r);
        tmem_ld_wait();
        if (m < p.M) {
          __half* yrow = p.y + static_cast<long long>(m) * p.ldy + n0 + col;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const int nb = n0 + col + v * 8;
            if (nb >= p.N) break;
            uint32_t packed[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __half lo = __float2half_rn(__uint_as_float(r[v * 8 + 2 * e]));
              __half hi = __float2half_rn(__uint_as_float(r[v * 8 + 2 * e + 1]));
              if (p.bias != nullptr) {
                lo = __float2half_rn(__half2float(lo) + __half2float(p.bias[nb + 2 * e]));
                hi = __float2half_rn(__half2float(hi) + __half2float(p.bias[nb + 2 * e + 1]));
              }
              packed[e] = static_cast<uint32_t>(__half_as_ushort(lo)) |
                          (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
            }
            if (p.vec_store) {
              *reinterpret_cast<uint4*>(yrow + v * 8) =
                  make_uint4(packed[0], packed[1], packed[2], packed[3]);
            } else {
              const __half* hp = reinterpret_cast<const __half*>(packed);
#pragma unroll
              for (int e = 0; e < 8; ++e) yrow[v * 8 + e] = hp[e];
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // The accumulator barrier completes once every issued MMA has finished.
    mbar_wait(accfull, 0);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace prefill
}  // namespace w4a16
