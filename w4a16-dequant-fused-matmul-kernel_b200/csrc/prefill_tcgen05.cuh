// prefill_tcgen05.cuh -- compute-bound W4A16 GEMM for M > 32 tokens (prefill)
// on the 5th-generation tensor cores (tcgen05, accumulators in TMEM).
//
// Replaces the reference's Triton kernel (w4a16-kernel/src/w4a16/triton_kernel.py:62-128)
// for large M. Persistent CTAs (one per SM) walk 256 x 128 output tiles; the
// K loop of a tile runs in 64-wide steps. Each dequantised weight tile feeds
// two M=128 MMAs (the two 128-row halves of the x tile), which halves the
// CUDA-core dequantisation work per tensor-core FLOP -- the dequantisation,
// not the MMA, is what bounds a W4A16 GEMM. Warp roles:
//
//   warp 0       TMA producer: per step the x tile [256 x 64] fp16 (128-byte
//                swizzle), the packed qweight tile [8 x 128] int32 and the
//                step's scale and zero rows [128] fp16 into a 4-deep ring, all
//                on one transaction-counted mbarrier.
//   warps 2..9   dequantisers: two threads per tile column, each unpacking
//                4 of the column's 8 words of the step (PRMT + LOP3 magic-number
//                nibble extraction, exact (q - z), one fp16 multiply by s: the
//                reference's rounding) and writes the fp16 weights K-major into
//                a 128-byte-swizzled B tile of a 3-deep ring, then
//                fence.proxy.async so the tensor core may read them.
//   warp 1       TMEM allocator (512 columns: two accumulator sets, each two
//                128x128 fp32 halves) and single-thread MMA issuer:
//                tcgen05.mma.cta_group::1.kind::f16, M=128 N=128 K=16, eight
//                per step; tcgen05.commit frees the ring slots and, after a
//                tile's last step, hands its accumulators to the epilogue.
//   warps 10..13 epilogue: each warp reads its 32-lane TMEM quarter of both
//                halves with tcgen05.ld, rounds to fp16, adds the optional bias
//                (rounded again, as W4A16Linear's separate add does) and
//                stores; the double-buffered accumulators let this overlap the
//                next tile's main loop.
//
// Every mbarrier wait is bounded; on expiry the role raises the sticky device
// error bit and leaves its loops, the producer drains its in-flight copies,
// the MMA issuer waits for its last MMAs, and TMEM is freed before exit.
#pragma once

#include "common.cuh"

namespace w4a16 {
namespace prefill {

constexpr int BM = 256;                      // two 128-row MMA halves
constexpr int BMH = 128;
constexpr int BN = 128;
constexpr int BK = 64;
constexpr int TSTAGES = 4;                   // TMA ring depth
constexpr int BSTAGES = 3;                   // dequantised-B ring depth
constexpr int A_BYTES = BM * BK * 2;         // 32768
constexpr int P_BYTES = (BK / 8) * BN * 4;   // 4096
constexpr int SZ_BYTES = BN * 2;             // 256
constexpr int T_BYTES = 37 * 1024;           // A + P + 2 SZ = 37376, padded to keep 1024-byte alignment
constexpr int TX_BYTES = A_BYTES + P_BYTES + 2 * SZ_BYTES;
constexpr int B_BYTES = BN * BK * 2;         // 16384
constexpr int DQ_WARPS = 8;                  // two threads per tile column, 4 words each
constexpr int EPI_WARPS = 4;
constexpr int NUM_WARPS = 2 + DQ_WARPS + EPI_WARPS;
constexpr int THREADS = NUM_WARPS * 32;
constexpr int EPI_WARP0 = 2 + DQ_WARPS;
constexpr uint32_t ACC_COLS = 2 * BN;        // one accumulator set: two 128-column halves
constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = 1024 + TSTAGES * T_BYTES + BSTAGES * B_BYTES + BAR_BYTES;
constexpr uint32_t IDESC = umma_idesc_f16_f32(BMH, BN);

static_assert(TX_BYTES <= T_BYTES, "TMA stage layout");
static_assert(T_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "tiles must keep 1024-byte alignment");
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

struct Params {
  const __half* bias;
  void* y;         // fp16, or fp32 when y_f32 (unrounded partial sums, no bias)
  int y_f32;
  int M, N, K, G;
  int g_shift;     // log2(G) when G is a power of two, else -1
  long long ldy;
  int m_tiles, n_tiles;
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

// Lane 0 waits, the warp follows: keeps mbarrier polling off the shared-memory pipe.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity);
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  __syncwarp();
  return ok;
}

struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void advance(int depth) {
    if (++slot == depth) { slot = 0; phase ^= 1u; }
  }
};

__global__ void __launch_bounds__(THREADS, 1)
    w4a16_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_x,
                         const __grid_constant__ CUtensorMap tm_p,
                         const __grid_constant__ CUtensorMap tm_s,
                         const __grid_constant__ CUtensorMap tm_z, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* tring = smem;                                   // TSTAGES x {A, P, S, Z}
  uint8_t* bring = smem + TSTAGES * T_BYTES;               // BSTAGES x B
  uint64_t* bars = reinterpret_cast<uint64_t*>(bring + BSTAGES * B_BYTES);
  uint64_t* tfull = bars;
  uint64_t* tempty = tfull + TSTAGES;
  uint64_t* bfull = tempty + TSTAGES;
  uint64_t* bempty = bfull + BSTAGES;
  uint64_t* accfull = bempty + BSTAGES;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KT = p.K / BK;
  const int ntiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TSTAGES; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 1);
    }
    for (int j = 0; j < BSTAGES; ++j) {
      mbar_init(&bfull[j], DQ_WARPS);
      mbar_init(&bempty[j], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accfull[a], 1);
      mbar_init(&accempty[a], EPI_WARPS);
    }
    mbar_init(drain, 1);
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
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_z);
      Ring r;
      long long issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
        const int m0 = (tile % p.m_tiles) * BM;
        const int n0 = (tile / p.m_tiles) * BN;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&tempty[r.slot], r.phase ^ 1u)) { ok = false; break; }
          uint8_t* st = tring + r.slot * T_BYTES;
          const int kk = kt * BK;
          const int grow = p.g_shift >= 0 ? kk >> p.g_shift : kk / p.G;
          mbar_arrive_expect_tx(&tfull[r.slot], TX_BYTES);
          tma_load_2d(st, &tm_x, &tfull[r.slot], kk, m0);
          tma_load_2d(st + A_BYTES, &tm_p, &tfull[r.slot], n0, kt * (BK / 8));
          tma_load_2d(st + A_BYTES + P_BYTES, &tm_s, &tfull[r.slot], n0, grow);
          tma_load_2d(st + A_BYTES + P_BYTES + SZ_BYTES, &tm_z, &tfull[r.slot], n0, grow);
          r.advance(TSTAGES);
          ++issued;
        }
      }
      // Never leave with copies in flight: wait for the newest phase of every slot used.
      const long long n = issued < TSTAGES ? issued : TSTAGES;
      for (long long i = 0; i < n; ++i) {
        if (r.slot == 0) { r.slot = TSTAGES; r.phase ^= 1u; }
        --r.slot;
        mbar_wait(&tfull[r.slot], r.phase);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0) {
      Ring t, b;
      bool ok = true;
      int local = 0;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++local) {
        const int a = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&accempty[a], aph ^ 1u)) { ok = false; break; }
        tc_fence_after();
        const uint32_t dtmem = tmem_base + a * ACC_COLS;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&tfull[t.slot], t.phase) || !mbar_wait(&bfull[b.slot], b.phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc0 = umma_desc_sw128(smem_u32(tring + t.slot * T_BYTES));
          const uint64_t adesc1 = umma_desc_sw128(smem_u32(tring + t.slot * T_BYTES + A_BYTES / 2));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(bring + b.slot * B_BYTES));
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // advance 16 fp16 = 32 bytes along K inside the swizzled rows
            const uint32_t acc = (kt | kk) != 0 ? 1u : 0u;
            tc_mma_f16(dtmem, adesc0 + static_cast<uint64_t>(kk * 2),
                       bdesc + static_cast<uint64_t>(kk * 2), IDESC, acc);
            tc_mma_f16(dtmem + BN, adesc1 + static_cast<uint64_t>(kk * 2),
                       bdesc + static_cast<uint64_t>(kk * 2), IDESC, acc);
          }
          tc_commit(&tempty[t.slot]);
          tc_commit(&bempty[b.slot]);
          t.advance(TSTAGES);
          b.advance(BSTAGES);
        }
        if (ok) tc_commit(&accfull[a]);
      }
      tc_commit(drain);   // completes once every MMA this thread issued has finished
    }
  } else if (warp < EPI_WARP0) {
    // ------------------------------ dequantisers --------------------------
    const int dt = threadIdx.x - 64;
    const int t = dt & (BN - 1);      // column of the tile owned by this thread
    const int c0 = (dt / BN) * 4;     // its 4 words (32 K) of the step's 8
    Ring tr, br;
    bool ok = true;
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      for (int kt = 0; kt < KT; ++kt) {
        if (!warp_wait(&tfull[tr.slot], tr.phase) || !warp_wait(&bempty[br.slot], br.phase ^ 1u)) {
          ok = false;
          break;
        }
        const uint8_t* st = tring + tr.slot * T_BYTES;
        const __half sv = reinterpret_cast<const __half*>(st + A_BYTES + P_BYTES)[t];
        const __half zv = reinterpret_cast<const __half*>(st + A_BYTES + P_BYTES + SZ_BYTES)[t];
        const uint32_t ss = static_cast<uint32_t>(__half_as_ushort(sv)) * 0x10001u;
        const uint32_t zc =
            static_cast<uint32_t>(__half_as_ushort(__hadd(zv, __float2half_rn(1024.0f)))) |
            (static_cast<uint32_t>(__half_as_ushort(__hadd(zv, __float2half_rn(64.0f)))) << 16);
        const uint32_t* pk = reinterpret_cast<const uint32_t*>(st + A_BYTES);
        uint32_t w[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) w[c] = pk[(c0 + c) * BN + t];
        uint8_t* brow = bring + br.slot * B_BYTES + t * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          *reinterpret_cast<uint4*>(brow + (((c0 + c) ^ (t & 7)) << 4)) =
              dequant_word_nat(w[c], zc, ss);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bfull[br.slot]);
        tr.advance(TSTAGES);
        br.advance(BSTAGES);
      }
    }
  } else {
    // ------------------------------ epilogue -------------------------------
    const int quarter = warp & 3;   // TMEM lanes this warp may access
    int local = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++local) {
      const int a = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!warp_wait(&accfull[a], aph)) break;
      tc_fence_after();
      const int n0 = (tile / p.m_tiles) * BN;
#pragma unroll 1
      for (int cc = 0; cc < 2 * BN / 32; ++cc) {
        const int h = cc / (BN / 32);                 // which 128-row half
        const int col = (cc % (BN / 32)) * 32;        // column within the tile
        const int m = (tile % p.m_tiles) * BM + h * BMH + quarter * 32 + lane;
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + a * ACC_COLS + h * BN + col +
                               (static_cast<uint32_t>(quarter * 32) << 16), r);
        tmem_ld_wait();
        if (m < p.M && p.y_f32) {
          float* yrow = static_cast<float*>(p.y) + static_cast<long long>(m) * p.ldy + n0 + col;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            if (n0 + col + v * 8 >= p.N) break;
            if (p.vec_store) {
              *reinterpret_cast<uint4*>(yrow + v * 8) = make_uint4(r[v * 8], r[v * 8 + 1], r[v * 8 + 2], r[v * 8 + 3]);
              *reinterpret_cast<uint4*>(yrow + v * 8 + 4) =
                  make_uint4(r[v * 8 + 4], r[v * 8 + 5], r[v * 8 + 6], r[v * 8 + 7]);
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) yrow[v * 8 + e] = __uint_as_float(r[v * 8 + e]);
            }
          }
        } else if (m < p.M) {
          __half* yrow = static_cast<__half*>(p.y) + static_cast<long long>(m) * p.ldy + n0 + col;
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
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[a]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    mbar_wait(drain, 0);   // every issued MMA has finished before TMEM is released
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace prefill
}  // namespace w4a16
