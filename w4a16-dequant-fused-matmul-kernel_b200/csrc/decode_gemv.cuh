// decode_gemv.cuh -- memory-bound W4A16 GEMM for M <= 32 tokens (decode).
//
// Replaces the reference's Triton K-loop (w4a16-kernel/src/w4a16/triton_kernel.py:99-124)
// for the decode regime, where the packed weights are read exactly once and
// the roofline is HBM bandwidth.
//
// Design (B200):
//  * One producer warp streams the CTA's column strip of qweight (128 columns x
//    32 packed rows = 16 KB per stage), its scale/zero rows and the matching
//    [M x 256] slice of x into a shared-memory ring with TMA; mbarriers with
//    transaction counts track each stage. TMA gives deep memory-level
//    parallelism without holding prefetched data in registers.
//  * Eight consumer warps dequantise in registers -- magic-number nibble
//    extraction (OR the nibble into the mantissa of fp16 1024 or 64, then
//    subtract 1024+z or 64+z: exact), then one fp16 multiply by the scale,
//    which reproduces the reference's fp16 (q - z) * s rounding bit for bit --
//    and feed the fp16 fragments straight into m16n8k16 tensor-core MMAs with
//    fp32 accumulation. The MMA is "swapped": 16 weight columns form the MMA's
//    M side and up to 8 tokens its N side. K is permuted inside each MMA so a
//    lane's 32-bit word supplies its fragment without shuffles; x is permuted
//    identically (a permutation of the summation index leaves the dot product
//    unchanged).
//  * Split-K: the 8 consumer warps split each stage (2 K halves x 4 column
//    quarters) and reduce through shared memory; when one resident wave can
//    hold more CTAs than there are column strips, S CTAs of a thread-block
//    cluster split K further and reduce through distributed shared memory --
//    no global scratch. The grid is sized to one resident wave so that every
//    CTA streams concurrently and none waits for a second wave.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace w4a16 {
namespace decode {

constexpr int BN = 128;             // columns per CTA (a "strip")
constexpr int ROWS = 32;            // packed rows (of 8 K each) per stage
constexpr int KSTAGE = ROWS * 8;    // 256 K per stage
constexpr int NCW = 8;              // consumer warps: 4 column quarters x 2 K halves
constexpr int KP = 2;               // K halves per stage
constexpr int THREADS = 32 * (NCW + 1);
constexpr int SZ_ROWS = 4;          // scale/zero rows per stage (G >= 64 => at most 4 groups)
constexpr int W_BYTES = ROWS * BN * 4;        // 16384
constexpr int SZ_BYTES = SZ_ROWS * BN * 2;    // 1024 (each of scales, zeros)

__host__ __device__ constexpr int x_bytes(int M) { return KSTAGE * 2 * M; }
__host__ __device__ constexpr int stage_bytes(int M) { return W_BYTES + 2 * SZ_BYTES + x_bytes(M); }
__host__ __device__ constexpr int red_bytes(int MT) { return KP * (MT * 8) * BN * 4; }

struct Params {
  const __half* bias;
  __half* y;
  int M, N, K, G;
  long long ldy;
  int stages_per_cta;   // K-stages handled by each CTA of a cluster
  int num_stages;       // ring depth
};

__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Dequantise one packed word into 4 half2 pairs in the K-permuted order the
// MMA fragments use: p[0] = (k0,k4), p[1] = (k1,k5), p[2] = (k2,k6), p[3] = (k3,k7).
// za = half2(1024+z), zb = half2(64+z), ss = half2(s).
__device__ __forceinline__ void dequant_word_perm(uint32_t w, uint32_t za, uint32_t zb, uint32_t ss,
                                                  uint32_t (&p)[4]) {
  const uint32_t w8 = w >> 8;
  p[0] = hmul2_u32(hsub2_u32(lop3_and_or(w, 0x000F000Fu, 0x64006400u), za), ss);
  p[1] = hmul2_u32(hsub2_u32(lop3_and_or(w, 0x00F000F0u, 0x54005400u), zb), ss);
  p[2] = hmul2_u32(hsub2_u32(lop3_and_or(w8, 0x000F000Fu, 0x64006400u), za), ss);
  p[3] = hmul2_u32(hsub2_u32(lop3_and_or(w8, 0x00F000F0u, 0x54005400u), zb), ss);
}

__device__ __forceinline__ uint32_t half2_bcast_u32(__half h) {
  const uint32_t u = __half_as_ushort(h);
  return u | (u << 16);
}

template <int MT>
__global__ void __launch_bounds__(THREADS, 1)
    decode_gemv_tma_kernel(const __grid_constant__ CUtensorMap tm_w,
                           const __grid_constant__ CUtensorMap tm_s,
                           const __grid_constant__ CUtensorMap tm_z,
                           const __grid_constant__ CUtensorMap tm_x, const Params p) {
  namespace cg = cooperative_groups;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int M = p.M;
  const int nst = p.num_stages;
  const int sbytes = stage_bytes(M);
  float* red = reinterpret_cast<float*>(smem + nst * sbytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + nst * sbytes + red_bytes(MT));
  uint64_t* empty = full + nst;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int col0 = blockIdx.x * BN;
  const int split = blockIdx.y;
  const int nsplit = gridDim.y;
  const int total_kst = (p.K + KSTAGE - 1) / KSTAGE;
  const int kst_begin = split * p.stages_per_cta;
  const int kst_end = min(total_kst, kst_begin + p.stages_per_cta);
  const int my_stages = max(0, kst_end - kst_begin);

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NCW);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_x);
      int issued = 0;
      for (int it = 0; it < my_stages; ++it) {
        const int s = it % nst;
        if (it >= nst) {
          if (!mbar_wait(&empty[s], ((it / nst) - 1) & 1)) break;
        }
        uint8_t* st = smem + s * sbytes;
        const int kst = kst_begin + it;
        mbar_arrive_expect_tx(&full[s], sbytes);
        tma_load_2d(st, &tm_w, &full[s], col0, kst * ROWS);
        tma_load_2d(st + W_BYTES, &tm_s, &full[s], col0, (kst * KSTAGE) / p.G);
        tma_load_2d(st + W_BYTES + SZ_BYTES, &tm_z, &full[s], col0, (kst * KSTAGE) / p.G);
        tma_load_2d(st + W_BYTES + 2 * SZ_BYTES, &tm_x, &full[s], kst * KSTAGE, 0);
        ++issued;
      }
      // Never leave with copies in flight: the newest stage of every slot.
      for (int it = max(0, issued - nst); it < issued; ++it) {
        mbar_wait(&full[it % nst], (it / nst) & 1);
      }
    }
  } else {
    // ------------------------------ consumers -----------------------------
    const int cw = warp - 1;
    const int cq = cw & 3;          // column quarter: 32 columns
    const int kp = cw >> 2;         // K half: packed rows [16kp, 16kp+16) of the stage
    const int q = lane >> 2;        // MMA group id: columns 4q..4q+3 of the quarter
    const int g = lane & 3;         // MMA thread-in-group: packed row within a quad
    const int ccol = cq * 32 + 4 * q;

    float acc[2][MT][4];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int tt = 0; tt < MT; ++tt)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[t][tt][r] = 0.0f;

    for (int it = 0; it < my_stages; ++it) {
      const int s = it % nst;
      if (!mbar_wait(&full[s], (it / nst) & 1)) break;
      const uint8_t* st = smem + s * sbytes;
      const int kst = kst_begin + it;
      const int g0 = (kst * KSTAGE) / p.G;   // first scale/zero row held by the stage

#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        // a pair of quads = 64 K: always inside one group since G % 64 == 0
        const int gloc = (kst * KSTAGE + kp * 128 + pr * 64) / p.G - g0;
        const uint2 s4 = *reinterpret_cast<const uint2*>(st + W_BYTES + (gloc * BN + ccol) * 2);
        const uint2 z4 =
            *reinterpret_cast<const uint2*>(st + W_BYTES + SZ_BYTES + (gloc * BN + ccol) * 2);
        uint32_t ss[4], za[4], zb[4];
        {
          const __half* sh = reinterpret_cast<const __half*>(&s4);
          const __half* zh = reinterpret_cast<const __half*>(&z4);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            ss[c] = half2_bcast_u32(sh[c]);
            za[c] = half2_bcast_u32(__hadd(zh[c], __float2half_rn(1024.0f)));
            zb[c] = half2_bcast_u32(__hadd(zh[c], __float2half_rn(64.0f)));
          }
        }
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
          const int iloc = kp * 16 + pr * 8 + qq * 4 + g;   // packed row within the stage
          const uint4 wv = *reinterpret_cast<const uint4*>(st + (iloc * BN + ccol) * 4);
          uint32_t d[4][4];
          dequant_word_perm(wv.x, za[0], zb[0], ss[0], d[0]);
          dequant_word_perm(wv.y, za[1], zb[1], ss[1], d[1]);
          dequant_word_perm(wv.z, za[2], zb[2], ss[2], d[2]);
          dequant_word_perm(wv.w, za[3], zb[3], ss[3], d[3]);
          uint32_t xb[MT][4];
#pragma unroll
          for (int tt = 0; tt < MT; ++tt) {
            const int tok = tt * 8 + q;
            if (tok < M) {
              const uint4 xv = *reinterpret_cast<const uint4*>(st + W_BYTES + 2 * SZ_BYTES +
                                                               tok * (KSTAGE * 2) + iloc * 16);
              xb[tt][0] = prmt(xv.x, xv.z, 0x5410);   // (k0, k4)
              xb[tt][1] = prmt(xv.x, xv.z, 0x7632);   // (k1, k5)
              xb[tt][2] = prmt(xv.y, xv.w, 0x5410);   // (k2, k6)
              xb[tt][3] = prmt(xv.y, xv.w, 0x7632);   // (k3, k7)
            } else {
              xb[tt][0] = xb[tt][1] = xb[tt][2] = xb[tt][3] = 0u;
            }
          }
#pragma unroll
          for (int t = 0; t < 2; ++t) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              // rows q / q+8 of the MMA = columns 2t / 2t+1 of the lane's four
              const uint32_t a[4] = {d[2 * t][2 * h], d[2 * t + 1][2 * h], d[2 * t][2 * h + 1],
                                     d[2 * t + 1][2 * h + 1]};
#pragma unroll
              for (int tt = 0; tt < MT; ++tt) {
                mma_16816(acc[t][tt], a, xb[tt][2 * h], xb[tt][2 * h + 1]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // partial sums of this K half -> red[kp][token][column]
#pragma unroll
    for (int tt = 0; tt < MT; ++tt) {
      const int t0 = tt * 8 + 2 * g;
      float4 v0 = make_float4(acc[0][tt][0], acc[0][tt][2], acc[1][tt][0], acc[1][tt][2]);
      float4 v1 = make_float4(acc[0][tt][1], acc[0][tt][3], acc[1][tt][1], acc[1][tt][3]);
      *reinterpret_cast<float4*>(&red[((kp * MT * 8) + t0) * BN + ccol]) = v0;
      *reinterpret_cast<float4*>(&red[((kp * MT * 8) + t0 + 1) * BN + ccol]) = v1;
    }
  }
  __syncthreads();

  // Reduce the K halves: red[0][t][c] += red[1][t][c].
  const int nout = M * BN;
  for (int idx = threadIdx.x; idx < nout; idx += THREADS) {
    const int t = idx / BN, c = idx % BN;
    red[t * BN + c] += red[(MT * 8 + t) * BN + c];
  }

  cg::cluster_group cluster = cg::this_cluster();
  if (nsplit > 1) cluster.sync();
  else __syncthreads();

  // Each cluster rank finishes a slice of the columns, summing every rank's partial.
  const int cpr = BN / nsplit;             // nsplit divides 128 (1, 2, 4 or 8)
  const int cbeg = split * cpr;
  for (int idx = threadIdx.x; idx < M * cpr; idx += THREADS) {
    const int t = idx / cpr, c = cbeg + idx % cpr;
    float v = 0.0f;
    if (nsplit > 1) {
      for (int r = 0; r < nsplit; ++r) {
        const float* rem = cluster.map_shared_rank(red, r);
        v += rem[t * BN + c];
      }
    } else {
      v = red[t * BN + c];
    }
    const int n = col0 + c;
    if (n < p.N) {
      __half h = __float2half_rn(v);
      if (p.bias != nullptr) h = __float2half_rn(__half2float(h) + __half2float(p.bias[n]));
      p.y[static_cast<long long>(t) * p.ldy + n] = h;
    }
  }
  if (nsplit > 1) cluster.sync();   // keep this CTA's shared memory alive for its peers
}

// ---------------------------------------------------------------------------
// Fallback for shapes the TMA kernel cannot take (N % 8 != 0 or unaligned
// pointers): plain loads, one thread per column, up to 32 tokens, x staged
// through shared memory. Same dequant rounding, fp32 accumulation.
// ---------------------------------------------------------------------------
constexpr int FB_THREADS = 128;
constexpr int FB_KCHUNK = 256;

__global__ void __launch_bounds__(FB_THREADS)
    decode_gemv_fallback_kernel(const __half* __restrict__ x, const int32_t* __restrict__ qw,
                                const __half* __restrict__ scales,
                                const __half* __restrict__ zeros, const __half* __restrict__ bias,
                                __half* __restrict__ y, int M, int N, int K, int G,
                                long long ldy) {
  __shared__ __half xs[32][FB_KCHUNK];
  const int n = blockIdx.x * FB_THREADS + threadIdx.x;
  float acc[32];
#pragma unroll
  for (int m = 0; m < 32; ++m) acc[m] = 0.0f;

  for (int k0 = 0; k0 < K; k0 += FB_KCHUNK) {
    const int kc = min(FB_KCHUNK, K - k0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < M * kc; idx += FB_THREADS) {
      const int m = idx / kc, kk = idx % kc;
      xs[m][kk] = x[static_cast<long long>(m) * K + k0 + kk];
    }
    __syncthreads();
    if (n < N) {
      for (int i = 0; i < kc / 8; ++i) {
        const int k = k0 + i * 8;
        const uint32_t word = static_cast<uint32_t>(qw[static_cast<long long>(k / 8) * N + n]);
        const int gi = k / G;
        const __half s = scales[static_cast<long long>(gi) * N + n];
        const __half z = zeros[static_cast<long long>(gi) * N + n];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const __half qh = __int2half_rn(static_cast<int>((word >> (4 * j)) & 0xFu));
          const float wv = __half2float(__hmul(__hsub(qh, z), s));
#pragma unroll
          for (int m = 0; m < 32; ++m) {
            if (m < M) acc[m] = fmaf(__half2float(xs[m][i * 8 + j]), wv, acc[m]);
          }
        }
      }
    }
  }
  if (n < N) {
#pragma unroll
    for (int m = 0; m < 32; ++m) {
      if (m < M) {
        __half h = __float2half_rn(acc[m]);
        if (bias != nullptr) h = __float2half_rn(__half2float(h) + __half2float(bias[n]));
        y[static_cast<long long>(m) * ldy + n] = h;
      }
    }
  }
}

}  // namespace decode
}  // namespace w4a16
