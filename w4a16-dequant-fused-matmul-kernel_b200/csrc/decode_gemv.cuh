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
//  * Stream-K: the work is a list of units (128-column strip, 256-K stage),
//    strip-major, dealt to one resident wave of CTAs in equal contiguous
//    ranges, so every SM streams the same number of bytes whatever N is.
//    Inside a CTA the 8 consumer warps split each stage (2 K halves x 4
//    column quarters) and reduce through shared memory. A strip whose K range
//    is split between CTAs is finished by the last CTA to arrive (an atomic
//    arrival counter per strip): it sums the pieces in CTA order -- so the
//    result is deterministic -- from a caller-provided workspace, writes y and
//    resets the counter, leaving the workspace clean for the next launch.
#pragma once

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
// Workspace layout: strip arrival counters in a fixed region at offset 0 (so
// that launches of any shape never write partial sums over another shape's
// counters), then the partial sums.
constexpr int MAX_STRIPS = 16384;             // N <= 2,097,152 on the decode path
constexpr size_t COUNTER_BYTES = MAX_STRIPS * sizeof(unsigned);
constexpr int SZ_BYTES = SZ_ROWS * BN * 2;    // 1024 (each of scales, zeros)

__host__ __device__ constexpr int x_bytes(int M) { return KSTAGE * 2 * M; }
__host__ __device__ constexpr int stage_bytes(int M) { return W_BYTES + 2 * SZ_BYTES + x_bytes(M); }
__host__ __device__ constexpr int red_bytes(int MT) { return KP * (MT * 8) * BN * 4; }

struct Params {
  const __half* bias;
  __half* y;
  float* partials;        // [gridDim.x][2][MT*8][BN] fp32 partial sums of split strips
  unsigned* counters;     // [strips] arrival counters, zero between launches
  int M, N, K, G;
  int g_shift;            // log2(G) when G is a power of two, else -1
  long long ldy;
  int kstages;            // K stages per strip (ceil(K / 256))
  long long units;        // strips * kstages
  int num_stages;         // ring depth
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

__device__ __forceinline__ uint32_t hadd2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// First unit of CTA p when U units are dealt to P CTAs in contiguous ranges.
__device__ __forceinline__ long long unit_begin(long long p, long long U, long long P) {
  return (p * U) / P;
}

// Consumer-warp-only barrier (named barrier 1; the producer warp does not take part).
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
}

template <int MT>
__global__ void __maxnreg__(MT <= 2 ? 96 : 168)
    decode_gemv_tma_kernel(const __grid_constant__ CUtensorMap tm_w,
                           const __grid_constant__ CUtensorMap tm_s,
                           const __grid_constant__ CUtensorMap tm_z,
                           const __grid_constant__ CUtensorMap tm_x, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int M = p.M;
  const int nst = p.num_stages;
  const int sbytes = stage_bytes(M);
  float* red = reinterpret_cast<float*>(smem + nst * sbytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + nst * sbytes + red_bytes(MT));
  uint64_t* empty = full + nst;
  int* flag = reinterpret_cast<int*>(empty + nst);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long P = gridDim.x;
  const long long U = p.units;
  const int KS = p.kstages;
  const long long u0 = unit_begin(blockIdx.x, U, P);
  const long long u1 = unit_begin(blockIdx.x + 1, U, P);

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
      int s = 0;
      uint32_t ph = 0;
      long long issued = 0;
      int c = static_cast<int>(u0 / KS);
      int k = static_cast<int>(u0 - static_cast<long long>(c) * KS);
      for (long long u = u0; u < u1; ++u, ++issued) {
        if (issued >= nst) {
          if (!mbar_wait(&empty[s], ph ^ 1)) break;
        }
        uint8_t* st = smem + s * sbytes;
        const int grow = p.g_shift >= 0 ? (k * KSTAGE) >> p.g_shift : (k * KSTAGE) / p.G;
        mbar_arrive_expect_tx(&full[s], sbytes);
        tma_load_2d(st, &tm_w, &full[s], c * BN, k * ROWS);
        tma_load_2d(st + W_BYTES, &tm_s, &full[s], c * BN, grow);
        tma_load_2d(st + W_BYTES + SZ_BYTES, &tm_z, &full[s], c * BN, grow);
        tma_load_2d(st + W_BYTES + 2 * SZ_BYTES, &tm_x, &full[s], k * KSTAGE, 0);
        if (++s == nst) { s = 0; ph ^= 1; }
        if (++k == KS) { k = 0; ++c; }
      }
      // Never leave with copies in flight: wait for the newest stage of every slot.
      const long long n_in_flight = issued < nst ? issued : nst;
      for (long long i = 0; i < n_in_flight; ++i) {
        if (s == 0) { s = nst; ph ^= 1; }
        --s;
        mbar_wait(&full[s], ph);
      }
    }
    return;   // the producer warp takes no part in the consumers' barriers below
  }

  // -------------------------------- consumers ---------------------------------
  const int cw = warp - 1;
  const int ctid = threadIdx.x - 32;
  const int cq = cw & 3;          // column quarter: 32 columns
  const int kp = cw >> 2;         // K half: packed rows [16kp, 16kp+16) of the stage
  const int q = lane >> 2;        // MMA group id: columns 4q..4q+3 of the quarter
  const int g = lane & 3;         // MMA thread-in-group: packed row within a quad
  const int ccol = cq * 32 + 4 * q;
  const bool has_x = q < M;       // lanes whose token of tile 0 exists

  float acc[2][MT][4];
  int s = 0;
  uint32_t ph = 0;
  bool ok = true;
  const int c_first = static_cast<int>(u0 / KS);
  int c = c_first;
  int k = static_cast<int>(u0 - static_cast<long long>(c) * KS);
  int kfirst = k;             // first stage of the current segment within its strip
  for (long long u = u0; u < u1; ++u) {
    if (k == kfirst) {
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int tt = 0; tt < MT; ++tt)
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[t][tt][r] = 0.0f;
    }
    if (ok) {
      // one lane waits, the warp follows (keeps shared-memory polling low)
      bool got = true;
      if (lane == 0) got = mbar_wait(&full[s], ph);
      ok = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
      __syncwarp();   // orders the other lanes' shared-memory reads after lane 0's acquire
    }
    if (ok) {
      const uint8_t* st = smem + s * sbytes;
      const int g0 = p.g_shift >= 0 ? (k * KSTAGE) >> p.g_shift : (k * KSTAGE) / p.G;
#pragma unroll
      for (int pr = 0; pr < 2; ++pr) {
        // a pair of quads = 64 K: always inside one group since G % 64 == 0
        const int kk = k * KSTAGE + kp * 128 + pr * 64;
        const int gloc = (p.g_shift >= 0 ? kk >> p.g_shift : kk / p.G) - g0;
        const uint2 s4 = *reinterpret_cast<const uint2*>(st + W_BYTES + (gloc * BN + ccol) * 2);
        const uint2 z4 =
            *reinterpret_cast<const uint2*>(st + W_BYTES + SZ_BYTES + (gloc * BN + ccol) * 2);
        const uint32_t za01 = hadd2_u32(z4.x, 0x64006400u), za23 = hadd2_u32(z4.y, 0x64006400u);
        const uint32_t zb01 = hadd2_u32(z4.x, 0x54005400u), zb23 = hadd2_u32(z4.y, 0x54005400u);
        const uint32_t ss[4] = {prmt(s4.x, 0, 0x1010), prmt(s4.x, 0, 0x3232),
                                prmt(s4.y, 0, 0x1010), prmt(s4.y, 0, 0x3232)};
        const uint32_t za[4] = {prmt(za01, 0, 0x1010), prmt(za01, 0, 0x3232),
                                prmt(za23, 0, 0x1010), prmt(za23, 0, 0x3232)};
        const uint32_t zb[4] = {prmt(zb01, 0, 0x1010), prmt(zb01, 0, 0x3232),
                                prmt(zb23, 0, 0x1010), prmt(zb23, 0, 0x3232)};
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
          const int iloc = kp * 16 + pr * 8 + qq * 4 + g;   // packed row within the stage
          const uint4 wv = *reinterpret_cast<const uint4*>(st + (iloc * BN + ccol) * 4);
          uint32_t xb[MT][4];
#pragma unroll
          for (int tt = 0; tt < MT; ++tt) {
            const int tok = tt * 8 + q;
            uint4 xv = make_uint4(0u, 0u, 0u, 0u);
            if (tt == 0 ? has_x : tok < M) {
              xv = *reinterpret_cast<const uint4*>(st + W_BYTES + 2 * SZ_BYTES +
                                                   tok * (KSTAGE * 2) + iloc * 16);
            }
            xb[tt][0] = prmt(xv.x, xv.z, 0x5410);   // (k0, k4)
            xb[tt][1] = prmt(xv.x, xv.z, 0x7632);   // (k1, k5)
            xb[tt][2] = prmt(xv.y, xv.w, 0x5410);   // (k2, k6)
            xb[tt][3] = prmt(xv.y, xv.w, 0x7632);   // (k3, k7)
          }
          uint32_t d[4][4];
          dequant_word_perm(wv.x, za[0], zb[0], ss[0], d[0]);
          dequant_word_perm(wv.y, za[1], zb[1], ss[1], d[1]);
          dequant_word_perm(wv.z, za[2], zb[2], ss[2], d[2]);
          dequant_word_perm(wv.w, za[3], zb[3], ss[3], d[3]);
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
    if (++s == nst) { s = 0; ph ^= 1; }

    // ---------------------- end of a segment: reduce and emit ----------------------
    if (k == KS - 1 || u == u1 - 1) {
#pragma unroll
      for (int tt = 0; tt < MT; ++tt) {
        const int t0 = tt * 8 + 2 * g;
        float4 v0 = make_float4(acc[0][tt][0], acc[0][tt][2], acc[1][tt][0], acc[1][tt][2]);
        float4 v1 = make_float4(acc[0][tt][1], acc[0][tt][3], acc[1][tt][1], acc[1][tt][3]);
        *reinterpret_cast<float4*>(&red[((kp * MT * 8) + t0) * BN + ccol]) = v0;
        *reinterpret_cast<float4*>(&red[((kp * MT * 8) + t0 + 1) * BN + ccol]) = v1;
      }
      consumer_sync();
      const bool whole = (kfirst == 0 && k == KS - 1);
      const int col0 = c * BN;
      const int nout = M * BN;
      if (whole) {
        for (int idx = ctid; idx < nout; idx += NCW * 32) {
          const int t = idx / BN, cc = idx % BN;
          const int n = col0 + cc;
          if (n < p.N) {
            const float v = red[t * BN + cc] + red[(MT * 8 + t) * BN + cc];
            __half h = __float2half_rn(v);
            if (p.bias != nullptr) h = __float2half_rn(__half2float(h) + __half2float(p.bias[n]));
            p.y[static_cast<long long>(t) * p.ldy + n] = h;
          }
        }
      } else {
        // This CTA holds one piece of strip c: publish it, and the last CTA to
        // arrive sums all pieces in CTA order (deterministic) and emits y.
        const int slot = (c == c_first) ? 0 : 1;
        float* mine = p.partials + (static_cast<long long>(blockIdx.x) * 2 + slot) * (MT * 8) * BN;
        for (int idx = ctid; idx < nout; idx += NCW * 32) {
          const int t = idx / BN, cc = idx % BN;
          mine[t * BN + cc] = red[t * BN + cc] + red[(MT * 8 + t) * BN + cc];
        }
        __threadfence();
        consumer_sync();
        if (ctid == 0) {
          // CTAs whose ranges touch strip c: first/last p with begin(p) <= unit < begin(p+1)
          const long long lo = static_cast<long long>(c) * KS, hi = lo + KS - 1;
          const long long pf = ((lo + 1) * P + U - 1) / U - 1;
          const long long pl = ((hi + 1) * P + U - 1) / U - 1;
          const unsigned nseg = static_cast<unsigned>(pl - pf + 1);
          const unsigned old = atomicAdd(&p.counters[c], 1u);
          flag[0] = (old == nseg - 1) ? 1 : 0;
          flag[1] = static_cast<int>(pf);
          flag[2] = static_cast<int>(pl);
        }
        consumer_sync();
        if (flag[0]) {
          __threadfence();
          const int pf = flag[1], pl = flag[2];
          for (int idx = ctid; idx < nout; idx += NCW * 32) {
            const int t = idx / BN, cc = idx % BN;
            const int n = col0 + cc;
            float v = 0.0f;
            for (int pp = pf; pp <= pl; ++pp) {
              const int sl = (c == static_cast<int>(unit_begin(pp, U, P) / KS)) ? 0 : 1;
              v += __ldcg(p.partials + ((static_cast<long long>(pp) * 2 + sl) * (MT * 8) + t) * BN + cc);
            }
            if (n < p.N) {
              __half h = __float2half_rn(v);
              if (p.bias != nullptr) h = __float2half_rn(__half2float(h) + __half2float(p.bias[n]));
              p.y[static_cast<long long>(t) * p.ldy + n] = h;
            }
          }
          if (ctid == 0) p.counters[c] = 0u;   // leave the workspace clean for the next launch
        }
      }
      consumer_sync();   // red[] is reused by the next segment
      kfirst = 0;          // any later segment starts at the top of its strip
    }
    if (++k == KS) { k = 0; ++c; }
  }
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
