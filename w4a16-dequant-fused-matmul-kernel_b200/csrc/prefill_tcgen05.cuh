// prefill_tcgen05.cuh -- compute-bound W4A16 GEMM for M > 32 tokens (prefill)
// on the 5th-generation tensor cores (tcgen05, accumulators in TMEM).
//
// Replaces the reference's Triton kernel (w4a16-kernel/src/w4a16/triton_kernel.py:62-128)
// for large M. Persistent CTAs (one per SM) walk 256 x bn output tiles (bn a
// multiple of 32 in [128, 224], chosen per shape by the host); the K loop of a
// tile runs in 64-wide steps.
//
// What bounds it on B200: shared-memory traffic. Per 64-K step a CTA writes the
// x tile (TMA) and the dequantised B tile, and the tensor core reads x once and
// B twice (once per 128-row half) -- ~150 KB per step against ~90 B/clk per SM,
// the rate a cuBLAS bf16 GEMM at 1.63 PF implies. Wider tiles amortise the x
// tile; the packed weights bypass shared memory. Under load a TMA load takes
// ~1.5 us to land, so the x ring is TSTAGES (4) steps deep. The two M=128 x N=bn
// accumulators fill most of TMEM, so the epilogue does not overlap the next
// tile's MMAs; 8 epilogue warps keep that drain short. bn below 224 only serves
// to round the tile count to whole waves of CTAs.
//
//   warp 0       TMA producer: per step the x tile [256 x 64] fp16 (128-byte
//                swizzle) into a 4-deep ring on a transaction-counted mbarrier.
//   warps 2..17  dequantisers: two threads per tile column each load 4 of the
//                column's 8 packed words of the step and its scale and zero
//                straight from global memory (L2-resident, two steps ahead),
//                unpack them (PRMT + LOP3 magic-number nibble
//                extraction, exact (q - z), one fp16 multiply by s: the
//                reference's rounding) and writes the fp16 weights K-major into
//                a 128-byte-swizzled B tile of a 2-deep ring, then
//                fence.proxy.async so the tensor core may read them.
//   warp 1       TMEM allocator (512 columns: two bn-column accumulator halves)
//                and single-thread MMA issuer: tcgen05.mma.cta_group::1.kind::f16,
//                M=128 N=bn K=16, eight per step (both 128-row halves of x
//                against one dequantised B tile); tcgen05.commit frees the ring
//                slots and, after a tile's last step, hands the accumulators to
//                the epilogue.
//   warps 18..25 epilogue: two warps per 32-lane TMEM quarter (one per 128-row
//                half) read the accumulators with tcgen05.ld, round to fp16,
//                add the optional bias (rounded again, as W4A16Linear's separate
//                add does), stage each 32 x 32 chunk in a swizzled shared-memory
//                tile and write it with a TMA tensor store (plain stores when y is
//                not 16-byte aligned).
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
constexpr int BN_MAX = 224;                  // tile columns: runtime bn in [128, 224], bn % 32 == 0
constexpr int BN_MIN = 128;                  // two halves; a single-half tile (M <= 128) goes down to 64
constexpr int BN_MIN_SINGLE = 64;
constexpr int BK = 64;
constexpr int TSTAGES = 4;                   // x-tile ring depth (covers ~1.5 us TMA latency under load)
constexpr int BSTAGES = 2;                   // dequantised-B ring depth
constexpr int A_BYTES = BM * BK * 2;         // 32768
constexpr int T_BYTES = A_BYTES;             // a TMA stage holds the x tile only
constexpr int B_BYTES = BN_MAX * BK * 2;     // 28672
constexpr int DQ_WARPS = 16;                 // two threads per tile column, 4 words each (256 columns of room)
constexpr int EPI_WARPS = 8;                 // two per TMEM lane quarter
constexpr int NUM_WARPS = 2 + DQ_WARPS + EPI_WARPS;
constexpr int THREADS = NUM_WARPS * 32;
constexpr int EPI_WARP0 = 2 + DQ_WARPS;
constexpr uint32_t TMEM_COLS = 512;          // two 128-row halves x bn columns (bn <= 224)
constexpr int STG_BYTES = 4096;              // per epilogue warp: a 32 x 32 output chunk (fp32 at most)
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES =
    1024 + TSTAGES * T_BYTES + BSTAGES * B_BYTES + EPI_WARPS * STG_BYTES + BAR_BYTES;

static_assert(T_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "tiles must keep 1024-byte alignment");
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
static_assert(DQ_WARPS * 32 >= 2 * BN_MAX, "two dequantiser threads per tile column");


struct Params {
  int tma_store;           // y written by TMA stores from a staging tile (y 16-byte aligned, ldy % 8 / % 4 == 0)
  const int32_t* qw;       // packed weights [K/8, N], read by the dequantisers with plain loads
  const __half* scales;    // [K/G, N]
  const __half* zeros;     // [K/G, N]
  const __half* bias;
  void* y;         // fp16, or fp32 when y_f32 (unrounded partial sums, no bias), or bf16 when y_bf16
  int y_f32;
  int y_bf16;      // y (and bias) bf16
  int M, N, K, G;
  int g_shift;     // log2(G) when G is a power of two, else -1
  long long ldy;
  int m_tiles, n_tiles;
  int halves;      // 128-row MMA halves per tile: 2 (256-row tiles), or 1 when M <= 128
  int bm;          // tile rows, 128 * halves
  int bn;          // tile columns
  uint32_t idesc;  // tcgen05 instruction descriptor for M=128, N=bn
  int vec_store;   // y and ldy allow 16-byte stores
  unsigned long long wait_ns;   // budget of every bounded wait (%globaltimer ns)
  int swiglu;      // (w4a16_tcgen05_kernel<true> only) fused gate/up columns interleaved in
                   // blocks of 16: y = h [M, N/2]
};

// Tile order: groups of RASTER_M row tiles, column-major inside a group, so that a
// wave of persistent CTAs reads a few row tiles of x (kept in L2) across many weight
// strips instead of every row tile of x per strip. Up to RASTER_M row tiles (M <=
// 4096) this is plain column-major order; at M = 8192 the groups measured 6% faster
// on B200, while groups of 8 were 1% slower at M = 4096.
constexpr int RASTER_M = 16;
__device__ __forceinline__ void tile_coords_mn(int m_tiles, int n_tiles, int tile, int& mt, int& nt) {
  const int per_group = RASTER_M * n_tiles;
  const int grp = tile / per_group;
  const int first = grp * RASTER_M;
  const int gm = m_tiles - first < RASTER_M ? m_tiles - first : RASTER_M;
  const int rem = tile - grp * per_group;
  mt = first + rem % gm;
  nt = rem / gm;
}
__device__ __forceinline__ void tile_coords(const Params& p, int tile, int& mt, int& nt) {
  tile_coords_mn(p.m_tiles, p.n_tiles, tile, mt, nt);
}

// Lane 0 waits, the warp follows: keeps mbarrier polling off the shared-memory pipe.
// sleep_ns > 0 backs the polling off (mbar_wait_backoff).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, uint64_t budget_ns,
                                          uint32_t sleep_ns = 0) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0)
    ok = sleep_ns ? mbar_wait_backoff(bar, parity, budget_ns, sleep_ns) : mbar_wait(bar, parity, budget_ns);
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  __syncwarp();
  return ok;
}

// Polling back-off of the roles that wait off the MMA issuer's critical path.
constexpr uint32_t kEpilogueSleepNs = 512;    // a tile's K loop lasts tens of microseconds
constexpr uint32_t kRunAheadSleepNs = 128;    // producers and dequantisers ahead of the MMAs

struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void advance(int depth) {
    if (++slot == depth) { slot = 0; phase ^= 1u; }
  }
};

// SWIGLU: the epilogue pairs each 32-column chunk's gate and up halves (see Params);
// a separate instantiation so the plain GEMM's epilogue is unchanged.
// NAT: qweight in the kernel nibble order (w4a16_repack): one shift and four LOP3s
// extract a word's natural-order pairs, instead of four PRMTs and four LOP3s.
template <bool SWIGLU, bool NAT>
__global__ void __launch_bounds__(THREADS, 1)
    w4a16_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_y,
                         const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* tring = smem;                                   // TSTAGES x x tile
  uint8_t* bring = smem + TSTAGES * T_BYTES;               // BSTAGES x B
  uint8_t* staging = bring + BSTAGES * B_BYTES;            // EPI_WARPS x STG_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + EPI_WARPS * STG_BYTES);
  uint64_t* tfull = bars;
  uint64_t* tempty = tfull + TSTAGES;
  uint64_t* bfull = tempty + TSTAGES;
  uint64_t* bempty = bfull + BSTAGES;
  uint64_t* accfull = bempty + BSTAGES;
  uint64_t* accempty = accfull + 1;
  uint64_t* drain = accempty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KT = p.K / BK;
  const int ntiles = p.m_tiles * p.n_tiles;
  const int bn = p.bn;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TSTAGES; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 1);
    }
    for (int j = 0; j < BSTAGES; ++j) {
      mbar_init(&bfull[j], DQ_WARPS);
      mbar_init(&bempty[j], 1);
    }
    mbar_init(accfull, 1);
    mbar_init(accempty, EPI_WARPS);
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
      Ring r;
      long long issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
        int mt, nt;
        tile_coords(p, tile, mt, nt);
        const int m0 = mt * p.bm;
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait_backoff(&tempty[r.slot], r.phase ^ 1u, p.wait_ns, kRunAheadSleepNs)) { ok = false; break; }
          uint8_t* st = tring + r.slot * T_BYTES;
          mbar_arrive_expect_tx(&tfull[r.slot], p.halves * (A_BYTES / 2));   // the x box is [bm x 64]
          tma_load_2d(st, &tm_x, &tfull[r.slot], kt * BK, m0);
          r.advance(TSTAGES);
          ++issued;
        }
      }
      // Never leave with copies in flight: wait for the newest phase of every slot used.
      const long long n = issued < TSTAGES ? issued : TSTAGES;
      for (long long i = 0; i < n; ++i) {
        if (r.slot == 0) { r.slot = TSTAGES; r.phase ^= 1u; }
        --r.slot;
        mbar_wait(&tfull[r.slot], r.phase, kWaitBudgetNs);   // default budget: never exit with copies in flight
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0) {
      Ring t, b;
      bool ok = true;
      int local = 0;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++local) {
        // the single accumulator set must have been drained by the epilogue
        if (!mbar_wait(accempty, (local & 1) ^ 1u, p.wait_ns)) { ok = false; break; }
        tc_fence_after();
        for (int kt = 0; kt < KT; ++kt) {
          if (!mbar_wait(&tfull[t.slot], t.phase, p.wait_ns) || !mbar_wait(&bfull[b.slot], b.phase, p.wait_ns)) {
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
            tc_mma_f16(tmem_base, adesc0 + static_cast<uint64_t>(kk * 2),
                       bdesc + static_cast<uint64_t>(kk * 2), p.idesc, acc);
            if (p.halves == 2)
              tc_mma_f16(tmem_base + bn, adesc1 + static_cast<uint64_t>(kk * 2),
                         bdesc + static_cast<uint64_t>(kk * 2), p.idesc, acc);
          }
          tc_commit(&tempty[t.slot]);
          tc_commit(&bempty[b.slot]);
          t.advance(TSTAGES);
          b.advance(BSTAGES);
        }
        if (ok) tc_commit(accfull);
      }
      tc_commit(drain);   // completes once every MMA this thread issued has finished
    }
  } else if (warp < EPI_WARP0) {
    // ------------------------------ dequantisers --------------------------
    // The packed words and the scale/zero of a step come straight from global
    // memory (L2-resident: every m-tile re-reads the n-tile's weights), loaded two
    // steps ahead into registers; only the dequantised B tile goes through shared
    // memory, which is what bounds this kernel.
    const int dt = threadIdx.x - 64;
    const int t = dt & 255;              // column of the tile owned by this thread
    const int c0 = (dt >> 8) * 4;        // its 4 words (32 K) of the step's 8
    const bool active = t < bn;
    const long long ldq = p.N;
    Ring br;
    bool ok = true;
    struct Step {
      uint32_t w[4];
      uint32_t s, z;
    };
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      int mt, nt;
      tile_coords(p, tile, mt, nt);
      const int n = nt * bn + t;
      const bool colok = active && n < p.N;
      auto fetch = [&](int kt, Step& f) {
        if (colok && kt < KT) {
          const int32_t* wp = p.qw + (static_cast<long long>(kt) * 8 + c0) * ldq + n;
#pragma unroll
          for (int c = 0; c < 4; ++c) f.w[c] = ldg_nc_u32(wp + c * ldq);
          const int kk = kt * BK;
          const long long grow = p.g_shift >= 0 ? kk >> p.g_shift : kk / p.G;
          f.s = ldg_nc_u16(p.scales + grow * ldq + n);
          f.z = ldg_nc_u16(p.zeros + grow * ldq + n);
        } else {
          f.w[0] = f.w[1] = f.w[2] = f.w[3] = 0u;
          f.s = f.z = 0u;
        }
      };
      Step cur, nxt, nnx;
      fetch(0, cur);
      fetch(1, nxt);
      for (int kt = 0; kt < KT; ++kt) {
        fetch(kt + 2, nnx);
        if (!warp_wait(&bempty[br.slot], br.phase ^ 1u, p.wait_ns, kRunAheadSleepNs)) {
          ok = false;
          break;
        }
        if (active) {
          const uint32_t ss = cur.s * 0x10001u;
          uint8_t* brow = bring + br.slot * B_BYTES + t * 128;
          if constexpr (NAT) {
            const uint32_t z2 = cur.z * 0x10001u;
            const uint32_t za = hadd2_u32(z2, 0x64006400u), zb = hadd2_u32(z2, 0x54005400u);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t q[4];
              dequant_word_perm(cur.w[c], za, zb, ss, q);
              *reinterpret_cast<uint4*>(brow + (((c0 + c) ^ (t & 7)) << 4)) = make_uint4(q[0], q[1], q[2], q[3]);
            }
          } else {
            const uint32_t zc = zero_pair_nat(cur.z);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              *reinterpret_cast<uint4*>(brow + (((c0 + c) ^ (t & 7)) << 4)) = dequant_word_nat(cur.w[c], zc, ss);
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bfull[br.slot]);
        br.advance(BSTAGES);
        cur = nxt;
        nxt = nnx;
      }
    }
  } else {
    // ------------------------------ epilogue -------------------------------
    const int quarter = warp & 3;                 // TMEM lanes this warp may access
    const int h = (warp - EPI_WARP0) >> 2;        // 128-row half of the tile
    uint8_t* stg = staging + (warp - EPI_WARP0) * STG_BYTES;
    // fp16 chunks (2 KB) alternate between the two halves of the warp's staging
    // buffer, so a chunk is staged while the previous one's store still reads
    int half_sel = 0;
    // y is written once and read by no CTA of this launch: first out of L2, so the
    // x and weight tiles that other CTAs re-read stay
    const uint64_t y_policy = l2_evict_first();
    if (p.tma_store && lane == 0) tma_prefetch_desc(&tm_y);
    int local = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++local) {
      if (!warp_wait(accfull, local & 1, p.wait_ns, kEpilogueSleepNs)) break;
      tc_fence_after();
      int mt, nt;
      tile_coords(p, tile, mt, nt);
      const int n0 = nt * bn;
      const int mrow0 = mt * p.bm + h * BMH + quarter * 32;
      const int m = mrow0 + lane;
#pragma unroll 1
      for (int col = 0; col < (h < p.halves ? bn : 0); col += 32) {   // (a missing half has no rows)
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + h * bn + col + (static_cast<uint32_t>(quarter * 32) << 16), r);
        tmem_ld_wait();
        if (p.tma_store) {
          // Stage the warp's 32 x 32 chunk (row = lane) in the TMA swizzle layout and
          // store it with one bulk tensor copy; rows >= M and columns >= N are clipped.
          // A chunk with no row below M or no column below N is neither staged nor
          // stored: a buffer is reused after waiting for all but the latest store group,
          // which holds only while every staged chunk commits a store.
          if (mrow0 >= p.M || n0 + col >= p.N) continue;
          uint8_t* sb = p.y_f32 ? stg : stg + half_sel * (STG_BYTES / 2);
          if (lane == 0) {
            // the chunk that last used this buffer has left it
            if (p.y_f32) bulk_wait_group_read0();
            else bulk_wait_group_read1();
          }
          __syncwarp();
          half_sel ^= 1;
          if (p.y_f32) {
            // 128-byte rows, 128-byte swizzle: 16-byte chunk c at c ^ (row & 7)
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<uint4*>(sb + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                  make_uint4(r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
          } else {
            uint32_t packed[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              // (columns past N are clipped by the store; their bias is not read)
              const int nb = n0 + col + 2 * e;
              packed[e] = out_bits(__uint_as_float(r[2 * e]), nb < p.N ? p.bias : nullptr, nb, p.y_bf16) |
                          (out_bits(__uint_as_float(r[2 * e + 1]), nb + 1 < p.N ? p.bias : nullptr, nb + 1,
                                    p.y_bf16) << 16);
            }
            // 64-byte rows, 64-byte swizzle: 16-byte chunk c at c ^ ((row >> 1) & 3)
#pragma unroll
            for (int c = 0; c < 4; ++c)
              *reinterpret_cast<uint4*>(sb + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) =
                  make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d_hint(&tm_y, sb, n0 + col, mrow0, y_policy);
            bulk_commit_group();
          }
          continue;
        }
        if constexpr (SWIGLU) {
          // 32-column chunk = 16 gate columns then the same 16 up columns (tiles start on
          // multiples of 32): 16 outputs of this row, columns (n0 + col) / 2 onwards
          const int no = (n0 + col) / 2;
          if (m < p.M && 2 * no < p.N) {
            uint32_t packed[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const __half lo = swiglu_h(__uint_as_float(r[2 * e]), __uint_as_float(r[16 + 2 * e]));
              const __half hi = swiglu_h(__uint_as_float(r[2 * e + 1]), __uint_as_float(r[16 + 2 * e + 1]));
              packed[e] = static_cast<uint32_t>(__half_as_ushort(lo)) |
                          (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
            }
            __half* hrow = static_cast<__half*>(p.y) + static_cast<long long>(m) * p.ldy + no;
            if (p.vec_store) {
              *reinterpret_cast<uint4*>(hrow) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
              *reinterpret_cast<uint4*>(hrow + 8) = make_uint4(packed[4], packed[5], packed[6], packed[7]);
            } else {
              const __half* hp = reinterpret_cast<const __half*>(packed);
#pragma unroll
              for (int e = 0; e < 16; ++e) hrow[e] = hp[e];
            }
          }
          continue;
        }
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
              packed[e] = out_bits(__uint_as_float(r[v * 8 + 2 * e]), p.bias, nb + 2 * e, p.y_bf16) |
                          (out_bits(__uint_as_float(r[v * 8 + 2 * e + 1]), p.bias, nb + 2 * e + 1, p.y_bf16)
                           << 16);
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
      if (lane == 0) mbar_arrive(accempty);
    }
    if (p.tma_store && lane == 0) bulk_wait_group0();   // every store of this warp has landed
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    mbar_wait(drain, 0, kWaitBudgetNs);   // every issued MMA has finished before TMEM is released
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace prefill
}  // namespace w4a16
