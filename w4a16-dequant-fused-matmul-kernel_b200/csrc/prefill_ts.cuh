// prefill_ts.cuh -- W4A16 GEMM for large M with the dequantised weights as the
// tensor-memory A operand of tcgen05.mma: the weights never pass through shared
// memory, which only carries the x tiles.
//
// Replaces the reference's Triton kernel (w4a16-kernel/src/w4a16/triton_kernel.py:62-128)
// for large M, like prefill_tcgen05.cuh, with the roles of the operands swapped:
//   D[n][m] = sum_k W[k][n] * x[m][k]      (D = y^T, one TMEM lane per weight column)
// A tile covers 256 weight columns (two M=128 MMA halves, A in TMEM) and mt tokens
// (the MMA's N, mt in {64, ..., 192}, a multiple of 32, chosen per shape by the host).
//
// Why: in the shared-memory operand form every 64-K step of a 256 x 224 tile moves
// ~148 KB through shared memory (x tile in, B tile in, x read once, B read twice),
// which bounds that kernel. Here a step of a 256 x mt tile moves the x tile in and
// reads it once per weight half: 3 * mt * 128 B, ~0.75 of the bytes per MAC.
//
//   warp 0       x producer: per step the x tile [mt x 64] fp16 (128-byte swizzle,
//                K-major: the MMA's B operand) into a ring of 144 KB (6 to 8 stages:
//                under load a tile takes ~2 us to land).
//   warp 2       weight producer: per step the packed words [8 x 256] int32 and the
//                group's scale and zero rows [256] into a WSTAGES-deep ring (TMA, so
//                the dequantisers never wait on DRAM latency: the weights of a tile
//                column are read from DRAM by its first row of tiles).
//   warps 3..18  dequantisers: warp w may only reach TMEM lanes 32*(w%4)..+31, so the
//                four warps of each lane quarter split the tile's two weight halves
//                and the step's two 4-word halves; a thread owns one weight column,
//                reads its 4 packed words and the scale/zero from the ring,
//                dequantises them (exact (q - z), one fp16 multiply by s: the
//                reference's rounding) into 16 registers of natural-order K pairs and
//                writes them into its lane of an A stage with one tcgen05.st.
//   warp 1       TMEM allocator (512 columns) and single-thread MMA issuer:
//                tcgen05.mma.cta_group::1.kind::f16 with A from TMEM, M=128, N=mt,
//                K=16, eight per step (two weight halves against one x tile).
//   warps 19..26 epilogue: two warps per TMEM lane quarter (one per weight half) read
//                the accumulators with tcgen05.ld (a thread holds one weight column
//                for 32 tokens), round to fp16 (+ bias, rounded again), transpose
//                through a swizzled staging tile into y's row-major order and write
//                it with TMA tensor stores (plain stores when y is not 16-byte aligned).
//
// TMEM columns: accumulator set s, half h at (2s + h) * mt (one or two sets, two when
// 4 * mt + 128 <= 512 so that the epilogue of a tile overlaps the next tile's MMAs),
// then the A stages: stage a, half h at a_col0 + 64a + 32h (32 columns = 64 K of fp16).
//
// Split K: the host may split the K loop of some tiles over several CTAs: of every tile
// when the tiles do not fill one wave of CTAs (whole = 0), or of the tiles of the last,
// partly filled wave (whole = the tiles of the full waves, a multiple of the grid, so
// every CTA runs the same number of whole tiles first). Each split's epilogue writes its
// fp32 partial tile to the workspace and takes an arrival ticket per (tile, epilogue
// warp); the last split sums every split's partial in split order (the bits do not
// depend on which split arrives last), applies the output form and resets the ticket.
//
// Every mbarrier wait is bounded; on expiry the role raises the sticky device error
// bit and leaves its loops; the producer drains its copies, the MMA issuer waits for
// its MMAs, and TMEM is freed before exit.
#pragma once

#include "common.cuh"
#include "prefill_tcgen05.cuh"

namespace w4a16 {
namespace prefill_ts {

constexpr int NT = 256;                      // weight columns per tile (two M=128 halves)
constexpr int BK = 64;
constexpr int MT_MAX = 192;                  // tokens per tile (the MMA's N)
constexpr int MT_MIN = 64;
constexpr int X_RING_BYTES = 147456;         // x-tile ring: as many [mt x 64] stages as fit (<= 8)
constexpr int TST_MAX = 8;
constexpr int WSTAGES = 4;                   // weight ring depth
constexpr int WQ_BYTES = (BK / 8) * NT * 4;  // 8 packed rows x 256 columns = 8192
constexpr int WSZ_BYTES = NT * 2;            // one scale (or zero) row of the tile = 512
constexpr int W_BYTES = WQ_BYTES + 2 * WSZ_BYTES;   // 9216
constexpr int AST_MAX = 4;                   // A stages in TMEM
constexpr int DQ_WARPS = 16;
constexpr int EPI_WARPS = 8;
constexpr int DQ_WARP0 = 3;
constexpr int EPI_WARP0 = DQ_WARP0 + DQ_WARPS;
constexpr int NUM_WARPS = EPI_WARP0 + EPI_WARPS;
constexpr int THREADS = NUM_WARPS * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr int STG_BYTES = 4096;              // per epilogue warp: a 32 x 32 chunk (fp32 at most)
constexpr int BAR_BYTES = 512;
constexpr int SMEM_BYTES = 1024 + X_RING_BYTES + WSTAGES * W_BYTES + EPI_WARPS * STG_BYTES + BAR_BYTES;

static_assert(X_RING_BYTES % 1024 == 0 && W_BYTES % 1024 == 0, "ring stages must keep 1024-byte alignment");
static_assert(X_RING_BYTES >= 6 * MT_MAX * BK * 2, "at least six x stages at the widest tile");
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
static_assert((2 * TST_MAX + 2 * WSTAGES + 2 * AST_MAX + 2 + 2 + 1) * 8 + 4 <= BAR_BYTES, "barrier area");

struct Params {
  int tma_store;           // y written by TMA stores (y 16-byte aligned, ldy % 8 / % 4 == 0)
  const void* bias;        // [N], fp16 (bf16 when y_bf16), or null
  void* y;                 // fp16, or fp32 when y_f32 (unrounded, no bias), or bf16 when y_bf16
  int y_f32;
  int y_bf16;
  int M, N, K, G;
  int g_shift;             // log2(G) when G is a power of two, else -1
  long long ldy;
  int m_tiles, n_tiles;
  int mt;                  // tokens per tile
  int dsets;               // accumulator sets (1 or 2)
  int a_col0;              // first TMEM column of the A stages
  int astages;             // A stages (2..AST_MAX)
  int xstages;             // x stages (X_RING_BYTES / (mt * 128), <= TST_MAX)
  uint32_t idesc;          // M=128, N=mt
  unsigned long long wait_ns;
  int splits;              // K splits of each tile past `whole` (1: no split)
  int whole;               // tiles [0, whole) run whole, one work item each; tile whole + t is
                           // split into items whole + t * splits + s (s < splits)
  float* partial;          // splits > 1: fp32 partial tiles [split item][epilogue warp][mt tokens][32 columns]
  unsigned int* counters;  // splits > 1: [split tile][epilogue warp] arrivals, left zero
};

__device__ __forceinline__ int num_items(const Params& p) {
  return p.whole + (p.m_tiles * p.n_tiles - p.whole) * p.splits;
}

// Work item -> tile and its K-step range [k0, k1) (K split evenly into p.splits parts for
// the tiles past p.whole); true for a split item.
__device__ __forceinline__ bool item_range(const Params& p, int item, int KT, int& tile, int& k0, int& k1) {
  if (item < p.whole) {
    tile = item;
    k0 = 0;
    k1 = KT;
    return false;
  }
  const int i = item - p.whole;
  const int t = i / p.splits;
  const int s = i - t * p.splits;
  tile = p.whole + t;
  k0 = static_cast<int>(static_cast<long long>(KT) * s / p.splits);
  k1 = static_cast<int>(static_cast<long long>(KT) * (s + 1) / p.splits);
  return p.splits > 1;
}

// SWIGLU: the weight columns are gate and up interleaved in blocks of 16, so a warp's
// 32 lanes hold 16 gate and the matching 16 up columns; y = h [M, N/2] (plain stores).
// NAT: qweight in the kernel nibble order (w4a16_repack).
template <bool SWIGLU, bool NAT>
__global__ void __launch_bounds__(THREADS, 1)
    w4a16_ts_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_y,
                    const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
                    const __grid_constant__ CUtensorMap tm_z, const Params p) {
  using prefill::Ring;
  using prefill::warp_wait;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* xring = smem;
  uint8_t* wring = xring + X_RING_BYTES;
  uint8_t* staging = wring + WSTAGES * W_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + EPI_WARPS * STG_BYTES);
  uint64_t* tfull = bars;
  uint64_t* tempty = tfull + TST_MAX;
  uint64_t* wfull = tempty + TST_MAX;
  uint64_t* wempty = wfull + WSTAGES;
  uint64_t* afull = wempty + WSTAGES;
  uint64_t* aempty = afull + AST_MAX;
  uint64_t* accfull = aempty + AST_MAX;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KT = p.K / BK;
  const int nitems = num_items(p);
  const int mt = p.mt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TST_MAX; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 1);
    }
    for (int w = 0; w < WSTAGES; ++w) {
      mbar_init(&wfull[w], 1);
      mbar_init(&wempty[w], DQ_WARPS);
    }
    for (int a = 0; a < AST_MAX; ++a) {
      mbar_init(&afull[a], DQ_WARPS);
      mbar_init(&aempty[a], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&accfull[s], 1);
      mbar_init(&accempty[s], EPI_WARPS);
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
    // ------------------------------ x producer ----------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      Ring r;
      long long issued = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < nitems; item += gridDim.x) {
        int tile, k0, k1, mi, ni;
        item_range(p, item, KT, tile, k0, k1);
        prefill::tile_coords_mn(p.m_tiles, p.n_tiles, tile, mi, ni);
        for (int kt = k0; kt < k1; ++kt) {
          if (!mbar_wait_backoff(&tempty[r.slot], r.phase ^ 1u, p.wait_ns, prefill::kRunAheadSleepNs)) { ok = false; break; }
          uint8_t* st = xring + r.slot * (mt * BK * 2);
          mbar_arrive_expect_tx(&tfull[r.slot], static_cast<uint32_t>(mt * BK * 2));   // the x box is [mt x 64]
          tma_load_2d(st, &tm_x, &tfull[r.slot], kt * BK, mi * mt);
          r.advance(p.xstages);
          ++issued;
        }
      }
      const long long n = issued < p.xstages ? issued : p.xstages;
      for (long long i = 0; i < n; ++i) {
        if (r.slot == 0) { r.slot = p.xstages; r.phase ^= 1u; }
        --r.slot;
        mbar_wait(&tfull[r.slot], r.phase, kWaitBudgetNs);   // default budget: never exit with copies in flight
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0) {
      Ring t, a, d;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < nitems; item += gridDim.x) {
        int tile, k0, k1;
        item_range(p, item, KT, tile, k0, k1);
        // this accumulator set must have been drained by the epilogue
        if (!mbar_wait(&accempty[d.slot], d.phase ^ 1u, p.wait_ns)) { ok = false; break; }
        tc_fence_after();
        const uint32_t dcol = tmem_base + static_cast<uint32_t>(d.slot * 2 * mt);
        for (int kt = k0; kt < k1; ++kt) {
          // afull also implies this step's x tile has landed (the first dequantiser warp
          // waits for it before arriving): one wait per step on this thread's path
          if (!mbar_wait(&afull[a.slot], a.phase, p.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = umma_desc_sw128(smem_u32(xring + t.slot * (mt * BK * 2)));
          const uint32_t acol = tmem_base + static_cast<uint32_t>(p.a_col0 + a.slot * 64);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint32_t acc = (kt != k0 || kk != 0) ? 1u : 0u;
            // K=16: 8 TMEM columns of A, 32 bytes along the swizzled x rows
            tc_mma_f16_ts(dcol, acol + kk * 8, bdesc + static_cast<uint64_t>(kk * 2), p.idesc, acc);
            tc_mma_f16_ts(dcol + mt, acol + 32 + kk * 8, bdesc + static_cast<uint64_t>(kk * 2), p.idesc, acc);
          }
          tc_commit(&tempty[t.slot]);
          tc_commit(&aempty[a.slot]);
          t.advance(p.xstages);
          a.advance(p.astages);
        }
        if (ok) tc_commit(&accfull[d.slot]);
        d.advance(p.dsets);
      }
      tc_commit(drain);   // completes once every MMA this thread issued has finished
    }
  } else if (warp == 2) {
    // ------------------------------ weight producer -----------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_z);
      Ring r;
      long long issued = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < nitems; item += gridDim.x) {
        int tile, k0, k1, mi, ni;
        item_range(p, item, KT, tile, k0, k1);
        prefill::tile_coords_mn(p.m_tiles, p.n_tiles, tile, mi, ni);
        for (int kt = k0; kt < k1; ++kt) {
          if (!mbar_wait_backoff(&wempty[r.slot], r.phase ^ 1u, p.wait_ns, prefill::kRunAheadSleepNs)) { ok = false; break; }
          uint8_t* st = wring + r.slot * W_BYTES;
          const int kk = kt * BK;
          const int grow = p.g_shift >= 0 ? kk >> p.g_shift : kk / p.G;
          mbar_arrive_expect_tx(&wfull[r.slot], static_cast<uint32_t>(W_BYTES));
          tma_load_2d(st, &tm_w, &wfull[r.slot], ni * NT, kt * (BK / 8));
          tma_load_2d(st + WQ_BYTES, &tm_s, &wfull[r.slot], ni * NT, grow);
          tma_load_2d(st + WQ_BYTES + WSZ_BYTES, &tm_z, &wfull[r.slot], ni * NT, grow);
          r.advance(WSTAGES);
          ++issued;
        }
      }
      const long long n = issued < WSTAGES ? issued : WSTAGES;
      for (long long i = 0; i < n; ++i) {
        if (r.slot == 0) { r.slot = WSTAGES; r.phase ^= 1u; }
        --r.slot;
        mbar_wait(&wfull[r.slot], r.phase, kWaitBudgetNs);   // default budget: never exit with copies in flight
      }
    }
  } else if (warp < EPI_WARP0) {
    // ------------------------------ dequantisers --------------------------
    const int dw = warp - DQ_WARP0;
    const int q = warp & 3;               // TMEM lane quarter this warp may reach
    const int h = (dw >> 2) & 1;          // weight half of the tile
    const int kp = dw >> 3;               // words 4kp..4kp+3 of the step
    const int nloc = h * 128 + q * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    Ring wr, ar, xr;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < nitems; item += gridDim.x) {
      int tile, k0, k1;
      item_range(p, item, KT, tile, k0, k1);
      for (int kt = k0; kt < k1; ++kt) {
        if (!warp_wait(&wfull[wr.slot], wr.phase, p.wait_ns, prefill::kRunAheadSleepNs)) {
          ok = false;
          break;
        }
        const uint8_t* st = wring + wr.slot * W_BYTES;
        uint32_t w[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) w[c] = *reinterpret_cast<const uint32_t*>(st + ((kp * 4 + c) * NT + nloc) * 4);
        const uint32_t sb = *reinterpret_cast<const unsigned short*>(st + WQ_BYTES + nloc * 2);
        const uint32_t zb = *reinterpret_cast<const unsigned short*>(st + WQ_BYTES + WSZ_BYTES + nloc * 2);
        uint32_t v[16];
        const uint32_t ss = sb * 0x10001u;
        if constexpr (NAT) {
          const uint32_t z2 = zb * 0x10001u;
          const uint32_t za = hadd2_u32(z2, 0x64006400u), zbb = hadd2_u32(z2, 0x54005400u);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t qv[4];
            dequant_word_perm(w[c], za, zbb, ss, qv);
#pragma unroll
            for (int j = 0; j < 4; ++j) v[4 * c + j] = qv[j];
          }
        } else {
          const uint32_t zc = zero_pair_nat(zb);
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 qv = dequant_word_nat(w[c], zc, ss);
            v[4 * c] = qv.x;
            v[4 * c + 1] = qv.y;
            v[4 * c + 2] = qv.z;
            v[4 * c + 3] = qv.w;
          }
        }
        // the ring slot's words are in registers (consumed above): hand it back
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty[wr.slot]);
        wr.advance(WSTAGES);
        if (!warp_wait(&aempty[ar.slot], ar.phase ^ 1u, p.wait_ns, prefill::kRunAheadSleepNs)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st_32x32b_x16(tmem_base + lane_addr + static_cast<uint32_t>(p.a_col0 + ar.slot * 64 + h * 32 + kp * 16), v);
        tmem_st_wait();
        tc_fence_before();
        if (warp == DQ_WARP0) {
          // the MMA issuer waits only on afull: this warp's arrival also vouches for the x tile
          if (!warp_wait(&tfull[xr.slot], xr.phase, p.wait_ns, prefill::kRunAheadSleepNs)) {
            ok = false;
            break;
          }
          xr.advance(p.xstages);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[ar.slot]);
        ar.advance(p.astages);
      }
    }
  } else {
    // ------------------------------ epilogue -------------------------------
    const int e = warp - EPI_WARP0;
    const int q = warp & 3;
    const int h = e >> 2;
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    uint8_t* stg = staging + e * STG_BYTES;
    int half_sel = 0;
    const uint64_t y_policy = l2_evict_first();
    if (p.tma_store && lane == 0) tma_prefetch_desc(&tm_y);
    Ring d;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
      int tile, k0, k1;
      const bool split = item_range(p, item, KT, tile, k0, k1);
      if (!warp_wait(&accfull[d.slot], d.phase, p.wait_ns, prefill::kEpilogueSleepNs)) break;
      tc_fence_after();
      int mi, ni;
      prefill::tile_coords_mn(p.m_tiles, p.n_tiles, tile, mi, ni);
      const int ncol0 = ni * NT + h * 128 + q * 32;   // first weight column of this warp
      const int n = ncol0 + lane;
      const int m0 = mi * mt;
      float bv = 0.0f;
      const bool has_bias = p.bias != nullptr && !p.y_f32;
      if (has_bias && n < p.N)
        bv = p.y_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[n])
                      : __half2float(static_cast<const __half*>(p.bias)[n]);
      const uint32_t dcol = tmem_base + lane_addr + static_cast<uint32_t>((d.slot * 2 + h) * mt);
      // One 32-token chunk of the warp's 32 columns (r[i] = fp32 y[m0 + mc + i][n]): round,
      // add the bias or apply SwiGLU, and store.
      auto emit_chunk = [&](uint32_t (&r)[32], int mc) {
        // A chunk with no token below M or no column below N has nothing to store, and it
        // must not touch the staging buffers either: the TMA-store path reuses a buffer
        // after waiting for all but the latest store group, which holds only while every
        // staged chunk commits a store.
        if (m0 + mc >= p.M || ncol0 >= p.N) return;
        if constexpr (SWIGLU) {
          // lanes l and l + 16 hold the gate and up values of output column ncol0 / 2 + l;
          // lane l finishes tokens 0..15 of the chunk, lane l + 16 tokens 16..31
          const bool up_lane = lane >= 16;
          const int no = ncol0 / 2 + (lane & 15);
          __half* ycol = static_cast<__half*>(p.y) + no;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint32_t recv = __shfl_xor_sync(0xffffffffu, up_lane ? r[j] : r[16 + j], 16);
            const float g = __uint_as_float(up_lane ? recv : r[j]);
            const float u = __uint_as_float(up_lane ? r[16 + j] : recv);
            const int m = m0 + mc + j + (up_lane ? 16 : 0);
            if (m < p.M && 2 * no < p.N) ycol[static_cast<long long>(m) * p.ldy] = swiglu_h(g, u);
          }
          return;
        }
        if (p.tma_store) {
          uint8_t* sb = p.y_f32 ? stg : stg + half_sel * (STG_BYTES / 2);
          if (lane == 0) {
            if (p.y_f32) bulk_wait_group_read0();
            else bulk_wait_group_read1();
          }
          __syncwarp();
          half_sel ^= 1;
          if (p.y_f32) {
            // row i = token, 32 fp32 columns = 128 B, 128-byte swizzle (16-byte chunk c at c ^ (i & 7))
#pragma unroll
            for (int i = 0; i < 32; ++i)
              *reinterpret_cast<uint32_t*>(sb + i * 128 + ((((lane >> 2) ^ (i & 7)) << 4) | ((lane & 3) << 2))) = r[i];
          } else {
            // row i = token, 32 16-bit columns = 64 B, 64-byte swizzle (chunk c at c ^ ((i >> 1) & 3))
            if (p.y_bf16) {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                __nv_bfloat16 o = __float2bfloat16_rn(__uint_as_float(r[i]));
                if (has_bias) o = __float2bfloat16_rn(__bfloat162float(o) + bv);
                r[i] = __bfloat16_as_ushort(o);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                __half o = __float2half_rn(__uint_as_float(r[i]));
                if (has_bias) o = __float2half_rn(__half2float(o) + bv);
                r[i] = __half_as_ushort(o);
              }
            }
            const uint32_t cb = static_cast<uint32_t>(lane >> 3), lo = static_cast<uint32_t>(lane & 7) << 1;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              *reinterpret_cast<unsigned short*>(sb + i * 64 + (((cb ^ ((i >> 1) & 3)) << 4) | lo)) =
                  static_cast<unsigned short>(r[i]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d_hint(&tm_y, sb, ncol0, m0 + mc, y_policy);
            bulk_commit_group();
          }
          return;
        }
        if (n < p.N) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int m = m0 + mc + i;
            if (m >= p.M) return;
            const float v = __uint_as_float(r[i]);
            if (p.y_f32) {
              static_cast<float*>(p.y)[static_cast<long long>(m) * p.ldy + n] = v;
            } else if (p.y_bf16) {
              __nv_bfloat16 o = __float2bfloat16_rn(v);
              if (has_bias) o = __float2bfloat16_rn(__bfloat162float(o) + bv);
              static_cast<__nv_bfloat16*>(p.y)[static_cast<long long>(m) * p.ldy + n] = o;
            } else {
              __half o = __float2half_rn(v);
              if (has_bias) o = __float2half_rn(__half2float(o) + bv);
              static_cast<__half*>(p.y)[static_cast<long long>(m) * p.ldy + n] = o;
            }
          }
        }
      };
      if (split) {
        // This split's fp32 partial of the warp's 32 columns x mt tokens, then TMEM is free.
        // Token-major ([token][32 columns] per warp): the warp's store or load of one token
        // is one 128-byte line.
        float* mine = p.partial + (static_cast<long long>(item - p.whole) * EPI_WARPS + e) * 32LL * mt + lane;
#pragma unroll 1
        for (int mc = 0; mc < mt; mc += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(dcol + mc, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) mine[(mc + i) * 32] = __uint_as_float(r[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&accempty[d.slot]);
        d.advance(p.dsets);
        // The split that arrives last for this warp's slice of the tile sums every split's
        // partial in split order (one summation order whoever arrives last) and stores y.
        __threadfence();
        __syncwarp();
        unsigned int* ctr = p.counters + static_cast<long long>(tile - p.whole) * EPI_WARPS + e;
        unsigned last = 0;
        if (lane == 0) last = atomicAdd(ctr, 1u) == static_cast<unsigned>(p.splits - 1) ? 1u : 0u;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence();
        const float* part0 =
            p.partial + static_cast<long long>(tile - p.whole) * p.splits * EPI_WARPS * 32LL * mt + e * 32LL * mt + lane;
        const long long sstride = static_cast<long long>(EPI_WARPS) * 32 * mt;
#pragma unroll 1
        for (int mc = 0; mc < mt; mc += 32) {
          uint32_t r[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__ldcg(part0 + (mc + i) * 32));
#pragma unroll 1
          for (int sp = 1; sp < p.splits; ++sp) {
            const float* src = part0 + sp * sstride + mc * 32;
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) + __ldcg(src + i * 32));
          }
          emit_chunk(r, mc);
        }
        __syncwarp();
        if (lane == 0) *ctr = 0u;   // left zero for the next launch
        continue;
      }
#pragma unroll 1
      for (int mc = 0; mc < mt; mc += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(dcol + mc, r);   // r[i] = y[m0 + mc + i][n]
        tmem_ld_wait();
        emit_chunk(r, mc);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[d.slot]);
      d.advance(p.dsets);
    }
    if (p.tma_store && lane == 0) bulk_wait_group0();
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

}  // namespace prefill_ts
}  // namespace w4a16
