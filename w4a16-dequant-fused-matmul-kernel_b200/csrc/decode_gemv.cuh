// decode_gemv.cuh -- memory-bound W4A16 GEMM for M <= 32 tokens (decode).
//
// Replaces the reference's Triton K-loop (w4a16-kernel/src/w4a16/triton_kernel.py:99-124)
// for the decode regime, where the packed weights are read exactly once and
// the roofline is HBM bandwidth.
//
// Design (B200):
//  * Stream-K over units of (128-column strip, 512-K stage), strip-major,
//    dealt in contiguous ranges (sizes differing by at most one unit, the longer
//    ones first) to one CTA per SM (two per SM for up to
//    8 tokens), so every SM streams the same number of bytes whatever N and K are.
//  * One producer thread streams each unit -- packed words [64 x 128] int32,
//    the scale and zero rows it needs and the matching x slice -- into a
//    shared-memory ring with TMA; one transaction-counted mbarrier per stage.
//  * Programmatic dependent launch: the kernel lets the next launch in the
//    stream start immediately, and its producer issues the weight loads of
//    the first stages BEFORE griddepcontrol.wait (weights never depend on the
//    previous kernel; x, y and the workspace do). Back-to-back GEMMs thus
//    overlap one launch's ramp-up with the previous launch's tail; measured
//    on B200, a 22.5 MB TMA stream drops from 5.8 to 4.1 us per launch.
//  * Consumers read each 8-element chunk of x (k0..k7) from shared memory and
//    reorder it to (k0,k4,k1,k5,k2,k6,k3,k7) with 4 PRMTs (ALU pipe, which has
//    slack) to match the K order of their weight fragments.
//  * Consumer warps dequantise in registers -- magic-number nibble extraction
//    (OR the nibble into the mantissa of fp16 1024 or 64, then subtract
//    1024+z or 64+z: exact), then one fp16 multiply by the scale, which
//    reproduces the reference's fp16 (q - z) * s rounding bit for bit -- and
//    feed m16n8k16 tensor-core MMAs (fp32 accumulation). The MMA is "swapped":
//    16 weight columns form its M side and up to 8 tokens its N side; K is
//    permuted inside each MMA so a lane's packed word supplies its fragment
//    without shuffles (x is permuted identically, which leaves the dot
//    product unchanged).
//  * A strip covered by one CTA is reduced in shared memory and written
//    directly. Each CTA shares at most two strips (its first and last) with
//    neighbours. A shared strip belongs to the CTA that holds its last K stage
//    (its "owner"); every earlier CTA of the strip ends its range inside it and
//    publishes its fp32 piece as 64-bit words (1 << 32 | bits) in its own
//    workspace slot: a 64-bit store is single-copy atomic, so the tag vouches
//    for the value and no fence or counter is needed. The owner parks its own
//    piece in shared memory when the strip ends mid-range, and at the end of its
//    range reads the other pieces until their tags are set, sums all pieces in
//    CTA order -- deterministic -- writes y and clears the tags, leaving the
//    workspace zeroed for the next launch. Only finished CTAs wait, and only on
//    other CTAs' units, so the launch completes even if its CTAs are not all
//    resident at once.
#pragma once

#include "common.cuh"

namespace w4a16 {
namespace decode {

constexpr int BN = 128;             // columns per strip
constexpr int ROWS = 64;            // packed rows (of 8 K each) per stage
constexpr int KSTAGE = ROWS * 8;    // 512 K per stage
constexpr int SZ_ROWS = 8;          // scale/zero rows per stage (G >= 64 => at most 8 groups)
constexpr int W_BYTES = ROWS * BN * 4;        // 32768
constexpr int SZ_BYTES = SZ_ROWS * BN * 2;    // 2048 (each of scales, zeros)
constexpr int XBOX = 256;                     // K width of one x box (TMA box sides <= 256)
// Workspace: one slot of tagged piece words per CTA, [gridDim.x][MT*8][BN]
// 64-bit words, all zero between launches.
constexpr int MAX_STRIPS = 16384;             // N <= 2,097,152 on the decode path
constexpr unsigned long long PIECE_TAG = 1ull << 32;

// Consumer warps: 4 column quarters x 2 K halves of 256 = 8 warps for every
// token count. (16 warps with K quarters were measured 5% slower at M = 1 on
// B200: the legacy MMA pipe, not warp count, bounds the consumers.)
__host__ __device__ constexpr int ncw_for(int /*MT*/) { return 8; }
__host__ __device__ constexpr int threads_for(int MT) { return 32 * (ncw_for(MT) + 1); }
// Up to 8 tokens two CTAs share each SM (grid = 2 x SMs, ~108 KB of shared memory and
// <= 113 registers per thread each): twice the consumer warps per SMSP to hide the
// dequantiser's latencies, measured 7-15% faster at K >= 8192 and K = 1024 and equal at
// the K = 4096 headline shape. Larger token tiles need more registers than that allows.
__host__ __device__ constexpr int ctas_per_sm(int MT) { return MT == 1 ? 2 : 1; }
__host__ __device__ constexpr int x_bytes(int M) { return KSTAGE * 2 * M; }
__host__ __device__ constexpr int stage_bytes(int M) { return W_BYTES + 2 * SZ_BYTES + x_bytes(M); }
__host__ __device__ constexpr int red_bytes(int MT) { return (ncw_for(MT) / 4) * (MT * 8) * BN * 4; }
// the owner's parked piece of its first strip: [MT*8][BN] fp32
__host__ __device__ constexpr int park_bytes(int MT) { return (MT * 8) * BN * 4; }
// TMA destinations within a stage (W, S, Z, x box 0, x box 1) are 128-byte aligned.
static_assert(W_BYTES % 128 == 0 && SZ_BYTES % 128 == 0 && (XBOX * 2) % 128 == 0 &&
                  stage_bytes(1) % 1024 == 0,
              "decode stage layout keeps TMA destinations 128-byte aligned");

struct Params {
  const __half* bias;
  void* y;                // fp16, or fp32 when y_f32 (unrounded partial sums, no bias), or bf16 when y_bf16
  int y_f32;
  int y_bf16;             // y (and bias) bf16
  unsigned long long* pieces;   // [gridDim.x][MT*8][BN] tagged piece words, zero between launches
  int M, N, K, G;
  int g_shift;            // log2(G) when G is a power of two, else -1
  long long ldy;
  int kstages;            // K stages per strip (ceil(K / 512))
  long long units;        // strips * kstages
  int num_stages;         // ring depth
  // Fused all-reduce (ar_world > 1): this rank's y is the sum over ranks of every
  // rank's partial GEMM (a row-parallel layer). Each rank owns one peer-to-peer
  // buffer (layout below); ar_peer[q] is rank q's buffer as mapped on this GPU.
  // Fused all-gather (ar_gather, same buffers): y is [M, ar_world * N], every rank's
  // columns in rank order; this rank computes columns [ar_rank * N, (ar_rank + 1) * N).
  int ar_world, ar_rank;
  int ar_gather;
  int ar_tail;                          // CTAs that finish the call: the last ar_tail to arrive
  int* ar_ctl;                          // this rank's control words: [0] epoch, [1] CTAs arrived
  long long ar_slot;                    // elements per rank slot (>= M * N)
  unsigned long long ar_peer[8];        // [ar_world] buffer addresses (kernel parameters)
  unsigned long long wait_ns;           // budget of every bounded wait (%globaltimer ns)
  // SwiGLU epilogue (w4a16_gemm_swiglu): the weight's columns are a fused gate/up
  // projection interleaved in blocks of 16 (16 gate columns, then the same 16 up
  // columns), and y is h [M, N/2] = fp16(silu(fp16(g)) * fp16(u)).
  int swiglu;
};

// Peer-to-peer all-reduce buffer (one per rank): two halves, selected by the
// epoch's parity, each holding one slot per rank of 64-bit words
//   word = (tag << 32) | fp32 bits,  tag = epoch + 1,   [2][world][slot]
// The CTA that finalises output element e writes its word into slot `rank` of
// every rank's buffer (one single-copy-atomic 64-bit store each, so the tag
// vouches for the value beside it: no fence, no separate flag). A rank reads its
// own buffer until every slot's word for its elements carries this epoch's tag.
// A rank can only be one epoch ahead of another (it needs every rank's words of
// the previous epoch to finish it), so the half it writes is never one a peer
// still reads.
constexpr int AR_MAX_RANKS = 8;
__host__ __device__ constexpr long long ar_buffer_bytes(int world, long long slot) {
  return 2ll * world * slot * 8;
}
// Output elements each finishing thread takes (sets how many CTAs finish).
constexpr int AR_ELEMS_PER_THREAD = 4;

__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// c (+)= a * b on the tensor core, m16n8k16, fp16 in, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}


// Programmatic dependent launch controls.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// First unit of CTA p when U units are dealt to P CTAs in contiguous ranges: every CTA
// gets U / P units and the first U % P CTAs one more. The lowest block indices are
// dispatched first -- under programmatic dependent launch they take the SM slots that
// free up first, so their weights are prefetched earliest -- and the last CTAs to
// start, whose first loads land latest, get the shorter ranges. (Spreading the extra
// units evenly over the indices put them on late starters too: measured on B200,
// those CTAs set the end of every launch.)
__device__ __forceinline__ long long unit_begin(long long p, long long U, long long P) {
  const long long b = U / P, e = U % P;
  return p * b + (p < e ? p : e);
}
// The CTA whose range holds unit u (the inverse of unit_begin).
__device__ __forceinline__ long long unit_owner(long long u, long long U, long long P) {
  const long long b = U / P, e = U % P;
  return u < e * (b + 1) ? u / (b + 1) : e + (u - e * (b + 1)) / b;
}

// Consumer-warp-only barrier (named barrier 1; the producer warp does not take part).
template <int NCW>
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
}

__device__ __forceinline__ unsigned long long ld_shared_u64_volatile(uint32_t addr) {
  unsigned long long v;
  asm volatile("ld.volatile.shared.u64 %0, [%1];" : "=l"(v) : "r"(addr) : "memory");
  return v;
}

// peer_s: shared-memory copy of ar_peer, read at each store (volatile, so the
// eight addresses are not hoisted into registers across the epilogue loops).
template <bool AR>
__device__ __forceinline__ void emit(const Params& p, int t, int n, float v, int ar_epoch,
                                     uint32_t peer_s) {
  if (AR) {
    // all-reduce: the unrounded partial; all-gather: the final fp16 value (with this
    // rank's bias), held exactly in fp32. Tagged, into this rank's slot of every rank's
    // buffer (the peers' first: they are the longer way).
    if (p.ar_gather) {
      __half h = __float2half_rn(v);
      if (p.bias != nullptr) h = __float2half_rn(__half2float(h) + __half2float(p.bias[n]));
      v = __half2float(h);
    }
    const uint32_t tag = static_cast<uint32_t>(ar_epoch) + 1u;
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    const long long slot0 = (static_cast<long long>(ar_epoch & 1) * p.ar_world + p.ar_rank) * p.ar_slot;
    const long long e8 = (slot0 + static_cast<long long>(t) * p.N + n) * 8;
#pragma unroll
    for (int q = 0; q < AR_MAX_RANKS; ++q)
      if (q < p.ar_world && q != p.ar_rank)
        st_relaxed_sys_u64(reinterpret_cast<unsigned long long*>(ld_shared_u64_volatile(peer_s + 8 * q) + e8), w);
    st_relaxed_sys_u64(reinterpret_cast<unsigned long long*>(ld_shared_u64_volatile(peer_s + 8 * p.ar_rank) + e8), w);
    return;
  }
  const long long o = static_cast<long long>(t) * p.ldy + n;
  if (p.y_f32) {
    static_cast<float*>(p.y)[o] = v;
    return;
  }
  static_cast<unsigned short*>(p.y)[o] = static_cast<unsigned short>(out_bits(v, p.bias, n, p.y_bf16));
}

// SwiGLU of a fused gate/up strip: output column o (0..63) of a 128-column strip
// reads the strip's column swiglu_gate_col(o) as gate and the one 16 further as up.
constexpr int SWIGLU_BLOCK = 16;
__device__ __forceinline__ int swiglu_gate_col(int o) { return ((o >> 4) << 5) | (o & 15); }

// AR: fused all-reduce (w4a16_gemm_allreduce); a separate instantiation so the
// plain GEMM's register allocation is not shaped by it.
// NAT: qweight in the kernel nibble order (w4a16_repack): the dequantised pairs come
// out in natural K order, so x is used as loaded, without the 4 PRMTs per chunk.
template <int MT, bool AR, bool NAT = false>
__global__ void __launch_bounds__(threads_for(MT), ctas_per_sm(MT))
    decode_gemv_tma_kernel(const __grid_constant__ CUtensorMap tm_w,
                           const __grid_constant__ CUtensorMap tm_s,
                           const __grid_constant__ CUtensorMap tm_z,
                           const __grid_constant__ CUtensorMap tm_x, const Params p) {
  constexpr int NCW = ncw_for(MT);
  constexpr int KQ = NCW / 4;             // K parts per stage
  constexpr int KPART = KSTAGE / KQ;      // K per warp per stage (128 or 256)
  constexpr int NPAIR = KPART / 64;       // 64-K slices per warp per stage
  static_assert(KPART == XBOX, "a warp's K part is one x box");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int M = p.M;
  const int nst = p.num_stages;
  const int sbytes = stage_bytes(M);
  float* red = reinterpret_cast<float*>(smem + nst * sbytes);
  float* park = reinterpret_cast<float*>(smem + nst * sbytes + red_bytes(MT));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + nst * sbytes + red_bytes(MT) + park_bytes(MT));
  uint64_t* empty = full + nst;
  int* flag = reinterpret_cast<int*>(empty + nst);                       // 16 ints
  unsigned long long* ar_peer_smem = reinterpret_cast<unsigned long long*>(flag + 16);   // AR: [8]
  // this CTA's unit range, worked out once (64-bit divisions) by thread 0:
  // u0, u1, then c_first, k_first, c_last, k_last and the first CTA of strip c_first
  long long* range = reinterpret_cast<long long*>(ar_peer_smem + AR_MAX_RANKS);
  int* range_i = reinterpret_cast<int*>(range + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long P = gridDim.x;
  const long long U = p.units;
  const int KS = p.kstages;

  if (threadIdx.x == 0) {
    pdl_launch_dependents();
    const long long a = unit_begin(blockIdx.x, U, P), b = unit_begin(blockIdx.x + 1, U, P);
    const int cf = static_cast<int>(a / KS), cl = static_cast<int>((b - 1) / KS);
    const long long lo = static_cast<long long>(cf) * KS;
    range[0] = a;
    range[1] = b;
    range_i[0] = cf;
    range_i[1] = static_cast<int>(a - lo);
    range_i[2] = cl;
    range_i[3] = static_cast<int>((b - 1) - static_cast<long long>(cl) * KS);
    range_i[4] = static_cast<int>(unit_owner(lo, U, P));
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NCW);
    }
    mbar_fence_init();
  }
  __syncthreads();
  const long long u0 = range[0];
  const long long u1 = range[1];
  const int c_first = range_i[0];
  const int k_first = range_i[1];
  const int c_last = range_i[2];
  const int k_last = range_i[3];
  // A strip is "split" when other CTAs hold part of its K range. This CTA owns
  // its first strip when that strip began in an earlier CTA and ends in this
  // range; it publishes its last segment when its last strip continues in a
  // later CTA. (Both can hold; when the range lies inside one strip that began
  // earlier and continues later, it only publishes.)
  const bool owns_first = k_first != 0 && (c_last > c_first || k_last == KS - 1);
  const bool publishes = k_last != KS - 1;

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_s);
      tma_prefetch_desc(&tm_z);
      tma_prefetch_desc(&tm_x);
      const long long total = u1 - u0;
      const long long pre = total < nst ? total : nst;
      // weights of the first `pre` stages do not depend on the previous kernel
      int c = c_first, k = k_first;
      for (long long i = 0; i < pre; ++i) {
        uint8_t* st = smem + i * sbytes;
        const int grow = p.g_shift >= 0 ? (k * KSTAGE) >> p.g_shift : (k * KSTAGE) / p.G;
        mbar_arrive_expect_tx(&full[i], sbytes);
        tma_load_2d(st, &tm_w, &full[i], c * BN, k * ROWS);
        tma_load_2d(st + W_BYTES, &tm_s, &full[i], c * BN, grow);
        tma_load_2d(st + W_BYTES + SZ_BYTES, &tm_z, &full[i], c * BN, grow);
        if (++k == KS) { k = 0; ++c; }
      }
      pdl_wait();
      c = c_first;
      k = k_first;
      for (long long i = 0; i < pre; ++i) {
        uint8_t* st = smem + i * sbytes;
        tma_load_2d(st + W_BYTES + 2 * SZ_BYTES, &tm_x, &full[i], k * KSTAGE, 0);
        tma_load_2d(st + W_BYTES + 2 * SZ_BYTES + XBOX * 2 * M, &tm_x, &full[i], k * KSTAGE + XBOX, 0);
        if (++k == KS) { k = 0; ++c; }
      }
      int s = static_cast<int>(pre % nst);
      uint32_t ph = pre == nst ? 1u : 0u;
      long long issued = pre;
      for (long long u = u0 + pre; u < u1; ++u, ++issued) {
        if (!mbar_wait(&empty[s], ph ^ 1, p.wait_ns)) break;
        uint8_t* st = smem + s * sbytes;
        const int grow = p.g_shift >= 0 ? (k * KSTAGE) >> p.g_shift : (k * KSTAGE) / p.G;
        mbar_arrive_expect_tx(&full[s], sbytes);
        tma_load_2d(st, &tm_w, &full[s], c * BN, k * ROWS);
        tma_load_2d(st + W_BYTES, &tm_s, &full[s], c * BN, grow);
        tma_load_2d(st + W_BYTES + SZ_BYTES, &tm_z, &full[s], c * BN, grow);
        // x slice [M x 512] as two [M x 256] boxes (a TMA box side is at most 256)
        tma_load_2d(st + W_BYTES + 2 * SZ_BYTES, &tm_x, &full[s], k * KSTAGE, 0);
        tma_load_2d(st + W_BYTES + 2 * SZ_BYTES + XBOX * 2 * M, &tm_x, &full[s], k * KSTAGE + XBOX, 0);
        if (++s == nst) { s = 0; ph ^= 1; }
        if (++k == KS) { k = 0; ++c; }
      }
      // Never leave with copies in flight: wait for the newest stage of every slot
      // (with the default budget, whatever budget the caller chose for the pipeline).
      const long long n_in_flight = issued < nst ? issued : nst;
      for (long long i = 0; i < n_in_flight; ++i) {
        if (s == 0) { s = nst; ph ^= 1; }
        --s;
        mbar_wait(&full[s], ph, kWaitBudgetNs);
      }
    }
    return;   // takes no part in the consumers' barriers below
  }
  pdl_wait();   // x, y and the workspace are only touched after the previous kernel

  // Fused all-reduce: this launch's epoch (the previous launch on this stream has
  // completed, so its epoch advance is visible) and this rank's slot in the half.
  const int ar_epoch = AR ? *reinterpret_cast<volatile int*>(p.ar_ctl) : 0;
  // the peers' addresses for emit (published to the consumers by their first barrier)
  if (AR && threadIdx.x - 32 < AR_MAX_RANKS) ar_peer_smem[threadIdx.x - 32] = p.ar_peer[threadIdx.x - 32];

  // -------------------------------- consumers ---------------------------------
  const int cw = warp - 1;
  const int ctid = threadIdx.x - 32;
  const int cq = cw & 3;          // column quarter: 32 columns
  const int kq = cw >> 2;         // K part: packed rows [kq*KPART/8, (kq+1)*KPART/8) of the stage
  const int q = lane >> 2;        // MMA group id: columns 4q..4q+3 of the quarter
  const int g = lane & 3;         // MMA thread-in-group: packed row within a quad
  const int ccol = cq * 32 + 4 * q;
  // x rows this lane feeds to its MMA column q of each token tile (token tt*8 + q;
  // token 0's row stands in for tokens that do not exist)
  int xoff[MT];
#pragma unroll
  for (int tt = 0; tt < MT; ++tt) xoff[tt] = tt * 8 + q < M ? (tt * 8 + q) * (XBOX * 2) : 0;

  // Scale/zero groups of the warp's 64-K slices in a stage: bit pr of gstart is set
  // when slice pr starts a group, byte pr of gpack holds its group relative to the
  // stage's first group. For G a power of two the pattern is the same in every stage
  // (a stage starts on a multiple of 512; G <= 512 divides it, a larger G holds the
  // whole stage); otherwise it is worked out per stage.
  auto group_plan = [&](int kbase, uint32_t& gstart, uint32_t& gpack) {
    gstart = 0u;
    gpack = 0u;
    const int g0 = p.g_shift >= 0 ? kbase >> p.g_shift : kbase / p.G;
    int prev = -1;
#pragma unroll
    for (int pr = 0; pr < NPAIR; ++pr) {
      const int kk = kbase + kq * KPART + pr * 64;
      const int gi = (p.g_shift >= 0 ? kk >> p.g_shift : kk / p.G) - g0;
      if (gi != prev) gstart |= 1u << pr;
      gpack |= static_cast<uint32_t>(gi) << (8 * pr);
      prev = gi;
    }
  };
  uint32_t gstart_fix = 0u, gpack_fix = 0u;
  if (p.g_shift >= 0) group_plan(0, gstart_fix, gpack_fix);

  float acc[2][2][MT][4];         // [quad parity][column tile][token tile][fragment]
  int s = 0;
  uint32_t ph = 0;
  bool ok = true;
  int c = c_first, k = k_first;
  for (long long u = u0; u < u1; ++u) {
    if (u == u0 || k == 0) {
#pragma unroll
      for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int tt = 0; tt < MT; ++tt)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[e][t][tt][r] = 0.0f;
    }
    if (ok) {
      bool got = true;
      if (lane == 0) got = mbar_wait(&full[s], ph, p.wait_ns);
      ok = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
      __syncwarp();   // orders the other lanes' shared-memory reads after lane 0's acquire
    }
    if (ok) {
      const uint8_t* st = smem + s * sbytes;
      // Per-stage load bases: every load below is base + a compile-time offset. The
      // warp's 32 packed rows all lie in x box kq (rows kq*32 .. kq*32+31 of the stage).
      const uint8_t* wq = st + ((kq * (KPART / 8) + g) * BN + ccol) * 4;
      const uint8_t* xq = st + W_BYTES + 2 * SZ_BYTES + kq * (XBOX * 2 * M) + g * 16;
      uint32_t gstart = gstart_fix, gpack = gpack_fix;
      if (p.g_shift < 0) group_plan(k * KSTAGE, gstart, gpack);
      const int kbase = k * KSTAGE;
      const int g0 = p.g_shift >= 0 ? kbase >> p.g_shift : kbase / p.G;
      int gcur = -1;
      uint32_t ss[4], za[4], zb[4];
#pragma unroll
      for (int pr = 0; pr < NPAIR; ++pr) {
        // a pair of quads = 64 K: always inside one group since G % 64 == 0
        bool starts;
        int gi;
        if constexpr (MT == 2) {
          // (two token tiles: the per-slice form below measured 8% faster at M = 16 on
          // B200 than the precomputed plan, a difference of register allocation)
          const int kk = kbase + kq * KPART + pr * 64;
          gi = (p.g_shift >= 0 ? kk >> p.g_shift : kk / p.G) - g0;
          starts = gi != gcur;
          gcur = gi;
        } else {
          starts = (gstart & (1u << pr)) != 0u;
          gi = static_cast<int>((gpack >> (8 * pr)) & 0xFFu);
        }
        if (starts) {
          const uint2 s4 = *reinterpret_cast<const uint2*>(st + W_BYTES + (gi * BN + ccol) * 2);
          const uint2 z4 =
              *reinterpret_cast<const uint2*>(st + W_BYTES + SZ_BYTES + (gi * BN + ccol) * 2);
          const uint32_t za01 = hadd2_u32(z4.x, 0x64006400u), za23 = hadd2_u32(z4.y, 0x64006400u);
          const uint32_t zb01 = hadd2_u32(z4.x, 0x54005400u), zb23 = hadd2_u32(z4.y, 0x54005400u);
          ss[0] = prmt(s4.x, 0, 0x1010);
          ss[1] = prmt(s4.x, 0, 0x3232);
          ss[2] = prmt(s4.y, 0, 0x1010);
          ss[3] = prmt(s4.y, 0, 0x3232);
          za[0] = prmt(za01, 0, 0x1010);
          za[1] = prmt(za01, 0, 0x3232);
          za[2] = prmt(za23, 0, 0x1010);
          za[3] = prmt(za23, 0, 0x3232);
          zb[0] = prmt(zb01, 0, 0x1010);
          zb[1] = prmt(zb01, 0, 0x3232);
          zb[2] = prmt(zb23, 0, 0x1010);
          zb[3] = prmt(zb23, 0, 0x3232);
        }
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
          // packed row kq*32 + roff + g of the stage
          const int roff = pr * 8 + qq * 4;
          const uint4 wv = *reinterpret_cast<const uint4*>(wq + roff * BN * 4);
          uint4 xv[MT];
#pragma unroll
          for (int tt = 0; tt < MT; ++tt) {
            // branch-free: lanes whose token does not exist read token 0's row; their MMA
            // columns are garbage that is never written out (an output column of the MMA
            // depends only on its own token column)
            const uint4 v = *reinterpret_cast<const uint4*>(xq + xoff[tt] + roff * 16);
            if constexpr (NAT) {
              xv[tt] = v;   // the weight fragments' pairs are (k0,k1) (k2,k3) (k4,k5) (k6,k7)
            } else {
              // (k0..k7) -> pairs (k0,k4) (k1,k5) (k2,k6) (k3,k7), the weight fragments' K order
              xv[tt] = make_uint4(prmt(v.x, v.z, 0x5410), prmt(v.x, v.z, 0x7632),
                                  prmt(v.y, v.w, 0x5410), prmt(v.y, v.w, 0x7632));
            }
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
                // permuted x: .x=(k0,k4) .y=(k1,k5) .z=(k2,k6) .w=(k3,k7)
                mma_16816(acc[qq][t][tt], a, h == 0 ? xv[tt].x : xv[tt].z, h == 0 ? xv[tt].y : xv[tt].w);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (++s == nst) { s = 0; ph ^= 1; }

    // ---------------------- end of a strip segment ----------------------
    if (k == KS - 1 || u == u1 - 1) {
      // reduce the K parts through shared memory
#pragma unroll
      for (int tt = 0; tt < MT; ++tt) {
        const int t0 = tt * 8 + 2 * g;
        const float4 v0 = make_float4(acc[0][0][tt][0] + acc[1][0][tt][0], acc[0][0][tt][2] + acc[1][0][tt][2],
                                      acc[0][1][tt][0] + acc[1][1][tt][0], acc[0][1][tt][2] + acc[1][1][tt][2]);
        const float4 v1 = make_float4(acc[0][0][tt][1] + acc[1][0][tt][1], acc[0][0][tt][3] + acc[1][0][tt][3],
                                      acc[0][1][tt][1] + acc[1][1][tt][1], acc[0][1][tt][3] + acc[1][1][tt][3]);
        *reinterpret_cast<float4*>(&red[((kq * MT * 8) + t0) * BN + ccol]) = v0;
        *reinterpret_cast<float4*>(&red[((kq * MT * 8) + t0 + 1) * BN + ccol]) = v1;
      }
      consumer_sync<NCW>();
      const bool whole = (k == KS - 1) && static_cast<long long>(c) * KS >= u0;
      if (whole && p.swiglu) {
        for (int idx = ctid; idx < M * (BN / 2); idx += NCW * 32) {
          const int t = idx / (BN / 2), o = idx % (BN / 2);
          const int cg = swiglu_gate_col(o);
          float vg = 0.0f, vu = 0.0f;
#pragma unroll
          for (int j = 0; j < KQ; ++j) {
            vg += red[(j * MT * 8 + t) * BN + cg];
            vu += red[(j * MT * 8 + t) * BN + cg + SWIGLU_BLOCK];
          }
          const int no = c * (BN / 2) + o;
          if (2 * no < p.N) static_cast<__half*>(p.y)[static_cast<long long>(t) * p.ldy + no] = swiglu_h(vg, vu);
        }
      } else if (whole) {
        for (int idx = ctid; idx < M * BN; idx += NCW * 32) {
          const int t = idx / BN, cc = idx % BN;
          float v = 0.0f;
#pragma unroll
          for (int j = 0; j < KQ; ++j) v += red[(j * MT * 8 + t) * BN + cc];
          const int n = c * BN + cc;
          if (n < p.N) emit<AR>(p, t, n, v, ar_epoch, smem_u32(ar_peer_smem));
        }
      } else if (u != u1 - 1) {
        // the first strip, which this CTA owns, ends here mid-range: park its piece
        for (int idx = ctid; idx < M * BN; idx += NCW * 32) {
          const int t = idx / BN, cc = idx % BN;
          float v = 0.0f;
#pragma unroll
          for (int j = 0; j < KQ; ++j) v += red[(j * MT * 8 + t) * BN + cc];
          park[t * BN + cc] = v;
        }
      }
      // (a final segment that is not a whole strip keeps its piece in red[] for below)
      if (u != u1 - 1) consumer_sync<NCW>();   // red[] is reused by the next segment
    }
    if (++k == KS) { k = 0; ++c; }
  }

  // ---------------- shared strips: publish the final piece, finish the owned strip ----------------
  const float* own_red = red;   // this CTA's piece of its final segment: sum over the K parts
  auto own_final = [&](int t, int cc) {
    float v = 0.0f;
#pragma unroll
    for (int j = 0; j < KQ; ++j) v += own_red[(j * MT * 8 + t) * BN + cc];
    return v;
  };
  if (publishes) {
    // the last strip continues in the next CTA: this segment is a piece for its owner
    unsigned long long* dst = p.pieces + static_cast<long long>(blockIdx.x) * (MT * 8) * BN;
    for (int idx = ctid; idx < M * BN; idx += NCW * 32) {
      const int t = idx / BN, cc = idx % BN;
      st_relaxed_gpu_u64(dst + t * BN + cc, PIECE_TAG | __float_as_uint(own_final(t, cc)));
    }
  }
  if (owns_first) {
    // y[:, strip c_first] = the pieces of CTAs pf .. this one, summed in CTA order
    const int cs = c_first;
    const int pf = range_i[4];
    const int me = static_cast<int>(blockIdx.x);
    const bool own_parked = c_last > c_first;   // else the strip is the final segment, in red[]
    bool waiting = true;                        // false once this thread's wait budget ran out
    for (int idx = ctid; idx < M * BN; idx += NCW * 32) {
      const int t = idx / BN, cc = idx % BN;
      const long long off = static_cast<long long>(t) * BN + cc;
      constexpr int MAXP = 8;   // pieces fetched before summing (more are summed in a loop)
      float v = 0.0f;
      for (int base = pf; base < me; base += MAXP) {
        unsigned long long w[MAXP];
#pragma unroll
        for (int i = 0; i < MAXP; ++i)
          w[i] = base + i < me ? ld_relaxed_gpu_u64(p.pieces + static_cast<long long>(base + i) * (MT * 8) * BN + off)
                               : PIECE_TAG;
#pragma unroll
        for (int i = 0; i < MAXP; ++i) {
          if (base + i >= me) break;
          unsigned long long* src = p.pieces + static_cast<long long>(base + i) * (MT * 8) * BN + off;
          uint64_t t0 = 0;
          for (uint32_t it = 0; waiting && (w[i] >> 32) != 1ull; ++it) {
            if (it == 0) {
              t0 = global_timer_ns();
            } else if ((it & 15u) == 0u && global_timer_ns() - t0 > p.wait_ns) {
              flag_error(kErrWaitTimeout);
              waiting = false;
              break;
            }
            __nanosleep(32);
            w[i] = ld_relaxed_gpu_u64(src);
          }
          v += __uint_as_float(static_cast<uint32_t>(w[i]));
          st_relaxed_gpu_u64(src, 0ull);   // consumed: the slot is zero for the next launch
        }
      }
      v += own_parked ? park[t * BN + cc] : own_final(t, cc);
      const int n = cs * BN + cc;
      if (p.swiglu) {
        park[t * BN + cc] = v;   // the strip's sums; paired below
      } else if (n < p.N) {
        emit<AR>(p, t, n, v, ar_epoch, smem_u32(ar_peer_smem));
      }
    }
    if (p.swiglu) {
      consumer_sync<NCW>();
      for (int idx = ctid; idx < M * (BN / 2); idx += NCW * 32) {
        const int t = idx / (BN / 2), o = idx % (BN / 2);
        const int cg = swiglu_gate_col(o);
        const int no = cs * (BN / 2) + o;
        if (2 * no < p.N)
          static_cast<__half*>(p.y)[static_cast<long long>(t) * p.ldy + no] =
              swiglu_h(park[t * BN + cg], park[t * BN + cg + SWIGLU_BLOCK]);
      }
    }
  }

  if (AR) {
    // ---------- fused all-reduce: the last ar_tail CTAs to arrive finish the call ----------
    // Every element's word reaches every rank's buffer from the CTA that finalised
    // it, so finishing needs no fence: a finishing CTA reads its share of the
    // elements in every rank's slot until each word carries this epoch's tag (the
    // words of this rank included), sums them in rank order and writes y. Only
    // CTAs that have finished their own units wait, and they wait only on other
    // CTAs' units, so the call completes whether or not the grid is co-resident.
    consumer_sync<NCW>();
    if (ctid == 0) {
      const int r = atomicAdd(p.ar_ctl + 1, 1);
      const int grid = static_cast<int>(gridDim.x);
      flag[3] = r - (grid - p.ar_tail);   // share index, negative: not finishing
      if (r == grid - 1) {
        // every CTA has read the epoch and arrived: advance both for the next launch
        p.ar_ctl[1] = 0;
        p.ar_ctl[0] = ar_epoch + 1;
      }
    }
    consumer_sync<NCW>();
    const int share = flag[3];
    if (share >= 0 && p.ar_gather) {
      // all-gather: y[t, q*N + n] = rank q's word (t, n), for this CTA's share of y.
      // A thread takes 4 consecutive elements per step (N % 8 == 0 keeps them in one
      // rank's row segment; shares start on multiples of 4) and issues their 4 loads
      // before polling any of them. (32-bit indices: the host keeps M * world * N
      // below 2^31; a thread's indices advance by the stride without divisions.)
      constexpr int VE = 4;
      const int NF = p.ar_world * p.N;
      const int total = M * NF;
      const int per = ((total + p.ar_tail - 1) / p.ar_tail + VE - 1) / VE * VE;
      const int lo = share * per;
      const int hi = lo + per < total ? lo + per : total;
      const unsigned long long* half_base =
          reinterpret_cast<const unsigned long long*>(p.ar_peer[p.ar_rank]) +
          static_cast<long long>(ar_epoch & 1) * p.ar_world * p.ar_slot;
      const uint32_t ar_tag = static_cast<uint32_t>(ar_epoch) + 1u;
      bool waiting = true;   // false once this thread's wait budget ran out
      const int e0 = lo + VE * ctid;
      int t = e0 / NF, q = (e0 - t * NF) / p.N;
      int n = e0 - t * NF - q * p.N;
      for (int e = e0; e < hi; e += VE * NCW * 32) {
        const int col = q * p.N + n;
        const unsigned long long* src = half_base + static_cast<long long>(q) * p.ar_slot + t * p.N + n;
        unsigned long long w[VE];
#pragma unroll
        for (int v = 0; v < VE; ++v) w[v] = ld_volatile_u64(src + v);
#pragma unroll
        for (int v = 0; v < VE; ++v) {
          uint64_t t0 = 0;
          for (uint32_t it = 0; waiting && static_cast<uint32_t>(w[v] >> 32) != ar_tag; ++it) {
            if (it == 0) {
              t0 = global_timer_ns();
            } else if ((it & 15u) == 0u && global_timer_ns() - t0 > p.wait_ns) {
              flag_error(kErrWaitTimeout);
              waiting = false;
              break;
            }
            __nanosleep(32);
            w[v] = ld_volatile_u64(src + v);
          }
        }
        __half* yrow = static_cast<__half*>(p.y) + static_cast<long long>(t) * p.ldy + col;
#pragma unroll
        for (int v = 0; v < VE; ++v) yrow[v] = __float2half_rn(__uint_as_float(static_cast<uint32_t>(w[v])));
        for (n += VE * NCW * 32; n >= p.N; n -= p.N) {
          if (++q == p.ar_world) {
            q = 0;
            ++t;
          }
        }
      }
    } else if (share >= 0) {
      // (32-bit indices: the host keeps M * N below 2^31)
      const int total = M * p.N;
      const int per = (total + p.ar_tail - 1) / p.ar_tail;
      const int lo = share * per;
      const int hi = lo + per < total ? lo + per : total;
      const unsigned long long* half_base =
          reinterpret_cast<const unsigned long long*>(p.ar_peer[p.ar_rank]) +
          static_cast<long long>(ar_epoch & 1) * p.ar_world * p.ar_slot;
      const uint32_t ar_tag = static_cast<uint32_t>(ar_epoch) + 1u;
      bool waiting = true;   // false once this thread's wait budget ran out
      int t = (lo + ctid) / p.N, n = lo + ctid - t * p.N;
      for (int e = lo + ctid; e < hi; e += NCW * 32) {
        unsigned long long w[AR_MAX_RANKS];
#pragma unroll
        for (int q = 0; q < AR_MAX_RANKS; ++q)
          if (q < p.ar_world) w[q] = ld_volatile_u64(half_base + q * p.ar_slot + e);
        float a = 0.0f;
#pragma unroll
        for (int q = 0; q < AR_MAX_RANKS; ++q) {
          if (q >= p.ar_world) break;
          uint64_t t0 = 0;
          for (uint32_t it = 0; waiting && static_cast<uint32_t>(w[q] >> 32) != ar_tag; ++it) {
            if (it == 0) {
              t0 = global_timer_ns();
            } else if ((it & 15u) == 0u && global_timer_ns() - t0 > p.wait_ns) {
              flag_error(kErrWaitTimeout);
              waiting = false;
              break;
            }
            __nanosleep(32);
            w[q] = ld_volatile_u64(half_base + q * p.ar_slot + e);
          }
          const float v = __uint_as_float(static_cast<uint32_t>(w[q]));
          a = q == 0 ? v : a + v;   // rank order
        }
        // y = fp16(sum) [+ bias, rounded again]
        __half h = __float2half_rn(a);
        if (p.bias != nullptr) h = __float2half_rn(__half2float(h) + __half2float(p.bias[n]));
        static_cast<__half*>(p.y)[static_cast<long long>(t) * p.ldy + n] = h;
        for (n += NCW * 32; n >= p.N; n -= p.N) ++t;
      }
    }
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
                                void* __restrict__ y, int y_f32, int M, int N, int K, int G,
                                long long ldy, int y_bf16) {
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
        const long long o = static_cast<long long>(m) * ldy + n;
        if (y_f32) {
          static_cast<float*>(y)[o] = acc[m];
        } else {
          static_cast<unsigned short*>(y)[o] = static_cast<unsigned short>(out_bits(acc[m], bias, n, y_bf16 != 0));
        }
      }
    }
  }
}

}  // namespace decode
}  // namespace w4a16
