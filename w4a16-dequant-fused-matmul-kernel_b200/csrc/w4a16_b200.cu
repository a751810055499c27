// w4a16_b200.cu -- the C ABI (include/w4a16_b200.h) over the sm_100a kernels.
//
// The library is a single translation unit: the kernels live in the .cuh
// files included below so that the one sticky device error word has exactly
// one definition without relocatable device code.
//
// Host-side duties: argument validation with the reference's rules
// (w4a16-kernel/src/w4a16/triton_kernel.py:153-182, quant.py:116-119), the
// per-device sm_100 check and kernel attributes, TMA tensor-map encoding, the
// M-bucket routing between the decode and prefill kernels, and turning CUDA
// launch errors into status codes. Nothing here allocates or synchronises
// (except w4a16_check_device_errors, which must read the device flag).

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "decode_gemv.cuh"
#include "prefill_tcgen05.cuh"
#include "prefill_ts.cuh"
#include "quantize.cuh"

namespace w4a16 {
namespace {

constexpr int kMaxDevices = 64;

struct DeviceState {
  bool checked = false;
  bool is_sm100 = false;
  bool attrs_set = false;
  int num_sms = 0;
  // set (release) once the fields above are final for an sm_100 device: later calls
  // read them without taking the mutex
  std::atomic<bool> ready{false};
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
// Budget of every bounded wait in the kernels launched from now on (process-wide).
std::atomic<unsigned long long> g_wait_budget_ns{kWaitBudgetNs};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int current_device_state(DeviceState** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return W4A16_ERR_DEVICE;
  }
  if (g_dev[dev].ready.load(std::memory_order_acquire)) {
    *out = &g_dev[dev];
    return W4A16_OK;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& d = g_dev[dev];
  if (!d.checked) {
    int major = 0, minor = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      cudaGetLastError();
      return W4A16_ERR_DEVICE;
    }
    d.is_sm100 = (major == 10 && minor == 0);
    d.num_sms = sms;
    d.checked = true;
  }
  if (!d.is_sm100) return W4A16_ERR_DEVICE;
  if (!d.attrs_set) {
    auto set_prefill = [](auto kern) {
      return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, prefill::SMEM_BYTES) ==
             cudaSuccess;
    };
    if (!set_prefill(prefill::w4a16_tcgen05_kernel<false, false>) ||
        !set_prefill(prefill::w4a16_tcgen05_kernel<true, false>) ||
        !set_prefill(prefill::w4a16_tcgen05_kernel<false, true>) ||
        !set_prefill(prefill::w4a16_tcgen05_kernel<true, true>)) {
      cudaGetLastError();
      return W4A16_ERR_LAUNCH;
    }
    auto set_ts = [](auto kern) {
      return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, prefill_ts::SMEM_BYTES) ==
             cudaSuccess;
    };
    if (!set_ts(prefill_ts::w4a16_ts_kernel<false, false>) || !set_ts(prefill_ts::w4a16_ts_kernel<false, true>) ||
        !set_ts(prefill_ts::w4a16_ts_kernel<true, false>) || !set_ts(prefill_ts::w4a16_ts_kernel<true, true>)) {
      cudaGetLastError();
      return W4A16_ERR_LAUNCH;
    }
    auto set_decode = [](auto kern) {
      return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) ==
                 cudaSuccess &&
             cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) ==
                 cudaSuccess;
    };
    if (!set_decode(decode::decode_gemv_tma_kernel<1, false>) ||
        !set_decode(decode::decode_gemv_tma_kernel<2, false>) ||
        !set_decode(decode::decode_gemv_tma_kernel<3, false>) ||
        !set_decode(decode::decode_gemv_tma_kernel<4, false>) ||
        !set_decode(decode::decode_gemv_tma_kernel<1, true>) ||
        !set_decode(decode::decode_gemv_tma_kernel<2, true>) ||
        !set_decode(decode::decode_gemv_tma_kernel<3, true>) ||
        !set_decode(decode::decode_gemv_tma_kernel<4, true>) ||
        !set_decode(decode::decode_gemv_tma_kernel<1, false, true>) ||
        !set_decode(decode::decode_gemv_tma_kernel<2, false, true>) ||
        !set_decode(decode::decode_gemv_tma_kernel<3, false, true>) ||
        !set_decode(decode::decode_gemv_tma_kernel<4, false, true>)) {
      cudaGetLastError();
      return W4A16_ERR_LAUNCH;
    }
    d.attrs_set = true;
  }
  d.ready.store(true, std::memory_order_release);
  *out = &d;
  return W4A16_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    } else {
      cudaGetLastError();
    }
  }
  return g_encode;
}

// Encoded tensor maps, cached per host thread. A map is a pure function of the
// encode arguments below (address, type, extents, pitch, box, swizzle), so a hit
// is exactly the map an encode would produce; decode GEMMs re-use the same
// weights every step, and the encode costs ~1 us of host time per map.
struct MapKey {
  const void* base;
  uint64_t cols, rows, ld;
  uint32_t box_cols, box_rows;
  int dt, swz;
  bool operator==(const MapKey& o) const {
    return base == o.base && cols == o.cols && rows == o.rows && ld == o.ld &&
           box_cols == o.box_cols && box_rows == o.box_rows && dt == o.dt && swz == o.swz;
  }
};
struct MapEntry {
  bool valid = false;
  MapKey key;
  CUtensorMap map;
};
constexpr int kMapCacheSlots = 64;   // direct-mapped
thread_local MapEntry t_map_cache[kMapCacheSlots];

inline size_t map_slot(const MapKey& k) {
  uint64_t h = reinterpret_cast<uintptr_t>(k.base) * 0x9E3779B97F4A7C15ull;
  h ^= (k.cols * 0x100000001B3ull) ^ (k.rows << 17) ^ (k.ld << 7) ^
       (static_cast<uint64_t>(k.box_cols) << 40) ^ (static_cast<uint64_t>(k.box_rows) << 52) ^
       (static_cast<uint64_t>(k.dt) << 3) ^ static_cast<uint64_t>(k.swz);
  h ^= h >> 29;
  return static_cast<size_t>(h % kMapCacheSlots);
}

// 2D row-major tensor map: `cols` contiguous elements per row, `rows` rows,
// row pitch `ld` elements; box [box_cols x box_rows]; out-of-range boxes
// read as zero.
bool make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t cols,
                 uint64_t rows, uint64_t ld, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swz) {
  const MapKey key{base, cols, rows, ld, box_cols, box_rows, static_cast<int>(dt), static_cast<int>(swz)};
  MapEntry& slot = t_map_cache[map_slot(key)];
  if (slot.valid && slot.key == key) {
    *m = slot.map;
    return true;
  }
  PFN_cuTensorMapEncodeTiled_v12000 enc = get_encode_fn();
  if (enc == nullptr) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * static_cast<uint64_t>(esize)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  if (enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  slot.valid = true;
  slot.key = key;
  slot.map = *m;
  return true;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

dim3 grid_2d(int64_t x, int64_t y) {
  return dim3(static_cast<unsigned>(x), static_cast<unsigned>(y), 1);
}

// ---------------------------------------------------------------------------
// GEMM launchers
// ---------------------------------------------------------------------------
// Decode launch plan: ring depth, grid (one resident wave) and workspace.
struct DecodePlan {
  int MT = 1, nst = 2, grid = 0, kstages = 0, chunks = 0;
  long long units = 0;
  size_t smem = 0;
  size_t piece_bytes = 0;
  size_t workspace() const { return piece_bytes; }
};

int plan_decode(DeviceState& dev, int M, int N, int K, DecodePlan* out) {
  DecodePlan d;
  d.MT = (M + 7) / 8;
  d.kstages = (K + decode::KSTAGE - 1) / decode::KSTAGE;
  d.chunks = (N + decode::BN - 1) / decode::BN;
  d.units = static_cast<long long>(d.chunks) * d.kstages;
  const int sbytes = decode::stage_bytes(M);
  // Ring depth: ~190 KB of stages plus the reduction buffer per SM, split between the CTAs
  // that share an SM (>= 2, <= 8 stages per CTA).
  const int ring_budget = (decode::ctas_per_sm(d.MT) == 2 ? 108 : 190) * 1024;
  int nst = (ring_budget - decode::red_bytes(d.MT) - decode::park_bytes(d.MT)) / sbytes;
  nst = nst < 2 ? 2 : (nst > 8 ? 8 : nst);
  d.nst = nst;
  d.smem = 1024 + static_cast<size_t>(nst) * sbytes + decode::red_bytes(d.MT) + decode::park_bytes(d.MT) +
           2 * nst * sizeof(uint64_t) + 64 + 64 + 64;
  long long grid = static_cast<long long>(dev.num_sms) * decode::ctas_per_sm(d.MT);
  if (grid > d.units) grid = d.units;
  d.grid = static_cast<int>(grid);
  d.piece_bytes = static_cast<size_t>(d.grid) * (d.MT * 8) * decode::BN * sizeof(unsigned long long);
  *out = d;
  return W4A16_OK;
}

// Fused all-reduce arguments of the decode kernel (world 0: off).
struct ArArgs {
  int world = 0, rank = 0;
  int gather = 0;                               // 1: all-gather instead of all-reduce
  const unsigned long long* peers = nullptr;   // host array [world]
  int* ctl = nullptr;
  long long slot = 0;
};

int launch_decode_tma(DeviceState& dev, const __half* x, const int32_t* qw, const __half* s,
                      const __half* z, const __half* bias, void* y, int y_f32, int M, int N, int K, int G,
                      long long ldy, void* workspace, int64_t workspace_bytes,
                      cudaStream_t stream, const ArArgs& ar = ArArgs(), int swiglu = 0, int nat = 0,
                      int y_bf16 = 0) {
  DecodePlan d;
  int st = plan_decode(dev, M, N, K, &d);
  if (st != W4A16_OK) return st;
  if (workspace == nullptr || workspace_bytes < static_cast<int64_t>(d.workspace()) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return W4A16_ERR_WORKSPACE;
  CUtensorMap tw, ts, tz, tx;
  if (!make_map_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, qw, N, K / 8, N, decode::BN,
                   decode::ROWS, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map_2d(&ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, s, N, K / G, N, decode::BN,
                   decode::SZ_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map_2d(&tz, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, z, N, K / G, N, decode::BN,
                   decode::SZ_ROWS, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x, K, M, K, decode::XBOX, M,
                   CU_TENSOR_MAP_SWIZZLE_NONE)) {
    return W4A16_ERR_ALIGNMENT;
  }
  decode::Params p;
  p.bias = bias;
  p.y = y;
  p.y_f32 = y_f32;
  p.pieces = static_cast<unsigned long long*>(workspace);
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = G;
  p.g_shift = ((G & (G - 1)) == 0) ? __builtin_ctz(static_cast<unsigned>(G)) : -1;
  p.ldy = ldy;
  p.kstages = d.kstages;
  p.units = d.units;
  p.num_stages = d.nst;
  p.ar_world = ar.world;
  p.ar_rank = ar.rank;
  p.ar_gather = ar.gather;
  p.ar_ctl = ar.ctl;
  p.ar_slot = ar.slot;
  p.ar_tail = 0;
  p.swiglu = swiglu;
  p.y_bf16 = y_bf16;
  p.wait_ns = g_wait_budget_ns.load(std::memory_order_relaxed);
  for (int q = 0; q < decode::AR_MAX_RANKS; ++q) p.ar_peer[q] = q < ar.world ? ar.peers[q] : 0ull;
  if (ar.world > 1) {
    // enough finishing CTAs that each thread finishes AR_ELEMS_PER_THREAD output elements
    const long long per_cta = static_cast<long long>(decode::ncw_for(d.MT)) * 32 * decode::AR_ELEMS_PER_THREAD;
    const long long elems = static_cast<long long>(M) * N * (ar.gather ? ar.world : 1);
    const long long tail = (elems + per_cta - 1) / per_cta;
    p.ar_tail = static_cast<int>(tail < 1 ? 1 : (tail > d.grid ? d.grid : tail));
  }

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(d.grid), 1, 1);
  cfg.blockDim = dim3(decode::threads_for(d.MT), 1, 1);
  cfg.dynamicSmemBytes = d.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  const bool fused = ar.world > 1;
  if (nat && !fused) {
    switch (d.MT) {
      case 1: e = cudaLaunchKernelEx(&cfg, decode::decode_gemv_tma_kernel<1, false, true>, tw, ts, tz, tx, p); break;
      case 2: e = cudaLaunchKernelEx(&cfg, decode::decode_gemv_tma_kernel<2, false, true>, tw, ts, tz, tx, p); break;
      case 3: e = cudaLaunchKernelEx(&cfg, decode::decode_gemv_tma_kernel<3, false, true>, tw, ts, tz, tx, p); break;
      default: e = cudaLaunchKernelEx(&cfg, decode::decode_gemv_tma_kernel<4, false, true>, tw, ts, tz, tx, p); break;
    }
  } else if (nat) {
    return W4A16_ERR_INVALID;   // the fused collectives read the reference nibble order
  } else switch (d.MT * 2 + (fused ? 1 : 0)) {
    case 2: e = cudaLaunchKernelEx(&cfg, decode::decode_gemv_tma_kernel<1, false>, tw, ts, tz, tx, p); break;
    case 3: e = cudaLaunchKernelEx(&cfg, decode::decode_gemv_tma_kernel<1, true>, tw, ts, tz, tx, p); break;
    case 4: e = cudaLaunchKernelEx(&cfg, decode::decode_gemv_tma_kernel<2, false>, tw, ts, tz, tx, p); break;
    case 5: e = cudaLaunchKernelEx(&cfg, decode::decode_gemv_tma_kernel<2, true>, tw, ts, tz, tx, p); break;
    case 6: e = cudaLaunchKernelEx(&cfg, decode::decode_gemv_tma_kernel<3, false>, tw, ts, tz, tx, p); break;
    case 7: e = cudaLaunchKernelEx(&cfg, decode::decode_gemv_tma_kernel<3, true>, tw, ts, tz, tx, p); break;
    case 8: e = cudaLaunchKernelEx(&cfg, decode::decode_gemv_tma_kernel<4, false>, tw, ts, tz, tx, p); break;
    default: e = cudaLaunchKernelEx(&cfg, decode::decode_gemv_tma_kernel<4, true>, tw, ts, tz, tx, p); break;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return W4A16_ERR_LAUNCH;
  }
  return W4A16_OK;
}

int launch_decode_fallback(const __half* x, const int32_t* qw, const __half* s, const __half* z,
                           const __half* bias, void* y, int y_f32, int64_t M, int N, int K, int G,
                           long long ldy, cudaStream_t stream, int y_bf16 = 0) {
  for (int64_t m0 = 0; m0 < M; m0 += 32) {
    const int mc = static_cast<int>(M - m0 < 32 ? M - m0 : 32);
    decode::decode_gemv_fallback_kernel<<<grid_2d((N + decode::FB_THREADS - 1) / decode::FB_THREADS, 1),
                                          decode::FB_THREADS, 0, stream>>>(
        x + m0 * K, qw, s, z, bias,
        static_cast<uint8_t*>(y) + m0 * ldy * (y_f32 ? sizeof(float) : sizeof(__half)), y_f32, mc,
        N, K, G, ldy, y_bf16);
    W4A16_RETURN_IF_LAUNCH_FAILED();
  }
  return W4A16_OK;
}

// Tile width of the prefill kernel for this shape: the candidate with the least
// modelled time = waves of tiles x cycles per K step, where a step costs the
// larger of its MMAs (4 * bn cycles) and its operand traffic (x tile 32 KB plus
// a per-column share, at the ~32 B/clk per SM measured on B200). Wider tiles
// reuse the x tile more; narrower ones can round the tile count to whole waves.
int choose_prefill_bn(int M, int N, int num_sms, int halves) {
  const int bm = prefill::BMH * halves;
  const long long m_tiles = (M + bm - 1) / bm;
  int best = prefill::BN_MAX;
  double best_t = 1e300;
  const int bn_min = halves == 2 ? prefill::BN_MIN : prefill::BN_MIN_SINGLE;
  for (int bn = prefill::BN_MAX; bn >= bn_min; bn -= 32) {
    const long long tiles = m_tiles * ((N + bn - 1) / bn);
    const long long waves = (tiles + num_sms - 1) / num_sms;
    const double step = std::max(2.0 * halves * bn, (prefill::A_BYTES / 2 * halves + 36.0 * bn) / 31.5);
    const double t = static_cast<double>(waves) * step;
    if (t < best_t * 0.999) {
      best_t = t;
      best = bn;
    }
  }
  return best;
}

int launch_prefill(const DeviceState& dev, const __half* x, const int32_t* qw, const __half* s,
                   const __half* z, const __half* bias, void* y, int y_f32, int M, int N, int K, int G,
                   long long ldy, cudaStream_t stream, int swiglu = 0, int nat = 0, int y_bf16 = 0) {
  // up to 128 tokens one 128-row MMA half per tile: no idle MMA rows, half the x traffic,
  // and narrower tiles (bn down to 64) so that one row of tiles spreads over the SMs
  const int halves = M <= prefill::BMH ? 1 : 2;
  const int bn = choose_prefill_bn(M, N, dev.num_sms, halves);
  CUtensorMap tx, ty;
  if (!make_map_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x, K, M, K, prefill::BK,
                   static_cast<uint32_t>(prefill::BMH * halves), CU_TENSOR_MAP_SWIZZLE_128B)) {
    return W4A16_ERR_ALIGNMENT;
  }
  // y through TMA stores when its base and row pitch are 16-byte aligned: 32 x 32
  // boxes, fp16 rows of 64 B (64-byte swizzle) or fp32 rows of 128 B (128-byte swizzle).
  const bool y_aligned = aligned16(y) && (ldy % (y_f32 ? 4 : 8)) == 0;
  const bool tma_store =
      !swiglu && y_aligned && (y_f32 ? make_map_2d(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, y, N, M, ldy, 32, 32,
                                        CU_TENSOR_MAP_SWIZZLE_128B)
                          : make_map_2d(&ty, y_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                        2, y, N, M, ldy, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B));
  if (!tma_store) ty = tx;   // unused by the kernel
  prefill::Params p;
  p.tma_store = tma_store ? 1 : 0;
  p.qw = qw;
  p.scales = s;
  p.zeros = z;
  p.bias = bias;
  p.y = y;
  p.y_f32 = y_f32;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = G;
  p.g_shift = ((G & (G - 1)) == 0) ? __builtin_ctz(static_cast<unsigned>(G)) : -1;
  p.ldy = ldy;
  p.halves = halves;
  p.bm = prefill::BMH * halves;
  p.m_tiles = (M + p.bm - 1) / p.bm;
  p.n_tiles = (N + bn - 1) / bn;
  p.bn = bn;
  p.idesc = umma_idesc_f16_f32(prefill::BMH, static_cast<uint32_t>(bn));
  p.vec_store = (aligned16(y) && (ldy % (y_f32 ? 4 : 8)) == 0) ? 1 : 0;
  p.swiglu = swiglu;
  p.y_bf16 = y_bf16;
  p.wait_ns = g_wait_budget_ns.load(std::memory_order_relaxed);
  const long long tiles = static_cast<long long>(p.m_tiles) * p.n_tiles;
  if (tiles > 0x7fffffffLL) return W4A16_ERR_INVALID;   // the kernels index tiles with int
  const int grid = static_cast<int>(tiles < dev.num_sms ? tiles : dev.num_sms);
  const dim3 blk(prefill::THREADS);
  if (swiglu && nat)
    prefill::w4a16_tcgen05_kernel<true, true><<<grid, blk, prefill::SMEM_BYTES, stream>>>(tx, ty, p);
  else if (swiglu)
    prefill::w4a16_tcgen05_kernel<true, false><<<grid, blk, prefill::SMEM_BYTES, stream>>>(tx, ty, p);
  else if (nat)
    prefill::w4a16_tcgen05_kernel<false, true><<<grid, blk, prefill::SMEM_BYTES, stream>>>(tx, ty, p);
  else
    prefill::w4a16_tcgen05_kernel<false, false><<<grid, blk, prefill::SMEM_BYTES, stream>>>(tx, ty, p);
  W4A16_RETURN_IF_LAUNCH_FAILED();
  return W4A16_OK;
}

// Which prefill kernel (and, for the TMEM-operand one, how many tokens per tile) a
// shape gets: the smaller of waves x K steps x step time, with the step times measured
// on B200 (M=8192, K=4096, N=14336 and the MLP block's shapes; L2 flushed):
//   shared-memory operand kernel, 256 x 224 tile: ~1.12 us per 64-K step, nearly flat
//     in bn (the x tile's shared-memory traffic dominates; the relative model of
//     choose_prefill_bn scales it);
//   TMEM-operand kernel, 256 weight columns x mt tokens: ~0.82 us at mt = 192, ~0.7 of
//     it independent of mt.
//   shared-memory operand kernel, single 128-row half (M <= 128): ~1.07 us per step,
//     latency-bound (its dequantisers prefetch only two steps ahead), whatever bn.
// The TMEM-operand tile does ~1.17x the work per unit time, so it wins unless its
// coarser wave quantisation loses more (N = 8192 at M = 2048), which its K splits
// (split_cost_us) partly recover. At 33-128 tokens it takes 42-46 vs 68.5 us (K=4096,
// N=14336) and 101-104 vs 138 us (K=8192, N=28672). w4a16_set_prefill_kernel()
// overrides the choice (tests exercise both).
std::atomic<int> g_prefill_kernel{W4A16_PREFILL_AUTO};

double ss_step_model(int bn, int halves) {
  return std::max(2.0 * halves * bn, (prefill::A_BYTES / 2 * halves + 36.0 * bn) / 31.5);
}

// The TMEM-operand kernel's split-K area starts at byte W4A16_NOALLOC_SCRATCH_BYTES of
// the workspace, past the decode kernel's piece words (one workspace serves every shape):
// a fixed region of arrival counters (left zero, and never overlapped by partials of any
// shape), then the fp32 partial tiles.
constexpr long long kSplitCounterBytes = 64 * 1024;   // 16384 counters = 2048 tiles of 8 slices

// The tiles that run whole ahead of the split ones: none when every tile is split (the
// tiles do not fill one wave of CTAs), else the tiles of the full waves of a grid of
// num_sms CTAs, so that each CTA runs the same number of whole tiles and then the split
// items of the last wave's tiles.
long long ts_whole_tiles(long long tiles, int splits, int num_sms) {
  if (splits <= 1) return tiles;
  return tiles < num_sms ? 0 : tiles / num_sms * num_sms;
}

long long ts_split_bytes(int M, int N, int mt, int splits, int num_sms) {
  if (splits <= 1) return 0;
  const long long tiles = static_cast<long long>((M + mt - 1) / mt) * ((N + prefill_ts::NT - 1) / prefill_ts::NT);
  const long long split_tiles = tiles - ts_whole_tiles(tiles, splits, num_sms);
  return kSplitCounterBytes + split_tiles * splits * prefill_ts::EPI_WARPS * 32LL * mt * 4;
}

// K splits of the TMEM-operand kernel: at most kMaxSplits parts of at least 8 steps. A split
// costs its pipeline restart plus, in the last split to arrive, one L2 round trip per
// 32-token chunk for each other split's partial: ~4 + 6.5 x sp x mt / 192 us, fitted on B200
// (K=4096, N=14336, mt=192, M=512..8192 with 2-7 splits of the last wave's tiles).
constexpr int kMaxSplits = 8;
double split_cost_us(int mt, int sp) { return 4.0 + 6.5 * sp * mt / 192.0; }

int choose_prefill_kernel(int M, int N, int K, int num_sms, int* ts_mt, int* ts_splits = nullptr) {
  const int force = g_prefill_kernel.load(std::memory_order_relaxed);
  const int KT = K / prefill::BK;
  const double kt = KT;
  auto waves = [num_sms](long long tiles) { return static_cast<double>((tiles + num_sms - 1) / num_sms); };
  int best_mt = prefill_ts::MT_MAX, best_splits = 1;
  double t_ts = 1e300;
  for (int mt = prefill_ts::MT_MAX; mt >= prefill_ts::MT_MIN; mt -= 32) {
    const long long tiles = static_cast<long long>((M + mt - 1) / mt) * ((N + prefill_ts::NT - 1) / prefill_ts::NT);
    const double step = 0.82 * (0.7 + 0.3 * mt / 192.0);
    // K split into `sp` parts when the tiles do not fill one wave of CTAs (every tile
    // split: each split writes a fp32 partial tile and the last one reads them all back).
    const bool may_split = tiles < num_sms && tiles * prefill_ts::EPI_WARPS * 4 <= kSplitCounterBytes;
    // With more tiles than CTAs, only the last, partly filled wave's tiles may be split,
    // into as many parts as keep that wave to one pass of the grid: the full waves' time
    // plus one split's steps plus the split's cost.
    const long long full = tiles / num_sms * num_sms, rem = tiles - full;
    const bool may_split_tail = full > 0 && rem > 0;
    for (int sp = 1; sp <= kMaxSplits && (sp == 1 || KT / sp >= 8); ++sp) {
      double t;
      if (sp == 1) {
        t = waves(tiles) * kt * step;
      } else if (may_split) {
        t = waves(tiles * sp) * ((KT + sp - 1) / sp) * step + split_cost_us(mt, sp);
      } else if (may_split_tail && rem * sp <= num_sms) {
        t = static_cast<double>(full / num_sms) * kt * step + ((KT + sp - 1) / sp) * step + split_cost_us(mt, sp);
      } else {
        break;
      }
      // 3 % margin for a different tile height; 1 % for K splits against the whole tiles of
      // the same height (measured on B200: splitting the last wave's tiles gained 1.3-1.9 % at
      // M=4096 and 8192, K=4096, N=14336, under the model's ~2 %)
      const double margin = sp > 1 && best_mt == mt ? 0.99 : 0.97;
      if (t < t_ts * margin) {
        t_ts = t;
        best_mt = mt;
        best_splits = sp;
      }
    }
  }
  *ts_mt = best_mt;
  if (ts_splits != nullptr) *ts_splits = best_splits;
  if (force == W4A16_PREFILL_TMEM_A) return W4A16_PREFILL_TMEM_A;
  if (force == W4A16_PREFILL_SMEM_B) return W4A16_PREFILL_SMEM_B;
  double t_ss;
  if (M <= prefill::BMH) {
    const int bn = choose_prefill_bn(M, N, num_sms, 1);
    t_ss = waves((N + bn - 1) / bn) * kt * 1.07;
  } else {
    const int bn = choose_prefill_bn(M, N, num_sms, 2);
    const long long ss_tiles = static_cast<long long>((M + prefill::BM - 1) / prefill::BM) * ((N + bn - 1) / bn);
    t_ss = waves(ss_tiles) * kt * 1.12 * ss_step_model(bn, 2) / ss_step_model(prefill::BN_MAX, 2);
  }
  return t_ts < t_ss ? W4A16_PREFILL_TMEM_A : W4A16_PREFILL_SMEM_B;
}

int launch_prefill_ts(const DeviceState& dev, const __half* x, const int32_t* qw, const __half* s,
                      const __half* z, const __half* bias, void* y, int y_f32, int M, int N, int K, int G,
                      long long ldy, cudaStream_t stream, int swiglu, int nat, int y_bf16, int mt, int splits,
                      void* workspace, int64_t workspace_bytes) {
  CUtensorMap tx, ty, tw, tsc, tz;
  if (!make_map_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x, K, M, K, prefill_ts::BK,
                   static_cast<uint32_t>(mt), CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_map_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, qw, N, K / 8, N, prefill_ts::NT, prefill_ts::BK / 8,
                   CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map_2d(&tsc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, s, N, K / G, N, prefill_ts::NT, 1,
                   CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !make_map_2d(&tz, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, z, N, K / G, N, prefill_ts::NT, 1,
                   CU_TENSOR_MAP_SWIZZLE_NONE)) {
    return W4A16_ERR_ALIGNMENT;
  }
  const bool y_aligned = aligned16(y) && (ldy % (y_f32 ? 4 : 8)) == 0;
  const bool tma_store =
      !swiglu && y_aligned && (y_f32 ? make_map_2d(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, y, N, M, ldy, 32, 32,
                                                   CU_TENSOR_MAP_SWIZZLE_128B)
                          : make_map_2d(&ty, y_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                                        2, y, N, M, ldy, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B));
  if (!tma_store) ty = tx;   // unused by the kernel
  prefill_ts::Params p;
  p.tma_store = tma_store ? 1 : 0;
  p.bias = bias;
  p.y = y;
  p.y_f32 = y_f32;
  p.y_bf16 = y_bf16;
  p.M = M;
  p.N = N;
  p.K = K;
  p.G = G;
  p.g_shift = ((G & (G - 1)) == 0) ? __builtin_ctz(static_cast<unsigned>(G)) : -1;
  p.ldy = ldy;
  p.mt = mt;
  p.m_tiles = (M + mt - 1) / mt;
  p.n_tiles = (N + prefill_ts::NT - 1) / prefill_ts::NT;
  p.dsets = 4 * mt + 128 <= static_cast<int>(prefill_ts::TMEM_COLS) ? 2 : 1;
  p.a_col0 = p.dsets * 2 * mt;
  p.astages = std::min(prefill_ts::AST_MAX, (static_cast<int>(prefill_ts::TMEM_COLS) - p.a_col0) / 64);
  if (p.astages < 2) return W4A16_ERR_INVALID;
  p.xstages = std::min(prefill_ts::TST_MAX, prefill_ts::X_RING_BYTES / (mt * prefill_ts::BK * 2));
  p.idesc = umma_idesc_f16_f32(128, static_cast<uint32_t>(mt));
  p.wait_ns = g_wait_budget_ns.load(std::memory_order_relaxed);
  const long long tiles = static_cast<long long>(p.m_tiles) * p.n_tiles;
  // split K only with room for the split area past the decode region of the workspace
  const long long need = W4A16_NOALLOC_SCRATCH_BYTES + ts_split_bytes(M, N, mt, splits, dev.num_sms);
  if (splits > 1 && (workspace == nullptr || workspace_bytes < need ||
                     (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0))
    splits = 1;
  p.splits = splits;
  p.counters = nullptr;
  p.partial = nullptr;
  if (splits > 1) {
    uint8_t* area = static_cast<uint8_t*>(workspace) + W4A16_NOALLOC_SCRATCH_BYTES;
    p.counters = reinterpret_cast<unsigned int*>(area);
    p.partial = reinterpret_cast<float*>(area + kSplitCounterBytes);
  }
  const long long whole = ts_whole_tiles(tiles, splits, dev.num_sms);
  p.whole = static_cast<int>(std::min<long long>(whole, 0x7fffffffLL));
  const long long items = whole + (tiles - whole) * splits;
  if (items > 0x7fffffffLL || tiles > 0x7fffffffLL) return W4A16_ERR_INVALID;   // the kernels index work items with int
  const int grid = static_cast<int>(items < dev.num_sms ? items : dev.num_sms);
  const dim3 blk(prefill_ts::THREADS);
  if (swiglu && nat)
    prefill_ts::w4a16_ts_kernel<true, true><<<grid, blk, prefill_ts::SMEM_BYTES, stream>>>(tx, ty, tw, tsc, tz, p);
  else if (swiglu)
    prefill_ts::w4a16_ts_kernel<true, false><<<grid, blk, prefill_ts::SMEM_BYTES, stream>>>(tx, ty, tw, tsc, tz, p);
  else if (nat)
    prefill_ts::w4a16_ts_kernel<false, true><<<grid, blk, prefill_ts::SMEM_BYTES, stream>>>(tx, ty, tw, tsc, tz, p);
  else
    prefill_ts::w4a16_ts_kernel<false, false><<<grid, blk, prefill_ts::SMEM_BYTES, stream>>>(tx, ty, tw, tsc, tz, p);
  W4A16_RETURN_IF_LAUNCH_FAILED();
  return W4A16_OK;
}

// h[m, n] = silu(g) * u with g = gate_up[m, n], u = gate_up[m, N + n]: the
// SwiGLU between the fused gate/up projection and the down projection of an
// MLP block, computed in fp32 and rounded once to fp16.
__global__ void swiglu_kernel(const __half* __restrict__ gu, __half* __restrict__ h, int64_t M,
                              int64_t N, int64_t ld_in, int64_t ld_out) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= M * N) return;
  const int64_t m = idx / N, n = idx % N;
  h[m * ld_out + n] = swiglu_h(__half2float(gu[m * ld_in + n]), __half2float(gu[m * ld_in + N + n]));
}

// dst[i] = round(src[i]) between fp16 / bf16 / fp32 (to fp16 or bf16): activations of a
// bf16 model are taken to fp16 this way before the GEMM (exact for |x| in [2^-14, 65504]).
__global__ void __launch_bounds__(256) convert_kernel(const void* src, int src_dtype, void* dst, int dst_dtype,
                                                      int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = src_dtype == W4A16_DTYPE_F16 ? __half2float(static_cast<const __half*>(src)[i])
                  : src_dtype == W4A16_DTYPE_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(src)[i])
                                                  : static_cast<const float*>(src)[i];
  if (dst_dtype == W4A16_DTYPE_BF16)
    static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(v);
  else
    static_cast<__half*>(dst)[i] = __float2half_rn(v);
}

// dst = src in 16-byte units, as a kernel that chains with the kernels around it
// under programmatic dependent launch (a memory-copy node in a CUDA graph would
// make the next GEMM wait for its predecessor's full completion instead). It lets
// the next kernel launch at once; with src_ready it reads its source before waiting
// for the previous kernel (the source must not be written by an earlier kernel, e.g.
// inputs the host placed in pinned memory), otherwise after; it writes only after
// that wait, so it completes after its predecessor, like the GEMMs.
constexpr int STAGE_THREADS = 256;
constexpr int STAGE_PER_THREAD = 4;   // 16-byte units per thread
__global__ void __launch_bounds__(STAGE_THREADS)
    stage_kernel(const uint4* src, uint4* dst, int64_t n16, int src_ready) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t base = static_cast<int64_t>(blockIdx.x) * STAGE_THREADS * STAGE_PER_THREAD + threadIdx.x;
  uint4 v[STAGE_PER_THREAD];
  if (!src_ready) asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll
  for (int i = 0; i < STAGE_PER_THREAD; ++i) {
    const int64_t j = base + static_cast<int64_t>(i) * STAGE_THREADS;
    if (j < n16) v[i] = src[j];
  }
  if (src_ready) asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll
  for (int i = 0; i < STAGE_PER_THREAD; ++i) {
    const int64_t j = base + static_cast<int64_t>(i) * STAGE_THREADS;
    if (j < n16) dst[j] = v[i];
  }
}

// The device address of p when the current device can dereference it (device or
// managed memory, or pinned host memory mapped into the device's address space),
// else nullptr.
const void* device_reachable(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  switch (a.type) {
    case cudaMemoryTypeDevice:
    case cudaMemoryTypeManaged:
      return p;
    case cudaMemoryTypeHost:
      return a.devicePointer;
    default:
      return nullptr;
  }
}

}  // namespace
}  // namespace w4a16

using namespace w4a16;

// Zero this device's w4a16_gemm_noalloc scratch on `stream` if it has been set up
// (defined with the scratch array below).
static int noalloc_scratch_zero(cudaStream_t stream, bool sync);

extern "C" {

int w4a16_version(void) { return 10000; }

const char* w4a16_strerror(int status) {
  switch (status) {
    case W4A16_OK: return "ok";
    case W4A16_ERR_INVALID: return "invalid argument (size, group size or null pointer)";
    case W4A16_ERR_ALIGNMENT: return "pointer or stride alignment not supported";
    case W4A16_ERR_LAUNCH: return "CUDA kernel launch failed";
    case W4A16_ERR_DEVICE: return "current CUDA device is not an sm_100 (B200) GPU";
    case W4A16_ERR_TIMEOUT: return "a kernel's bounded pipeline wait expired (device error flag set)";
    case W4A16_ERR_WORKSPACE: return "workspace missing, too small or not 256-byte aligned";
    case W4A16_ERR_SCRATCH_LIMIT:
      return "shape needs more scratch than w4a16_gemm_noalloc's static buffer holds "
             "(use w4a16_gemm with a workspace)";
    default: return "unknown w4a16 status";
  }
}

int w4a16_gemm_workspace_size(int64_t M, int64_t N, int64_t K, int64_t group_size,
                              int64_t* bytes_out) {
  if (bytes_out == nullptr) return W4A16_ERR_INVALID;
  *bytes_out = 0;
  if (M < 0 || N < 0 || K <= 0 || group_size <= 0) return W4A16_ERR_INVALID;
  if (K % 8 != 0 || K % group_size != 0 || group_size % 64 != 0) return W4A16_ERR_INVALID;
  if (M == 0 || N == 0 || N % 8 != 0) return W4A16_OK;   // routes without workspace
  if (M > 32) {
    // the TMEM-operand prefill kernel's K splits (none: no workspace)
    if (M > 0x7fffffffLL || N > (1ll << 30) || K > (1ll << 30)) return W4A16_ERR_INVALID;
    DeviceState* dev = nullptr;
    int st = current_device_state(&dev);
    if (st != W4A16_OK) return st;
    int mt = 0, splits = 1;
    if (choose_prefill_kernel(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), dev->num_sms, &mt,
                              &splits) == W4A16_PREFILL_TMEM_A && splits > 1)
      *bytes_out = W4A16_NOALLOC_SCRATCH_BYTES +
                   ts_split_bytes(static_cast<int>(M), static_cast<int>(N), mt, splits, dev->num_sms);
    return W4A16_OK;
  }
  if ((N + decode::BN - 1) / decode::BN > decode::MAX_STRIPS) return W4A16_OK;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  DecodePlan d;
  st = plan_decode(*dev, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), &d);
  if (st != W4A16_OK) return st;
  *bytes_out = static_cast<int64_t>(d.workspace());
  return W4A16_OK;
}

}  // extern "C"

static int gemm_impl(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                     const void* bias, void* y, int y_f32, int64_t M, int64_t N, int64_t K,
                     int64_t group_size, int64_t ldy, void* workspace, int64_t workspace_bytes,
                     void* stream, uint32_t flags = 0) {
  const int nat = (flags & W4A16_FLAG_KERNEL_ORDER) ? 1 : 0;
  const int swiglu = (flags & W4A16_FLAG_SWIGLU) ? 1 : 0;
  const int y_bf16 = (flags & W4A16_FLAG_BF16_OUT) ? 1 : 0;
  if ((flags & ~(W4A16_FLAG_KERNEL_ORDER | W4A16_FLAG_SWIGLU | W4A16_FLAG_F32_OUT | W4A16_FLAG_BF16_OUT)) != 0)
    return W4A16_ERR_INVALID;
  if ((flags & W4A16_FLAG_F32_OUT) != 0) y_f32 = 1;
  if (y_bf16 && (y_f32 || swiglu)) return W4A16_ERR_INVALID;
  if (M < 0 || N < 0 || K <= 0 || group_size <= 0) return W4A16_ERR_INVALID;
  if (K % 8 != 0 || K % group_size != 0 || group_size % 64 != 0) return W4A16_ERR_INVALID;
  if (swiglu && (y_f32 || bias != nullptr || N % (2 * decode::SWIGLU_BLOCK) != 0)) return W4A16_ERR_INVALID;
  if (y_f32 && bias != nullptr) return W4A16_ERR_INVALID;
  if (ldy < (swiglu ? N / 2 : N)) return W4A16_ERR_INVALID;
  if (M == 0 || N == 0) return W4A16_OK;
  if (x == nullptr || qweight == nullptr || scales == nullptr || zeros == nullptr || y == nullptr)
    return W4A16_ERR_INVALID;
  if (N > (1ll << 30) || K > (1ll << 30) || M > (1ll << 31) - 1) return W4A16_ERR_INVALID;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* xh = static_cast<const __half*>(x);
  const __half* sh = static_cast<const __half*>(scales);
  const __half* zh = static_cast<const __half*>(zeros);
  const __half* bh = static_cast<const __half*>(bias);
  const bool tma_ok = (N % 8 == 0) && aligned16(x) && aligned16(qweight) && aligned16(scales) &&
                      aligned16(zeros);
  const int n = static_cast<int>(N), k = static_cast<int>(K), g = static_cast<int>(group_size);
  if (!tma_ok) {
    // the plain-load fallback reads the reference layout and writes the plain output
    if (nat || swiglu) return W4A16_ERR_ALIGNMENT;
    return launch_decode_fallback(xh, qweight, sh, zh, bh, y, y_f32, M, n, k, g, ldy, s, y_bf16);
  }
  if (M <= 32 && (N + decode::BN - 1) / decode::BN <= decode::MAX_STRIPS) {
    return launch_decode_tma(*dev, xh, qweight, sh, zh, bh, y, y_f32, static_cast<int>(M), n, k, g,
                             ldy, workspace, workspace_bytes, s, ArArgs(), swiglu, nat, y_bf16);
  }
  int ts_mt = 0, ts_splits = 1;
  if (choose_prefill_kernel(static_cast<int>(M), n, k, dev->num_sms, &ts_mt, &ts_splits) == W4A16_PREFILL_TMEM_A)
    return launch_prefill_ts(*dev, xh, qweight, sh, zh, bh, y, y_f32, static_cast<int>(M), n, k, g, ldy, s, swiglu,
                             nat, y_bf16, ts_mt, ts_splits, workspace, workspace_bytes);
  return launch_prefill(*dev, xh, qweight, sh, zh, bh, y, y_f32, static_cast<int>(M), n, k, g, ldy, s,
                        swiglu, nat, y_bf16);
}

extern "C" {

int w4a16_gemm(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
               const void* bias, void* y, int64_t M, int64_t N, int64_t K, int64_t group_size,
               int64_t ldy, void* workspace, int64_t workspace_bytes, void* stream) {
  return gemm_impl(x, qweight, scales, zeros, bias, y, 0, M, N, K, group_size, ldy, workspace,
                   workspace_bytes, stream);
}

int w4a16_gemm_f32(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                   float* y, int64_t M, int64_t N, int64_t K, int64_t group_size, int64_t ldy,
                   void* workspace, int64_t workspace_bytes, void* stream) {
  return gemm_impl(x, qweight, scales, zeros, nullptr, y, 1, M, N, K, group_size, ldy, workspace,
                   workspace_bytes, stream);
}

int w4a16_swiglu(const void* gate_up, void* h, int64_t M, int64_t N, int64_t ld_in,
                 int64_t ld_out, void* stream) {
  if (M < 0 || N < 0 || ld_in < 2 * N || ld_out < N) return W4A16_ERR_INVALID;
  if (M == 0 || N == 0) return W4A16_OK;
  if (gate_up == nullptr || h == nullptr) return W4A16_ERR_INVALID;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  const int64_t total = M * N;
  const int64_t blocks = (total + 255) / 256;
  if (blocks > 0x7fffffffLL) return W4A16_ERR_INVALID;
  swiglu_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(gate_up), static_cast<__half*>(h), M, N, ld_in, ld_out);
  W4A16_RETURN_IF_LAUNCH_FAILED();
  return W4A16_OK;
}

int w4a16_gemm_swiglu(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                      void* h, int64_t M, int64_t N, int64_t K, int64_t group_size, int64_t ldh,
                      void* workspace, int64_t workspace_bytes, void* stream) {
  return gemm_impl(x, qweight, scales, zeros, nullptr, h, 0, M, N, K, group_size, ldh, workspace,
                   workspace_bytes, stream, W4A16_FLAG_SWIGLU);
}

int w4a16_gemm_ex(const void* x, const int32_t* qweight, const void* scales, const void* zeros,
                  const void* bias, void* y, int64_t M, int64_t N, int64_t K, int64_t group_size,
                  int64_t ldy, uint32_t flags, void* workspace, int64_t workspace_bytes, void* stream) {
  return gemm_impl(x, qweight, scales, zeros, bias, y, 0, M, N, K, group_size, ldy, workspace,
                   workspace_bytes, stream, flags);
}

int w4a16_convert(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n, void* stream) {
  if (n < 0) return W4A16_ERR_INVALID;
  if (n == 0) return W4A16_OK;
  if (src == nullptr || dst == nullptr) return W4A16_ERR_INVALID;
  if (src_dtype < W4A16_DTYPE_F16 || src_dtype > W4A16_DTYPE_BF16) return W4A16_ERR_INVALID;
  if (dst_dtype != W4A16_DTYPE_F16 && dst_dtype != W4A16_DTYPE_BF16) return W4A16_ERR_INVALID;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  const int64_t blocks = (n + 255) / 256;
  if (blocks > 0x7fffffffLL) return W4A16_ERR_INVALID;
  convert_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      src, src_dtype, dst, dst_dtype, n);
  W4A16_RETURN_IF_LAUNCH_FAILED();
  return W4A16_OK;
}

int w4a16_repack(const int32_t* qweight, int32_t* out, int64_t K, int64_t N, int to_kernel_order,
                 void* stream) {
  if (K < 0 || N < 0 || K % 8 != 0) return W4A16_ERR_INVALID;
  if (K == 0 || N == 0) return W4A16_OK;
  if (qweight == nullptr || out == nullptr) return W4A16_ERR_INVALID;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  const int64_t words = K / 8 * N;
  const int64_t blocks = (words + 255) / 256;
  if (blocks > 0x7fffffffLL) return W4A16_ERR_INVALID;
  repack_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      qweight, out, words, to_kernel_order ? 1 : 0);
  W4A16_RETURN_IF_LAUNCH_FAILED();
  return W4A16_OK;
}

}  // extern "C"

// The staging kernel between two device-visible addresses (checked by the caller).
static int launch_stage(const void* s, void* d, int64_t bytes, int src_ready, void* stream) {
  const int64_t n16 = bytes / 16;
  const int64_t per_cta = static_cast<int64_t>(STAGE_THREADS) * STAGE_PER_THREAD;
  const int64_t blocks = (n16 + per_cta - 1) / per_cta;
  if (blocks > 0x7fffffffLL) return W4A16_ERR_INVALID;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
  cfg.blockDim = dim3(STAGE_THREADS, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, stage_kernel, static_cast<const uint4*>(s), static_cast<uint4*>(d), n16,
                         src_ready ? 1 : 0) != cudaSuccess) {
    cudaGetLastError();
    return W4A16_ERR_LAUNCH;
  }
  return W4A16_OK;
}

extern "C" {

int w4a16_stage(const void* src, void* dst, int64_t bytes, int src_ready, void* stream) {
  if (bytes < 0 || (bytes & 15) != 0) return W4A16_ERR_INVALID;
  if (bytes == 0) return W4A16_OK;
  if (src == nullptr || dst == nullptr) return W4A16_ERR_INVALID;
  if (!aligned16(src) || !aligned16(dst)) return W4A16_ERR_ALIGNMENT;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  const void* s = device_reachable(src);
  void* d = const_cast<void*>(device_reachable(dst));
  if (s == nullptr || d == nullptr) return W4A16_ERR_INVALID;
  return launch_stage(s, d, bytes, src_ready, stream);
}

static int quantize_impl(const void* w, int w_dtype, int32_t* qweight, void* scales, void* zeros,
                         int64_t K, int64_t N, int64_t group_size, int symmetric, void* stream) {
  if (K < 0 || N < 0 || group_size <= 0) return W4A16_ERR_INVALID;
  if (K % 8 != 0 || K % group_size != 0) return W4A16_ERR_INVALID;
  if (K == 0 || N == 0) return W4A16_OK;
  if (w == nullptr || qweight == nullptr || scales == nullptr || zeros == nullptr)
    return W4A16_ERR_INVALID;
  if (K / group_size > 65535 || K / 8 > 65535) return W4A16_ERR_INVALID;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid = grid_2d((N + 255) / 256, K / group_size);
  __half* sh = static_cast<__half*>(scales);
  __half* zh = static_cast<__half*>(zeros);
  switch (w_dtype) {
    case W4A16_DTYPE_F16:
      quantize_pack_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(w), qweight, sh,
                                                         zh, N, group_size, symmetric);
      break;
    case W4A16_DTYPE_F32:
      quantize_pack_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(w), qweight, sh,
                                                        zh, N, group_size, symmetric);
      break;
    case W4A16_DTYPE_BF16:
      quantize_pack_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(w), qweight, sh, zh, N, group_size, symmetric);
      break;
    default:
      return W4A16_ERR_INVALID;
  }
  W4A16_RETURN_IF_LAUNCH_FAILED();
  if (group_size % 8 != 0) {
    const dim3 pg = grid_2d((N + 255) / 256, K / 8);
    switch (w_dtype) {
      case W4A16_DTYPE_F16:
        pack_ragged_groups_kernel<__half><<<pg, 256, 0, s>>>(static_cast<const __half*>(w), qweight,
                                                              N, K, group_size, symmetric);
        break;
      case W4A16_DTYPE_F32:
        pack_ragged_groups_kernel<float><<<pg, 256, 0, s>>>(static_cast<const float*>(w), qweight,
                                                             N, K, group_size, symmetric);
        break;
      default:
        pack_ragged_groups_kernel<__nv_bfloat16><<<pg, 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(w), qweight, N, K, group_size, symmetric);
        break;
    }
    W4A16_RETURN_IF_LAUNCH_FAILED();
  }
  return W4A16_OK;
}

int w4a16_quantize(const void* w, int w_dtype, int32_t* qweight, void* scales, void* zeros,
                   int64_t K, int64_t N, int64_t group_size, void* stream) {
  return quantize_impl(w, w_dtype, qweight, scales, zeros, K, N, group_size, 0, stream);
}

int w4a16_quantize_ex(const void* w, int w_dtype, int32_t* qweight, void* scales, void* zeros,
                      int64_t K, int64_t N, int64_t group_size, uint32_t flags, void* stream) {
  if ((flags & ~W4A16_QUANT_SYMMETRIC) != 0) return W4A16_ERR_INVALID;
  return quantize_impl(w, w_dtype, qweight, scales, zeros, K, N, group_size,
                       (flags & W4A16_QUANT_SYMMETRIC) ? 1 : 0, stream);
}

int w4a16_pack_int4(const int32_t* q, int32_t* qweight, int64_t K, int64_t N, void* stream) {
  if (K < 0 || N < 0 || K % 8 != 0) return W4A16_ERR_INVALID;
  if (K == 0 || N == 0) return W4A16_OK;
  if (q == nullptr || qweight == nullptr || K / 8 > 65535) return W4A16_ERR_INVALID;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  pack_int4_kernel<<<grid_2d((N + 255) / 256, K / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      q, qweight, N);
  W4A16_RETURN_IF_LAUNCH_FAILED();
  return W4A16_OK;
}

int w4a16_unpack_int4(const int32_t* qweight, int32_t* q, int64_t K, int64_t N, void* stream) {
  if (K < 0 || N < 0 || K % 8 != 0) return W4A16_ERR_INVALID;
  if (K == 0 || N == 0) return W4A16_OK;
  if (q == nullptr || qweight == nullptr || K / 8 > 65535) return W4A16_ERR_INVALID;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  unpack_int4_kernel<<<grid_2d((N + 255) / 256, K / 8), 256, 0,
                       static_cast<cudaStream_t>(stream)>>>(qweight, q, N);
  W4A16_RETURN_IF_LAUNCH_FAILED();
  return W4A16_OK;
}

int w4a16_dequantize(const int32_t* qweight, const void* scales, const void* zeros, void* w,
                     int64_t K, int64_t N, int64_t group_size, void* stream) {
  if (K < 0 || N < 0 || group_size <= 0 || K % 8 != 0 || K % group_size != 0)
    return W4A16_ERR_INVALID;
  if (K == 0 || N == 0) return W4A16_OK;
  if (qweight == nullptr || scales == nullptr || zeros == nullptr || w == nullptr ||
      K / 8 > 65535)
    return W4A16_ERR_INVALID;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  dequantize_kernel<<<grid_2d((N + 255) / 256, K / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      qweight, static_cast<const __half*>(scales), static_cast<const __half*>(zeros),
      static_cast<__half*>(w), N, group_size);
  W4A16_RETURN_IF_LAUNCH_FAILED();
  return W4A16_OK;
}

int w4a16_check_device_errors(void* stream, uint32_t* flags_out) {
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t flags = 0;
  const uint32_t zero = 0;
  if (cudaMemcpyFromSymbolAsync(&flags, g_device_error, sizeof(flags), 0,
                                cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice,
                              s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    cudaGetLastError();
    return W4A16_ERR_LAUNCH;
  }
  if (flags_out != nullptr) *flags_out = flags;
  if (flags != 0) {
    // A launch abandoned on a timeout may have left tagged piece words in the
    // allocation-free entry point's static scratch, whose callers cannot clear
    // it themselves: zero it here (a no-op if it was never set up).
    const int zst = noalloc_scratch_zero(s, true);
    if (zst != W4A16_OK) return zst;
  }
  return flags == 0 ? W4A16_OK : W4A16_ERR_TIMEOUT;
}

int w4a16_set_wait_budget_ns(int64_t ns) {
  if (ns < 0 || (ns > 0 && ns < 1000 * 1000) || ns > 600ll * 1000 * 1000 * 1000) return W4A16_ERR_INVALID;
  g_wait_budget_ns.store(ns == 0 ? kWaitBudgetNs : static_cast<unsigned long long>(ns),
                         std::memory_order_relaxed);
  return W4A16_OK;
}

int w4a16_gemm_host(const void* x_host, const int32_t* qweight, const void* scales, const void* zeros,
                    const void* bias, void* y_host, int64_t M, int64_t N, int64_t K, int64_t group_size,
                    uint32_t flags, void* x_dev, void* y_dev, void* workspace, int64_t workspace_bytes,
                    void* stream) {
  if (M < 0 || N < 0 || K <= 0) return W4A16_ERR_INVALID;
  if (M == 0 || N == 0) return W4A16_OK;
  if (x_host == nullptr || y_host == nullptr || x_dev == nullptr || y_dev == nullptr) return W4A16_ERR_INVALID;
  const int64_t ncols = (flags & W4A16_FLAG_SWIGLU) ? N / 2 : N;
  const int64_t esize = (flags & W4A16_FLAG_F32_OUT) ? 4 : 2;
  const int64_t xbytes = M * K * 2, ybytes = M * ncols * esize;
  if ((xbytes & 15) != 0 || (ybytes & 15) != 0) return W4A16_ERR_ALIGNMENT;
  if (!aligned16(x_host) || !aligned16(y_host) || !aligned16(x_dev) || !aligned16(y_dev))
    return W4A16_ERR_ALIGNMENT;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  const void* xs = device_reachable(x_host);
  void* yd = const_cast<void*>(device_reachable(y_host));
  if (xs == nullptr || yd == nullptr) return W4A16_ERR_INVALID;
  // x in (read at once: the host filled it before the call), the GEMM, y out (after
  // the GEMM): kernels chained under programmatic dependent launch. Up to 32 tokens the
  // GEMM (decode or plain-load kernel, plain stores) writes y straight into the mapped
  // host buffer and no stage-out kernel is needed; the prefill kernels store y with TMA,
  // which needs device memory.
  st = launch_stage(xs, x_dev, xbytes, 1, stream);
  if (st != W4A16_OK) return st;
  const bool direct = M <= 32;
  st = gemm_impl(x_dev, qweight, scales, zeros, bias, direct ? yd : y_dev, 0, M, N, K, group_size, ncols,
                 workspace, workspace_bytes, stream, flags);
  if (st != W4A16_OK || direct) return st;
  return launch_stage(y_dev, yd, ybytes, 0, stream);
}

int w4a16_prefill_choice(int64_t M, int64_t N, int64_t K, int* which) {
  if (which == nullptr || M <= 0 || N <= 0 || K <= 0 || M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff)
    return W4A16_ERR_INVALID;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  int mt = 0;
  *which = M <= 32 ? W4A16_PREFILL_AUTO
                   : choose_prefill_kernel(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                                           dev->num_sms, &mt);
  return W4A16_OK;
}

int w4a16_prefill_plan(int64_t M, int64_t N, int64_t K, int num_sms, int* which, int* tokens_per_tile,
                       int* splits) {
  if (which == nullptr || tokens_per_tile == nullptr || splits == nullptr || num_sms <= 0 || num_sms > 4096 ||
      M <= 0 || N <= 0 || K <= 0 || K % prefill::BK != 0 || M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff)
    return W4A16_ERR_INVALID;
  if (M <= 32) {
    *which = W4A16_PREFILL_AUTO;
    *tokens_per_tile = 0;
    *splits = 1;
    return W4A16_OK;
  }
  int mt = 0, sp = 1;
  *which = choose_prefill_kernel(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), num_sms, &mt, &sp);
  *tokens_per_tile = *which == W4A16_PREFILL_TMEM_A ? mt : 0;
  *splits = *which == W4A16_PREFILL_TMEM_A ? sp : 1;
  return W4A16_OK;
}

int w4a16_set_prefill_kernel(int which) {
  if (which != W4A16_PREFILL_AUTO && which != W4A16_PREFILL_SMEM_B && which != W4A16_PREFILL_TMEM_A)
    return W4A16_ERR_INVALID;
  g_prefill_kernel.store(which, std::memory_order_relaxed);
  return W4A16_OK;
}

int w4a16_reset_scratch(void* workspace, int64_t workspace_bytes, void* stream) {
  if (workspace_bytes < 0 || (workspace == nullptr && workspace_bytes != 0)) return W4A16_ERR_INVALID;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (workspace != nullptr && workspace_bytes > 0 &&
      cudaMemsetAsync(workspace, 0, static_cast<size_t>(workspace_bytes), s) != cudaSuccess) {
    cudaGetLastError();
    return W4A16_ERR_LAUNCH;
  }
  return noalloc_scratch_zero(s, false);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free GEMM (w4a16_gemm_noalloc)
// ---------------------------------------------------------------------------
// For callers that cannot allocate device memory when they launch (a C/FFI
// host without a device allocator, an engine whose planner owns all device
// memory, a plugin call that passes no scratch): the decode kernel's scratch
// is this static array instead of a caller workspace, used exactly as one: the
// tagged piece words of shared strips, which must be zero when a launch starts
// (every launch leaves them zero). One array per device, so launches that
// overlap in time race on it; callers keep them ordered.
static __device__ __align__(256) unsigned char g_noalloc_scratch[W4A16_NOALLOC_SCRATCH_BYTES];

namespace {
struct NoallocScratch {
  bool ready = false;
  void* ptr = nullptr;
};
NoallocScratch g_noalloc[w4a16::kMaxDevices];
std::mutex g_noalloc_mu;

// Once per device, with that device current: the array's device address
// (host code never passes the symbol itself to a kernel) and the whole array
// zeroed on `stream`, which is then synchronised. Refused while
// `stream` is capturing, since neither step belongs in a graph.
int noalloc_scratch(cudaStream_t stream, void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= w4a16::kMaxDevices) {
    cudaGetLastError();
    return W4A16_ERR_DEVICE;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoallocScratch& sc = g_noalloc[dev];
  if (!sc.ready) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
      cudaGetLastError();
      return W4A16_ERR_LAUNCH;
    }
    if (cap != cudaStreamCaptureStatusNone) return W4A16_ERR_INVALID;
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr ||
        (reinterpret_cast<uintptr_t>(ptr) & 255u) != 0) {
      cudaGetLastError();
      return W4A16_ERR_LAUNCH;
    }
    if (cudaMemsetAsync(ptr, 0, W4A16_NOALLOC_SCRATCH_BYTES, stream) != cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess) {
      cudaGetLastError();
      return W4A16_ERR_LAUNCH;
    }
    sc.ptr = ptr;
    sc.ready = true;
  }
  *out = sc.ptr;
  return W4A16_OK;
}
}  // namespace

static int noalloc_scratch_zero(cudaStream_t stream, bool sync) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= w4a16::kMaxDevices) {
    cudaGetLastError();
    return W4A16_ERR_DEVICE;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoallocScratch& sc = g_noalloc[dev];
  if (!sc.ready) return W4A16_OK;   // set-up zeroes it before its first use
  if (cudaMemsetAsync(sc.ptr, 0, W4A16_NOALLOC_SCRATCH_BYTES, stream) != cudaSuccess ||
      (sync && cudaStreamSynchronize(stream) != cudaSuccess)) {
    cudaGetLastError();
    return W4A16_ERR_LAUNCH;
  }
  return W4A16_OK;
}

extern "C" int w4a16_gemm_noalloc(const void* x, const int32_t* qweight, const void* scales,
                                  const void* zeros, const void* bias, void* y, int64_t M,
                                  int64_t N, int64_t K, int64_t group_size, int64_t ldy,
                                  void* stream) {
  // The argument rules of w4a16_gemm, checked before any device work.
  if (M < 0 || N < 0 || K <= 0 || group_size <= 0) return W4A16_ERR_INVALID;
  if (K % 8 != 0 || K % group_size != 0 || group_size % 64 != 0) return W4A16_ERR_INVALID;
  if (ldy < N) return W4A16_ERR_INVALID;
  if (M == 0 || N == 0) return W4A16_OK;
  if (x == nullptr || qweight == nullptr || scales == nullptr || zeros == nullptr || y == nullptr)
    return W4A16_ERR_INVALID;
  int64_t need = 0;
  int st = w4a16_gemm_workspace_size(M, N, K, group_size, &need);
  if (st != W4A16_OK) return st;
  // (prefill shapes run without K splits here: their split area lies past the array)
  if (M <= 32 && need > W4A16_NOALLOC_SCRATCH_BYTES) return W4A16_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  st = noalloc_scratch(static_cast<cudaStream_t>(stream), &scratch);
  if (st != W4A16_OK) return st;
  return gemm_impl(x, qweight, scales, zeros, bias, y, 0, M, N, K, group_size, ldy, scratch,
                   W4A16_NOALLOC_SCRATCH_BYTES, stream);
}

// ---------------------------------------------------------------------------
// Row-parallel decode GEMM fused with its all-reduce over NVLink peer memory
// ---------------------------------------------------------------------------
extern "C" int w4a16_gemm_allreduce(const void* x, const int32_t* qweight, const void* scales,
                                    const void* zeros, const void* bias, void* y, int64_t M, int64_t N,
                                    int64_t K, int64_t group_size, int64_t ldy, void* workspace,
                                    int64_t workspace_bytes, const unsigned long long* peers,
                                    int world, int rank, int* ctl, int64_t slot, void* stream) {
  if (M < 0 || N < 0 || K <= 0 || group_size <= 0) return W4A16_ERR_INVALID;
  if (K % 8 != 0 || K % group_size != 0 || group_size % 64 != 0) return W4A16_ERR_INVALID;
  if (ldy < N || M > 32 || N % 8 != 0) return W4A16_ERR_INVALID;
  if (world < 2 || world > decode::AR_MAX_RANKS || rank < 0 || rank >= world) return W4A16_ERR_INVALID;
  if (M * N > 0x7fffffffLL) return W4A16_ERR_INVALID;   // the finishing CTAs index y in 32 bits
  if (peers == nullptr || ctl == nullptr || slot < M * N) return W4A16_ERR_INVALID;
  for (int q = 0; q < world; ++q)
    if (peers[q] == 0ull || (peers[q] & 15ull) != 0ull) return W4A16_ERR_ALIGNMENT;
  if (M == 0 || N == 0) return W4A16_OK;
  if (x == nullptr || qweight == nullptr || scales == nullptr || zeros == nullptr || y == nullptr)
    return W4A16_ERR_INVALID;
  if (N > (1ll << 30) || K > (1ll << 30) || (N + decode::BN - 1) / decode::BN > decode::MAX_STRIPS)
    return W4A16_ERR_INVALID;
  if (!aligned16(x) || !aligned16(qweight) || !aligned16(scales) || !aligned16(zeros))
    return W4A16_ERR_ALIGNMENT;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  ArArgs ar;
  ar.world = world;
  ar.rank = rank;
  ar.peers = peers;
  ar.ctl = ctl;
  ar.slot = slot;
  return launch_decode_tma(*dev, static_cast<const __half*>(x), qweight, static_cast<const __half*>(scales),
                           static_cast<const __half*>(zeros), static_cast<const __half*>(bias), y, 0,
                           static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                           static_cast<int>(group_size), ldy, workspace, workspace_bytes,
                           static_cast<cudaStream_t>(stream), ar);
}

extern "C" int w4a16_gemm_allgather(const void* x, const int32_t* qweight, const void* scales,
                                    const void* zeros, const void* bias, void* y, int64_t M, int64_t N,
                                    int64_t K, int64_t group_size, int64_t ldy, void* workspace,
                                    int64_t workspace_bytes, const unsigned long long* peers,
                                    int world, int rank, int* ctl, int64_t slot, void* stream) {
  if (M < 0 || N < 0 || K <= 0 || group_size <= 0) return W4A16_ERR_INVALID;
  if (K % 8 != 0 || K % group_size != 0 || group_size % 64 != 0) return W4A16_ERR_INVALID;
  if (M > 32 || N % 8 != 0) return W4A16_ERR_INVALID;
  if (world < 2 || world > decode::AR_MAX_RANKS || rank < 0 || rank >= world) return W4A16_ERR_INVALID;
  if (ldy < static_cast<int64_t>(world) * N) return W4A16_ERR_INVALID;
  if (M * world * N > 0x7fffffffLL) return W4A16_ERR_INVALID;   // 32-bit indices into y
  if (peers == nullptr || ctl == nullptr || slot < M * N) return W4A16_ERR_INVALID;
  for (int q = 0; q < world; ++q)
    if (peers[q] == 0ull || (peers[q] & 15ull) != 0ull) return W4A16_ERR_ALIGNMENT;
  if (M == 0 || N == 0) return W4A16_OK;
  if (x == nullptr || qweight == nullptr || scales == nullptr || zeros == nullptr || y == nullptr)
    return W4A16_ERR_INVALID;
  if (N > (1ll << 30) || K > (1ll << 30) || (N + decode::BN - 1) / decode::BN > decode::MAX_STRIPS)
    return W4A16_ERR_INVALID;
  if (!aligned16(x) || !aligned16(qweight) || !aligned16(scales) || !aligned16(zeros))
    return W4A16_ERR_ALIGNMENT;
  DeviceState* dev = nullptr;
  int st = current_device_state(&dev);
  if (st != W4A16_OK) return st;
  ArArgs ar;
  ar.world = world;
  ar.rank = rank;
  ar.gather = 1;
  ar.peers = peers;
  ar.ctl = ctl;
  ar.slot = slot;
  return launch_decode_tma(*dev, static_cast<const __half*>(x), qweight, static_cast<const __half*>(scales),
                           static_cast<const __half*>(zeros), static_cast<const __half*>(bias), y, 0,
                           static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                           static_cast<int>(group_size), ldy, workspace, workspace_bytes,
                           static_cast<cudaStream_t>(stream), ar);
}

extern "C" int w4a16_p2p_buffer_bytes(int world, int64_t slot, int64_t* bytes_out) {
  if (bytes_out == nullptr || world < 2 || world > decode::AR_MAX_RANKS || slot <= 0)
    return W4A16_ERR_INVALID;
  *bytes_out = decode::ar_buffer_bytes(world, slot);
  return W4A16_OK;
}

extern "C" int w4a16_p2p_alloc(int64_t bytes, void** ptr_out, void* handle_out) {
  if (bytes <= 0 || ptr_out == nullptr || handle_out == nullptr) return W4A16_ERR_INVALID;
  void* p = nullptr;
  if (cudaMalloc(&p, static_cast<size_t>(bytes)) != cudaSuccess) {
    cudaGetLastError();
    return W4A16_ERR_DEVICE;
  }
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, static_cast<size_t>(bytes)) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(p);
    return W4A16_ERR_DEVICE;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  *ptr_out = p;
  return W4A16_OK;
}

extern "C" int w4a16_p2p_open(const void* handle, void** ptr_out) {
  if (handle == nullptr || ptr_out == nullptr) return W4A16_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return W4A16_ERR_DEVICE;
  }
  *ptr_out = p;
  return W4A16_OK;
}

extern "C" int w4a16_p2p_close(void* ptr) {
  if (ptr == nullptr) return W4A16_ERR_INVALID;
  if (cudaIpcCloseMemHandle(ptr) != cudaSuccess) {
    cudaGetLastError();
    return W4A16_ERR_DEVICE;
  }
  return W4A16_OK;
}

extern "C" int w4a16_p2p_free(void* ptr) {
  if (ptr == nullptr) return W4A16_ERR_INVALID;
  if (cudaFree(ptr) != cudaSuccess) {
    cudaGetLastError();
    return W4A16_ERR_DEVICE;
  }
  return W4A16_OK;
}
