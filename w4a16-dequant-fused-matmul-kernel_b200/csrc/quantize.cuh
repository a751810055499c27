// quantize.cuh -- quantise/pack, pack, unpack and dequantise kernels.
//
// These are the load-path halves of the format (w4a16-kernel/src/w4a16/quant.py).
// They are HBM-bound elementwise/reduction work: one thread per (group, column)
// or per packed word, consecutive threads on consecutive columns so every
// global access is a coalesced row segment.
#pragma once

#include "common.cuh"

namespace w4a16 {

template <typename T>
__device__ __forceinline__ float load_as_f32(const T* p);
template <>
__device__ __forceinline__ float load_as_f32<__half>(const __half* p) {
  return __half2float(*p);
}
template <>
__device__ __forceinline__ float load_as_f32<float>(const float* p) {
  return *p;
}
template <>
__device__ __forceinline__ float load_as_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

// clamp(x, 0, 15) with the reference's (torch CPU) semantics: comparisons,
// so NaN and -0.0 pass through unchanged (quant.py:134, :139).
__device__ __forceinline__ float clamp_0_15(float x) {
  x = (x < 0.0f) ? 0.0f : x;
  return (x > 15.0f) ? 15.0f : x;
}

// A group's fp32 scale and zero-point from its min and max.
// Asymmetric (the reference, quant.py:125-136): scale = (max - min) / 15 (1 when not
// > 0), zero = clamp(rint(-min / scale), 0, 15).
// Symmetric (the code layout GPTQ-style checkpoints use for sym=True; no counterpart
// in the reference): scale = 2 * max(|min|, |max|) / 15 (1 when not > 0), zero = 8.
// Codes are clamp(rint(w / scale) + zero, 0, 15) either way, in the same format.
__device__ __forceinline__ void group_scale_zero(float mx, float mn, bool symmetric, float& scale,
                                                 float& zero) {
  if (symmetric) {
    const float amax = fmaxf(fabsf(mx), fabsf(mn));
    scale = __fdiv_rn(__fmul_rn(2.0f, amax), 15.0f);
    scale = (scale > 0.0f) ? scale : 1.0f;
    zero = 8.0f;
  } else {
    scale = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
    scale = (scale > 0.0f) ? scale : 1.0f;
    zero = clamp_0_15(rintf(__fdiv_rn(-mn, scale)));
  }
}

// One thread per (group g, column n): fp32 min/max over the G rows of the
// group, then scale / zero, then the group's codes packed 8 rows per word.
// Bit-exact with quant.py:101-144 (IEEE division, round-half-even rintf).
template <typename T>
__global__ void __launch_bounds__(256) quantize_pack_kernel(const T* __restrict__ w,
                                                            int32_t* __restrict__ qweight,
                                                            __half* __restrict__ scales,
                                                            __half* __restrict__ zeros,
                                                            int64_t N, int64_t G, int symmetric) {
  const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t g = blockIdx.y;
  if (n >= N) return;
  const T* col = w + g * G * N + n;

  float mx = load_as_f32(col);
  float mn = mx;
  for (int64_t r = 1; r < G; ++r) {
    const float v = load_as_f32(col + r * N);
    mx = (v > mx) ? v : mx;
    mn = (v < mn) ? v : mn;
  }
  float scale, zero;
  group_scale_zero(mx, mn, symmetric != 0, scale, zero);

  scales[g * N + n] = __float2half_rn(scale);
  zeros[g * N + n] = __float2half_rn(zero);

  // G % 8 == 0 is not required by the format, only K % 8 == 0 and K % G == 0;
  // when G is not a multiple of 8 a packed word straddles groups, so the
  // packing pass below walks words and looks up each row's group.
  if (G % 8 == 0) {
    int32_t* out = qweight + (g * G / 8) * N + n;
    for (int64_t i = 0; i < G / 8; ++i) {
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v = load_as_f32(col + (i * 8 + j) * N);
        const float q = clamp_0_15(__fadd_rn(rintf(__fdiv_rn(v, scale)), zero));
        word |= (static_cast<uint32_t>(static_cast<int>(q)) & 0xFu) << (4 * j);
      }
      out[i * N] = static_cast<int32_t>(word);
    }
  }
}

// Packing pass for group sizes that are not a multiple of 8: one thread per
// packed word, reading each row's scale/zero back (already rounded to fp16 is
// NOT what the reference uses, so the fp32 values are recomputed per group).
template <typename T>
__global__ void __launch_bounds__(256) pack_ragged_groups_kernel(const T* __restrict__ w,
                                                                 int32_t* __restrict__ qweight,
                                                                 int64_t N, int64_t K,
                                                                 int64_t G, int symmetric) {
  const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t i = blockIdx.y;  // packed row
  if (n >= N) return;
  uint32_t word = 0;
  int64_t cur_g = -1;
  float scale = 1.0f, zero = 0.0f;
  for (int j = 0; j < 8; ++j) {
    const int64_t k = i * 8 + j;
    const int64_t g = k / G;
    if (g != cur_g) {
      cur_g = g;
      const T* col = w + g * G * N + n;
      float mx = load_as_f32(col), mn = mx;
      for (int64_t r = 1; r < G; ++r) {
        const float v = load_as_f32(col + r * N);
        mx = (v > mx) ? v : mx;
        mn = (v < mn) ? v : mn;
      }
      group_scale_zero(mx, mn, symmetric != 0, scale, zero);
    }
    const float v = load_as_f32(w + k * N + n);
    const float q = clamp_0_15(__fadd_rn(rintf(__fdiv_rn(v, scale)), zero));
    word |= (static_cast<uint32_t>(static_cast<int>(q)) & 0xFu) << (4 * j);
  }
  qweight[i * N + n] = static_cast<int32_t>(word);
}

__global__ void __launch_bounds__(256) pack_int4_kernel(const int32_t* __restrict__ q,
                                                        int32_t* __restrict__ packed,
                                                        int64_t N) {
  const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t i = blockIdx.y;
  if (n >= N) return;
  uint32_t word = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    word |= (static_cast<uint32_t>(q[(i * 8 + j) * N + n]) & 0xFu) << (4 * j);
  }
  packed[i * N + n] = static_cast<int32_t>(word);
}

__global__ void __launch_bounds__(256) unpack_int4_kernel(const int32_t* __restrict__ packed,
                                                          int32_t* __restrict__ q, int64_t N) {
  const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t i = blockIdx.y;
  if (n >= N) return;
  const uint32_t word = static_cast<uint32_t>(packed[i * N + n]);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    q[(i * 8 + j) * N + n] = static_cast<int32_t>((word >> (4 * j)) & 0xFu);
  }
}

// Nibble order of a packed word: the reference keeps row 8i+j in nibble j; the kernel
// order keeps rows (k0, k2, k4, k6, k1, k3, k5, k7) in nibbles 0..7, so that a mask
// with 0x000F000F (and the same after a shift by 4 or 8 or 12) extracts consecutive
// row pairs. Elementwise over the [K/8, N] words; `to_kernel` selects the direction.
// In-place use (in == out) is allowed.
__device__ __forceinline__ uint32_t repack_word(uint32_t w, bool to_kernel) {
  // reference nibble j sits at kernel nibble pos[j] = {0, 4, 1, 5, 2, 6, 3, 7}[j]
  uint32_t r = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int pos = (j >> 1) | ((j & 1) << 2);
    if (to_kernel)
      r |= ((w >> (4 * j)) & 0xFu) << (4 * pos);
    else
      r |= ((w >> (4 * pos)) & 0xFu) << (4 * j);
  }
  return r;
}

__global__ void __launch_bounds__(256) repack_kernel(const int32_t* in, int32_t* out, int64_t n_words,
                                                     int to_kernel) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n_words) return;
  out[i] = static_cast<int32_t>(repack_word(static_cast<uint32_t>(in[i]), to_kernel != 0));
}

// w = fp16(fp16(q - z) * s): two correctly rounded fp16 operations, the same
// as the reference's fp16 tensor arithmetic (quant.py:177).
__global__ void __launch_bounds__(256) dequantize_kernel(const int32_t* __restrict__ packed,
                                                         const __half* __restrict__ scales,
                                                         const __half* __restrict__ zeros,
                                                         __half* __restrict__ w, int64_t N,
                                                         int64_t G) {
  const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t i = blockIdx.y;
  if (n >= N) return;
  const uint32_t word = static_cast<uint32_t>(packed[i * N + n]);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int64_t k = i * 8 + j;
    const int64_t g = k / G;
    const __half s = scales[g * N + n];
    const __half z = zeros[g * N + n];
    const __half qh = __int2half_rn(static_cast<int>((word >> (4 * j)) & 0xFu));
    w[k * N + n] = __hmul(__hsub(qh, z), s);
  }
}

}  // namespace w4a16
