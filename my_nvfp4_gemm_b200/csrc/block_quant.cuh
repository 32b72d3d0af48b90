// block_quant.cuh — the NVFP4 block-quantization arithmetic shared by quantize_kernel and the
// GEMM's quantized-output epilogue, so both produce the same bytes for the same bf16 values.
//
// Per 16 consecutive bf16 values x_i and the per-tensor scale s (the reference's arithmetic,
// csrc/quantize/quantize_nvfp4.cu:15-34):
//   amax  = NaN-propagating max of |x_i|, seeded with bf16 0x0001
//   sf    = e4m3_rn_satfinite((f32(amax) * s) * (1/6))
//   os    = rcp_rn(f32(sf) * rcp_rn(s))
//   q_i   = e2m1_rn_satfinite(f32(x_i) * os)
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

#include "ptx.cuh"

namespace nvfp4 {
namespace bq {

constexpr float kRcpE2m1Max = 1.0f / 6.0f;  // 0.16666667f, as the reference

__device__ __forceinline__ float bf16lo_to_f32(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi_to_f32(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Running NaN-propagating max of |x| over bf16 pairs.
__device__ __forceinline__ uint32_t abs_max_bf16x2(uint32_t acc, uint32_t w) {
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&acc);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&w);
  __nv_bfloat162 r = __hmax2_nan(a, __habs2(b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t max_bf16x2(uint32_t acc, uint32_t w) {
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&acc);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&w);
  __nv_bfloat162 r = __hmax2_nan(a, b);
  return *reinterpret_cast<uint32_t*>(&r);
}

constexpr uint32_t kAmaxSeed = 0x00010001u;  // bf16x2 {0x0001, 0x0001}: the non-zero floor

// amax of a block from the pairwise running max m (both halves of the pair folded).
__device__ __forceinline__ float block_amax(uint32_t m) {
  const __nv_bfloat162 m2 = *reinterpret_cast<__nv_bfloat162*>(&m);
  return __bfloat162float(__hmax_nan(m2.x, m2.y));
}

// Scale byte of a block and the multiplier its values are encoded with.
__device__ __forceinline__ uint8_t block_scale(float amax, float s, float rcp_s, float& os) {
  const float t = __fmul_rn(__fmul_rn(amax, s), kRcpE2m1Max);
  const uint8_t sfb = static_cast<uint8_t>(ptx::f32x2_to_e4m3x2(t, 0.0f) & 0xFFu);
  os = __frcp_rn(__fmul_rn(ptx::e4m3_to_f32(sfb), rcp_s));
  return sfb;
}

// 8 bf16 (4 words, element 0 in the low half of word 0) -> 8 E2M1 codes, element 0 in the
// low nibble.
__device__ __forceinline__ uint32_t encode8(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3,
                                           float os) {
  return ptx::f32x8_to_e2m1x8(__fmul_rn(bf16lo_to_f32(w0), os), __fmul_rn(bf16hi_to_f32(w0), os),
                              __fmul_rn(bf16lo_to_f32(w1), os), __fmul_rn(bf16hi_to_f32(w1), os),
                              __fmul_rn(bf16lo_to_f32(w2), os), __fmul_rn(bf16hi_to_f32(w2), os),
                              __fmul_rn(bf16lo_to_f32(w3), os), __fmul_rn(bf16hi_to_f32(w3), os));
}

// A whole block held by one thread: 16 bf16 in w0..w7 (by value, so callers' arrays stay in
// registers) -> 8 code bytes (lo, hi words) + scale byte.
__device__ __forceinline__ uint8_t quantize_block16(uint32_t w0, uint32_t w1, uint32_t w2,
                                                    uint32_t w3, uint32_t w4, uint32_t w5,
                                                    uint32_t w6, uint32_t w7, float s, float rcp_s,
                                                    uint32_t& lo, uint32_t& hi) {
  uint32_t m = kAmaxSeed;
  m = abs_max_bf16x2(m, w0);
  m = abs_max_bf16x2(m, w1);
  m = abs_max_bf16x2(m, w2);
  m = abs_max_bf16x2(m, w3);
  m = abs_max_bf16x2(m, w4);
  m = abs_max_bf16x2(m, w5);
  m = abs_max_bf16x2(m, w6);
  m = abs_max_bf16x2(m, w7);
  float os;
  const uint8_t sfb = block_scale(block_amax(m), s, rcp_s, os);
  lo = encode8(w0, w1, w2, w3, os);
  hi = encode8(w4, w5, w6, w7, os);
  return sfb;
}

// The block's encode multiplier os depends only on its scale byte (for a fixed s), so a caller
// that quantizes many blocks can tabulate it once: tab[b] = rcp_rn(f32(b) * rcp_rn(s)), the same
// expression block_scale evaluates.
__device__ __forceinline__ float os_of_scale_byte(uint32_t b, float rcp_s) {
  return __frcp_rn(__fmul_rn(ptx::e4m3_to_f32(uint8_t(b)), rcp_s));
}

// quantize_block16 with the multiplier read from such a table.
__device__ __forceinline__ uint8_t quantize_block16_tab(uint32_t w0, uint32_t w1, uint32_t w2,
                                                        uint32_t w3, uint32_t w4, uint32_t w5,
                                                        uint32_t w6, uint32_t w7, float s,
                                                        const float* tab, uint32_t& lo,
                                                        uint32_t& hi) {
  uint32_t m = kAmaxSeed;
  m = abs_max_bf16x2(m, w0);
  m = abs_max_bf16x2(m, w1);
  m = abs_max_bf16x2(m, w2);
  m = abs_max_bf16x2(m, w3);
  m = abs_max_bf16x2(m, w4);
  m = abs_max_bf16x2(m, w5);
  m = abs_max_bf16x2(m, w6);
  m = abs_max_bf16x2(m, w7);
  const float t = __fmul_rn(__fmul_rn(block_amax(m), s), kRcpE2m1Max);
  const uint8_t sfb = static_cast<uint8_t>(ptx::f32x2_to_e4m3x2(t, 0.0f) & 0xFFu);
  const float os = tab[sfb];
  lo = encode8(w0, w1, w2, w3, os);
  hi = encode8(w4, w5, w6, w7, os);
  return sfb;
}

}  // namespace bq
}  // namespace nvfp4
