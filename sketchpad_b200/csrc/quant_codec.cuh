// quant_codec.cuh -- device codecs for the quantized weight formats.
//
// e4m3 (OCP FP8, "E4M3FN"): 1 sign, 4 exponent (bias 7), 3 mantissa bits; normals
// (1 + m/8) * 2^(e-7) for e in 1..15 (e=15, m=7 is NaN), subnormals m/8 * 2^-6.
// Written from the bit-layout definition; every e4m3 value is exact in f32 and in bf16.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace sp {

__host__ __device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  const uint32_t sign = (uint32_t)(b & 0x80u) << 24;
  const uint32_t e = (b >> 3) & 0xFu;
  const uint32_t m = b & 0x7u;
  uint32_t bits;
  if (e == 0xFu && m == 0x7u) {
    bits = sign | 0x7FC00000u;  // NaN
  } else if (e == 0) {
    // subnormal: m * 2^-9 (m in 0..7), exact
    if (m == 0) {
      bits = sign;
    } else {
      const int lz = m >= 4 ? 0 : (m >= 2 ? 1 : 2);  // normalise m into 1.xx
      const uint32_t mm = (m << (lz + 1)) & 0x7u;    // drop the leading one
      bits = sign | ((uint32_t)(127 - 7 - lz) << 23) | (mm << 20);
    }
  } else {
    bits = sign | ((e + 120u) << 23) | (m << 20);
  }
#ifdef __CUDA_ARCH__
  return __uint_as_float(bits);
#else
  float f;
  __builtin_memcpy(&f, &bits, 4);
  return f;
#endif
}

// Encode with the rounding rule of the reference's quantize_fp8_scalar
// (crates/sketchpad-core/src/quantization.rs:451-492): NaN stays NaN, |v| > 448 saturates
// to 448, |v| < 2^-9 goes to zero, otherwise the mantissa is rounded to 3 bits to nearest
// with ties away from zero.  Below 2^-6 the reference keeps 3 mantissa bits that e4m3
// cannot store; there the value is rounded (ties away) to the e4m3 subnormal grid k * 2^-9.
__device__ __forceinline__ uint8_t f32_to_e4m3_ref(float v) {
  const uint32_t bits = __float_as_uint(v);
  const uint8_t sign = (uint8_t)((bits >> 24) & 0x80u);
  const float a = fabsf(v);
  if (a != a) return 0x7F;                 // NaN
  if (a > 448.0f) return sign | 0x7E;      // saturate (inf included)
  if (a < 0.001953125f) return 0;          // < 2^-9 -> +0 as the reference returns 0.0
  if (a < 0.015625f) {                     // [2^-9, 2^-6): subnormal grid
    const float k = floorf(a * 512.0f + 0.5f);  // exact scaling by 2^9, ties away from zero
    return sign | (uint8_t)k;              // k in 1..8; k == 8 encodes 2^-6 as 0x08
  }
  int e = (int)((__float_as_uint(a) >> 23) & 0xFFu) - 127;  // floor(log2 a), a normal f32
  const float normalized = a * __uint_as_float((uint32_t)(127 - e) << 23);  // a / 2^e, exact
  int q = (int)floorf((normalized - 1.0f) * 8.0f + 0.5f);  // round half away (value >= 0)
  if (q == 8) {
    q = 0;
    e += 1;
  }
  return sign | (uint8_t)(((e + 7) << 3) | q);
}

}  // namespace sp
