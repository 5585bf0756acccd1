// kquant.cu -- GGUF K-quant weights (Q4_K, Q2_K, Q3_K): lossless repack into the planar
// layout of the fused dequant-GEMM, and the dequantization kernel.
//
// Decode semantics follow the reference's CPU decode, the parity oracle:
//   Q4_K  crates/sketchpad-convert/src/gguf.rs:821-871  (144 B / 256 values: f16 d, f16 dmin,
//         12 B of 6-bit scales/mins, 128 B of nibbles; sub-block j of 32 values uses bytes
//         16j..16j+15: low nibbles are values 0..15, high nibbles 16..31);
//         w = d * sc * q - dmin * m
//   Q2_K  gguf.rs:737-758  (84 B: 16 B of (scale, min) nibbles per 16 values, 64 B of 2-bit
//         quants, 4 per byte from the low bits up, f16 d, f16 dmin); w = d * sc * q - dmin * m
//   Q3_K  gguf.rs:760-819  (110 B: 32 B high-bit mask, 64 B low 2 bits, 12 B scales, f16 d);
//         w = d * scale * (q - 4) with q = low2 | hbit << 2 and scale = 6-bit field - 32, the
//         6-bit fields extracted as that function does (its `utmp` words)
// The reference's GPU kernels (crates/sketchpad-cubecl/src/quantized_matmul.rs:113-360)
// agree with these for Q4_K and Q2_K; for Q3_K their scale extraction for sub-blocks 8..15
// differs from the CPU decode, and the CPU decode is the one followed here.  d and dmin
// decode as IEEE f16 including subnormals (the CPU `half` crate behaviour).
//
// Repacked layout (all three formats): `qpack` [N, K/2] bytes holding one 4-bit unsigned
// quant per value (value k of a row at byte k/2, low nibble for even k); per sub-block of
// `sub` values (32 for Q4_K, 16 for Q2_K/Q3_K) two f32 factors in k-block-major arrays
// a[K/sub][N] = f32(d) * sc and b[K/sub][N] = f32(dmin) * m (b = 0 for Q3_K), each rounded
// to f32 as the reference's left-to-right product does.  Then w = a * (q - off) - b
// reproduces the reference's f32 value exactly (off = 4 for Q3_K, else 0).
#include <cstring>

#include "common.cuh"

namespace sp {
namespace {

constexpr int kBlockBytes[3] = {144, 84, 110};  // Q4_K, Q2_K, Q3_K

int kq_index(int fmt) {
  switch (fmt) {
    case SP_QK_Q4_K: return 0;
    case SP_QK_Q2_K: return 1;
    case SP_QK_Q3_K: return 2;
    default: return -1;
  }
}

// IEEE binary16 -> binary32, exact (normals, subnormals, inf, NaN), from the bit layout.
float f16_bits_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu;
  uint32_t bits;
  if (e == 0x1F) {
    bits = sign | 0x7F800000u | (m << 13);
  } else if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {  // subnormal m * 2^-24: normalise
      int sh = 0;
      while (!(m & 0x400u)) {
        m <<= 1;
        ++sh;
      }
      bits = sign | ((uint32_t)(127 - 15 + 1 - sh) << 23) | ((m & 0x3FFu) << 13);
    }
  } else {
    bits = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// The reference's product `d * sc` (or `dmin * m`): one f32 multiplication, rounded.
inline float mul_f32(float a, float b) { return a * b; }

// 6-bit scale/min of Q4_K sub-block j (gguf.rs:854-871).
inline void q4k_scale_min(const uint8_t* buf, int j, int& sc, int& m) {
  if (j < 4) {
    sc = buf[j] & 63;
    m = buf[j + 4] & 63;
  } else {
    sc = (buf[j + 4] & 0x0F) | ((buf[j - 4] >> 6) << 4);
    m = (buf[j + 4] >> 4) | ((buf[j] >> 6) << 4);
  }
}

// The 16 signed 6-bit Q3_K scales as gguf.rs:767-810 extracts them.
inline void q3k_scales(const uint8_t* s, int out[16]) {
  const uint32_t w0 = (uint32_t)s[0] | ((uint32_t)s[1] << 8) | ((uint32_t)s[2] << 16) |
                      ((uint32_t)s[3] << 24);
  const uint32_t w1 = (uint32_t)s[4] | ((uint32_t)s[5] << 8) | ((uint32_t)s[6] << 16) |
                      ((uint32_t)s[7] << 24);
  const uint32_t u[4] = {w0 & 0x3f3f3f3fu, w1 & 0x3f3f3f3fu, (w0 >> 6) & 0x3f3f3f3fu,
                         (w1 >> 6) & 0x3f3f3f3fu};
  for (int i = 0; i < 4; ++i)
    for (int b = 0; b < 4; ++b) out[i * 4 + b] = (int)((u[i] >> (8 * b)) & 0xFFu) - 32;
}

inline void put_nibble(uint8_t* row, int64_t k, uint32_t q) {
  uint8_t& byte = row[k >> 1];
  byte = (k & 1) ? (uint8_t)((byte & 0x0F) | (q << 4)) : (uint8_t)((byte & 0xF0) | q);
}

// One super-block (256 values of row n starting at column k0) -> nibbles + factors.
void repack_block(int fi, const uint8_t* blk, int64_t N, int64_t n, int64_t k0, uint8_t* qrow,
                  float* a, float* b) {
  if (fi == 0) {  // Q4_K
    const float d = f16_bits_to_f32(rd16(blk)), dmin = f16_bits_to_f32(rd16(blk + 2));
    const uint8_t* sbuf = blk + 4;
    const uint8_t* qs = blk + 16;
    for (int j = 0; j < 8; ++j) {
      int sc, m;
      q4k_scale_min(sbuf, j, sc, m);
      const int64_t kb = (k0 >> 5) + j;
      a[kb * N + n] = mul_f32(d, (float)sc);
      b[kb * N + n] = mul_f32(dmin, (float)m);
      for (int i = 0; i < 16; ++i) {
        const uint8_t byte = qs[j * 16 + i];
        put_nibble(qrow, k0 + j * 32 + i, byte & 0x0F);
        put_nibble(qrow, k0 + j * 32 + i + 16, (byte >> 4) & 0x0F);
      }
    }
  } else if (fi == 1) {  // Q2_K
    const uint8_t* sbuf = blk;
    const uint8_t* qs = blk + 16;
    const float d = f16_bits_to_f32(rd16(blk + 80)), dmin = f16_bits_to_f32(rd16(blk + 82));
    for (int j = 0; j < 16; ++j) {
      const int64_t kb = (k0 >> 4) + j;
      a[kb * N + n] = mul_f32(d, (float)(sbuf[j] & 0x0F));
      b[kb * N + n] = mul_f32(dmin, (float)((sbuf[j] >> 4) & 0x0F));
    }
    for (int i = 0; i < 256; ++i) put_nibble(qrow, k0 + i, (qs[i / 4] >> (2 * (i % 4))) & 0x3);
  } else {  // Q3_K
    const uint8_t* hmask = blk;
    const uint8_t* qs = blk + 32;
    const float d = f16_bits_to_f32(rd16(blk + 108));
    int sc[16];
    q3k_scales(blk + 96, sc);
    for (int j = 0; j < 16; ++j) {
      const int64_t kb = (k0 >> 4) + j;
      a[kb * N + n] = mul_f32(d, (float)sc[j]);
      b[kb * N + n] = 0.0f;
    }
    for (int i = 0; i < 256; ++i) {
      const uint32_t low2 = (qs[i / 4] >> (2 * (i % 4))) & 0x3;
      const uint32_t hbit = (hmask[i / 8] >> (i % 8)) & 1;
      put_nibble(qrow, k0 + i, low2 | (hbit << 2));
    }
  }
}

template <typename T>
__device__ __forceinline__ T kq_out(float v);
template <>
__device__ __forceinline__ float kq_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half kq_out<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 kq_out<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// One thread per byte of qpack (two values): w = a * (q - off) - b, f32, then cast.
template <typename T>
__global__ void kquant_dequant_kernel(const uint8_t* __restrict__ qpack, const float* __restrict__ a,
                                      const float* __restrict__ b, int64_t N, int64_t K, int sub_shift,
                                      float off, T* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // byte index
  if (i >= N * (K >> 1)) return;
  const int64_t n = i / (K >> 1), k = (i - n * (K >> 1)) * 2;
  const uint8_t byte = qpack[i];
  const int64_t f = (k >> sub_shift) * N + n;  // both values share a sub-block (sub >= 16)
  const float fa = a[f], fb = b[f];
  const float q0 = (float)(byte & 0x0F) - off, q1 = (float)(byte >> 4) - off;  // exact
  out[n * K + k] = kq_out<T>(__fsub_rn(__fmul_rn(fa, q0), fb));
  out[n * K + k + 1] = kq_out<T>(__fsub_rn(__fmul_rn(fa, q1), fb));
}

}  // namespace
}  // namespace sp

extern "C" {

int sp_kquant_repack_host(int fmt, const uint8_t* gguf_host, size_t nbytes, int64_t out_f,
                          int64_t in_f, uint8_t* qpack_host, float* a_host, float* b_host) {
  using namespace sp;
  clear_error();
  const int fi = kq_index(fmt);
  if (fi < 0) return set_error(SP_ERR_DTYPE, "k-quant repack: unknown format %d", fmt);
  if (!gguf_host || !qpack_host || !a_host || !b_host)
    return set_error(SP_ERR_INVALID_ARG, "k-quant repack: null pointer");
  if (out_f <= 0 || in_f <= 0 || in_f % 256)
    return set_error(SP_ERR_SHAPE, "k-quant repack: in_features (%lld) must be a positive multiple of 256",
                     (long long)in_f);
  const int64_t spr = in_f / 256;  // super-blocks per row
  const int64_t nblocks = out_f * spr;
  if (nbytes < (size_t)nblocks * kBlockBytes[fi])
    return set_error(SP_ERR_SHAPE, "k-quant repack: %zu bytes < %lld super-blocks x %d", nbytes,
                     (long long)nblocks, kBlockBytes[fi]);
  std::memset(qpack_host, 0, (size_t)out_f * (size_t)(in_f / 2));
  for (int64_t n = 0; n < out_f; ++n)
    for (int64_t s = 0; s < spr; ++s)
      repack_block(fi, gguf_host + (n * spr + s) * kBlockBytes[fi], out_f, n, s * 256,
                   qpack_host + n * (in_f / 2), a_host, b_host);
  return SP_OK;
}

int sp_kquant_dequant(int fmt, const void* qpack, const float* a, const float* b, int64_t out_f,
                      int64_t in_f, void* out, int out_dtype, void* stream) {
  using namespace sp;
  clear_error();
  const int fi = kq_index(fmt);
  if (fi < 0) return set_error(SP_ERR_DTYPE, "k-quant dequant: unknown format %d", fmt);
  if (!qpack || !a || !b || !out) return set_error(SP_ERR_INVALID_ARG, "k-quant dequant: null pointer");
  if (out_f <= 0 || in_f <= 0 || in_f % 256)
    return set_error(SP_ERR_SHAPE, "k-quant dequant: in_features (%lld) must be a positive multiple of 256",
                     (long long)in_f);
  if (int rc = require_sm100()) return rc;
  const int sub_shift = fi == 0 ? 5 : 4;
  const float off = fi == 2 ? 4.0f : 0.0f;
  const int64_t nbytes = out_f * (in_f / 2);
  const unsigned grid = (unsigned)((nbytes + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* qp = static_cast<const uint8_t*>(qpack);
  switch (out_dtype) {
    case SP_F32:
      kquant_dequant_kernel<float><<<grid, 256, 0, s>>>(qp, a, b, out_f, in_f, sub_shift, off,
                                                        static_cast<float*>(out));
      break;
    case SP_F16:
      kquant_dequant_kernel<__half><<<grid, 256, 0, s>>>(qp, a, b, out_f, in_f, sub_shift, off,
                                                         static_cast<__half*>(out));
      break;
    case SP_BF16:
      kquant_dequant_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          qp, a, b, out_f, in_f, sub_shift, off, static_cast<__nv_bfloat16*>(out));
      break;
    default: return set_error(SP_ERR_DTYPE, "k-quant dequant: unknown out dtype %d", out_dtype);
  }
  return check_launch("k-quant dequant");
}

}  // extern "C"
