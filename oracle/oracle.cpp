// oracle.cpp -- CPU restatement (C++17 + OpenMP, fp32) of the reference's Burn-ndarray
// semantics for the denoiser hot path.  TEST INFRASTRUCTURE ONLY: loaded by tests/,
// __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs, never by the
// product library.  See oracle.h for the per-function parity status ("parity unpinned"
// for GroupNorm and attention, which have no reference golden vectors).
//
// Built with -ffp-contract=off so that every `a*b + c` written here rounds twice, as Rust
// code without fast-math does; GEMM-shaped loops that model a BLAS micro-kernel (which
// does use FMA in the reference's `matrixmultiply`/`gemm` crates) call fmaf explicitly.
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

int g_threads = 0;

inline int nthreads() {
#ifdef _OPENMP
  return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
  return 1;
#endif
}

inline float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

// burn `sigmoid` on ndarray: 1 / (1 + exp(-x)) evaluated in f32.
inline float sigmoidf_ref(float x) { return 1.0f / (1.0f + std::exp(-x)); }

// ---------------------------------------------------------------------------------------
// f16 <-> f32 (IEEE binary16; the `half` crate's to_f32 / from_f32 semantics)
// ---------------------------------------------------------------------------------------
inline float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  const uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      // subnormal: value = man * 2^-24, renormalise
      int e = -1;
      uint32_t m = man;
      do {
        ++e;
        m <<= 1;
      } while ((m & 0x400u) == 0);
      m &= 0x3FFu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (m << 13);
    }
  } else if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);  // inf / nan (payload kept)
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline uint16_t float_to_half_rne(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t absx = x & 0x7FFFFFFFu;
  if (absx >= 0x7F800000u) {  // inf or nan
    if (absx > 0x7F800000u) return (uint16_t)(sign | 0x7E00u | ((absx >> 13) & 0x3FFu));
    return (uint16_t)(sign | 0x7C00u);
  }
  const int e = (int)(absx >> 23) - 127;
  if (e > 15) return (uint16_t)(sign | 0x7C00u);  // overflow -> inf
  if (e >= -14) {
    // normal half: keep 10 mantissa bits, round to nearest even on the 13 dropped bits
    uint32_t m = absx & 0x7FFFFFu;
    uint32_t h = ((uint32_t)(e + 15) << 10) | (m >> 13);
    const uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;  // may carry into exponent
    return (uint16_t)(sign | h);
  }
  if (e < -25) return sign;  // rounds to zero (below half of the smallest subnormal)
  // subnormal half: value = round(|f| * 2^24) as an integer mantissa
  const uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;  // 24-bit significand
  const int shift = -e - 14 + 13;                     // bits dropped: 13 + (-14 - e)
  uint32_t h = m >> shift;
  const uint32_t rem = m & ((1u << shift) - 1u);
  const uint32_t halfway = 1u << (shift - 1);
  if (rem > halfway || (rem == halfway && (h & 1u))) h += 1;
  return (uint16_t)(sign | h);
}

// ---------------------------------------------------------------------------------------
// A small cache-blocked SGEMM modelled on a BLAS micro-kernel (f32 FMA accumulate).
// C[M,N] = A[M,K] * B  (+ C if accumulate), B either [K,N] (nn) or [N,K] (nt).
// ---------------------------------------------------------------------------------------
void sgemm_nn(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
              int64_t lda, int64_t ldb, int64_t ldc, bool accumulate) {
  const int64_t KB = 256, NB = 512;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads())
  for (int64_t i0 = 0; i0 < M; i0 += 4) {
    const int64_t i1 = std::min<int64_t>(i0 + 4, M);
    for (int64_t j0 = 0; j0 < N; j0 += NB) {
      const int64_t j1 = std::min<int64_t>(j0 + NB, N);
      const int64_t nj = j1 - j0;
      float acc[4][NB];
      for (int64_t i = i0; i < i1; ++i)
        for (int64_t j = 0; j < nj; ++j) acc[i - i0][j] = accumulate ? C[i * ldc + j0 + j] : 0.f;
      for (int64_t k0 = 0; k0 < K; k0 += KB) {
        const int64_t k1 = std::min<int64_t>(k0 + KB, K);
        for (int64_t i = i0; i < i1; ++i) {
          float* __restrict__ a = acc[i - i0];
          for (int64_t k = k0; k < k1; ++k) {
            const float av = A[i * lda + k];
            const float* __restrict__ b = B + k * ldb + j0;
            for (int64_t j = 0; j < nj; ++j) a[j] = std::fmaf(av, b[j], a[j]);
          }
        }
      }
      for (int64_t i = i0; i < i1; ++i)
        std::memcpy(C + i * ldc + j0, acc[i - i0], sizeof(float) * nj);
    }
  }
}

// Dot product with 8 interleaved f32 FMA partial sums (a vector micro-kernel's order).
inline float dot_blas(const float* __restrict__ a, const float* __restrict__ b, int64_t n) {
  float p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int64_t k = 0;
  for (; k + 8 <= n; k += 8)
    for (int u = 0; u < 8; ++u) p[u] = std::fmaf(a[k + u], b[k + u], p[u]);
  float s = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
  for (; k < n; ++k) s = std::fmaf(a[k], b[k], s);
  return s;
}

void sgemm_nt(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
              int64_t lda, int64_t ldb, int64_t ldc) {
#pragma omp parallel for collapse(2) schedule(static) num_threads(nthreads())
  for (int64_t i = 0; i < M; ++i)
    for (int64_t j = 0; j < N; ++j) C[i * ldc + j] = dot_blas(A + i * lda, B + j * ldb, K);
}

}  // namespace

extern "C" {

int or_set_threads(int n) {
  g_threads = n;
  return nthreads();
}
int or_get_threads(void) { return nthreads(); }

void or_f16_to_f32(const uint16_t* h, float* f, int64_t n) {
  for (int64_t i = 0; i < n; ++i) f[i] = half_to_float(h[i]);
}
void or_f32_to_f16(const float* f, uint16_t* h, int64_t n) {
  for (int64_t i = 0; i < n; ++i) h[i] = float_to_half_rne(f[i]);
}

// Rounding of an f32 value to the tensor dtype and back: 0 = f32 (no-op), 1 = f16 (the
// `half` crate's f16::from_f32, round to nearest even), 2 = bf16 (half's bf16::from_f32,
// round to nearest even).
inline float bf16_round(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return f;  // nan stays nan
  u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}
inline float round_to_dtype(float v, int dtype) {
  if (dtype == 1) return half_to_float(float_to_half_rne(v));
  if (dtype == 2) return bf16_round(v);
  return v;
}

// crates/sketchpad-core/src/groupnorm.rs:62-102 (+ silu.rs:5-7).  dtype is the tensor dtype
// of x, weight and bias (0 f32, 1 f16, 2 bf16); their values arrive here as f32 (exact).
//  * :68 clamp x to +-65000 (in the tensor dtype; exact for f16/bf16 inputs)
//  * :76-87 f32 mean, biased variance (mean of squared deviations), (x - mean)/sqrt(var+eps)
//  * :88 cast the normalised value back to the tensor dtype  <- rounding for f16/bf16
//  * :95 x * weight + bias as two tensor ops in the tensor dtype, each rounded
//  * :99 clamp +-65000
//  * silu.rs:5-7 x * sigmoid(x): burn's sigmoid evaluates in f32 and casts back to the
//    tensor dtype (burn-tensor 0.20.0-pre.6 ActivationOps::sigmoid default; burn is not
//    vendored with the reference, so this step is restated from its published code), then
//    the product is one more tensor op in the tensor dtype.
int or_groupnorm_act_dtype(const float* x, const float* gamma, const float* beta, float* y,
                           int64_t B, int64_t C, int64_t H, int64_t W, int64_t G, float eps,
                           int act, int dtype) {
  if (!x || !gamma || !beta || !y || B <= 0 || C <= 0 || H <= 0 || W <= 0 || G <= 0) return -1;
  if (dtype < 0 || dtype > 2) return -1;
  if (C % G != 0) return -2;  // the reference asserts channels % num_groups == 0
  const int64_t cg = C / G, hw = H * W, n = cg * hw;
#pragma omp parallel for collapse(2) schedule(dynamic, 1) num_threads(nthreads())
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t g = 0; g < G; ++g) {
      const float* xs = x + (b * C + g * cg) * hw;
      float* ys = y + (b * C + g * cg) * hw;
      // x.clamp(-65000, 65000); mean_dim(2) in f32 (accumulated in double, rounded once)
      double s = 0.0;
      for (int64_t i = 0; i < n; ++i) s += (double)clampf(xs[i], -65000.f, 65000.f);
      const float mean = (float)(s / (double)n);
      // var = mean((x - mean)^2)  -- the BIASED variance (divide by n)
      double ss = 0.0;
      for (int64_t i = 0; i < n; ++i) {
        const float d = clampf(xs[i], -65000.f, 65000.f) - mean;
        ss += (double)(d * d);
      }
      const float var = (float)(ss / (double)n);
      const float denom = std::sqrt(var + eps);
      for (int64_t c = 0; c < cg; ++c) {
        const float w = gamma[g * cg + c], bb = beta[g * cg + c];
        for (int64_t i = 0; i < hw; ++i) {
          const float d = clampf(xs[c * hw + i], -65000.f, 65000.f) - mean;
          const float xn = round_to_dtype(d / denom, dtype);  // x_f32.cast(original_dtype)
          float v = round_to_dtype(round_to_dtype(xn * w, dtype) + bb, dtype);
          v = clampf(v, -65000.f, 65000.f);
          if (act == 1) v = round_to_dtype(v * round_to_dtype(sigmoidf_ref(v), dtype), dtype);
          ys[c * hw + i] = v;
        }
      }
    }
  }
  return 0;
}

int or_groupnorm_act(const float* x, const float* gamma, const float* beta, float* y, int64_t B,
                     int64_t C, int64_t H, int64_t W, int64_t G, float eps, int act) {
  return or_groupnorm_act_dtype(x, gamma, beta, y, B, C, H, W, G, eps, act, 0);
}

// crates/sketchpad-unet/src/blocks.rs:393-401 (variant 0) and
// crates/sketchpad-core/src/attention.rs:4-27 (variant 1).
int or_attention(const float* q, const float* k, const float* v, const float* mask, float* out,
                 int64_t BH, int64_t Sq, int64_t Skv, int64_t D, int64_t Dv, int causal,
                 float scale, int variant) {
  if (!q || !k || !v || !out || BH <= 0 || Sq <= 0 || Skv <= 0 || D <= 0 || Dv <= 0) return -1;
  const float sc = scale > 0.f ? scale : (float)std::pow((double)D, -0.5);
  const float sc4 = scale > 0.f ? std::sqrt(scale) : (float)std::pow((double)D, -0.25);
  const float ninf = -std::numeric_limits<float>::infinity();
#pragma omp parallel num_threads(nthreads())
  {
    std::vector<float> srow(Skv), qrow(D), acc(Dv);
    std::vector<float> kscaled;
#pragma omp for collapse(2) schedule(dynamic, 16)
    for (int64_t bh = 0; bh < BH; ++bh) {
      for (int64_t i = 0; i < Sq; ++i) {
        const float* qi = q + (bh * Sq + i) * D;
        const float* kb = k + bh * Skv * D;
        const float* vb = v + bh * Skv * Dv;
        if (variant == 1) {
          for (int64_t d = 0; d < D; ++d) qrow[d] = qi[d] * sc4;
          for (int64_t j = 0; j < Skv; ++j) {
            float p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int64_t d = 0;
            for (; d + 8 <= D; d += 8)
              for (int u = 0; u < 8; ++u) p[u] = std::fmaf(qrow[d + u], kb[j * D + d + u] * sc4, p[u]);
            float s = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
            for (; d < D; ++d) s = std::fmaf(qrow[d], kb[j * D + d] * sc4, s);
            srow[j] = s;
          }
        } else {
          for (int64_t j = 0; j < Skv; ++j) srow[j] = dot_blas(qi, kb + j * D, D) * sc;
        }
        for (int64_t j = 0; j < Skv; ++j) {
          if (mask) srow[j] += mask[i * Skv + j];
          if (causal && j > i) srow[j] = ninf;
        }
        float m = ninf;
        for (int64_t j = 0; j < Skv; ++j) m = std::max(m, srow[j]);
        double sum = 0.0;
        for (int64_t j = 0; j < Skv; ++j) {
          srow[j] = std::exp(srow[j] - m);
          sum += srow[j];
        }
        const float fsum = (float)sum;
        for (int64_t d = 0; d < Dv; ++d) acc[d] = 0.f;
        for (int64_t j = 0; j < Skv; ++j) {
          const float p = srow[j] / fsum;
          const float* vj = vb + j * Dv;
          for (int64_t d = 0; d < Dv; ++d) acc[d] = std::fmaf(p, vj[d], acc[d]);
        }
        float* oi = out + (bh * Sq + i) * Dv;
        for (int64_t d = 0; d < Dv; ++d) oi[d] = acc[d];
      }
    }
  }
  return 0;
}

// crates/sketchpad-convert/src/gguf.rs:638-656
int or_q8_0_dequantize(const uint8_t* data, int64_t nblocks, float* out) {
  if (!data || !out || nblocks < 0) return -1;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t bi = 0; bi < nblocks; ++bi) {
    const uint8_t* blk = data + bi * 34;
    const uint16_t bits = (uint16_t)(blk[0] | (blk[1] << 8));
    const float scale = half_to_float(bits);
    for (int i = 0; i < 32; ++i) out[bi * 32 + i] = scale * (float)(int8_t)blk[2 + i];
  }
  return 0;
}

// K-quant super-blocks of 256 values, the reference's CPU decode
// (crates/sketchpad-convert/src/gguf.rs:737-871).  Products are evaluated left to right in
// f32 as the Rust expressions are (`d * sc * q - dmin * m`, `d * scale * raw`).
// fmt: 10 = Q2_K (84 B), 11 = Q3_K (110 B), 12 = Q4_K (144 B).
int or_kquant_dequantize(int fmt, const uint8_t* data, int64_t nblocks, float* out) {
  if (!data || !out || nblocks < 0 || fmt < 10 || fmt > 12) return -1;
  const int bytes = fmt == 12 ? 144 : (fmt == 10 ? 84 : 110);
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t bi = 0; bi < nblocks; ++bi) {
    const uint8_t* blk = data + bi * bytes;
    float* o = out + bi * 256;
    if (fmt == 12) {  // gguf.rs:821-852, scales/mins gguf.rs:854-871
      const float d = half_to_float((uint16_t)(blk[0] | (blk[1] << 8)));
      const float dmin = half_to_float((uint16_t)(blk[2] | (blk[3] << 8)));
      const uint8_t* sb = blk + 4;
      const uint8_t* qs = blk + 16;
      uint8_t scales[8], mins[8];
      for (int i = 0; i < 4; ++i) {
        scales[i] = sb[i] & 63;
        mins[i] = sb[i + 4] & 63;
      }
      for (int i = 4; i < 8; ++i) {
        scales[i] = (uint8_t)((sb[i + 4] & 0x0F) | ((sb[i - 4] >> 6) << 4));
        mins[i] = (uint8_t)((sb[i + 4] >> 4) | ((sb[i] >> 6) << 4));
      }
      for (int j = 0; j < 8; ++j) {
        const float sc = (float)scales[j], m = (float)mins[j];
        for (int i = 0; i < 16; ++i) {
          const uint8_t byte = qs[j * 16 + i];
          const float lo = (float)(byte & 0x0F), hi = (float)((byte >> 4) & 0x0F);
          const float dsc = d * sc, dm = dmin * m;
          o[j * 32 + i] = dsc * lo - dm;
          o[j * 32 + i + 16] = dsc * hi - dm;
        }
      }
    } else if (fmt == 10) {  // gguf.rs:737-758
      const uint8_t* sb = blk;
      const uint8_t* qs = blk + 16;
      const float d = half_to_float((uint16_t)(blk[80] | (blk[81] << 8)));
      const float dmin = half_to_float((uint16_t)(blk[82] | (blk[83] << 8)));
      for (int i = 0; i < 256; ++i) {
        const int ib = i / 16;
        const float sc = (float)(sb[ib] & 0x0F), m = (float)((sb[ib] >> 4) & 0x0F);
        const float q = (float)((qs[i / 4] >> (2 * (i % 4))) & 0x3);
        const float dsc = d * sc, dm = dmin * m;
        o[i] = dsc * q - dm;
      }
    } else {  // Q3_K, gguf.rs:760-819
      const uint8_t* hmask = blk;
      const uint8_t* qs = blk + 32;
      const uint8_t* sr = blk + 96;
      const float d = half_to_float((uint16_t)(blk[108] | (blk[109] << 8)));
      const uint32_t w0 = (uint32_t)sr[0] | ((uint32_t)sr[1] << 8) | ((uint32_t)sr[2] << 16) |
                          ((uint32_t)sr[3] << 24);
      const uint32_t w1 = (uint32_t)sr[4] | ((uint32_t)sr[5] << 8) | ((uint32_t)sr[6] << 16) |
                          ((uint32_t)sr[7] << 24);
      const uint32_t utmp[4] = {w0 & 0x3f3f3f3fu, w1 & 0x3f3f3f3fu, (w0 >> 6) & 0x3f3f3f3fu,
                                (w1 >> 6) & 0x3f3f3f3fu};
      int scales[16];
      for (int i = 0; i < 4; ++i)
        for (int b = 0; b < 4; ++b) scales[i * 4 + b] = (int)((utmp[i] >> (b * 8)) & 0xFF) - 32;
      for (int i = 0; i < 256; ++i) {
        const int low2 = (qs[i / 4] >> (2 * (i % 4))) & 0x3;
        const int hbit = (hmask[i / 8] >> (i % 8)) & 1;
        const int raw = (low2 | (hbit << 2)) - 4;
        const float ds = d * (float)scales[i / 16];
        o[i] = ds * (float)raw;
      }
    }
  }
  return 0;
}

// crates/sketchpad-llm/src/quantized.rs:70-92 (QuantizedTensor::matmul_f32): row dequant into
// a buffer, then for every token a sequential f32 dot (Iterator::sum folds from -0.0).
int or_q8_0_matmul(const uint8_t* data, int64_t N, int64_t K, const float* x, int64_t M,
                   float* y) {
  if (!data || !x || !y || N <= 0 || K <= 0 || M <= 0 || K % 32 != 0) return -1;
  const int64_t row_bytes = K / 32 * 34;
#pragma omp parallel num_threads(nthreads())
  {
    std::vector<float> row(K);
#pragma omp for schedule(dynamic, 4)
    for (int64_t n = 0; n < N; ++n) {
      or_q8_0_dequantize(data + n * row_bytes, K / 32, row.data());
      for (int64_t t = 0; t < M; ++t) {
        const float* xi = x + t * K;
        float s = -0.0f;
        for (int64_t kk = 0; kk < K; ++kk) {
          const float prod = xi[kk] * row[kk];
          s = s + prod;
        }
        y[t * N + n] = s;
      }
    }
  }
  return 0;
}

// crates/sketchpad-core/src/quantization.rs:451-492 (quantize_fp8_scalar)
float or_fp8_quantize_scalar(float value, int format) {
  const float max_val = format == 0 ? 448.0f : 57344.0f;
  const float min_sub = format == 0 ? std::ldexp(1.0f, -9) : std::ldexp(1.0f, -16);
  const int mant_bits = format == 0 ? 3 : 2;
  if (std::isnan(value)) return std::numeric_limits<float>::quiet_NaN();
  if (std::isinf(value)) return value > 0 ? max_val : -max_val;
  const float sign = std::signbit(value) ? -1.0f : 1.0f;  // f32::signum (+0 -> 1, -0 -> -1)
  const float a = std::fabs(value);
  if (a > max_val) return sign * max_val;
  if (a < min_sub) return 0.0f;
  const int e = (int)std::floor(std::log2(a));
  const float ms = std::ldexp(1.0f, e);                 // 2f32.powi(e), exact
  const float normalized = a / ms;
  const float steps = (float)(1u << mant_bits);
  const float qm = std::round((normalized - 1.0f) * steps) / steps + 1.0f;  // half away from 0
  return sign * qm * ms;
}

// crates/sketchpad-core/src/quantization.rs:495-577 (quantize_fp8)
int or_fp8_quantize(const float* w, int64_t rows, int64_t cols, int format, int per_channel,
                    int has_explicit_scale, float explicit_scale, float* data_out,
                    float* scale_out) {
  if (!w || !data_out || !scale_out || rows <= 0 || cols <= 0) return -1;
  const float max_fp8 = format == 0 ? 448.0f : 57344.0f;
  if (per_channel) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
    for (int64_t r = 0; r < rows; ++r) {
      float mx = 0.f;
      for (int64_t c = 0; c < cols; ++c) mx = std::max(mx, std::fabs(w[r * cols + c]));
      const float scale = mx > 0.f ? mx / max_fp8 : 1.0f;
      scale_out[r] = scale;
      for (int64_t c = 0; c < cols; ++c)
        data_out[r * cols + c] = or_fp8_quantize_scalar(w[r * cols + c] / scale, format);
    }
  } else {
    float scale;
    if (has_explicit_scale) {
      scale = explicit_scale;
    } else {
      float mx = 0.f;
      for (int64_t i = 0; i < rows * cols; ++i) mx = std::max(mx, std::fabs(w[i]));
      scale = mx > 0.f ? mx / max_fp8 : 1.0f;
    }
    scale_out[0] = scale;
#pragma omp parallel for schedule(static) num_threads(nthreads())
    for (int64_t i = 0; i < rows * cols; ++i) data_out[i] = or_fp8_quantize_scalar(w[i] / scale, format);
  }
  return 0;
}

// crates/sketchpad-core/src/quantization.rs:435-447 (Fp8Tensor::dequantize)
int or_fp8_dequantize(const float* data, const float* scale, int64_t nscale, int64_t rows,
                      int64_t cols, float* out) {
  if (!data || !scale || !out || rows <= 0 || cols <= 0) return -1;
  if (nscale != 1 && nscale != rows) return -2;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t r = 0; r < rows; ++r) {
    const float s = nscale == 1 ? scale[0] : scale[r];
    for (int64_t c = 0; c < cols; ++c) out[r * cols + c] = data[r * cols + c] * s;
  }
  return 0;
}

int or_linear_nt(const float* x, const float* w_nk, const float* b, float* y, int64_t M,
                 int64_t K, int64_t N) {
  if (!x || !w_nk || !y || M <= 0 || K <= 0 || N <= 0) return -1;
  sgemm_nt(x, w_nk, y, M, N, K, K, K, N);
  if (b) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
    for (int64_t i = 0; i < M; ++i)
      for (int64_t j = 0; j < N; ++j) y[i * N + j] += b[j];
  }
  return 0;
}

int or_linear_kn(const float* x, const float* w_kn, const float* b, float* y, int64_t M,
                 int64_t K, int64_t N) {
  if (!x || !w_kn || !y || M <= 0 || K <= 0 || N <= 0) return -1;
  sgemm_nn(x, w_kn, y, M, N, K, K, N, N, false);
  if (b) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
    for (int64_t i = 0; i < M; ++i)
      for (int64_t j = 0; j < N; ++j) y[i * N + j] += b[j];
  }
  return 0;
}

// crates/sketchpad-core/src/layernorm.rs:63-73 -- burn `var` is the unbiased (n-1) variance.
int or_layernorm(const float* x, const float* gamma, const float* beta, float* y, int64_t rows,
                 int64_t n, float eps) {
  if (!x || !gamma || !beta || !y || rows <= 0 || n <= 1) return -1;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * n;
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += xr[i];
    const float mean = (float)(s / (double)n);
    double ss = 0.0;
    for (int64_t i = 0; i < n; ++i) {
      const float d = xr[i] - mean;
      ss += (double)(d * d);
    }
    const float var = (float)(ss / (double)(n - 1));
    const float denom = std::sqrt(var + eps);
    for (int64_t i = 0; i < n; ++i) y[r * n + i] = (xr[i] - mean) / denom * gamma[i] + beta[i];
  }
  return 0;
}

int or_activation(const float* x, float* y, int64_t n, int kind) {
  if (!x || !y || n < 0) return -1;
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t i = 0; i < n; ++i) {
    const float v = x[i];
    if (kind == 0)
      y[i] = v * sigmoidf_ref(v);
    else if (kind == 1)
      y[i] = (float)((double)v * 0.5 * (1.0 + std::erf((double)v / std::sqrt(2.0))));
    else
      y[i] = sigmoidf_ref(v);
  }
  return 0;
}

// NCHW conv2d via im2col + SGEMM (burn-ndarray conv2d semantics: cross-correlation, zero pad).
int or_conv2d(const float* x, const float* w, const float* b, float* y, int64_t B, int64_t Cin,
              int64_t H, int64_t W, int64_t Cout, int64_t kh, int64_t kw, int64_t stride,
              int64_t pad) {
  if (!x || !w || !y || B <= 0 || Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0 || stride <= 0)
    return -1;
  const int64_t Ho = (H + 2 * pad - kh) / stride + 1, Wo = (W + 2 * pad - kw) / stride + 1;
  const int64_t Kc = Cin * kh * kw, P = Ho * Wo;
  std::vector<float> col((size_t)(Kc * P));
  for (int64_t bi = 0; bi < B; ++bi) {
    const float* xb = x + bi * Cin * H * W;
#pragma omp parallel for collapse(2) schedule(static) num_threads(nthreads())
    for (int64_t c = 0; c < Cin; ++c)
      for (int64_t u = 0; u < kh; ++u)
        for (int64_t vv = 0; vv < kw; ++vv) {
          float* dst = col.data() + ((c * kh + u) * kw + vv) * P;
          for (int64_t oy = 0; oy < Ho; ++oy) {
            const int64_t iy = oy * stride - pad + u;
            for (int64_t ox = 0; ox < Wo; ++ox) {
              const int64_t ix = ox * stride - pad + vv;
              dst[oy * Wo + ox] =
                  (iy >= 0 && iy < H && ix >= 0 && ix < W) ? xb[(c * H + iy) * W + ix] : 0.f;
            }
          }
        }
    float* yb = y + bi * Cout * P;
    sgemm_nn(w, col.data(), yb, Cout, P, Kc, Kc, P, P, false);
    if (b) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
      for (int64_t co = 0; co < Cout; ++co)
        for (int64_t p = 0; p < P; ++p) yb[co * P + p] += b[co];
    }
  }
  return 0;
}

}  // extern "C"
