// quant.cu -- Q8_0 repack/dequantize and FP8 (e4m3) quantize/dequantize kernels.
//
// Q8_0: crates/sketchpad-convert/src/gguf.rs:643-656 (CPU decode: f16 scale incl. subnormals)
//       crates/sketchpad-cubecl/src/quantized_matmul.rs:85-110, :376-408 (GPU decode).
// FP8:  crates/sketchpad-core/src/quantization.rs:435-447 (dequantize), :495-577 (quantize).
#include <cstring>

#include "common.cuh"
#include "quant_codec.cuh"

namespace sp {
namespace {

// One thread per 34-byte GGUF block -> 32 int8 quants (8 x u32) + one f16 scale.  Block i
// is (row n = i / kb, k-block i % kb); its scale goes to scale[i % kb][n] (k-block-major, so
// the GEMM loads a k-tile's scales for 256 consecutive rows as one 512-byte TMA row).
__global__ void q8_0_repack_kernel(const uint8_t* __restrict__ gguf, int64_t nblocks, int64_t kb,
                                   int64_t rows, int8_t* __restrict__ q,
                                   uint16_t* __restrict__ scale) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nblocks) return;
  const uint8_t* blk = gguf + i * 34;
  scale[(i % kb) * rows + i / kb] = (uint16_t)(blk[0] | (blk[1] << 8));
  uint32_t w[8];
#pragma unroll
  for (int t = 0; t < 8; ++t)
    w[t] = (uint32_t)blk[2 + 4 * t] | ((uint32_t)blk[3 + 4 * t] << 8) |
           ((uint32_t)blk[4 + 4 * t] << 16) | ((uint32_t)blk[5 + 4 * t] << 24);
  uint4* dst = reinterpret_cast<uint4*>(q + i * 32);  // 32-byte aligned
  dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
  dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

template <typename T>
__device__ __forceinline__ T cvt_out(float v);
template <>
__device__ __forceinline__ float cvt_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half cvt_out<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// One thread per 4 consecutive quants: out = f32(f16 scale) * int8, exact in f32.
template <typename T>
__global__ void q8_0_dequant_kernel(const int8_t* __restrict__ q, const uint16_t* __restrict__ scale,
                                    int64_t n4, int64_t rows, int64_t cols, T* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  const char4 v = reinterpret_cast<const char4*>(q)[i];
  const int64_t n = (i * 4) / cols, k = (i * 4) % cols;
  const float s = __half2float(__ushort_as_half(scale[(k >> 5) * rows + n]));
  T* o = out + i * 4;
  o[0] = cvt_out<T>(s * (float)v.x);
  o[1] = cvt_out<T>(s * (float)v.y);
  o[2] = cvt_out<T>(s * (float)v.z);
  o[3] = cvt_out<T>(s * (float)v.w);
}

// quantize_fp8, E4M3: one CTA per row (per channel) or a grid-stride pass (per tensor).
constexpr int kQThreads = 256;

__global__ void fp8_rowmax_kernel(const float* __restrict__ w, int64_t K, float* __restrict__ scale) {
  __shared__ float red[kQThreads / 32];
  const int64_t r = blockIdx.x;
  float m = 0.f;
  for (int64_t k = threadIdx.x; k < K; k += kQThreads) m = fmaxf(m, fabsf(w[r * K + k]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < kQThreads / 32; ++i) t = fmaxf(t, red[i]);
    scale[r] = t > 0.f ? t / 448.0f : 1.0f;  // quantization.rs:514-518
  }
}

__global__ void fp8_tensormax_kernel(const float* __restrict__ w, int64_t n, unsigned int* __restrict__ mx_bits) {
  float m = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(w[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(mx_bits, __float_as_uint(m));  // non-negative floats
}

__global__ void fp8_tensorscale_kernel(const unsigned int* __restrict__ mx_bits, float* __restrict__ scale) {
  const float t = __uint_as_float(*mx_bits);
  scale[0] = t > 0.f ? t / 448.0f : 1.0f;  // quantization.rs:550-556
}

__global__ void fp8_encode_kernel(const float* __restrict__ w, int64_t N, int64_t K, int per_channel,
                                  const float* __restrict__ scale, uint8_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N * K) return;
  const float s = scale[per_channel ? i / K : 0];
  out[i] = f32_to_e4m3_ref(__fdiv_rn(w[i], s));  // `row / scale` then quantize_fp8_scalar
}

template <typename T>
__global__ void fp8_dequant_kernel(const uint8_t* __restrict__ w, const float* __restrict__ scale,
                                   int64_t nscale, int64_t N, int64_t K, T* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N * K) return;
  const float s = scale[nscale == 1 ? 0 : i / K];
  out[i] = cvt_out<T>(e4m3_to_f32(w[i]) * s);
}

inline unsigned grid_for(int64_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

}  // namespace
}  // namespace sp

extern "C" {

int sp_q8_0_repack_host(const uint8_t* gguf_host, size_t nbytes, int64_t out_f, int64_t in_f,
                        int8_t* q_host, uint16_t* scale_host) {
  using namespace sp;
  clear_error();
  if (!gguf_host || !q_host || !scale_host) return set_error(SP_ERR_INVALID_ARG, "q8_0 repack: null pointer");
  if (out_f <= 0 || in_f <= 0 || in_f % 32)
    return set_error(SP_ERR_SHAPE, "q8_0 repack: in_features (%lld) must be a positive multiple of 32",
                     (long long)in_f);
  const int64_t nblocks = out_f * (in_f / 32);
  if (nbytes < (size_t)nblocks * 34)
    return set_error(SP_ERR_SHAPE, "q8_0 repack: %zu bytes < %lld blocks x 34", nbytes, (long long)nblocks);
  const int64_t kb = in_f / 32;
  for (int64_t i = 0; i < nblocks; ++i) {
    const uint8_t* blk = gguf_host + i * 34;
    scale_host[(i % kb) * out_f + i / kb] = (uint16_t)(blk[0] | (blk[1] << 8));
    std::memcpy(q_host + i * 32, blk + 2, 32);
  }
  return SP_OK;
}

int sp_q8_0_repack(const void* gguf, size_t nbytes, int64_t out_f, int64_t in_f, void* q, void* scale,
                   void* stream) {
  using namespace sp;
  clear_error();
  if (!gguf || !q || !scale) return set_error(SP_ERR_INVALID_ARG, "q8_0 repack: null pointer");
  if (out_f <= 0 || in_f <= 0 || in_f % 32)
    return set_error(SP_ERR_SHAPE, "q8_0 repack: in_features (%lld) must be a positive multiple of 32",
                     (long long)in_f);
  const int64_t nblocks = out_f * (in_f / 32);
  if (nbytes < (size_t)nblocks * 34)
    return set_error(SP_ERR_SHAPE, "q8_0 repack: %zu bytes < %lld blocks x 34", nbytes, (long long)nblocks);
  if (!aligned(q, 16) || !aligned(scale, 2)) return set_error(SP_ERR_ALIGN, "q8_0 repack: output misaligned");
  if (int rc = require_sm100()) return rc;
  q8_0_repack_kernel<<<grid_for(nblocks, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(gguf), nblocks, in_f / 32, out_f, static_cast<int8_t*>(q),
      static_cast<uint16_t*>(scale));
  return check_launch("q8_0 repack");
}

int sp_q8_0_dequant(const void* q, const void* scale, int64_t out_f, int64_t in_f, void* out, int out_dtype,
                    void* stream) {
  using namespace sp;
  clear_error();
  if (!q || !scale || !out) return set_error(SP_ERR_INVALID_ARG, "q8_0 dequant: null pointer");
  if (out_f <= 0 || in_f <= 0 || in_f % 32)
    return set_error(SP_ERR_SHAPE, "q8_0 dequant: in_features (%lld) must be a positive multiple of 32",
                     (long long)in_f);
  if (!aligned(q, 4)) return set_error(SP_ERR_ALIGN, "q8_0 dequant: q must be 4-byte aligned");
  if (int rc = require_sm100()) return rc;
  const int64_t n4 = out_f * in_f / 4;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int8_t* qq = static_cast<const int8_t*>(q);
  const uint16_t* ss = static_cast<const uint16_t*>(scale);
  switch (out_dtype) {
    case SP_F32: q8_0_dequant_kernel<float><<<grid_for(n4, 256), 256, 0, s>>>(qq, ss, n4, out_f, in_f, static_cast<float*>(out)); break;
    case SP_F16: q8_0_dequant_kernel<__half><<<grid_for(n4, 256), 256, 0, s>>>(qq, ss, n4, out_f, in_f, static_cast<__half*>(out)); break;
    case SP_BF16: q8_0_dequant_kernel<__nv_bfloat16><<<grid_for(n4, 256), 256, 0, s>>>(qq, ss, n4, out_f, in_f, static_cast<__nv_bfloat16*>(out)); break;
    default: return set_error(SP_ERR_DTYPE, "q8_0 dequant: unknown dtype %d", out_dtype);
  }
  return check_launch("q8_0 dequant");
}

int sp_fp8_quantize(const float* w, int64_t N, int64_t K, int scale_mode, void* w_e4m3, float* scale,
                    void* stream) {
  using namespace sp;
  clear_error();
  if (!w || !w_e4m3 || !scale) return set_error(SP_ERR_INVALID_ARG, "fp8 quantize: null pointer");
  if (N <= 0 || K <= 0) return set_error(SP_ERR_INVALID_ARG, "fp8 quantize: bad shape");
  if (N > 2147483647LL) return set_error(SP_ERR_SHAPE, "fp8 quantize: too many rows");
  if (scale_mode < SP_FP8_PER_TENSOR || scale_mode > SP_FP8_GIVEN_SCALE)
    return set_error(SP_ERR_INVALID_ARG, "fp8 quantize: unknown scale mode %d", scale_mode);
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int per_channel = scale_mode == SP_FP8_PER_CHANNEL;
  if (scale_mode == SP_FP8_GIVEN_SCALE) {
    // the caller's scale is used as is
  } else if (per_channel) {
    fp8_rowmax_kernel<<<(unsigned)N, kQThreads, 0, s>>>(w, K, scale);
  } else {
    // the running max is kept as float bits inside `scale` itself before becoming the scale
    unsigned int* mx = reinterpret_cast<unsigned int*>(scale);
    if (cudaMemsetAsync(mx, 0, sizeof(unsigned int), s) != cudaSuccess)
      return set_error(SP_ERR_LAUNCH, "fp8 quantize: memset failed");
    fp8_tensormax_kernel<<<(unsigned)std::min<int64_t>(grid_for(N * K, 256), 4096), 256, 0, s>>>(w, N * K, mx);
    fp8_tensorscale_kernel<<<1, 1, 0, s>>>(mx, scale);
  }
  if (int rc = check_launch("fp8 scale")) return rc;
  fp8_encode_kernel<<<grid_for(N * K, 256), 256, 0, s>>>(w, N, K, per_channel, scale,
                                                         static_cast<uint8_t*>(w_e4m3));
  return check_launch("fp8 encode");
}

int sp_fp8_dequant(const void* w_e4m3, const float* scale, int64_t nscale, int64_t N, int64_t K, void* out,
                   int out_dtype, void* stream) {
  using namespace sp;
  clear_error();
  if (!w_e4m3 || !scale || !out) return set_error(SP_ERR_INVALID_ARG, "fp8 dequant: null pointer");
  if (N <= 0 || K <= 0) return set_error(SP_ERR_INVALID_ARG, "fp8 dequant: bad shape");
  if (nscale != 1 && nscale != N)
    return set_error(SP_ERR_SHAPE, "fp8 dequant: scale count %lld must be 1 or N=%lld", (long long)nscale,
                     (long long)N);
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* wq = static_cast<const uint8_t*>(w_e4m3);
  const unsigned g = grid_for(N * K, 256);
  switch (out_dtype) {
    case SP_F32: fp8_dequant_kernel<float><<<g, 256, 0, s>>>(wq, scale, nscale, N, K, static_cast<float*>(out)); break;
    case SP_F16: fp8_dequant_kernel<__half><<<g, 256, 0, s>>>(wq, scale, nscale, N, K, static_cast<__half*>(out)); break;
    case SP_BF16: fp8_dequant_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(wq, scale, nscale, N, K, static_cast<__nv_bfloat16*>(out)); break;
    default: return set_error(SP_ERR_DTYPE, "fp8 dequant: unknown dtype %d", out_dtype);
  }
  return check_launch("fp8 dequant");
}

}  // extern "C"
