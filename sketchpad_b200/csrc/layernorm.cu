// layernorm.cu -- row LayerNorm with the reference's UNBIASED variance.
//
// crates/sketchpad-core/src/layernorm.rs:63-73: y = (x - mean) / sqrt(var + eps) * w + b with
// burn `var` = sum((x - mean)^2) / (n - 1).  One warp per row; the row is held in registers
// (16-byte loads) so it is read from HBM once, statistics are two-pass in registers.
#include "common.cuh"

namespace sp {
namespace {

__device__ __forceinline__ float ln_to_f32(float v) { return v; }
__device__ __forceinline__ float ln_to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float ln_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T ln_from_f32(float v);
template <>
__device__ __forceinline__ float ln_from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half ln_from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 ln_from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

__device__ __forceinline__ float ln_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int kLnWarps = 8;

// VPL = 16-byte vectors per lane; row length n = nvec * (16 / sizeof(T)), nvec <= 32 * VPL.
template <typename T, int VPL>
__global__ void __launch_bounds__(kLnWarps * 32) ln_reg_kernel(const T* __restrict__ x,
                                                               const T* __restrict__ xadd,
                                                               const T* __restrict__ w,
                                                               const T* __restrict__ bias,
                                                               T* __restrict__ y, int64_t rows,
                                                               int n, float eps, int unbiased) {
  constexpr int VE = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kLnWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = n / VE;
  const uint4* xv = reinterpret_cast<const uint4*>(x + row * n);
  uint4 buf[VPL];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int vi = lane + 32 * j;
    if (vi < nvec) {
      buf[j] = __ldg(xv + vi);
      if (xadd) {  // x + xadd[column], rounded back to T like a separate add would
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(xadd) + vi);
        T* e = reinterpret_cast<T*>(&buf[j]);
        const T* ea = reinterpret_cast<const T*>(&a);
#pragma unroll
        for (int t = 0; t < VE; ++t) e[t] = ln_from_f32<T>(ln_to_f32(e[t]) + ln_to_f32(ea[t]));
      }
      const T* e = reinterpret_cast<const T*>(&buf[j]);
#pragma unroll
      for (int t = 0; t < VE; ++t) s += ln_to_f32(e[t]);
    }
  }
  const float mean = ln_warp_sum(s) / (float)n;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int vi = lane + 32 * j;
    if (vi < nvec) {
      const T* e = reinterpret_cast<const T*>(&buf[j]);
#pragma unroll
      for (int t = 0; t < VE; ++t) {
        const float d = ln_to_f32(e[t]) - mean;
        ss += d * d;
      }
    }
  }
  const float var = ln_warp_sum(ss) / (float)(unbiased ? n - 1 : n);
  const float rstd = rsqrtf(var + eps);
  uint4* yv = reinterpret_cast<uint4*>(y + row * n);
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int vi = lane + 32 * j;
    if (vi < nvec) {
      const T* e = reinterpret_cast<const T*>(&buf[j]);
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int t = 0; t < VE; ++t) {
        const int c = vi * VE + t;
        oe[t] = ln_from_f32<T>((ln_to_f32(e[t]) - mean) * rstd * ln_to_f32(w[c]) +
                               ln_to_f32(bias[c]));
      }
      yv[vi] = o;
    }
  }
}

// Any n: two reads of the row, one warp per row.
template <typename T>
__global__ void __launch_bounds__(kLnWarps * 32) ln_generic_kernel(const T* __restrict__ x,
                                                                   const T* __restrict__ xadd,
                                                                   const T* __restrict__ w,
                                                                   const T* __restrict__ bias,
                                                                   T* __restrict__ y,
                                                                   int64_t rows, int n, float eps,
                                                                   int unbiased) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kLnWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * n;
  auto xi = [&](int i) {
    return xadd ? ln_to_f32(ln_from_f32<T>(ln_to_f32(xr[i]) + ln_to_f32(xadd[i])))
                : ln_to_f32(xr[i]);
  };
  float s = 0.f;
  for (int i = lane; i < n; i += 32) s += xi(i);
  const float mean = ln_warp_sum(s) / (float)n;
  float ss = 0.f;
  for (int i = lane; i < n; i += 32) {
    const float d = xi(i) - mean;
    ss += d * d;
  }
  const float rstd = rsqrtf(ln_warp_sum(ss) / (float)(unbiased ? n - 1 : n) + eps);
  for (int i = lane; i < n; i += 32)
    y[row * n + i] = ln_from_f32<T>((xi(i) - mean) * rstd * ln_to_f32(w[i]) + ln_to_f32(bias[i]));
}

template <typename T>
int launch_ln(const void* x, const void* xadd, const void* w, const void* b, void* y, int64_t rows,
              int n, float eps, int unbiased, cudaStream_t s) {
  constexpr int VE = 16 / sizeof(T);
  const dim3 grid((unsigned)((rows + kLnWarps - 1) / kLnWarps));
  const T* xt = static_cast<const T*>(x);
  const T* at = static_cast<const T*>(xadd);
  const T* wt = static_cast<const T*>(w);
  const T* bt = static_cast<const T*>(b);
  T* yt = static_cast<T*>(y);
  const bool vec = n % VE == 0 && aligned(x, 16) && aligned(y, 16) && aligned(xadd, 16);
  const int nvec = n / VE;
  if (vec && nvec <= 32 * 2)
    ln_reg_kernel<T, 2><<<grid, kLnWarps * 32, 0, s>>>(xt, at, wt, bt, yt, rows, n, eps, unbiased);
  else if (vec && nvec <= 32 * 4)
    ln_reg_kernel<T, 4><<<grid, kLnWarps * 32, 0, s>>>(xt, at, wt, bt, yt, rows, n, eps, unbiased);
  else if (vec && nvec <= 32 * 8)
    ln_reg_kernel<T, 8><<<grid, kLnWarps * 32, 0, s>>>(xt, at, wt, bt, yt, rows, n, eps, unbiased);
  else
    ln_generic_kernel<T><<<grid, kLnWarps * 32, 0, s>>>(xt, at, wt, bt, yt, rows, n, eps, unbiased);
  return check_launch("layernorm");
}

}  // namespace
}  // namespace sp

namespace sp {
namespace {
int layernorm_entry(const void* x, const void* xadd, const void* gamma, const void* beta, void* y,
                    int64_t rows, int64_t n, float eps, int unbiased, int dtype, void* stream) {
  clear_error();
  if (!x || !gamma || !beta || !y) return set_error(SP_ERR_INVALID_ARG, "layernorm: null pointer");
  if (rows <= 0 || n <= 1 || n > (1LL << 30))
    return set_error(SP_ERR_INVALID_ARG, "layernorm: bad shape rows=%lld n=%lld",
                     (long long)rows, (long long)n);
  if (rows > (int64_t)kLnWarps * 2147483647LL) return set_error(SP_ERR_SHAPE, "layernorm: too many rows");
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SP_F32: return launch_ln<float>(x, xadd, gamma, beta, y, rows, (int)n, eps, unbiased, s);
    case SP_F16: return launch_ln<__half>(x, xadd, gamma, beta, y, rows, (int)n, eps, unbiased, s);
    case SP_BF16:
      return launch_ln<__nv_bfloat16>(x, xadd, gamma, beta, y, rows, (int)n, eps, unbiased, s);
    default: return set_error(SP_ERR_DTYPE, "layernorm: unknown dtype %d", dtype);
  }
}
}  // namespace
}  // namespace sp

extern "C" int sp_layernorm(const void* x, const void* gamma, const void* beta, void* y,
                            int64_t rows, int64_t n, float eps, int unbiased, int dtype,
                            void* stream) {
  return sp::layernorm_entry(x, nullptr, gamma, beta, y, rows, n, eps, unbiased, dtype, stream);
}

extern "C" int sp_layernorm_add(const void* x, const void* x_add, const void* gamma,
                                const void* beta, void* y, int64_t rows, int64_t n, float eps,
                                int unbiased, int dtype, void* stream) {
  if (!x_add) return sp::set_error(SP_ERR_INVALID_ARG, "layernorm_add: x_add is NULL");
  return sp::layernorm_entry(x, x_add, gamma, beta, y, rows, n, eps, unbiased, dtype, stream);
}
