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

// One launch's operands.  gamma/beta are either the affine vectors of LayerNorm::forward
// (w, b: [n]) or, with `modulate`, the DiT blocks' per-group `scale` / `shift` vectors:
// y = LN(x) * (1 + scale[g]) + shift[g], g = row / rows_per_group, vectors mod_stride apart
// (flux.rs:479-481, wan.rs:541-542 after a LayerNorm::new, i.e. gamma 1 and beta 0).  A null
// gamma reads as 1 and a null beta as 0 (so modulate with neither is the plain LN::new).
template <typename T>
struct LnArgs {
  const T* x;
  const T* xadd;  // [n] added to every row before the statistics, or null
  const T* w;
  const T* b;
  T* y;
  int64_t rows;
  int64_t rows_per_group;
  int64_t mod_stride;
  int n;
  float eps;
  int unbiased;
  int modulate;
};

// VPL = 16-byte vectors per lane; row length n = nvec * (16 / sizeof(T)), nvec <= 32 * VPL.
template <typename T, int VPL>
__global__ void __launch_bounds__(kLnWarps * 32) ln_reg_kernel(const LnArgs<T> a) {
  constexpr int VE = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kLnWarps + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const int n = a.n;
  const int nvec = n / VE;
  const uint4* xv = reinterpret_cast<const uint4*>(a.x + row * n);
  // gamma / beta rows are loaded together with x, so their latency overlaps the statistics
  const int64_t goff = a.modulate ? (row / a.rows_per_group) * a.mod_stride : 0;
  const T* wr = a.w ? a.w + goff : nullptr;
  const T* br = a.b ? a.b + goff : nullptr;
  uint4 buf[VPL], wbuf[VPL], bbuf[VPL];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int vi = lane + 32 * j;
    if (vi < nvec) {
      buf[j] = __ldg(xv + vi);
      if (wr) wbuf[j] = __ldg(reinterpret_cast<const uint4*>(wr) + vi);
      if (br) bbuf[j] = __ldg(reinterpret_cast<const uint4*>(br) + vi);
    }
  }
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int vi = lane + 32 * j;
    if (vi < nvec) {
      if (a.xadd) {  // x + xadd[column], rounded back to T like a separate add would
        const uint4 av = __ldg(reinterpret_cast<const uint4*>(a.xadd) + vi);
        T* e = reinterpret_cast<T*>(&buf[j]);
        const T* ea = reinterpret_cast<const T*>(&av);
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
  const float var = ln_warp_sum(ss) / (float)(a.unbiased ? n - 1 : n);
  const float rstd = rsqrtf(var + a.eps);
  uint4* yv = reinterpret_cast<uint4*>(a.y + row * n);
  const float gbase = a.modulate ? 1.f : 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const int vi = lane + 32 * j;
    if (vi < nvec) {
      float g[VE], bb[VE];
      const T* we = reinterpret_cast<const T*>(&wbuf[j]);
      const T* be = reinterpret_cast<const T*>(&bbuf[j]);
#pragma unroll
      for (int t = 0; t < VE; ++t) {
        g[t] = wr ? gbase + ln_to_f32(we[t]) : 1.f;
        bb[t] = br ? ln_to_f32(be[t]) : 0.f;
      }
      const T* e = reinterpret_cast<const T*>(&buf[j]);
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int t = 0; t < VE; ++t) oe[t] = ln_from_f32<T>((ln_to_f32(e[t]) - mean) * rstd * g[t] + bb[t]);
      yv[vi] = o;
    }
  }
}

// Any n (and unaligned rows): two reads of the row, one warp per row.
template <typename T>
__global__ void __launch_bounds__(kLnWarps * 32) ln_generic_kernel(const LnArgs<T> a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kLnWarps + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const int n = a.n;
  const T* xr = a.x + row * n;
  auto xi = [&](int i) {
    return a.xadd ? ln_to_f32(ln_from_f32<T>(ln_to_f32(xr[i]) + ln_to_f32(a.xadd[i])))
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
  const float rstd = rsqrtf(ln_warp_sum(ss) / (float)(a.unbiased ? n - 1 : n) + a.eps);
  const int64_t goff = a.modulate ? (row / a.rows_per_group) * a.mod_stride : 0;
  const float base = a.modulate ? 1.f : 0.f;
  for (int i = lane; i < n; i += 32) {
    const float g = a.w ? base + ln_to_f32(a.w[goff + i]) : 1.f;
    const float bb = a.b ? ln_to_f32(a.b[goff + i]) : 0.f;
    a.y[row * n + i] = ln_from_f32<T>((xi(i) - mean) * rstd * g + bb);
  }
}

template <typename T>
int launch_ln(const LnArgs<T>& a, cudaStream_t s) {
  constexpr int VE = 16 / sizeof(T);
  const dim3 grid((unsigned)((a.rows + kLnWarps - 1) / kLnWarps));
  const dim3 block(kLnWarps * 32);
  const bool vec = a.n % VE == 0 && aligned(a.x, 16) && aligned(a.y, 16) &&
                   aligned(a.xadd, 16) && aligned(a.w, 16) && aligned(a.b, 16) &&
                   (a.mod_stride * (int64_t)sizeof(T)) % 16 == 0;
  const int nvec = a.n / VE;
  // the row stays in registers up to 32 x 20 vectors (5120 bf16: Flux 3072, Wan 5120)
  if (vec && nvec <= 32 * 2) ln_reg_kernel<T, 2><<<grid, block, 0, s>>>(a);
  else if (vec && nvec <= 32 * 4) ln_reg_kernel<T, 4><<<grid, block, 0, s>>>(a);
  else if (vec && nvec <= 32 * 8) ln_reg_kernel<T, 8><<<grid, block, 0, s>>>(a);
  else if (vec && nvec <= 32 * 12) ln_reg_kernel<T, 12><<<grid, block, 0, s>>>(a);
  else if (vec && nvec <= 32 * 16) ln_reg_kernel<T, 16><<<grid, block, 0, s>>>(a);
  else if (vec && nvec <= 32 * 20) ln_reg_kernel<T, 20><<<grid, block, 0, s>>>(a);
  else ln_generic_kernel<T><<<grid, block, 0, s>>>(a);
  return check_launch("layernorm");
}

}  // namespace
}  // namespace sp

namespace sp {
namespace {
template <typename T>
LnArgs<T> ln_args(const void* x, const void* xadd, const void* w, const void* b, void* y,
                  int64_t rows, int64_t n, int64_t rows_per_group, int64_t mod_stride, float eps,
                  int unbiased, int modulate) {
  return LnArgs<T>{static_cast<const T*>(x), static_cast<const T*>(xadd),
                   static_cast<const T*>(w), static_cast<const T*>(b), static_cast<T*>(y), rows,
                   rows_per_group, mod_stride, (int)n, eps, unbiased, modulate};
}

int layernorm_entry(const void* x, const void* xadd, const void* gamma, const void* beta, void* y,
                    int64_t rows, int64_t n, int64_t rows_per_group, int64_t mod_stride,
                    float eps, int unbiased, int modulate, int dtype, void* stream) {
  if (!x || !y) return set_error(SP_ERR_INVALID_ARG, "layernorm: null pointer");
  if (rows <= 0 || n <= 1 || n > (1LL << 30))
    return set_error(SP_ERR_INVALID_ARG, "layernorm: bad shape rows=%lld n=%lld",
                     (long long)rows, (long long)n);
  if (rows > (int64_t)kLnWarps * 2147483647LL) return set_error(SP_ERR_SHAPE, "layernorm: too many rows");
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define SP_LN_ARGS(T) \
  ln_args<T>(x, xadd, gamma, beta, y, rows, n, rows_per_group, mod_stride, eps, unbiased, modulate)
  switch (dtype) {
    case SP_F32: return launch_ln<float>(SP_LN_ARGS(float), s);
    case SP_F16: return launch_ln<__half>(SP_LN_ARGS(__half), s);
    case SP_BF16: return launch_ln<__nv_bfloat16>(SP_LN_ARGS(__nv_bfloat16), s);
    default: return set_error(SP_ERR_DTYPE, "layernorm: unknown dtype %d", dtype);
  }
#undef SP_LN_ARGS
}
}  // namespace
}  // namespace sp

extern "C" int sp_layernorm(const void* x, const void* gamma, const void* beta, void* y,
                            int64_t rows, int64_t n, float eps, int unbiased, int dtype,
                            void* stream) {
  sp::clear_error();
  if (!gamma || !beta) return sp::set_error(SP_ERR_INVALID_ARG, "layernorm: null pointer");
  return sp::layernorm_entry(x, nullptr, gamma, beta, y, rows, n, 1, 0, eps, unbiased, 0, dtype,
                             stream);
}

extern "C" int sp_layernorm_add(const void* x, const void* x_add, const void* gamma,
                                const void* beta, void* y, int64_t rows, int64_t n, float eps,
                                int unbiased, int dtype, void* stream) {
  sp::clear_error();
  if (!x_add) return sp::set_error(SP_ERR_INVALID_ARG, "layernorm_add: x_add is NULL");
  if (!gamma || !beta) return sp::set_error(SP_ERR_INVALID_ARG, "layernorm: null pointer");
  return sp::layernorm_entry(x, x_add, gamma, beta, y, rows, n, 1, 0, eps, unbiased, 0, dtype,
                             stream);
}

extern "C" int sp_layernorm_modulate(const void* x, const void* scale, const void* shift,
                                     void* y, int64_t rows, int64_t n, int64_t rows_per_group,
                                     int64_t mod_stride, float eps, int unbiased, int dtype,
                                     void* stream) {
  sp::clear_error();
  if (rows_per_group <= 0 || mod_stride < 0)
    return sp::set_error(SP_ERR_INVALID_ARG, "layernorm_modulate: bad rows_per_group / stride");
  return sp::layernorm_entry(x, nullptr, scale, shift, y, rows, n, rows_per_group, mod_stride,
                             eps, unbiased, 1, dtype, stream);
}
