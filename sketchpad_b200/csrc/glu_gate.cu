// glu_gate.cu -- gated-linear-unit gates of the feed-forwards, one pass over the [M, 2F] hidden:
//   GEGLU  y = x[:, :F] * gelu(x[:, F:])   (UNet FeedForward::forward,
//          crates/sketchpad-unet/src/blocks.rs:446-458; erf GELU 0.5*g*(1 + erf(g/sqrt(2))))
//   SwiGLU y = silu(x[:, :F]) * x[:, F:]   (SwiGluFfn::forward, crates/sketchpad-core/src/
//          glu.rs:91-96, used by the Flux blocks; WanExpert::forward,
//          crates/sketchpad-dit/src/wan.rs:330-337; gate and up stacked in one GEMM)
// As two element-wise passes the hidden tensor is read 1.5 times and 1.5 times the output
// written; here it is read once and y written once.
#include "common.cuh"

namespace sp {
namespace {

constexpr int kGegluThreads = 256;

__device__ __forceinline__ float gelu_erf(float g) {
  return 0.5f * g * (1.0f + erff(g * 0.70710678118654752f));
}

// x * sigmoid(x) with an IEEE division, as the reference's silu
__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

template <typename T>
__device__ __forceinline__ float ld_f32(const T* p);
template <>
__device__ __forceinline__ float ld_f32<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_f32<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ld_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

template <typename T>
__device__ __forceinline__ T to_t(float v);
template <>
__device__ __forceinline__ float to_t<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half to_t<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 to_t<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// One thread per 16-byte vector of the output row: VE values and their VE gates.
template <typename T, int KIND>
__global__ void __launch_bounds__(kGegluThreads) glu_kernel(const T* __restrict__ x,
                                                            T* __restrict__ y, int64_t rows,
                                                            int64_t F, int64_t xs, int64_t ys) {
  constexpr int VE = 16 / sizeof(T);
  const int64_t fv = F / VE;  // vectors per output row
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * fv) return;
  const int64_t r = i / fv, c = (i - r * fv) * VE;
  const T* xr = x + r * xs;
  const uint4 va = __ldg(reinterpret_cast<const uint4*>(xr + c));
  const uint4 vg = __ldg(reinterpret_cast<const uint4*>(xr + F + c));
  const T* a = reinterpret_cast<const T*>(&va);
  const T* g = reinterpret_cast<const T*>(&vg);
  uint4 o;
  T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
  for (int t = 0; t < VE; ++t) {
    const float lo = ld_f32<T>(a + t), hi = ld_f32<T>(g + t);
    oe[t] = to_t<T>(KIND == SP_GLU_GEGLU ? lo * gelu_erf(hi) : silu_f(lo) * hi);
  }
  *reinterpret_cast<uint4*>(y + r * ys + c) = o;
}

}  // namespace
}  // namespace sp

extern "C" {

int sp_glu_gate(const void* x, void* y, int64_t rows, int64_t F, int64_t x_row_stride,
                int64_t y_row_stride, int kind, int dtype, void* stream) {
  using namespace sp;
  clear_error();
  if (!x || !y) return set_error(SP_ERR_INVALID_ARG, "glu gate: null pointer");
  if (rows <= 0 || F <= 0) return set_error(SP_ERR_INVALID_ARG, "glu gate: non-positive shape");
  if (kind != SP_GLU_GEGLU && kind != SP_GLU_SWIGLU)
    return set_error(SP_ERR_INVALID_ARG, "glu gate: unknown kind %d", kind);
  const int es = dtype_size(dtype);
  if (!es) return set_error(SP_ERR_DTYPE, "glu gate: unknown dtype %d", dtype);
  const int VE = 16 / es;
  if (F % VE || x_row_stride % VE || y_row_stride % VE || x_row_stride < 2 * F ||
      y_row_stride < F)
    return set_error(SP_ERR_SHAPE,
                     "glu gate: F and the row strides must be multiples of %d elements (x "
                     "stride >= 2F, y stride >= F)",
                     VE);
  if (!aligned(x, 16) || !aligned(y, 16))
    return set_error(SP_ERR_ALIGN, "glu gate: x and y must be 16-byte aligned");
  if (int rc = require_sm100()) return rc;
  const int64_t n = rows * (F / VE);
  const unsigned grid = (unsigned)((n + kGegluThreads - 1) / kGegluThreads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define SP_GLU_LAUNCH(T)                                                                   \
  (kind == SP_GLU_GEGLU                                                                    \
       ? glu_kernel<T, SP_GLU_GEGLU><<<grid, kGegluThreads, 0, s>>>(                       \
             static_cast<const T*>(x), static_cast<T*>(y), rows, F, x_row_stride, y_row_stride) \
       : glu_kernel<T, SP_GLU_SWIGLU><<<grid, kGegluThreads, 0, s>>>(                      \
             static_cast<const T*>(x), static_cast<T*>(y), rows, F, x_row_stride, y_row_stride))
  switch (dtype) {
    case SP_F32: SP_GLU_LAUNCH(float); break;
    case SP_F16: SP_GLU_LAUNCH(__half); break;
    default: SP_GLU_LAUNCH(__nv_bfloat16); break;
  }
#undef SP_GLU_LAUNCH
  return check_launch("glu gate");
}

}  // extern "C"
