// residual.cu -- out = y + bias[c] (+ r): the convolution bias and the ResBlock's residual
// add of ResBlock::forward (crates/sketchpad-unet/src/blocks.rs:123-150: conv2(h) + skip(x)),
// in one pass over channels-last [rows, C] activations.
//
// Running the convolutions without their bias and adding it here (together with the
// residual, and with the skip convolution's bias folded into the same vector) replaces a
// broadcast bias pass per convolution plus a separate residual pass.
#include "common.cuh"

namespace sp {
namespace {

constexpr int kResThreads = 256;

template <typename T>
__device__ __forceinline__ float rs_f32(T v);
template <>
__device__ __forceinline__ float rs_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float rs_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float rs_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T>
__device__ __forceinline__ T rs_from(float v);
template <>
__device__ __forceinline__ float rs_from<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half rs_from<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 rs_from<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// One thread per 16-byte vector; rows are C contiguous values (C a multiple of the vector).
template <typename T, bool HAS_R>
__global__ void __launch_bounds__(kResThreads) add_bias_residual_kernel(
    const T* __restrict__ y, const T* __restrict__ r, const T* __restrict__ bias,
    T* __restrict__ out, int64_t nvec, int cvec) {
  constexpr int VE = 16 / sizeof(T);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nvec) return;
  const int c = (int)(i % cvec) * VE;
  const uint4 vy = __ldg(reinterpret_cast<const uint4*>(y) + i);
  const uint4 vb = __ldg(reinterpret_cast<const uint4*>(bias + c));
  uint4 vr = make_uint4(0, 0, 0, 0);
  if constexpr (HAS_R) vr = __ldg(reinterpret_cast<const uint4*>(r) + i);
  const T* ey = reinterpret_cast<const T*>(&vy);
  const T* eb = reinterpret_cast<const T*>(&vb);
  const T* er = reinterpret_cast<const T*>(&vr);
  uint4 o;
  T* eo = reinterpret_cast<T*>(&o);
#pragma unroll
  for (int t = 0; t < VE; ++t) {
    float v = rs_f32<T>(ey[t]) + rs_f32<T>(eb[t]);
    if constexpr (HAS_R) v += rs_f32<T>(er[t]);
    eo[t] = rs_from<T>(v);
  }
  reinterpret_cast<uint4*>(out)[i] = o;
}

template <typename T>
int launch_abr(const void* y, const void* r, const void* bias, void* out, int64_t rows, int64_t C,
               cudaStream_t s) {
  constexpr int VE = 16 / sizeof(T);
  const int64_t nvec = rows * C / VE;
  const unsigned grid = (unsigned)((nvec + kResThreads - 1) / kResThreads);
  if (r)
    add_bias_residual_kernel<T, true><<<grid, kResThreads, 0, s>>>(
        static_cast<const T*>(y), static_cast<const T*>(r), static_cast<const T*>(bias),
        static_cast<T*>(out), nvec, (int)(C / VE));
  else
    add_bias_residual_kernel<T, false><<<grid, kResThreads, 0, s>>>(
        static_cast<const T*>(y), nullptr, static_cast<const T*>(bias), static_cast<T*>(out),
        nvec, (int)(C / VE));
  return check_launch("add bias residual");
}

}  // namespace
}  // namespace sp

extern "C" {

int sp_add_bias_residual(const void* y, const void* r, const void* bias, void* out, int64_t rows,
                         int64_t C, int dtype, void* stream) {
  using namespace sp;
  clear_error();
  if (!y || !bias || !out) return set_error(SP_ERR_INVALID_ARG, "add bias residual: null pointer");
  if (rows <= 0 || C <= 0) return set_error(SP_ERR_INVALID_ARG, "add bias residual: bad shape");
  const int es = dtype_size(dtype);
  if (!es) return set_error(SP_ERR_DTYPE, "add bias residual: unknown dtype %d", dtype);
  if (C % (16 / es))
    return set_error(SP_ERR_SHAPE, "add bias residual: C (%lld) must be a multiple of %d",
                     (long long)C, 16 / es);
  if (!aligned(y, 16) || !aligned(bias, 16) || !aligned(out, 16) || (r && !aligned(r, 16)))
    return set_error(SP_ERR_ALIGN, "add bias residual: pointers must be 16-byte aligned");
  if (rows * C / (16 / es) >= (1LL << 31) * 256)
    return set_error(SP_ERR_SHAPE, "add bias residual: tensor too large");
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SP_F32: return launch_abr<float>(y, r, bias, out, rows, C, s);
    case SP_F16: return launch_abr<__half>(y, r, bias, out, rows, C, s);
    default: return launch_abr<__nv_bfloat16>(y, r, bias, out, rows, C, s);
  }
}

}  // extern "C"
