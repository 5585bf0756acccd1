// sampler.cu -- the per-step latent update of the denoising loop, fused with classifier-free
// guidance, on the device (one pass over the latent instead of a chain of tensor ops).
//
//   guidance  crates/sketchpad-samplers/src/ddim.rs:158-164 (apply_guidance):
//             eps = uncond + (cond - uncond) * guidance_scale
//   DDIM      ddim.rs:72-133 (DdimSampler::step):
//             pred_x0 = (x - eps * sqrt(1 - a_t)) / sqrt(a_t)
//             prev    = pred_x0 * sqrt(a_prev) + dir_xt * eps  [+ noise * sigma when eta > 0]
//   DPM++ 2M  crates/sketchpad-samplers/src/dpm.rs:101-171 (DpmPlusPlusSampler::step):
//             denoised = x - eps * sigma
//             first order:  x' = x * (sigma_next / sigma) + denoised * (1 - exp(-h))
//             second order: d  = denoised * (1 + c) - prev_denoised * c,  x' = x * r + d * (1 - exp(-h))
// out may be x (an in-place update).  The step's scalars (square roots, ratios, exponentials)
// are host values, computed as the reference computes them; every element operation below
// is one f32 operation in the reference's order (no contraction), so f32 inputs give the
// reference's f32 result.
#include "common.cuh"

namespace sp {
namespace {

template <typename T>
__device__ __forceinline__ float sm_ld(const T* p, int64_t i);
template <>
__device__ __forceinline__ float sm_ld<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float sm_ld<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }
template <>
__device__ __forceinline__ float sm_ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}
template <typename T>
__device__ __forceinline__ T sm_st(float v);
template <>
__device__ __forceinline__ float sm_st<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half sm_st<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 sm_st<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

struct DdimArgs {
  float guidance, sqrt_one_minus_at, sqrt_at, sqrt_at_prev, dir_xt, sigma;
};

template <typename T>
__device__ __forceinline__ float guided_eps(const T* u, const T* c, float g, int64_t i) {
  const float eu = sm_ld<T>(u, i);
  if (!c) return eu;
  return __fadd_rn(eu, __fmul_rn(__fsub_rn(sm_ld<T>(c, i), eu), g));
}

template <typename T>
__global__ void ddim_step_kernel(const T* x, const T* __restrict__ eps_u,
                                 const T* __restrict__ eps_c, const T* __restrict__ noise, T* out,
                                 int64_t n, DdimArgs a) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float eps = guided_eps(eps_u, eps_c, a.guidance, i);
    const float px0 = __fdiv_rn(__fsub_rn(sm_ld<T>(x, i), __fmul_rn(eps, a.sqrt_one_minus_at)), a.sqrt_at);
    float prev = __fadd_rn(__fmul_rn(px0, a.sqrt_at_prev), __fmul_rn(a.dir_xt, eps));
    if (noise) prev = __fadd_rn(prev, __fmul_rn(sm_ld<T>(noise, i), a.sigma));
    out[i] = sm_st<T>(prev);
  }
}

struct DpmArgs {
  float guidance, sigma, ratio, c1, c2, coeff;
  int second_order;
};

template <typename T>
__global__ void dpmpp_2m_step_kernel(const T* x, const T* __restrict__ eps_u,
                                     const T* __restrict__ eps_c, float* prev_denoised, T* out,
                                     int64_t n, DpmArgs a) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float eps = guided_eps(eps_u, eps_c, a.guidance, i);
    const float xv = sm_ld<T>(x, i);
    const float den = __fsub_rn(xv, __fmul_rn(eps, a.sigma));
    float d = den;
    if (a.second_order) d = __fsub_rn(__fmul_rn(den, a.c2), __fmul_rn(prev_denoised[i], a.coeff));
    if (prev_denoised) prev_denoised[i] = den;
    out[i] = sm_st<T>(__fadd_rn(__fmul_rn(xv, a.ratio), __fmul_rn(d, a.c1)));
  }
}

inline unsigned sm_grid(int64_t n) {
  const int64_t blocks = (n + 255) / 256;
  return (unsigned)(blocks < 4096 ? blocks : 4096);
}

template <typename T>
int launch_ddim(const void* x, const void* u, const void* c, const void* noise, void* out, int64_t n,
                const DdimArgs& a, cudaStream_t s) {
  ddim_step_kernel<T><<<sm_grid(n), 256, 0, s>>>(static_cast<const T*>(x), static_cast<const T*>(u),
                                                 static_cast<const T*>(c), static_cast<const T*>(noise),
                                                 static_cast<T*>(out), n, a);
  return check_launch("ddim step");
}

template <typename T>
int launch_dpm(const void* x, const void* u, const void* c, float* prev, void* out, int64_t n,
               const DpmArgs& a, cudaStream_t s) {
  dpmpp_2m_step_kernel<T><<<sm_grid(n), 256, 0, s>>>(static_cast<const T*>(x), static_cast<const T*>(u),
                                                     static_cast<const T*>(c), prev,
                                                     static_cast<T*>(out), n, a);
  return check_launch("dpm++ 2m step");
}

}  // namespace
}  // namespace sp

extern "C" {

int sp_cfg_ddim_step(const void* x, const void* eps_uncond, const void* eps_cond, const void* noise,
                     void* out, int64_t n, float guidance, float sqrt_one_minus_at, float sqrt_at,
                     float sqrt_at_prev, float dir_xt, float sigma, int dtype, void* stream) {
  using namespace sp;
  clear_error();
  if (!x || !eps_uncond || !out) return set_error(SP_ERR_INVALID_ARG, "ddim step: null pointer");
  if (n <= 0) return set_error(SP_ERR_INVALID_ARG, "ddim step: n must be positive");
  if (int rc = require_sm100()) return rc;
  const DdimArgs a{guidance, sqrt_one_minus_at, sqrt_at, sqrt_at_prev, dir_xt, sigma};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SP_F32: return launch_ddim<float>(x, eps_uncond, eps_cond, noise, out, n, a, s);
    case SP_F16: return launch_ddim<__half>(x, eps_uncond, eps_cond, noise, out, n, a, s);
    case SP_BF16: return launch_ddim<__nv_bfloat16>(x, eps_uncond, eps_cond, noise, out, n, a, s);
    default: return set_error(SP_ERR_DTYPE, "ddim step: unknown dtype %d", dtype);
  }
}

int sp_cfg_dpmpp_2m_step(const void* x, const void* eps_uncond, const void* eps_cond,
                         float* prev_denoised, void* out, int64_t n, float guidance, float sigma,
                         float sigma_ratio, float one_minus_exp_neg_h, float one_plus_coeff,
                         float coeff, int second_order, int dtype, void* stream) {
  using namespace sp;
  clear_error();
  if (!x || !eps_uncond || !out) return set_error(SP_ERR_INVALID_ARG, "dpm++ 2m step: null pointer");
  if (second_order && !prev_denoised)
    return set_error(SP_ERR_INVALID_ARG, "dpm++ 2m step: the second-order update needs prev_denoised");
  if (n <= 0) return set_error(SP_ERR_INVALID_ARG, "dpm++ 2m step: n must be positive");
  if (int rc = require_sm100()) return rc;
  const DpmArgs a{guidance, sigma, sigma_ratio, one_minus_exp_neg_h, one_plus_coeff, coeff,
                  second_order ? 1 : 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SP_F32: return launch_dpm<float>(x, eps_uncond, eps_cond, prev_denoised, out, n, a, s);
    case SP_F16: return launch_dpm<__half>(x, eps_uncond, eps_cond, prev_denoised, out, n, a, s);
    case SP_BF16: return launch_dpm<__nv_bfloat16>(x, eps_uncond, eps_cond, prev_denoised, out, n, a, s);
    default: return set_error(SP_ERR_DTYPE, "dpm++ 2m step: unknown dtype %d", dtype);
  }
}

}  // extern "C"
