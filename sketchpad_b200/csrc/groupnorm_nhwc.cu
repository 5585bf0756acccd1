// groupnorm_nhwc.cu -- GroupNorm(+SiLU) for channels-last (NHWC) activations.
//
// Same semantics as the NCHW kernels in groupnorm_act.cu (crates/sketchpad-core/src/
// groupnorm.rs:62-102: clamp +-65000, f32 statistics, biased variance, clamp after the
// affine, optional SiLU).  Channels-last is what cuDNN's implicit-GEMM convolutions on
// sm_100 read and write, so a UNet kept channels-last runs no layout conversions.
//
// x is viewed as a row-major [B*H*W, C] matrix; group g owns channels [g*Cg, (g+1)*Cg) of
// every row of its batch image.  Two kernels:
//   stats  grid (chunks, B): each CTA reduces a chunk of rows to per-group (count, mean, M2)
//          (two passes over the chunk, the second from L1/L2).
//   apply  grid (chunks, B): every CTA merges its image's chunk partials (lanes of a warp
//          split the chunks, then a shuffle tree; Chan's pairwise update), then normalises +
//          affine + activation with 16-byte loads and stores.
// HBM sees one read and one write of x at UNet sizes (the second read is an L2 hit).
#include <algorithm>

#include "common.cuh"

namespace sp {

namespace {

constexpr int kNhwcThreads = 256;

__device__ __forceinline__ float nh_to_f32(float v) { return v; }
__device__ __forceinline__ float nh_to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float nh_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T nh_from_f32(float v);
template <>
__device__ __forceinline__ float nh_from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half nh_from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 nh_from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

__device__ __forceinline__ float nh_clamp(float v) { return fminf(fmaxf(v, -65000.0f), 65000.0f); }

__device__ __forceinline__ float nh_act(float v, int act) {
  v = nh_clamp(v);
  if (act == SP_ACT_SILU) {
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(0.5f * v));
    v = v * fmaf(0.5f, t, 0.5f);
  }
  return v;
}

struct NhwcParams {
  const void* x;
  const void* gamma;
  const void* beta;
  void* y;
  int P;               // pixels per image (H*W)
  int C, G, Cg;        // channels, groups, channels per group
  int CV;              // 16-byte channel vectors per row
  int TX, TY;          // block shape: TX channel-vector lanes x TY row lanes
  int rows_per_chunk;  // rows of one batch image per CTA
  int nchunks;         // chunks per batch image
  float* part;         // [B, nchunks, G, 3] (count, mean, M2)
  float eps;
  int act;
};

// Deterministic block reduction of per-thread channel accumulators: every thread stores
// its values into red[ty][c], then each channel is summed over ty in a fixed order.
template <int NV, int VE>
__device__ __forceinline__ void stage_channels(float* red, const float (&acc)[NV][VE], int tx,
                                               int ty, int TX, int CV, int C) {
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int cv = tx + k * TX;
    if (cv < CV)
#pragma unroll
      for (int t = 0; t < VE; ++t) red[ty * C + cv * VE + t] = acc[k][t];
  }
}

// Per-thread channel vectors: cv = tx + k*TX (k < NV).
template <typename T, int NV>
__global__ void __launch_bounds__(kNhwcThreads) gn_nhwc_stats_kernel(NhwcParams p) {
  constexpr int VE = 16 / sizeof(T);
  extern __shared__ float red[];  // [TY][C] staging for the fixed-order reductions
  __shared__ float gval[1024];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int tid = ty * p.TX + tx;
  const int nthr = p.TX * p.TY;
  const int b = blockIdx.y, chunk = blockIdx.x;
  const int r0 = chunk * p.rows_per_chunk;
  const int r1 = min(p.P, r0 + p.rows_per_chunk);
  const T* xb = static_cast<const T*>(p.x) + (int64_t)b * p.P * p.C;

  float acc[NV][VE];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int e = 0; e < VE; ++e) acc[k][e] = 0.f;
  for (int r = r0 + ty; r < r1; r += p.TY) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int cv = tx + k * p.TX;
      if (cv < p.CV) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(xb + (int64_t)r * p.C) + cv);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int t = 0; t < VE; ++t) acc[k][t] += nh_clamp(nh_to_f32(e[t]));
      }
    }
  }
  stage_channels<NV, VE>(red, acc, tx, ty, p.TX, p.CV, p.C);
  __syncthreads();
  const int rows = r1 - r0;
  const float cnt = (float)rows * (float)p.Cg;
  for (int g = tid; g < p.G; g += nthr) {
    float s = 0.f;
    for (int c = g * p.Cg; c < (g + 1) * p.Cg; ++c)
      for (int y = 0; y < p.TY; ++y) s += red[y * p.C + c];
    gval[g] = s / cnt;  // chunk mean of group g
  }
  __syncthreads();
  // second pass: centred sum of squares around the chunk mean (rows are L1/L2 resident)
  float mine[NV][VE];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int cv = tx + k * p.TX;
#pragma unroll
    for (int t = 0; t < VE; ++t) {
      acc[k][t] = 0.f;
      mine[k][t] = cv < p.CV ? gval[(cv * VE + t) / p.Cg] : 0.f;
    }
  }
  for (int r = r0 + ty; r < r1; r += p.TY) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int cv = tx + k * p.TX;
      if (cv < p.CV) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(xb + (int64_t)r * p.C) + cv);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int t = 0; t < VE; ++t) {
          const float d = nh_clamp(nh_to_f32(e[t])) - mine[k][t];
          acc[k][t] += d * d;
        }
      }
    }
  }
  __syncthreads();  // red is rewritten below
  stage_channels<NV, VE>(red, acc, tx, ty, p.TX, p.CV, p.C);
  __syncthreads();
  float* part = p.part + ((int64_t)b * p.nchunks + chunk) * p.G * 3;
  for (int g = tid; g < p.G; g += nthr) {
    float m2 = 0.f;
    for (int c = g * p.Cg; c < (g + 1) * p.Cg; ++c)
      for (int y = 0; y < p.TY; ++y) m2 += red[y * p.C + c];
    part[g * 3 + 0] = cnt;
    part[g * 3 + 1] = gval[g];
    part[g * 3 + 2] = m2;
  }
}

template <typename T, int NV>
__global__ void __launch_bounds__(kNhwcThreads) gn_nhwc_apply_kernel(NhwcParams p) {
  constexpr int VE = 16 / sizeof(T);
  extern __shared__ float pst[];  // this image's chunk partials [nchunks][G][3]
  __shared__ float st[2048];      // (mean, rstd) per group
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int tid = ty * p.TX + tx;
  const int nthr = p.TX * p.TY;
  const int b = blockIdx.y, chunk = blockIdx.x;
  const int r0 = chunk * p.rows_per_chunk;
  const int r1 = min(p.P, r0 + p.rows_per_chunk);
  const T* xb = static_cast<const T*>(p.x) + (int64_t)b * p.P * p.C;
  T* yb = static_cast<T*>(p.y) + (int64_t)b * p.P * p.C;
  const T* gam = static_cast<const T*>(p.gamma);
  const T* bet = static_cast<const T*>(p.beta);
  {
    // coalesced copy of the partials, then per group (fixed order, no divisions in the loop):
    // mean = sum(n_i mean_i) / N;  M2 = sum(M2_i + n_i (mean_i - mean)^2)   (Chan et al.)
    const int nfl = p.nchunks * p.G * 3;
    const float* pb = p.part + (int64_t)b * nfl;
    for (int i = tid; i < nfl; i += nthr) pst[i] = pb[i];
    __syncthreads();
    for (int g = tid; g < p.G; g += nthr) {
      float n = 0.f, s = 0.f;
      for (int i = 0; i < p.nchunks; ++i) {
        const float* q = pst + (i * p.G + g) * 3;
        n += q[0];
        s += q[0] * q[1];
      }
      const float mean = s / n;
      float m2 = 0.f;
      for (int i = 0; i < p.nchunks; ++i) {
        const float* q = pst + (i * p.G + g) * 3;
        const float d = q[1] - mean;
        m2 += q[2] + q[0] * d * d;
      }
      st[2 * g] = mean;
      st[2 * g + 1] = rsqrtf(m2 / n + p.eps);
    }
    __syncthreads();
  }
  // per-channel multiplier / offset: y = (x - mean) * (rstd * gamma) + beta
  float mul[NV][VE], sub[NV][VE], add[NV][VE];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int cv = tx + k * p.TX;
#pragma unroll
    for (int t = 0; t < VE; ++t) {
      const int c = min(cv * VE + t, p.C - 1);
      const int g = c / p.Cg;
      sub[k][t] = st[g * 2];
      mul[k][t] = st[g * 2 + 1] * nh_to_f32(gam[c]);
      add[k][t] = nh_to_f32(bet[c]);
    }
  }
  for (int r = r0 + ty; r < r1; r += p.TY) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int cv = tx + k * p.TX;
      if (cv < p.CV) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(xb + (int64_t)r * p.C) + cv);
        const T* e = reinterpret_cast<const T*>(&u);
        uint4 o;
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int t = 0; t < VE; ++t)
          oe[t] = nh_from_f32<T>(nh_act((nh_clamp(nh_to_f32(e[t])) - sub[k][t]) * mul[k][t] + add[k][t], p.act));
        reinterpret_cast<uint4*>(yb + (int64_t)r * p.C)[cv] = o;
      }
    }
  }
}

struct NhwcPlan {
  int CV, NV, TX, TY, rows_per_chunk, nchunks;
};

NhwcPlan plan_nhwc(int64_t B, int64_t P, int64_t C, int es, int64_t groups) {
  NhwcPlan pl{};
  const int VE = 16 / es;
  pl.CV = (int)(C / VE);
  pl.NV = (pl.CV + kNhwcThreads - 1) / kNhwcThreads;
  if (pl.NV == 3) pl.NV = 4;
  pl.TX = (pl.CV + pl.NV - 1) / pl.NV;
  pl.TY = std::max(1, kNhwcThreads / pl.TX);
  const int64_t target_ctas = 2LL * num_sms();
  int64_t per_image = std::max<int64_t>(1, (target_ctas + B - 1) / B);
  // the apply kernel stages [chunks][groups][3] floats in shared memory: keep it <= 40 KB
  per_image = std::min<int64_t>(per_image, std::max<int64_t>(1, 40960 / (groups * 12)));
  int64_t rows = (P + per_image - 1) / per_image;
  rows = ((rows + pl.TY - 1) / pl.TY) * pl.TY;
  rows = std::max<int64_t>(rows, pl.TY);
  pl.rows_per_chunk = (int)rows;
  pl.nchunks = (int)((P + rows - 1) / rows);
  return pl;
}

}  // namespace

bool gn_nhwc_applicable(int64_t B, int64_t C, int64_t H, int64_t W, const int64_t* st, int es,
                        int64_t groups) {
  if (!st) return false;
  const int64_t want[4] = {H * W * C, 1, W * C, C};
  const int64_t dims[4] = {B, C, H, W};
  for (int i = 0; i < 4; ++i)
    if (dims[i] > 1 && st[i] != want[i]) return false;
  if (C == 1 && H * W > 1) return false;  // ambiguous with NCHW; leave it to the NCHW path
  const int VE = 16 / es;
  // blocks always hold >= 32 threads (TX <= 256 and TY = 256 / TX), which the merge needs
  return C % VE == 0 && C / VE <= 4 * kNhwcThreads && groups <= 1024 && H * W < (1LL << 31);
}

size_t gn_nhwc_workspace_bytes(int64_t B, int64_t C, int64_t H, int64_t W, int es, int64_t groups) {
  const NhwcPlan pl = plan_nhwc(B, H * W, C, es, groups);
  return (size_t)B * pl.nchunks * groups * 3 * sizeof(float);
}

template <typename T>
static int launch_nhwc_t(const NhwcParams& p, int NV, int64_t B, cudaStream_t s) {
  dim3 block(p.TX, p.TY), grid(p.nchunks, (unsigned)B);
  const size_t smem_stats = (size_t)p.TY * p.C * sizeof(float);
  const size_t smem_apply = (size_t)p.nchunks * p.G * 3 * sizeof(float);
  if (NV == 1) {
    gn_nhwc_stats_kernel<T, 1><<<grid, block, smem_stats, s>>>(p);
    if (int rc = check_launch("groupnorm nhwc stats")) return rc;
    gn_nhwc_apply_kernel<T, 1><<<grid, block, smem_apply, s>>>(p);
  } else if (NV == 2) {
    gn_nhwc_stats_kernel<T, 2><<<grid, block, smem_stats, s>>>(p);
    if (int rc = check_launch("groupnorm nhwc stats")) return rc;
    gn_nhwc_apply_kernel<T, 2><<<grid, block, smem_apply, s>>>(p);
  } else {
    gn_nhwc_stats_kernel<T, 4><<<grid, block, smem_stats, s>>>(p);
    if (int rc = check_launch("groupnorm nhwc stats")) return rc;
    gn_nhwc_apply_kernel<T, 4><<<grid, block, smem_apply, s>>>(p);
  }
  return check_launch("groupnorm nhwc apply");
}

int gn_nhwc_launch(const void* x, const void* gamma, const void* beta, void* y, int64_t B,
                   int64_t C, int64_t H, int64_t W, int64_t groups, float eps, int act, int dtype,
                   void* workspace, size_t workspace_bytes, cudaStream_t s) {
  const int es = dtype_size(dtype);
  const size_t need = gn_nhwc_workspace_bytes(B, C, H, W, es, groups);
  if (!workspace || workspace_bytes < need)
    return set_error(SP_ERR_WORKSPACE, "groupnorm (channels-last): needs %zu bytes of workspace (got %zu)",
                     need, workspace_bytes);
  if (!aligned(workspace, 16) || !aligned(x, 16) || !aligned(y, 16))
    return set_error(SP_ERR_ALIGN, "groupnorm (channels-last): x, y and workspace must be 16-byte aligned");
  const NhwcPlan pl = plan_nhwc(B, H * W, C, es, groups);
  NhwcParams p{};
  p.x = x;
  p.gamma = gamma;
  p.beta = beta;
  p.y = y;
  p.P = (int)(H * W);
  p.C = (int)C;
  p.G = (int)groups;
  p.Cg = (int)(C / groups);
  p.CV = pl.CV;
  p.TX = pl.TX;
  p.TY = pl.TY;
  p.rows_per_chunk = pl.rows_per_chunk;
  p.nchunks = pl.nchunks;
  p.part = static_cast<float*>(workspace);
  p.eps = eps;
  p.act = act;
  switch (dtype) {
    case SP_F32: return launch_nhwc_t<float>(p, pl.NV, B, s);
    case SP_F16: return launch_nhwc_t<__half>(p, pl.NV, B, s);
    default: return launch_nhwc_t<__nv_bfloat16>(p, pl.NV, B, s);
  }
}

}  // namespace sp
