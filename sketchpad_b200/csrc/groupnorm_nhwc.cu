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

#include <cooperative_groups.h>

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
  const void* x_add;   // optional [B, C] per-(image, channel) addend, applied before the norm
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
  const T* addb = p.x_add ? static_cast<const T*>(p.x_add) + (int64_t)b * p.C : nullptr;
  float addv[NV][VE];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int cv = tx + k * p.TX;
#pragma unroll
    for (int t = 0; t < VE; ++t) addv[k][t] = (addb && cv < p.CV) ? nh_to_f32(addb[cv * VE + t]) : 0.f;
  }

  float acc[NV][VE];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int e = 0; e < VE; ++e) acc[k][e] = 0.f;
#pragma unroll 4
  for (int r = r0 + ty; r < r1; r += p.TY) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int cv = tx + k * p.TX;
      if (cv < p.CV) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(xb + (int64_t)r * p.C) + cv);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int t = 0; t < VE; ++t) acc[k][t] += nh_clamp(nh_to_f32(e[t]) + addv[k][t]);
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
          const float d = nh_clamp(nh_to_f32(e[t]) + addv[k][t]) - mine[k][t];
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
    // eight loads in flight per thread (the copy is latency-bound, not bandwidth-bound)
    for (int i0 = tid; i0 < nfl; i0 += 8 * nthr) {
      float tmp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * nthr;
        tmp[u] = i < nfl ? __ldcg(pb + i) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * nthr;
        if (i < nfl) pst[i] = tmp[u];
      }
    }
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
  const T* addb = p.x_add ? static_cast<const T*>(p.x_add) + (int64_t)b * p.C : nullptr;
  float mul[NV][VE], sub[NV][VE], add[NV][VE], pre[NV][VE];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int cv = tx + k * p.TX;
#pragma unroll
    for (int t = 0; t < VE; ++t) {
      const int c = min(cv * VE + t, p.C - 1);
      const int g = c / p.Cg;
      pre[k][t] = addb ? nh_to_f32(addb[c]) : 0.f;
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
          oe[t] = nh_from_f32<T>(nh_act((nh_clamp(nh_to_f32(e[t]) + pre[k][t]) - sub[k][t]) * mul[k][t] + add[k][t], p.act));
        reinterpret_cast<uint4*>(yb + (int64_t)r * p.C)[cv] = o;
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// Single-launch variant (cooperative launch, every CTA resident): each thread loads its R rows
// x NV channel vectors into registers at once; the CTA reduces them to per-group (count,
// mean, M2) -- channel sums over the row lanes, then one warp per group -- with the centred
// pass reading the registers, and writes the chunk partial; a grid-wide barrier; then one
// warp per group merges the image's chunk partials (lanes take chunks i = lane mod 32 in
// order, then a fixed shuffle tree: Chan's pairwise update, identical in every CTA), and every
// thread normalises its registers.  HBM sees one read and one write of x in one launch.
// With x_add, x + x_add[b, c] is normalised (the ResBlock's time-embedding add folded in).
template <typename T>
__device__ __forceinline__ void nh_unpack(const uint4& u, float* f) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int t = 0; t < 16 / (int)sizeof(T); ++t) f[t] = nh_to_f32(e[t]);
}

// Sum of the staged per-thread channel values over the row lanes, then per group (one warp
// per group, lanes over the group's channels).  out[g] = group sum.  Fixed order.
__device__ __forceinline__ void nh_group_sums(const float* stage, float* chan, float* out,
                                              const NhwcParams& p, int tid, int nthr) {
  for (int c = tid; c < p.C; c += nthr) {
    float s = 0.f;
    for (int y = 0; y < p.TY; ++y) s += stage[y * p.C + c];
    chan[c] = s;
  }
  __syncthreads();
  // full warps only (a block of TX x TY threads may end in a partial warp; it idles here)
  const int lane = tid & 31, warp = tid >> 5, nwarps = nthr >> 5;
  for (int g = warp < nwarps ? warp : p.G; g < p.G; g += nwarps) {
    float s = 0.f;
    for (int c = lane; c < p.Cg; c += 32) s += chan[g * p.Cg + c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[g] = s;
  }
  __syncthreads();
}

template <typename T, int NV, int R>
__global__ void __launch_bounds__(kNhwcThreads, 2) gn_nhwc_fused_kernel(NhwcParams p) {
  constexpr int VE = 16 / sizeof(T);
  extern __shared__ float sbuf[];  // [TY][C] staging | [C] channel sums | [G] | [G] | [2G]
  float* chan = sbuf + p.TY * p.C;
  float* gsum = chan + p.C;
  float* gm2 = gsum + p.G;
  float* st = gm2 + p.G;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int tid = ty * p.TX + tx;
  const int nthr = p.TX * p.TY;
  const int b = blockIdx.y, chunk = blockIdx.x;
  const int r0 = chunk * p.rows_per_chunk;
  const int r1 = min(p.P, r0 + p.rows_per_chunk);
  const T* xb = static_cast<const T*>(p.x) + (int64_t)b * p.P * p.C;
  T* yb = static_cast<T*>(p.y) + (int64_t)b * p.P * p.C;
  const T* addb = p.x_add ? static_cast<const T*>(p.x_add) + (int64_t)b * p.C : nullptr;

  // ---- load: every row of this thread at once (all loads in flight)
  uint4 v[R][NV];
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const int r = r0 + ty + k * p.TY;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int cv = tx + j * p.TX;
      v[k][j] = (r < r1 && cv < p.CV)
                    ? __ldg(reinterpret_cast<const uint4*>(xb + (int64_t)r * p.C) + cv)
                    : make_uint4(0, 0, 0, 0);
    }
  }
  float addv[NV][VE];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int cv = tx + j * p.TX;
#pragma unroll
    for (int t = 0; t < VE; ++t)
      addv[j][t] = (addb && cv < p.CV) ? nh_to_f32(addb[cv * VE + t]) : 0.f;
  }
  // ---- chunk statistics per group: mean, then M2 about it (from the registers)
  float acc[NV][VE];
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int t = 0; t < VE; ++t) acc[j][t] = 0.f;
#pragma unroll
  for (int k = 0; k < R; ++k) {
    if (r0 + ty + k * p.TY < r1) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        float f[VE];
        nh_unpack<T>(v[k][j], f);
#pragma unroll
        for (int t = 0; t < VE; ++t) acc[j][t] += nh_clamp(f[t] + addv[j][t]);
      }
    }
  }
  stage_channels<NV, VE>(sbuf, acc, tx, ty, p.TX, p.CV, p.C);
  __syncthreads();
  nh_group_sums(sbuf, chan, gsum, p, tid, nthr);
  const float cnt = (float)(r1 - r0) * (float)p.Cg;
  float gmean[NV][VE];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int cv = tx + j * p.TX;
#pragma unroll
    for (int t = 0; t < VE; ++t) {
      acc[j][t] = 0.f;
      gmean[j][t] = cv < p.CV ? gsum[(cv * VE + t) / p.Cg] / cnt : 0.f;
    }
  }
#pragma unroll
  for (int k = 0; k < R; ++k) {
    if (r0 + ty + k * p.TY < r1) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        float f[VE];
        nh_unpack<T>(v[k][j], f);
#pragma unroll
        for (int t = 0; t < VE; ++t) {
          const float d = nh_clamp(f[t] + addv[j][t]) - gmean[j][t];
          acc[j][t] = fmaf(d, d, acc[j][t]);
        }
      }
    }
  }
  stage_channels<NV, VE>(sbuf, acc, tx, ty, p.TX, p.CV, p.C);
  __syncthreads();
  nh_group_sums(sbuf, chan, gm2, p, tid, nthr);
  float4* part = reinterpret_cast<float4*>(p.part) + ((int64_t)b * p.nchunks + chunk) * p.G;
  for (int g = tid; g < p.G; g += nthr) part[g] = make_float4(cnt, gsum[g] / cnt, gm2[g], 0.f);

  // ---- every chunk of every image has published its partial
  __threadfence();
  cooperative_groups::this_grid().sync();

  // ---- merge this image's partials: one warp per group (fixed order in every CTA)
  {
    const int lane = tid & 31, warp = tid >> 5, nwarps = nthr >> 5;  // full warps only
    const float4* pb = reinterpret_cast<const float4*>(p.part) + (int64_t)b * p.nchunks * p.G;
    for (int g = warp < nwarps ? warp : p.G; g < p.G; g += nwarps) {
      float n = 0.f, mean = 0.f, m2 = 0.f;
      for (int i = lane; i < p.nchunks; i += 32) {
        const float4 q = __ldcg(pb + (int64_t)i * p.G + g);
        const float nn = n + q.x, d = q.y - mean, f = q.x / nn;
        mean = fmaf(d, f, mean);
        m2 = m2 + q.z + d * d * n * f;
        n = nn;
      }
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float n2 = __shfl_xor_sync(0xffffffffu, n, o);
        const float mean2 = __shfl_xor_sync(0xffffffffu, mean, o);
        const float m22 = __shfl_xor_sync(0xffffffffu, m2, o);
        // merge in lane order so both partners compute the same value
        const bool lo = (lane & o) == 0;
        const float na = lo ? n : n2, ma = lo ? mean : mean2, qa = lo ? m2 : m22;
        const float nb = lo ? n2 : n, mb = lo ? mean2 : mean, qb = lo ? m22 : m2;
        const float nn = na + nb;
        if (nn > 0.f) {
          const float d = mb - ma, f = nb / nn;
          mean = fmaf(d, f, ma);
          m2 = qa + qb + d * d * na * f;
        } else {
          mean = 0.f;
          m2 = 0.f;
        }
        n = nn;
      }
      if (lane == 0) {
        st[2 * g] = mean;
        st[2 * g + 1] = rsqrtf(m2 / n + p.eps);
      }
    }
    __syncthreads();
  }
  const T* gam = static_cast<const T*>(p.gamma);
  const T* bet = static_cast<const T*>(p.beta);
  float mul[NV][VE], sub[NV][VE], add[NV][VE];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int cv = tx + j * p.TX;
#pragma unroll
    for (int t = 0; t < VE; ++t) {
      const int c = min(cv * VE + t, p.C - 1);
      const int g = c / p.Cg;
      sub[j][t] = st[g * 2];
      mul[j][t] = st[g * 2 + 1] * nh_to_f32(gam[c]);
      add[j][t] = nh_to_f32(bet[c]);
    }
  }
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const int r = r0 + ty + k * p.TY;
    if (r < r1) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int cv = tx + j * p.TX;
        if (cv < p.CV) {
          float f[VE];
          nh_unpack<T>(v[k][j], f);
          uint4 o;
          T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
          for (int t = 0; t < VE; ++t)
            oe[t] = nh_from_f32<T>(nh_act(
                (nh_clamp(f[t] + addv[j][t]) - sub[j][t]) * mul[j][t] + add[j][t], p.act));
          reinterpret_cast<uint4*>(yb + (int64_t)r * p.C)[cv] = o;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// Cluster variant (the UNet's shapes): a thread-block cluster of CS CTAs owns one image x a
// slice of gpc consecutive groups (a 16-byte-aligned channel range of every row); CTA rank r
// owns rows [r*RP, (r+1)*RP).  Each thread loads its R rows of one channel vector into
// registers at once; the CTA forms per-group (count, mean, M2) about its own mean (both passes
// from the registers; one warp per group over the staged [TY][SC] values); the cluster
// exchanges them through distributed shared memory and every CTA merges the CS partials in
// rank order (Chan), so all agree; then each thread normalises its registers and stores.
// One read and one write of x, one launch, no workspace and no grid-wide barrier.
struct NhwcClusterParams {
  const void* x;
  const void* x_add;
  const void* gamma;
  const void* beta;
  void* y;
  int P, C, G, Cg;
  int gpc, SC, SV;  // groups per cluster, channels and 16-byte vectors per row slice
  int TY, RP;       // row lanes per CTA, rows per CTA
  int R;            // rows per thread (staged in shared memory)
  float eps;
  int act;
};

constexpr int kClMaxGpc = 16;
constexpr int kClMaxCluster = 8;  // CTAs per cluster (8: portable; 16 measured slower)
constexpr int kClMaxRows = 32;     // rows per thread staged in shared memory

// Per-group sums of the staged [TY][SC] values (fixed order): Q threads per channel sum
// strided row subsets into col[Q][SC], one thread per channel adds its Q partials, then one
// thread per group adds its Cg channels.  Every level is a short serial chain.
__device__ __forceinline__ void cl_group_sums(const float* red, float* col, float* out,
                                              const NhwcClusterParams& p, int tid, int nthr) {
  const int Q = max(1, min(8, nthr / p.SC));
  if (tid < Q * p.SC) {
    const int c = tid % p.SC, q = tid / p.SC;
    float s = 0.f;
    for (int y = q; y < p.TY; y += Q) s += red[y * p.SC + c];
    col[q * p.SC + c] = s;
  }
  __syncthreads();
  if (tid < p.SC) {
    float s = col[tid];
    for (int q = 1; q < Q; ++q) s += col[q * p.SC + tid];
    col[8 * p.SC + tid] = s;
  }
  __syncthreads();
  if (tid < p.gpc) {
    float s = 0.f;
    for (int c = 0; c < p.Cg; ++c) s += col[8 * p.SC + tid * p.Cg + c];
    out[tid] = s;
  }
  __syncthreads();
}

// Register variant for few rows per thread (R <= 8): each thread loads its R rows of one
// channel vector into registers at once and every pass reads the registers.
template <typename T, int R>
__global__ void __launch_bounds__(kNhwcThreads) gn_nhwc_cluster_reg_kernel(NhwcClusterParams p) {
  constexpr int VE = 16 / sizeof(T);
  extern __shared__ float red_reg[];  // [TY][SC] staging, then col [9][SC]
  float* red = red_reg;
  float* col = red + p.TY * p.SC;
  __shared__ float gsum[kClMaxGpc];
  __shared__ float part[kClMaxGpc][3];       // this CTA's (n, mean, M2) per group
  __shared__ float gst[kClMaxGpc][2];        // merged (mean, rstd) per group
  cooperative_groups::cluster_group cluster = cooperative_groups::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int cs = (int)cluster.num_blocks();
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int TX = p.SV;
  const int tid = ty * TX + tx;
  const int b = blockIdx.z, slice = blockIdx.y;
  const int c0 = slice * p.SC;  // first channel of the slice
  const int r0 = rank * p.RP;
  const int r1 = min(p.P, r0 + p.RP);
  const T* xb = static_cast<const T*>(p.x) + (int64_t)b * p.P * p.C + c0;
  T* yb = static_cast<T*>(p.y) + (int64_t)b * p.P * p.C + c0;

  uint4 v[R];
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const int r = r0 + ty + k * p.TY;
    v[k] = r < r1 ? __ldg(reinterpret_cast<const uint4*>(xb + (int64_t)r * p.C) + tx)
                  : make_uint4(0, 0, 0, 0);
  }
  float addv[VE], gmv[VE], btv[VE];  // issued now, used after the exchange
  {
    const T* gam = static_cast<const T*>(p.gamma) + c0 + tx * VE;
    const T* bet = static_cast<const T*>(p.beta) + c0 + tx * VE;
#pragma unroll
    for (int t = 0; t < VE; ++t) {
      addv[t] = p.x_add ? nh_to_f32(static_cast<const T*>(p.x_add)[(int64_t)b * p.C + c0 + tx * VE + t])
                        : 0.f;
      gmv[t] = nh_to_f32(gam[t]);
      btv[t] = nh_to_f32(bet[t]);
    }
  }
  const int rows = max(0, r1 - r0);
  const float cnt = (float)rows * (float)p.Cg;

  // pass 1: per-channel sums of this thread's rows -> per-group sums (warp g, fixed order)
  float acc[VE];
#pragma unroll
  for (int t = 0; t < VE; ++t) acc[t] = 0.f;
#pragma unroll
  for (int k = 0; k < R; ++k) {
    if (r0 + ty + k * p.TY < r1) {
      float f[VE];
      nh_unpack<T>(v[k], f);
#pragma unroll
      for (int t = 0; t < VE; ++t) acc[t] += nh_clamp(f[t] + addv[t]);
    }
  }
#pragma unroll
  for (int t = 0; t < VE; ++t) red[ty * p.SC + tx * VE + t] = acc[t];
  __syncthreads();
  const int nthr = TX * p.TY;
  cl_group_sums(red, col, gsum, p, tid, nthr);
  if (tid < p.gpc) part[tid][1] = cnt > 0.f ? gsum[tid] / cnt : 0.f;
  __syncthreads();
  // pass 2: M2 about this CTA's group means, from the registers
  float gmean[VE];
#pragma unroll
  for (int t = 0; t < VE; ++t) {
    gmean[t] = part[(tx * VE + t) / p.Cg][1];
    acc[t] = 0.f;
  }
#pragma unroll
  for (int k = 0; k < R; ++k) {
    if (r0 + ty + k * p.TY < r1) {
      float f[VE];
      nh_unpack<T>(v[k], f);
#pragma unroll
      for (int t = 0; t < VE; ++t) {
        const float d = nh_clamp(f[t] + addv[t]) - gmean[t];
        acc[t] = fmaf(d, d, acc[t]);
      }
    }
  }
  __syncthreads();  // red is rewritten
#pragma unroll
  for (int t = 0; t < VE; ++t) red[ty * p.SC + tx * VE + t] = acc[t];
  __syncthreads();
  cl_group_sums(red, col, gsum, p, tid, nthr);
  if (tid < p.gpc) {
    part[tid][0] = cnt;
    part[tid][2] = gsum[tid];
  }
  // exchange: every CTA reads every peer's partials (rank order) after the cluster barrier
  cluster.sync();
  if (tid < p.gpc) {
    // every peer's partial first (independent loads in flight), then the rank-order merge
    float pn[kClMaxCluster], pm[kClMaxCluster], pq2[kClMaxCluster];
#pragma unroll
    for (int q = 0; q < kClMaxCluster; ++q) {
      if (q < cs) {
        const float* pq = cluster.map_shared_rank(&part[tid][0], q);
        pn[q] = pq[0];
        pm[q] = pq[1];
        pq2[q] = pq[2];
      }
    }
    float n = 0.f, mean = 0.f, m2 = 0.f;
#pragma unroll
    for (int q = 0; q < kClMaxCluster; ++q) {
      if (q < cs) {
        const float nn = n + pn[q];
        if (nn > 0.f) {
          const float d = pm[q] - mean, f = pn[q] / nn;
          mean = fmaf(d, f, mean);
          m2 = m2 + pq2[q] + d * d * n * f;
        }
        n = nn;
      }
    }
    gst[tid][0] = mean;
    gst[tid][1] = rsqrtf(m2 / n + p.eps);
  }
  // peers may still read this CTA's `part`: arrive now, wait before leaving
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  __syncthreads();
  float mul[VE], sub[VE];
#pragma unroll
  for (int t = 0; t < VE; ++t) {
    const int g = (tx * VE + t) / p.Cg;
    sub[t] = gst[g][0];
    mul[t] = gst[g][1] * gmv[t];
  }
#pragma unroll
  for (int k = 0; k < R; ++k) {
    const int r = r0 + ty + k * p.TY;
    if (r < r1) {
      float f[VE];
      nh_unpack<T>(v[k], f);
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int t = 0; t < VE; ++t)
        oe[t] = nh_from_f32<T>(nh_act((nh_clamp(f[t] + addv[t]) - sub[t]) * mul[t] + btv[t], p.act));
      reinterpret_cast<uint4*>(yb + (int64_t)r * p.C)[tx] = o;
    }
  }
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared-memory variant (R > 8): the CTA's slice is staged by cp.async (all rows in flight at
// once) and the passes loop over it; the fully unrolled register variant was bound by
// instruction-cache misses at 16+ rows per thread.
__device__ __forceinline__ uint32_t smem_u32_nh(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32_nh(dst)), "l"(src)
               : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kNhwcThreads) gn_nhwc_cluster_kernel(NhwcClusterParams p) {
  constexpr int VE = 16 / sizeof(T);
  extern __shared__ uint4 dsm[];  // [R][nthr] x vectors | red [TY][SC] | col [9][SC] (floats)
  __shared__ float part[kClMaxGpc][3];  // this CTA's (n, mean, M2) per group
  __shared__ float gst[kClMaxGpc][2];   // merged (mean, rstd) per group
  __shared__ float gsum[kClMaxGpc];
  cooperative_groups::cluster_group cluster = cooperative_groups::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int cs = (int)cluster.num_blocks();
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int TX = p.SV;
  const int tid = ty * TX + tx;
  const int nthr = TX * p.TY;
  const int R = p.R;
  uint4* xs = dsm;
  float* red = reinterpret_cast<float*>(dsm + (size_t)R * nthr);
  float* col = red + p.TY * p.SC;
  const int b = blockIdx.z, slice = blockIdx.y;
  const int c0 = slice * p.SC;  // first channel of the slice
  const int r0 = rank * p.RP;
  const int r1 = min(p.P, r0 + p.RP);
  const T* xb = static_cast<const T*>(p.x) + (int64_t)b * p.P * p.C + c0;
  T* yb = static_cast<T*>(p.y) + (int64_t)b * p.P * p.C + c0;
  // rows of this thread: r0 + ty + k * TY, k < R (those < r1)
  const int kmax = r1 > r0 + ty ? min(R, (r1 - r0 - ty + p.TY - 1) / p.TY) : 0;

  for (int k = 0; k < kmax; ++k) {
    const int r = r0 + ty + k * p.TY;
    cp_async16(xs + k * nthr + tid, reinterpret_cast<const uint4*>(xb + (int64_t)r * p.C) + tx);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  float addv[VE], gmv[VE], btv[VE];  // issued while the copies fly, used later
  {
    const T* gam = static_cast<const T*>(p.gamma) + c0 + tx * VE;
    const T* bet = static_cast<const T*>(p.beta) + c0 + tx * VE;
#pragma unroll
    for (int t = 0; t < VE; ++t) {
      addv[t] = p.x_add ? nh_to_f32(static_cast<const T*>(p.x_add)[(int64_t)b * p.C + c0 + tx * VE + t])
                        : 0.f;
      gmv[t] = nh_to_f32(gam[t]);
      btv[t] = nh_to_f32(bet[t]);
    }
  }
  const int rows = max(0, r1 - r0);
  const float cnt = (float)rows * (float)p.Cg;
  asm volatile("cp.async.wait_all;" ::: "memory");  // each thread reads only its own vectors

  // pass 1: per-channel sums of this thread's rows -> per-group sums
  float acc[VE];
#pragma unroll
  for (int t = 0; t < VE; ++t) acc[t] = 0.f;
#pragma unroll 2
  for (int k = 0; k < kmax; ++k) {
    float f[VE];
    nh_unpack<T>(xs[k * nthr + tid], f);
#pragma unroll
    for (int t = 0; t < VE; ++t) acc[t] += nh_clamp(f[t] + addv[t]);
  }
#pragma unroll
  for (int t = 0; t < VE; ++t) red[ty * p.SC + tx * VE + t] = acc[t];
  __syncthreads();
  cl_group_sums(red, col, gsum, p, tid, nthr);
  if (tid < p.gpc) part[tid][1] = cnt > 0.f ? gsum[tid] / cnt : 0.f;
  __syncthreads();
  // pass 2: M2 about this CTA's group means
  float gmean[VE];
#pragma unroll
  for (int t = 0; t < VE; ++t) {
    gmean[t] = part[(tx * VE + t) / p.Cg][1];
    acc[t] = 0.f;
  }
#pragma unroll 2
  for (int k = 0; k < kmax; ++k) {
    float f[VE];
    nh_unpack<T>(xs[k * nthr + tid], f);
#pragma unroll
    for (int t = 0; t < VE; ++t) {
      const float d = nh_clamp(f[t] + addv[t]) - gmean[t];
      acc[t] = fmaf(d, d, acc[t]);
    }
  }
  __syncthreads();  // red is rewritten
#pragma unroll
  for (int t = 0; t < VE; ++t) red[ty * p.SC + tx * VE + t] = acc[t];
  __syncthreads();
  cl_group_sums(red, col, gsum, p, tid, nthr);
  if (tid < p.gpc) {
    part[tid][0] = cnt;
    part[tid][2] = gsum[tid];
  }
  // exchange: every CTA reads every peer's partials (rank order) after the cluster barrier
  cluster.sync();
  if (tid < p.gpc) {
    float pn[kClMaxCluster], pm[kClMaxCluster], pq2[kClMaxCluster];
#pragma unroll
    for (int q = 0; q < kClMaxCluster; ++q) {
      if (q < cs) {
        const float* pq = cluster.map_shared_rank(&part[tid][0], q);
        pn[q] = pq[0];
        pm[q] = pq[1];
        pq2[q] = pq[2];
      }
    }
    float n = 0.f, mean = 0.f, m2 = 0.f;
#pragma unroll
    for (int q = 0; q < kClMaxCluster; ++q) {
      if (q < cs) {
        const float nn = n + pn[q];
        if (nn > 0.f) {
          const float d = pm[q] - mean, f = pn[q] / nn;
          mean = fmaf(d, f, mean);
          m2 = m2 + pq2[q] + d * d * n * f;
        }
        n = nn;
      }
    }
    gst[tid][0] = mean;
    gst[tid][1] = rsqrtf(m2 / n + p.eps);
  }
  // peers may still read this CTA's `part`: arrive now, wait before leaving
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  __syncthreads();
  float mul[VE], sub[VE];
#pragma unroll
  for (int t = 0; t < VE; ++t) {
    const int g = (tx * VE + t) / p.Cg;
    sub[t] = gst[g][0];
    mul[t] = gst[g][1] * gmv[t];
  }
#pragma unroll 2
  for (int k = 0; k < kmax; ++k) {
    const int r = r0 + ty + k * p.TY;
    float f[VE];
    nh_unpack<T>(xs[k * nthr + tid], f);
    uint4 o;
    T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int t = 0; t < VE; ++t)
      oe[t] = nh_from_f32<T>(nh_act((nh_clamp(f[t] + addv[t]) - sub[t]) * mul[t] + btv[t], p.act));
    reinterpret_cast<uint4*>(yb + (int64_t)r * p.C)[tx] = o;
  }
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

struct ClusterPlan {
  bool ok;
  int gpc, SC, SV, TY, CS, RP, R;
  size_t smem;
};

constexpr int kClRegRows = 8;  // up to this many rows per thread: the register variant

// dynamic shared memory: [TY][SC] staging floats and [9][SC] column sums, after the staged
// slice [R][threads] of 16-byte vectors in the shared-memory variant
size_t cluster_smem_bytes(const ClusterPlan& pl) {
  const size_t sums = (size_t)(pl.TY + 9) * pl.SC * sizeof(float);
  return pl.R <= kClRegRows ? sums : (size_t)pl.R * pl.SV * pl.TY * 16 + sums;
}

ClusterPlan plan_cluster(int64_t B, int64_t P, int64_t C, int es, int64_t G) {
  ClusterPlan pl{};
  const int VE = 16 / es;
  const int64_t Cg = C / G;
  // the smallest group slice whose rows are whole 16-byte vectors (measured faster than
  // rounding slices up to 32-byte sectors, which leaves fewer, larger slices)
  int gpc = 0;
  for (int align : {16}) {
    for (int d = 1; d <= kClMaxGpc && !gpc; ++d)
      if (G % d == 0 && (d * Cg * es) % align == 0) gpc = d;
    if (gpc) break;
  }
  if (!gpc || (C * es) % 16) return pl;
  const int SC = (int)(gpc * Cg), SV = SC / VE;
  if (SV > kNhwcThreads) return pl;
  const int TY = std::max(1, kNhwcThreads / SV);
  if (SV * TY < 32) return pl;  // at least one full warp
  auto rows_per_thread = [&](int cs) {
    const int64_t rp = (P + cs - 1) / cs;
    return (int)((rp + TY - 1) / TY);
  };
  const int max_rows = kClMaxRows;
  int cs = 1;
  while (cs < kClMaxCluster && rows_per_thread(cs) > max_rows) cs *= 2;
  if (rows_per_thread(cs) > max_rows) return pl;
  // more CTAs while the grid is under two per SM and each thread keeps >= 2 rows
  const int64_t slices = B * (G / gpc);
  while (cs < kClMaxCluster && slices * cs < 2LL * num_sms() && rows_per_thread(cs * 2) >= 2)
    cs *= 2;
  pl.gpc = gpc;
  pl.SC = SC;
  pl.SV = SV;
  pl.TY = TY;
  pl.CS = cs;
  pl.RP = (int)((P + cs - 1) / cs);
  pl.R = rows_per_thread(cs);
  pl.smem = cluster_smem_bytes(pl);
  pl.ok = slices <= 65535 && pl.smem <= 200 * 1024;
  return pl;
}

constexpr int kFusedRows = 8;  // rows per thread held in registers by the fused kernel

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

struct FusedPlan {
  bool ok;
  int rows_per_chunk, nchunks;
  size_t smem;
};

FusedPlan plan_fused(int64_t P, int64_t C, int es, int64_t groups) {
  FusedPlan f{};
  const NhwcPlan pl = plan_nhwc(1, P, C, es, groups);
  if (pl.NV > 2) return f;  // R * NV register vectors per thread: keep it at 8
  const int R = kFusedRows / pl.NV;
  f.rows_per_chunk = pl.TY * R;
  f.nchunks = (int)((P + f.rows_per_chunk - 1) / f.rows_per_chunk);
  f.smem = ((size_t)pl.TY * C + C + 4 * groups) * sizeof(float);
  f.ok = f.smem <= 48 * 1024;
  return f;
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
  const FusedPlan f = plan_fused(H * W, C, es, groups);
  // two-kernel path: 3 floats per (image, chunk, group); fused path: one float4
  const size_t two = (size_t)B * pl.nchunks * groups * 3 * sizeof(float);
  const size_t one = f.ok ? (size_t)B * f.nchunks * groups * 4 * sizeof(float) : 0;
  return std::max(two, one);
}

template <typename T>
static int launch_cluster_nhwc(const NhwcClusterParams& p, const ClusterPlan& pl, int64_t B,
                               cudaStream_t s) {
  void (*kern)(NhwcClusterParams) =
      pl.R > kClRegRows ? gn_nhwc_cluster_kernel<T>
      : pl.R > 4        ? gn_nhwc_cluster_reg_kernel<T, 8>
      : pl.R > 2        ? gn_nhwc_cluster_reg_kernel<T, 4>
      : pl.R > 1        ? gn_nhwc_cluster_reg_kernel<T, 2>
                        : gn_nhwc_cluster_reg_kernel<T, 1>;
  if (pl.R > kClRegRows) {
    static unsigned long long attr_set = 0;
    if (first_time_on_device(&attr_set)) {
      cudaError_t e = cudaFuncSetAttribute(gn_nhwc_cluster_kernel<T>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (e != cudaSuccess) {
        __atomic_fetch_and(&attr_set, ~(1ull << current_device()), __ATOMIC_ACQ_REL);
        return set_error(SP_ERR_LAUNCH, "groupnorm (channels-last): smem attribute failed: %s",
                         cudaGetErrorString(e));
      }
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pl.CS, (unsigned)(p.G / pl.gpc), (unsigned)B);
  cfg.blockDim = dim3((unsigned)pl.SV, (unsigned)pl.TY, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)pl.CS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess)
    return set_error(SP_ERR_LAUNCH, "groupnorm (channels-last) cluster launch failed: %s",
                     cudaGetErrorString(e));
  return SP_OK;
}

// The single-launch kernel when every CTA of its grid can be resident at once (checked with
// the occupancy API; the launch is cooperative, so the runtime guarantees it).  Returns
// SP_OK when launched, 1 when the two-kernel path must run instead, < 0 on error.
template <typename T>
static int try_launch_fused(NhwcParams p, const FusedPlan& f, int NV, int64_t B, cudaStream_t s) {
  p.rows_per_chunk = f.rows_per_chunk;
  p.nchunks = f.nchunks;
  void (*kern)(NhwcParams) = NV == 1 ? gn_nhwc_fused_kernel<T, 1, kFusedRows>
                                     : gn_nhwc_fused_kernel<T, 2, kFusedRows / 2>;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, p.TX * p.TY, f.smem) !=
      cudaSuccess) {
    cudaGetLastError();
    return 1;
  }
  if ((int64_t)per_sm * num_sms() < (int64_t)f.nchunks * B) return 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)f.nchunks, (unsigned)B, 1);
  cfg.blockDim = dim3((unsigned)p.TX, (unsigned)p.TY, 1);
  cfg.dynamicSmemBytes = f.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess)
    return set_error(SP_ERR_LAUNCH, "groupnorm (channels-last) fused launch failed: %s",
                     cudaGetErrorString(e));
  return SP_OK;
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

int gn_nhwc_launch(const void* x, const void* x_add, const void* gamma, const void* beta, void* y,
                   int64_t B, int64_t C, int64_t H, int64_t W, int64_t groups, float eps, int act,
                   int dtype, void* workspace, size_t workspace_bytes, cudaStream_t s) {
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
  p.x_add = x_add;
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
  const ClusterPlan cpl = plan_cluster(B, H * W, C, es, groups);
  if (cpl.ok) {
    NhwcClusterParams cp{x,   x_add,          gamma,      beta, y, (int)(H * W), (int)C, (int)groups,
                         (int)(C / groups), cpl.gpc, cpl.SC, cpl.SV, cpl.TY, cpl.RP, cpl.R, eps,
                         act};
    switch (dtype) {
      case SP_F32: return launch_cluster_nhwc<float>(cp, cpl, B, s);
      case SP_F16: return launch_cluster_nhwc<__half>(cp, cpl, B, s);
      default: return launch_cluster_nhwc<__nv_bfloat16>(cp, cpl, B, s);
    }
  }
  const FusedPlan f = plan_fused(H * W, C, es, groups);
  if (f.ok) {
    int rc = 1;
    switch (dtype) {
      case SP_F32: rc = try_launch_fused<float>(p, f, pl.NV, B, s); break;
      case SP_F16: rc = try_launch_fused<__half>(p, f, pl.NV, B, s); break;
      default: rc = try_launch_fused<__nv_bfloat16>(p, f, pl.NV, B, s); break;
    }
    if (rc <= 0) return rc;
  }
  switch (dtype) {
    case SP_F32: return launch_nhwc_t<float>(p, pl.NV, B, s);
    case SP_F16: return launch_nhwc_t<__half>(p, pl.NV, B, s);
    default: return launch_nhwc_t<__nv_bfloat16>(p, pl.NV, B, s);
  }
}

}  // namespace sp
