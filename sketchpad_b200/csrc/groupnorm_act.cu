// groupnorm_act.cu -- fused GroupNorm (+SiLU) for NCHW activations on sm_100a.
//
// Semantics: crates/sketchpad-core/src/groupnorm.rs:62-102 + crates/sketchpad-core/src/silu.rs:5-7
//   x <- clamp(x, +-65000); per (batch, group): mean, BIASED variance (f32 statistics);
//   y <- clamp((x - mean) / sqrt(var + eps) * gamma[c] + beta[c], +-65000); y <- y*sigmoid(y).
// Replaces the reference's two-kernel GPU path (groupnorm_silu.rs:64-211), whose statistics
// kernel runs one thread per (batch, group).
//
// Fast path (contiguous x): ONE read and ONE write of HBM.  A (batch, group) is split over a
// thread-block cluster of CS CTAs (CS <= 16); each CTA keeps its slice in registers (16-byte
// vector loads), the cluster reduces the sum and then the centred sum of squares through
// distributed shared memory, and every CTA normalises its slice straight from registers.
//
// General path (strided x, or a group larger than a 16-CTA cluster holds): two kernels.
// Pass 1 writes per-chunk (count, mean, M2) partials to a caller workspace; pass 2 merges
// its group's partials (Chan et al.'s pairwise update) and normalises (x is read twice).
#include <algorithm>

#include <cooperative_groups.h>

#include "common.cuh"
#include "tc.cuh"

namespace cg = cooperative_groups;

namespace sp {
namespace {

constexpr int kGnThreads = 256;
constexpr int kMaxCluster = 16;
constexpr float kClamp = 65000.0f;

template <typename T>
struct VecTraits;
template <>
struct VecTraits<float> {
  static constexpr int kElems = 4;
};
template <>
struct VecTraits<__half> {
  static constexpr int kElems = 8;
};
template <>
struct VecTraits<__nv_bfloat16> {
  static constexpr int kElems = 8;
};

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Unpack a 16-byte vector into f32 lanes.
template <typename T>
__device__ __forceinline__ void unpack(const uint4& u, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  } else {
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = to_f32(h[i]);
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack(const float* f) {
  uint4 u;
  if constexpr (sizeof(T) == 4) {
    u.x = __float_as_uint(f[0]);
    u.y = __float_as_uint(f[1]);
    u.z = __float_as_uint(f[2]);
    u.w = __float_as_uint(f[3]);
  } else {
    T* h = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = from_f32<T>(f[i]);
  }
  return u;
}

__device__ __forceinline__ float clamp65k(float v) { return fminf(fmaxf(v, -kClamp), kClamp); }

__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// SiLU as x * sigmoid(x) with sigmoid(x) = 0.5 * tanh(x / 2) + 0.5: one MUFU op per element
// instead of an exponential plus an IEEE division (tanh.approx: ~2^-11 relative error).
__device__ __forceinline__ float apply_act(float v, int act) {
  v = clamp65k(v);
  if (act == SP_ACT_SILU) v = v * fmaf(0.5f, tanh_approx(0.5f * v), 0.5f);
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum over kGnThreads threads; result valid in every thread.
__device__ __forceinline__ float block_sum(float v, float* scratch /* >= 32 floats */) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();  // scratch may still be read from a previous call
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < (kGnThreads / 32) ? scratch[lane] : 0.f;
  return warp_sum(t);
}

struct GnParams {
  int resident;  // streaming path: the slice stays in shared memory between the passes
  const void* x;
  const void* gamma;
  const void* beta;
  void* y;
  int64_t C, HW, G, cg;       // channels, H*W, groups, channels per group
  int64_t n;                   // elements per group = cg * HW
  int64_t chunk_vecs;          // 16-byte vectors per CTA slice
  float eps;
  int act;
};

// grid = (CS, B*G), cluster = (CS, 1, 1); x and y contiguous, n % vec == 0, 16-B aligned.
template <typename T, int VPT>
__global__ void __launch_bounds__(kGnThreads, 2) gn_cluster_kernel(GnParams p) {
  constexpr int VE = VecTraits<T>::kElems;
  __shared__ float red[2];          // this CTA's partial (sum, centred sum of squares)
  __shared__ float scratch[32];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int cs = (int)cluster.num_blocks();

  const int64_t bg = blockIdx.y;  // b * G + g
  const int64_t g = bg % p.G;
  const int64_t base = bg * p.n;  // contiguous NCHW: a group is one contiguous range
  const uint4* xv = reinterpret_cast<const uint4*>(static_cast<const T*>(p.x) + base);
  uint4* yv = reinterpret_cast<uint4*>(static_cast<T*>(p.y) + base);
  const int64_t nvec = p.n / VE;
  const int64_t v0 = (int64_t)rank * p.chunk_vecs;
  const int64_t v1 = min(nvec, v0 + p.chunk_vecs);

  uint4 buf[VPT];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t vi = v0 + threadIdx.x + (int64_t)j * kGnThreads;
    if (vi < v1) buf[j] = __ldg(xv + vi);
  }
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t vi = v0 + threadIdx.x + (int64_t)j * kGnThreads;
    if (vi < v1) {
      float f[VE];
      unpack<T>(buf[j], f);
#pragma unroll
      for (int e = 0; e < VE; ++e) s += clamp65k(f[e]);
    }
  }
  s = block_sum(s, scratch);
  if (threadIdx.x == 0) red[0] = s;
  cluster.sync();
  float tot = 0.f;
  for (int r = 0; r < cs; ++r) tot += *cluster.map_shared_rank(&red[0], r);
  const float mean = tot / (float)p.n;

  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t vi = v0 + threadIdx.x + (int64_t)j * kGnThreads;
    if (vi < v1) {
      float f[VE];
      unpack<T>(buf[j], f);
#pragma unroll
      for (int e = 0; e < VE; ++e) {
        const float d = clamp65k(f[e]) - mean;
        ss += d * d;
      }
    }
  }
  ss = block_sum(ss, scratch);
  if (threadIdx.x == 0) red[1] = ss;
  cluster.sync();
  float tss = 0.f;
  for (int r = 0; r < cs; ++r) tss += *cluster.map_shared_rank(&red[1], r);
  // Every remote read of this CTA's `red` is done once all CTAs pass this arrive; the
  // matching wait sits at the end so the normalisation overlaps it.
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  const float var = tss / (float)p.n;
  const float rstd = rsqrtf(var + p.eps);

  const T* gam = static_cast<const T*>(p.gamma);
  const T* bet = static_cast<const T*>(p.beta);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t vi = v0 + threadIdx.x + (int64_t)j * kGnThreads;
    if (vi < v1) {
      float f[VE];
      unpack<T>(buf[j], f);
      // HW % VE == 0 on this path, so one vector never straddles two channels.
      const int c = (int)g * (int)p.cg + (int)((uint32_t)(vi * VE) / (uint32_t)p.HW);
      const float w = to_f32(gam[c]) * rstd;
      const float b = to_f32(bet[c]);
#pragma unroll
      for (int e = 0; e < VE; ++e) f[e] = apply_act((clamp65k(f[e]) - mean) * w + b, p.act);
      yv[vi] = pack<T>(f);
    }
  }
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------------------
// Streaming path for large contiguous groups (hundreds of KB and up).  Holding such a group
// in registers takes a 16-CTA cluster per group, few of which fit on the GPU at once, and
// each serialises load -> reduce -> store.  Here a persistent cluster of CS CTAs owns a
// sequence of (batch, group)s; each CTA owns one contiguous slice of every group.
//   warp 8 (producers): bulk-copies the slice into shared memory twice per group: lane 0
//     through ring A from HBM (L2 evict-last), lane 1 through ring B from L2 (evict-first);
//     each runs ahead across groups as far as its ring allows.
//   warps 0-7 (consumers): pass 1 forms per-thread (count, mean, M2) of clamp(x) from sums
//     shifted by the thread's first value, and max |x|; the partials merge (Chan et al.)
//     over the warps, then every CTA pushes its partial into every cluster peer's shared
//     memory and arrives on the peer's mbarrier; each CTA merges the CS partials in rank
//     order (so all agree on mean and rstd) and tabulates gamma_c * rstd, beta_c for the
//     group's channels.  Pass 2 normalises, applies the affine map and SiLU (packed f32x2
//     arithmetic, and no clamps when max |x| and the affine bound show none can bite), and
//     stores.
// HBM sees one read and one write of x.
// ---------------------------------------------------------------------------------------
constexpr int kGrConsumers = 256;
constexpr int kGrThreads = kGrConsumers + 32;
constexpr int kGrChunk = 32768;  // bytes per ring stage
// Two rings: A carries pass-1 chunks (from HBM), B pass-2 chunks (from L2), so the HBM
// stream of the next group's pass 1 never waits behind the current group's pass 2.
constexpr int kGrStagesA = 2;
constexpr int kGrStagesB = 1;
constexpr int kGrStages = kGrStagesA + kGrStagesB;  // 96 KB: two CTAs per SM
constexpr int kGrMaxCluster = 16;
constexpr int kGrMaxCg = 1024;   // channels per group the shared affine table holds

struct Welford {
  float n, mean, m2;
};

__device__ __forceinline__ Welford welford_merge(Welford a, Welford b) {
  const float n = a.n + b.n;
  if (n == 0.f) return a;
  const float d = b.mean - a.mean;
  const float fb = b.n / n;
  return {n, fmaf(d, fb, a.mean), a.m2 + b.m2 + d * d * a.n * fb};
}

// packed f32x2 arithmetic (sm_100): two lanes per instruction
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

__device__ __forceinline__ uint64_t l2_policy(bool keep) {
  uint64_t pol;
  if (keep)
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  else
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// contiguous global -> shared copy completing on an mbarrier (bytes % 16 == 0, both 16-B
// aligned)
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

__device__ __forceinline__ uint32_t map_rank(const void* p, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ void arrive_cluster(uint32_t bar_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_addr)
               : "memory");
}

// bounded wait with cluster-scope acquire (the arrivals come from peer CTAs)
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort) {
  const long long t0 = clock64();
  uint32_t spins = 0;
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((++spins & 255u) == 0) {
      if (*abort) return false;
      if (clock64() - t0 > kWaitBudgetCycles) {
        atomicCAS(&g_watchdog, 0, WD_CLUSTER_WAIT);
        *abort = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kGrConsumers) : "memory");
}

// grid = (n_clusters * CS), cluster = (CS, 1, 1), kGrThreads threads, dynamic smem =
// kGrStages * kGrChunk (+ alignment).  x, y contiguous NCHW, HW % VE == 0, 16-B aligned.
// p.chunk_vecs = vectors per CTA slice.
template <typename T>
__global__ void __launch_bounds__(kGrThreads, 2) gn_ring_kernel(GnParams p, int64_t BG) {
  constexpr int VE = VecTraits<T>::kElems;
  constexpr int kCWarps = kGrConsumers / 32;
  extern __shared__ uint8_t gr_smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gr_smem_raw) + 127) &
                                             ~uintptr_t(127));
  __shared__ uint64_t full[kGrStages], empty[kGrStages], stats_bar[2];  // A stages first
  // partials (n, mean, M2, max|x|) pushed by every rank, per parity
  __shared__ float slot[2][kGrMaxCluster][4];
  __shared__ Welford wpart[kCWarps];
  __shared__ float wamax[kCWarps];
  __shared__ float2 aff[kGrMaxCg];  // this group's (gamma_c * rstd, beta_c)
  __shared__ float gb_max[2];       // max |gamma|, max |beta| over all channels
  __shared__ int abort_flag_s;
  volatile int* abort_flag = &abort_flag_s;

  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int cs = (int)cluster.num_blocks();
  const int64_t cid = blockIdx.x / cs, ncl = gridDim.x / cs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kGrStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kCWarps);
    }
    mbar_init(&stats_bar[0], cs);
    mbar_init(&stats_bar[1], cs);
    abort_flag_s = 0;
    fence_mbar_init();
  }
  // peers arrive on these barriers: they must be initialised cluster-wide first
  cluster.sync();

  // n < 2^31 on this path: slice indices fit 32 bits
  const int nvec = (int)(p.n / VE);
  const int v0 = min(nvec, rank * (int)p.chunk_vecs);
  const int v1 = min(nvec, v0 + (int)p.chunk_vecs);
  const uint32_t slice_bytes = (uint32_t)(v1 - v0) * 16u;
  const uint32_t nchunks = (slice_bytes + kGrChunk - 1) / kGrChunk;
  // the whole slice fits the stages: load it once per group, both passes read it
  const bool resident = p.resident != 0;

  if (warp == kCWarps) {
    // ------------------------------------------------------------------ producers
    // lane 0 feeds ring A (pass 1, HBM, L2 evict-last); lane 1 feeds ring B (pass 2, the
    // same bytes again from L2, evict-first).  Each runs ahead as far as its ring allows.
    if (resident && lane == 0) {
      // resident: chunk c of every group lives in stage c and is read by both passes; the
      // stage is refilled once the consumers have finished pass 2 of the previous group
      const uint64_t pol = l2_policy(false);
      int it = 0;
      bool ok = true;
      for (int64_t bg = cid; ok && bg < BG; bg += ncl, ++it) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(static_cast<const T*>(p.x) + bg * p.n) +
                             (size_t)v0 * 16;
        for (uint32_t c = 0; c < nchunks; ++c) {
          if (it > 0 && !mbar_wait(&empty[c], (it - 1) & 1, abort_flag, WD_TMA_WAIT)) {
            ok = false;
            break;
          }
          const uint32_t bytes = min((uint32_t)kGrChunk, slice_bytes - c * kGrChunk);
          mbar_arrive_expect_tx(&full[c], bytes);
          bulk_load(ring + c * kGrChunk, src + (size_t)c * kGrChunk, bytes, &full[c], pol);
        }
      }
      if (!ok)  // let the copies in flight land before the CTA can exit (bounded)
        for (uint32_t c = 0; c < nchunks; ++c) mbar_wait(&full[c], (it & 1), nullptr, WD_TMA_WAIT);
    } else if (!resident && lane < 2) {
      const int pass = lane;
      const uint32_t nst = pass == 0 ? kGrStagesA : kGrStagesB;
      const uint32_t base = pass == 0 ? 0 : kGrStagesA;
      const uint64_t pol = l2_policy(pass == 0);
      uint32_t k = 0;
      bool ok = true;
      for (int64_t bg = cid; ok && bg < BG; bg += ncl) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(static_cast<const T*>(p.x) + bg * p.n) +
                             (size_t)v0 * 16;
        for (uint32_t c = 0; c < nchunks; ++c, ++k) {
          const uint32_t st = base + k % nst, ph = (k / nst) & 1;
          if (k >= nst && !mbar_wait(&empty[st], ph ^ 1, abort_flag, WD_TMA_WAIT)) {
            ok = false;
            break;
          }
          const uint32_t bytes = min((uint32_t)kGrChunk, slice_bytes - c * kGrChunk);
          mbar_arrive_expect_tx(&full[st], bytes);
          bulk_load(ring + st * kGrChunk, src + (size_t)c * kGrChunk, bytes, &full[st], pol);
        }
      }
      if (!ok) {
        // let the copies in flight land before the CTA can exit (bounded)
        for (uint32_t j = k > nst ? k - nst : 0; j < k; ++j)
          mbar_wait(&full[base + j % nst], (j / nst) & 1, nullptr, WD_TMA_WAIT);
      }
    }
  } else {
    // ------------------------------------------------------------------ consumers
    // A failed (expired) wait sets the shared abort flag before it returns.  Warps never
    // leave the group loop on their own: they skip work once `ok` is false and leave
    // together right after a named barrier, where every consumer sees the flag.
    const T* gam = static_cast<const T*>(p.gamma);
    const T* bet = static_cast<const T*>(p.beta);
    // max |gamma|, max |beta| over all channels: bounds the affine output of a group
    {
      float gm = 0.f, bm = 0.f;
      for (int64_t c = threadIdx.x; c < p.C; c += kGrConsumers) {
        gm = fmaxf(gm, fabsf(to_f32(gam[c])));
        bm = fmaxf(bm, fabsf(to_f32(bet[c])));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
        bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
      }
      if (lane == 0) wpart[warp] = Welford{gm, bm, 0.f};
      consumer_sync();
      if (threadIdx.x == 0) {
        for (int i = 1; i < kCWarps; ++i) {
          gm = fmaxf(gm, wpart[i].n);
          bm = fmaxf(bm, wpart[i].mean);
        }
        gb_max[0] = fmaxf(gm, wpart[0].n);
        gb_max[1] = fmaxf(bm, wpart[0].mean);
      }
      consumer_sync();
    }
    const float gmax = gb_max[0], bmax = gb_max[1];
    const uint32_t vpc = (uint32_t)(p.HW / VE);  // vectors per channel
    const float inv_vpc = 1.0f / (float)vpc;
    uint32_t ka = 0, kb = 0;  // chunks taken from ring A / ring B
    int it = 0;
    bool ok = true;  // warp-uniform
    for (int64_t bg = cid; bg < BG; bg += ncl, ++it) {
      const int64_t g = bg % p.G;
      uint4* yv = reinterpret_cast<uint4*>(static_cast<T*>(p.y) + bg * p.n) + v0;

      // ---- pass 1: statistics of clamp(x) and max |x|
      const uint64_t zero2 = f2(0.f, 0.f);
      uint64_t sh2 = zero2, s1 = zero2, s2 = zero2;
      float amax = 0.f, cnt = 0.f;
      bool first = true;
      for (uint32_t c = 0; ok && c < nchunks; ++c, ++ka) {
        const uint32_t st = resident ? c : ka % kGrStagesA;
        const uint32_t ph = resident ? (uint32_t)(it & 1) : (ka / kGrStagesA) & 1;
        if (!mbar_wait_warp(&full[st], ph, abort_flag, WD_CONVERT_WAIT)) {
          ok = false;
          break;
        }
        const uint32_t cv = min((uint32_t)kGrChunk, slice_bytes - c * kGrChunk) / 16u;
        const uint4* sv = reinterpret_cast<const uint4*>(ring + st * kGrChunk);
        for (uint32_t i = threadIdx.x; i < cv; i += kGrConsumers) {
          float f[VE];
          unpack<T>(sv[i], f);
#pragma unroll
          for (int e = 0; e < VE; ++e) {
            amax = fmaxf(amax, fabsf(f[e]));
            f[e] = clamp65k(f[e]);
          }
          if (first) {
            sh2 = f2(f[0], f[0]);
            first = false;
          }
#pragma unroll
          for (int e = 0; e < VE; e += 2) {
            const uint64_t d = f2_sub(f2(f[e], f[e + 1]), sh2);
            s1 = f2_add(s1, d);
            s2 = f2_fma(d, d, s2);
          }
          cnt += (float)VE;
        }
        __syncwarp();
        if (lane == 0 && !resident) mbar_arrive(&empty[st]);
      }
      Welford w{cnt, 0.f, 0.f};
      if (cnt > 0.f) {
        float a, b, shift, dummy;
        f2_split(s1, a, b);
        const float t1 = a + b;
        f2_split(s2, a, b);
        const float t2 = a + b;
        f2_split(sh2, shift, dummy);
        const float m = t1 / cnt;
        w.mean = shift + m;
        w.m2 = fmaxf(t2 - t1 * m, 0.f);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        Welford b{__shfl_xor_sync(0xffffffffu, w.n, o), __shfl_xor_sync(0xffffffffu, w.mean, o),
                  __shfl_xor_sync(0xffffffffu, w.m2, o)};
        w = welford_merge(w, b);
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      }
      if (lane == 0) {
        wpart[warp] = w;
        wamax[warp] = amax;
      }
      consumer_sync();
      if (*abort_flag) break;  // uniform across the consumer warps
      const int par = it & 1;
      if (threadIdx.x == 0) {
        Welford t = wpart[0];
        float am = wamax[0];
        for (int i = 1; i < kCWarps; ++i) {
          t = welford_merge(t, wpart[i]);
          am = fmaxf(am, wamax[i]);
        }
        // push the partial into every rank's slot[par][rank], then arrive there
        for (int r = 0; r < cs; ++r) {
          const uint32_t a = map_rank(&slot[par][rank][0], r);
          st_cluster_f32(a, t.n);
          st_cluster_f32(a + 4, t.mean);
          st_cluster_f32(a + 8, t.m2);
          st_cluster_f32(a + 12, am);
          arrive_cluster(map_rank(&stats_bar[par], r));
        }
      }
      __syncwarp();
      ok = __all_sync(0xffffffffu, mbar_wait_cluster(&stats_bar[par], (it >> 1) & 1, abort_flag));
      float mean = 0.f, rstd = 0.f, gamax = 0.f;
      if (ok) {
        Welford t{slot[par][0][0], slot[par][0][1], slot[par][0][2]};
        gamax = slot[par][0][3];
        for (int r = 1; r < cs; ++r) {
          t = welford_merge(t, Welford{slot[par][r][0], slot[par][r][1], slot[par][r][2]});
          gamax = fmaxf(gamax, slot[par][r][3]);
        }
        mean = t.mean;
        rstd = rsqrtf(t.m2 / t.n + p.eps);
        for (int c = threadIdx.x; c < (int)p.cg; c += kGrConsumers)
          aff[c] = make_float2(to_f32(gam[g * p.cg + c]) * rstd, to_f32(bet[g * p.cg + c]));
      }
      consumer_sync();
      if (!ok) continue;  // leaves at the next named barrier (or at the end)
      // no clamp can bite when |x| <= 65000 and |(x - mean) * w + b| <= 65000 for all x, c
      const bool no_clamp =
          gamax <= kClamp && (gamax + fabsf(mean)) * gmax * rstd + bmax <= kClamp;
      const uint64_t mean2 = f2(mean, mean);
      const uint64_t half2 = f2(0.5f, 0.5f);

      // ---- pass 2: normalise, affine, activation, store
      for (uint32_t c = 0; c < nchunks; ++c, ++kb) {
        const uint32_t st = resident ? c : kGrStagesA + kb % kGrStagesB;
        const uint32_t ph = (kb / kGrStagesB) & 1;
        // resident: the chunk is still in its stage from pass 1
        if (!resident && !mbar_wait_warp(&full[st], ph, abort_flag, WD_CONVERT_WAIT)) {
          ok = false;
          break;
        }
        const uint32_t c0 = c * (kGrChunk / 16);  // first vector of this chunk in the slice
        const uint32_t cv = min((uint32_t)kGrChunk, slice_bytes - c * kGrChunk) / 16u;
        const uint4* sv = reinterpret_cast<const uint4*>(ring + st * kGrChunk);
        for (uint32_t i = threadIdx.x; i < cv; i += kGrConsumers) {
          float f[VE];
          unpack<T>(sv[i], f);
          // channel of this vector: vi / vpc via a float estimate and one correction step
          const uint32_t vi = (uint32_t)v0 + c0 + i;
          uint32_t q = __float2uint_rz((float)vi * inv_vpc);
          const int32_t rem = (int32_t)(vi - q * vpc);
          q = rem < 0 ? q - 1 : (rem >= (int32_t)vpc ? q + 1 : q);
          const float2 ab = aff[q];
          const uint64_t w2 = f2(ab.x, ab.x), b2 = f2(ab.y, ab.y);
          if (no_clamp) {
#pragma unroll
            for (int e = 0; e < VE; e += 2) {
              uint64_t v = f2_fma(f2_sub(f2(f[e], f[e + 1]), mean2), w2, b2);
              if (p.act == SP_ACT_SILU) {
                float t0, t1;
                f2_split(f2_mul(v, half2), t0, t1);
                const uint64_t sg = f2_fma(f2(tanh_approx(t0), tanh_approx(t1)), half2, half2);
                v = f2_mul(v, sg);
              }
              f2_split(v, f[e], f[e + 1]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < VE; ++e)
              f[e] = apply_act((clamp65k(f[e]) - mean) * ab.x + ab.y, p.act);
          }
          yv[c0 + i] = pack<T>(f);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
      }
    }
  }
  // no CTA may leave while a peer could still push into its shared memory (the barrier is
  // warp-aligned: reconverge the producer warp and any consumer lanes first)
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------------------
// General path: strided input, or groups beyond one cluster's capacity.
// ---------------------------------------------------------------------------------------
struct GnGeneralParams {
  const void* x;
  const void* gamma;
  const void* beta;
  void* y;
  int64_t B, C, H, W, G, cg, n;
  int64_t sb, sc, sh, sw;  // element strides of x
  int64_t yb, yc, yh, yw;  // element strides of y (NCHW-contiguous, or x's NHWC layout)
  int64_t chunk;           // elements per chunk
  int64_t nchunks;         // chunks per group
  float* part;             // [B*G, nchunks, 3] : count, mean, M2
  float eps;
  int act;
};

__device__ __forceinline__ int64_t gn_offset(const GnGeneralParams& p, int64_t b, int64_t g,
                                             int64_t e) {
  const int64_t cl = e / (p.H * p.W);
  const int64_t hw = e - cl * p.H * p.W;
  const int64_t h = hw / p.W, w = hw - h * p.W;
  return b * p.sb + (g * p.cg + cl) * p.sc + h * p.sh + w * p.sw;
}

template <typename T>
__global__ void __launch_bounds__(kGnThreads) gn_partial_kernel(GnGeneralParams p) {
  __shared__ float scratch[32];
  const int64_t bg = blockIdx.y, b = bg / p.G, g = bg % p.G;
  const int64_t e0 = (int64_t)blockIdx.x * p.chunk;
  const int64_t e1 = min(p.n, e0 + p.chunk);
  const T* x = static_cast<const T*>(p.x);
  float s = 0.f;
  for (int64_t e = e0 + threadIdx.x; e < e1; e += kGnThreads) s += clamp65k(to_f32(x[gn_offset(p, b, g, e)]));
  s = block_sum(s, scratch);
  const float cnt = (float)(e1 - e0);
  const float m = s / cnt;
  float ss = 0.f;
  for (int64_t e = e0 + threadIdx.x; e < e1; e += kGnThreads) {
    const float d = clamp65k(to_f32(x[gn_offset(p, b, g, e)])) - m;
    ss += d * d;
  }
  ss = block_sum(ss, scratch);
  if (threadIdx.x == 0) {
    float* o = p.part + (bg * p.nchunks + blockIdx.x) * 3;
    o[0] = cnt;
    o[1] = m;
    o[2] = ss;
  }
}

template <typename T>
__global__ void __launch_bounds__(kGnThreads) gn_apply_kernel(GnGeneralParams p) {
  __shared__ float stats[2];
  const int64_t bg = blockIdx.y, b = bg / p.G, g = bg % p.G;
  if (threadIdx.x == 0) {
    // Chan's pairwise merge of (count, mean, M2), in chunk order.
    const float* q = p.part + bg * p.nchunks * 3;
    double n = 0.0, mean = 0.0, m2 = 0.0;
    for (int64_t i = 0; i < p.nchunks; ++i) {
      const double nb = q[3 * i], mb = q[3 * i + 1], m2b = q[3 * i + 2];
      const double nn = n + nb, d = mb - mean;
      mean += d * nb / nn;
      m2 += m2b + d * d * n * nb / nn;
      n = nn;
    }
    stats[0] = (float)mean;
    stats[1] = rsqrtf((float)(m2 / n) + p.eps);
  }
  __syncthreads();
  const float mean = stats[0], rstd = stats[1];
  const int64_t e0 = (int64_t)blockIdx.x * p.chunk;
  const int64_t e1 = min(p.n, e0 + p.chunk);
  const T* x = static_cast<const T*>(p.x);
  const T* gam = static_cast<const T*>(p.gamma);
  const T* bet = static_cast<const T*>(p.beta);
  T* y = static_cast<T*>(p.y);
  for (int64_t e = e0 + threadIdx.x; e < e1; e += kGnThreads) {
    const int64_t cl = e / (p.H * p.W);
    const int64_t hw = e - cl * p.H * p.W;
    const int64_t hh = hw / p.W, ww = hw - hh * p.W;
    const int64_t c = g * p.cg + cl;
    const float v = (clamp65k(to_f32(x[gn_offset(p, b, g, e)])) - mean) * rstd;
    y[b * p.yb + c * p.yc + hh * p.yh + ww * p.yw] =
        from_f32<T>(apply_act(v * to_f32(gam[c]) + to_f32(bet[c]), p.act));
  }
}

constexpr int64_t kGeneralChunk = 16384;

struct GnPlan {
  bool cluster_path;
  bool stream_path;  // persistent streaming clusters (large groups)
  bool resident;     // streaming path with the whole slice held in shared memory
  int cs;      // cluster size
  int vpt;     // vectors per thread
  int64_t chunk_vecs;
  int64_t nchunks;  // general path
};

// Groups of at least this many bytes take the streaming path.
constexpr int64_t kStreamMinGroupBytes = 256 * 1024;

GnPlan plan_gn(int64_t B, int64_t G, int64_t cg, int64_t n, bool contiguous, bool vec_ok,
               int vec_elems) {
  GnPlan pl{};
  const int64_t nvec = n / vec_elems;
  // 16 vectors (64 f32) per thread for f32, 8 vectors (64 halves) for 16-bit types: both
  // stay within the 128 registers that two resident CTAs per SM allow.
  const int max_vpt = vec_elems == 4 ? 16 : 8;
  const int64_t group_bytes = n * (16 / vec_elems);
  if (contiguous && vec_ok && n < (1LL << 31) && group_bytes >= kStreamMinGroupBytes &&
      cg <= kGrMaxCg) {
    // two CTAs per SM; the smallest cluster (>= 2) that still gives every CTA slot a slice
    // (measured on B200: larger slices per CTA beat keeping fewer groups in flight, and
    // clusters grown just to shrink slices into shared memory ran slower)
    int cs = 2;
    while (cs < 8 && B * G * cs < (2LL * num_sms() * 7) / 8) cs *= 2;  // 16: measured slower
    // when the slice fits the stages: one HBM read, both passes from shared memory
    pl.resident = (nvec + cs - 1) / cs * 16 <= (int64_t)kGrStages * kGrChunk;
    pl.stream_path = true;
    pl.cs = cs;
    pl.chunk_vecs = (nvec + cs - 1) / cs;
    return pl;
  }
  if (contiguous && vec_ok && n < (1LL << 31)) {
    static const int kVpts[] = {1, 2, 4, 8, 16};
    int best_cs = 0, best_vpt = 0;
    // smallest cluster whose slices fit max_vpt vectors per thread
    for (int cs = 1; cs <= kMaxCluster; cs *= 2) {
      const int64_t per = (nvec + cs - 1) / cs;
      if (per <= (int64_t)kGnThreads * max_vpt) {
        best_cs = cs;
        break;
      }
    }
    if (best_cs) {
      // widen the cluster while the grid is small and the slices stay >= 2 vectors/thread
      const int64_t target_ctas = 2LL * num_sms();
      while (best_cs < kMaxCluster && B * G * best_cs < target_ctas &&
             (nvec + 2 * best_cs - 1) / (2 * best_cs) >= (int64_t)kGnThreads * 2)
        best_cs *= 2;
      const int64_t per = (nvec + best_cs - 1) / best_cs;
      for (int v : kVpts)
        if ((int64_t)v * kGnThreads >= per) {
          best_vpt = v;
          break;
        }
      pl.cluster_path = true;
      pl.cs = best_cs;
      pl.vpt = best_vpt;
      pl.chunk_vecs = per;
      return pl;
    }
  }
  pl.cluster_path = false;
  pl.nchunks = (n + kGeneralChunk - 1) / kGeneralChunk;
  return pl;
}

template <typename T, int VPT>
int launch_cluster(const GnParams& p, int cs, int64_t BG, cudaStream_t stream) {
  auto kern = gn_cluster_kernel<T, VPT>;
  static unsigned long long attr_set = 0;
  if (cs > 8 && first_time_on_device(&attr_set)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) {
      __atomic_fetch_and(&attr_set, ~(1ull << current_device()), __ATOMIC_ACQ_REL);
      return set_error(SP_ERR_LAUNCH, "groupnorm: cluster size %d not allowed: %s", cs,
                       cudaGetErrorString(e));
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)cs, (unsigned)BG, 1);
  cfg.blockDim = dim3(kGnThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess)
    return set_error(SP_ERR_LAUNCH, "groupnorm cluster launch (cs=%d, vpt=%d) failed: %s", cs,
                     VPT, cudaGetErrorString(e));
  return SP_OK;
}

template <typename T>
int launch_cluster_vpt(const GnParams& p, int cs, int vpt, int64_t BG, cudaStream_t s) {
  switch (vpt) {
    case 1: return launch_cluster<T, 1>(p, cs, BG, s);
    case 2: return launch_cluster<T, 2>(p, cs, BG, s);
    case 4: return launch_cluster<T, 4>(p, cs, BG, s);
    case 8: return launch_cluster<T, 8>(p, cs, BG, s);
    default:
      if constexpr (sizeof(T) == 4) return launch_cluster<T, 16>(p, cs, BG, s);
      return set_error(SP_ERR_SHAPE, "groupnorm: internal plan error (vpt %d)", vpt);
  }
}

constexpr int kGrSmem = kGrStages * kGrChunk + 128;

template <typename T>
int launch_stream(const GnParams& p, int cs, int64_t BG, cudaStream_t stream) {
  auto kern = gn_ring_kernel<T>;
  static unsigned long long attr_set = 0;
  if (first_time_on_device(&attr_set)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGrSmem);
    if (e != cudaSuccess) {
      __atomic_fetch_and(&attr_set, ~(1ull << current_device()), __ATOMIC_ACQ_REL);
      return set_error(SP_ERR_LAUNCH, "groupnorm: kernel attribute failed: %s",
                       cudaGetErrorString(e));
    }
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kGrThreads, 1, 1);
  cfg.dynamicSmemBytes = kGrSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // as many clusters as can be resident at once (each loops over groups), found once per
  // device and cluster size
  static int resident[64][5] = {};
  const int dev = current_device();
  int lg = 0;
  while ((1 << lg) < cs) ++lg;
  int ncl = (dev >= 0 && dev < 64) ? __atomic_load_n(&resident[dev][lg], __ATOMIC_ACQUIRE) : 0;
  if (ncl <= 0) {
    cfg.gridDim = dim3((unsigned)(cs * (2 * num_sms() / cs)), 1, 1);
    if (cudaOccupancyMaxActiveClusters(&ncl, kern, &cfg) != cudaSuccess || ncl <= 0) {
      cudaGetLastError();
      ncl = 2 * num_sms() / cs;
    }
    if (dev >= 0 && dev < 64) __atomic_store_n(&resident[dev][lg], ncl, __ATOMIC_RELEASE);
  }
  const int64_t nclusters = std::min<int64_t>(ncl, BG);
  cfg.gridDim = dim3((unsigned)(nclusters * cs), 1, 1);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p, BG);
  if (e != cudaSuccess)
    return set_error(SP_ERR_LAUNCH, "groupnorm stream launch (cs=%d) failed: %s", cs,
                     cudaGetErrorString(e));
  return SP_OK;
}

template <typename T>
int launch_general(const GnGeneralParams& p, int64_t BG, cudaStream_t s) {
  dim3 grid((unsigned)p.nchunks, (unsigned)BG, 1);
  gn_partial_kernel<T><<<grid, kGnThreads, 0, s>>>(p);
  int rc = check_launch("groupnorm partial");
  if (rc) return rc;
  gn_apply_kernel<T><<<grid, kGnThreads, 0, s>>>(p);
  return check_launch("groupnorm apply");
}

}  // namespace
}  // namespace sp

extern "C" {

namespace sp {
namespace {
size_t general_workspace_bytes(int64_t B, int64_t C, int64_t H, int64_t W, int64_t groups) {
  const int64_t n = C / groups * H * W;
  const int64_t nchunks = (n + kGeneralChunk - 1) / kGeneralChunk;
  return (size_t)(B * groups * nchunks * 3 * sizeof(float));
}
// y follows x when x is dense channels-last (NHWC), else it is contiguous NCHW.
void output_strides(int64_t B, int64_t C, int64_t H, int64_t W, const int64_t* xs, int64_t* ys) {
  bool nhwc = xs != nullptr;
  if (nhwc) {
    const int64_t want[4] = {H * W * C, 1, W * C, C};
    const int64_t dims[4] = {B, C, H, W};
    for (int i = 0; i < 4; ++i)
      if (dims[i] > 1 && xs[i] != want[i]) nhwc = false;
    if (C == 1) nhwc = false;
  }
  if (nhwc) {
    ys[0] = H * W * C; ys[1] = 1; ys[2] = W * C; ys[3] = C;
  } else {
    ys[0] = C * H * W; ys[1] = H * W; ys[2] = W; ys[3] = 1;
  }
}

bool is_contiguous_nchw(int64_t B, int64_t C, int64_t H, int64_t W, const int64_t* st) {
  if (!st) return true;
  const int64_t want[4] = {C * H * W, H * W, W, 1};
  const int64_t dims[4] = {B, C, H, W};
  for (int i = 0; i < 4; ++i)
    if (dims[i] > 1 && st[i] != want[i]) return false;
  return true;
}
}  // namespace
}  // namespace sp

size_t sp_groupnorm_act_workspace_size(int64_t B, int64_t C, int64_t H, int64_t W,
                                       const int64_t x_strides[4], int64_t groups, int dtype) {
  const int es = sp::dtype_size(dtype);
  if (!es || B <= 0 || C <= 0 || H <= 0 || W <= 0 || groups <= 0 || C % groups) return 0;
  if (sp::gn_nhwc_applicable(B, C, H, W, x_strides, es, groups))
    return sp::gn_nhwc_workspace_bytes(B, C, H, W, es, groups);
  const bool contiguous = sp::is_contiguous_nchw(B, C, H, W, x_strides);
  const int vec = 16 / es;
  const sp::GnPlan pl = sp::plan_gn(B, groups, C / groups, C / groups * H * W, contiguous,
                                    contiguous && (H * W) % vec == 0, vec);
  return (pl.cluster_path || pl.stream_path) ? 0 : sp::general_workspace_bytes(B, C, H, W, groups);
}

int sp_groupnorm_act_output_strides(int64_t B, int64_t C, int64_t H, int64_t W,
                                    const int64_t x_strides[4], int64_t y_strides[4]) {
  sp::clear_error();
  if (!y_strides || B <= 0 || C <= 0 || H <= 0 || W <= 0)
    return sp::set_error(SP_ERR_INVALID_ARG, "groupnorm output strides: bad arguments");
  sp::output_strides(B, C, H, W, x_strides, y_strides);
  return SP_OK;
}

int sp_groupnorm_act(const void* x, const void* gamma, const void* beta, void* y, int64_t B,
                     int64_t C, int64_t H, int64_t W, const int64_t x_strides[4], int64_t groups,
                     float eps, int act, int dtype, void* workspace, size_t workspace_bytes,
                     void* stream) {
  using namespace sp;
  clear_error();
  if (!x || !gamma || !beta || !y)
    return set_error(SP_ERR_INVALID_ARG, "groupnorm: null tensor pointer");
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0 || groups <= 0)
    return set_error(SP_ERR_INVALID_ARG, "groupnorm: non-positive dimension");
  if (C % groups != 0)
    return set_error(SP_ERR_SHAPE, "channels (%lld) must be divisible by num_groups (%lld)",
                     (long long)C, (long long)groups);
  if (act != SP_ACT_NONE && act != SP_ACT_SILU)
    return set_error(SP_ERR_INVALID_ARG, "groupnorm: unknown activation %d", act);
  const int es = dtype_size(dtype);
  if (!es) return set_error(SP_ERR_DTYPE, "groupnorm: unknown dtype %d", dtype);
  if (B * groups > 65535)
    return set_error(SP_ERR_SHAPE, "groupnorm: batch*groups (%lld) exceeds 65535",
                     (long long)(B * groups));
  if (int rc = require_sm100()) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  const int64_t HW = H * W, cg = C / groups, n = cg * HW;
  if (gn_nhwc_applicable(B, C, H, W, x_strides, es, groups))
    return gn_nhwc_launch(x, nullptr, gamma, beta, y, B, C, H, W, groups, eps, act, dtype,
                          workspace, workspace_bytes, s);
  int64_t st[4] = {C * HW, HW, W, 1};
  const bool contiguous = is_contiguous_nchw(B, C, H, W, x_strides);
  if (!contiguous)
    for (int i = 0; i < 4; ++i) st[i] = x_strides[i];
  const int vec_elems = 16 / es;
  const bool vec_ok = contiguous && (HW % vec_elems == 0) && aligned(x, 16) && aligned(y, 16);
  const GnPlan pl = plan_gn(B, groups, cg, n, contiguous, vec_ok, vec_elems);

  if (pl.stream_path) {
    GnParams p{pl.resident ? 1 : 0, x, gamma, beta, y, C, HW, groups, cg, n, pl.chunk_vecs, eps,
               act};
    switch (dtype) {
      case SP_F32: return launch_stream<float>(p, pl.cs, B * groups, s);
      case SP_F16: return launch_stream<__half>(p, pl.cs, B * groups, s);
      default: return launch_stream<__nv_bfloat16>(p, pl.cs, B * groups, s);
    }
  }
  if (pl.cluster_path) {
    GnParams p{0, x, gamma, beta, y, C, HW, groups, cg, n, pl.chunk_vecs, eps, act};
    switch (dtype) {
      case SP_F32: return launch_cluster_vpt<float>(p, pl.cs, pl.vpt, B * groups, s);
      case SP_F16: return launch_cluster_vpt<__half>(p, pl.cs, pl.vpt, B * groups, s);
      default: return launch_cluster_vpt<__nv_bfloat16>(p, pl.cs, pl.vpt, B * groups, s);
    }
  }
  const size_t need = general_workspace_bytes(B, C, H, W, groups);
  if (!workspace || workspace_bytes < need)
    return set_error(SP_ERR_WORKSPACE,
                     "groupnorm: this shape/layout takes the two-pass path and needs %zu bytes "
                     "of workspace (got %zu)",
                     need, workspace_bytes);
  if (!aligned(workspace, 4)) return set_error(SP_ERR_ALIGN, "groupnorm: workspace misaligned");
  int64_t ys[4];
  output_strides(B, C, H, W, x_strides, ys);
  GnGeneralParams p{x,     gamma, beta,  y,     B,     C,     H,     W,     groups, cg, n,
                    st[0], st[1], st[2], st[3], ys[0], ys[1], ys[2], ys[3], kGeneralChunk,
                    pl.nchunks, static_cast<float*>(workspace), eps, act};
  switch (dtype) {
    case SP_F32: return launch_general<float>(p, B * groups, s);
    case SP_F16: return launch_general<__half>(p, B * groups, s);
    default: return launch_general<__nv_bfloat16>(p, B * groups, s);
  }
}

int sp_groupnorm_add_act(const void* x, const void* x_add, const void* gamma, const void* beta,
                         void* y, int64_t B, int64_t C, int64_t H, int64_t W,
                         const int64_t x_strides[4], int64_t groups, float eps, int act,
                         int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace sp;
  clear_error();
  if (!x || !x_add || !gamma || !beta || !y)
    return set_error(SP_ERR_INVALID_ARG, "groupnorm_add: null tensor pointer");
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0 || groups <= 0)
    return set_error(SP_ERR_INVALID_ARG, "groupnorm_add: non-positive dimension");
  if (C % groups != 0)
    return set_error(SP_ERR_SHAPE, "channels (%lld) must be divisible by num_groups (%lld)",
                     (long long)C, (long long)groups);
  if (act != SP_ACT_NONE && act != SP_ACT_SILU)
    return set_error(SP_ERR_INVALID_ARG, "groupnorm_add: unknown activation %d", act);
  const int es = dtype_size(dtype);
  if (!es) return set_error(SP_ERR_DTYPE, "groupnorm_add: unknown dtype %d", dtype);
  if (B * groups > 65535)
    return set_error(SP_ERR_SHAPE, "groupnorm_add: batch*groups (%lld) exceeds 65535",
                     (long long)(B * groups));
  if (!gn_nhwc_applicable(B, C, H, W, x_strides, es, groups))
    return set_error(SP_ERR_SHAPE,
                     "groupnorm_add: x must be dense channels-last (NHWC) with C a multiple of "
                     "the 16-byte vector and at most 1024 groups");
  if (int rc = require_sm100()) return rc;
  return gn_nhwc_launch(x, x_add, gamma, beta, y, B, C, H, W, groups, eps, act, dtype, workspace,
                        workspace_bytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// GroupNorm(+SiLU) for callers that cannot allocate device memory.
//
// sp_groupnorm_act needs caller-provided workspace whenever it takes the two-pass path.
// Some callers have no way to provide it: a host whose allocator must not be touched while
// it runs (a real-time or pre-reserved memory budget), or an FFI host that holds raw device
// pointers for its tensors but no handle to any CUDA allocator.  This variant runs the same
// two-pass kernels with their per-chunk statistics in a fixed array compiled into the
// library, so it allocates nothing and needs no workspace argument.
//
// The array lives in every device that loads the library, until the process exits.  Its
// device address is looked up (cudaGetSymbolAddress) the first time the entry point runs on
// a device, with that device current; make that first call outside any stream capture.
// All calls on a device share the array: calls that can overlap on the GPU (different
// streams without ordering between them) race on it.  Every slot a call reads is written
// earlier by the same call, so nothing needs clearing between calls.
// ---------------------------------------------------------------------------------------
#include <mutex>

namespace sp {
namespace {

constexpr size_t kNoAllocScratchBytes = 256 * 1024;
constexpr size_t kNoAllocScratchFloats = kNoAllocScratchBytes / sizeof(float);
static __device__ __align__(256) float g_gn_noalloc_scratch[kNoAllocScratchFloats];

std::mutex g_noalloc_mutex;
float* g_noalloc_ptr[64] = {};

int noalloc_scratch(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return set_error(SP_ERR_DEVICE, "groupnorm (no-alloc): no usable current device");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gn_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(SP_ERR_LAUNCH, "groupnorm (no-alloc): scratch address lookup failed: %s",
                       cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return SP_OK;
}

}  // namespace
}  // namespace sp

extern "C" size_t sp_groupnorm_act_noalloc_max_scratch_bytes(void) {
  return sp::kNoAllocScratchBytes;
}

extern "C" int sp_groupnorm_act_noalloc(const void* x, const void* gamma, const void* beta, void* y,
                                        int64_t B, int64_t C, int64_t H, int64_t W,
                                        const int64_t x_strides[4], int64_t groups, float eps,
                                        int act, int dtype, void* stream) {
  using namespace sp;
  clear_error();
  if (!x || !gamma || !beta || !y)
    return set_error(SP_ERR_INVALID_ARG, "groupnorm (no-alloc): null tensor pointer");
  if (B <= 0 || C <= 0 || H <= 0 || W <= 0 || groups <= 0)
    return set_error(SP_ERR_INVALID_ARG, "groupnorm (no-alloc): non-positive dimension");
  if (C % groups != 0)
    return set_error(SP_ERR_SHAPE, "channels (%lld) must be divisible by num_groups (%lld)",
                     (long long)C, (long long)groups);
  if (act != SP_ACT_NONE && act != SP_ACT_SILU)
    return set_error(SP_ERR_INVALID_ARG, "groupnorm (no-alloc): unknown activation %d", act);
  if (!dtype_size(dtype)) return set_error(SP_ERR_DTYPE, "groupnorm (no-alloc): unknown dtype %d", dtype);
  if (B * groups > 65535)
    return set_error(SP_ERR_SHAPE, "groupnorm (no-alloc): batch*groups (%lld) exceeds 65535",
                     (long long)(B * groups));
  const size_t need = general_workspace_bytes(B, C, H, W, groups);
  if (need > kNoAllocScratchBytes)
    return set_error(SP_ERR_WORKSPACE,
                     "groupnorm (no-alloc): this shape needs %zu bytes of statistics but the fixed "
                     "scratch holds %zu; use sp_groupnorm_act with a workspace",
                     need, kNoAllocScratchBytes);
  if (int rc = require_sm100()) return rc;
  float* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;

  const int64_t HW = H * W, cg = C / groups, n = cg * HW;
  int64_t st[4] = {C * HW, HW, W, 1};
  if (!is_contiguous_nchw(B, C, H, W, x_strides))
    for (int i = 0; i < 4; ++i) st[i] = x_strides[i];
  const int64_t nchunks = (n + kGeneralChunk - 1) / kGeneralChunk;
  int64_t ys[4];
  output_strides(B, C, H, W, x_strides, ys);
  GnGeneralParams p{x,     gamma, beta,  y,     B,     C,     H,     W,     groups, cg, n,
                    st[0], st[1], st[2], st[3], ys[0], ys[1], ys[2], ys[3], kGeneralChunk,
                    nchunks, scratch, eps, act};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SP_F32: return launch_general<float>(p, B * groups, s);
    case SP_F16: return launch_general<__half>(p, B * groups, s);
    default: return launch_general<__nv_bfloat16>(p, B * groups, s);
  }
}
