// groupnorm_act.cu -- fused GroupNorm (+SiLU) for NCHW activations on sm_100a.
//
// Semantics: crates/sketchpad-core/src/groupnorm.rs:62-102 + crates/sketchpad-core/src/silu.rs:5-7
//   x <- clamp(x, +-65000); per (batch, group): mean, BIASED variance (f32 statistics);
//   y <- clamp((x - mean) / sqrt(var + eps) * gamma[c] + beta[c], +-65000); y <- y*sigmoid(y).
// Replaces the reference's two-kernel GPU path (groupnorm_silu.rs:64-211), whose statistics
// kernel runs one thread per (batch, group).
//
// Fast path (contiguous x, groups below 256 KB): ONE read and ONE write of HBM.  A (batch,
// group) is split over a thread-block cluster of CS CTAs (CS <= 16); each CTA keeps its slice
// in registers (16-byte vector loads), the cluster reduces the sum and then the centred sum
// of squares through distributed shared memory, and every CTA normalises its slice straight
// from registers.
//
// Streaming path (contiguous x, groups of 256 KB and more): a persistent grid of slice units
// (statistics of a slice, then normalisation of it once its group's statistics are known);
// x is read once from HBM and once more from L2, y written once.  Described at
// gn_slice_kernel.
//
// General path (strided x): two kernels.  Pass 1 writes per-chunk (count, mean, M2) partials
// to a caller workspace; pass 2 merges its group's partials (Chan et al.'s pairwise update)
// and normalises (x is read twice).
#include <algorithm>
#include <type_traits>

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
    // two lanes per conversion (cvt.rn.{f16x2,bf16x2}.f32), same rounding as one at a time
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (std::is_same<T, __half>::value) {
        const __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
  }
  return u;
}

__device__ __forceinline__ float clamp65k(float v) { return fminf(fmaxf(v, -kClamp), kClamp); }

__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two 16-bit lanes (f16x2 / bf16x2 by T): round a pair of f32 values, tanh, fused h*t + h.
template <typename T>
__device__ __forceinline__ uint32_t cvt2_16(float lo, float hi) {
  uint32_t r;
  if constexpr (std::is_same<T, __half>::value)
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
template <typename T>
__device__ __forceinline__ uint32_t tanh2_16(uint32_t x) {
  uint32_t r;
  if constexpr (std::is_same<T, __half>::value)
    asm("tanh.approx.f16x2 %0, %1;" : "=r"(r) : "r"(x));
  else
    asm("tanh.approx.bf16x2 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}
template <typename T>
__device__ __forceinline__ uint32_t fma2_16(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  if constexpr (std::is_same<T, __half>::value)
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  else
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
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
// Streaming path for large contiguous groups (hundreds of KB and up): a persistent,
// cooperatively launched grid walks one fixed sequence of slice units.  A group is cut into
// S slices of SlCfg::kBytes.  Unit (pass 0, g, s) reads slice s of group g from HBM once and
// writes its (count, mean, M2, max |x|) partial to global memory; unit (pass 1, g, s) takes
// the group's statistics merged from the S partials in slice order (so every slice of a group
// gets the same mean and rstd), re-reads the slice (from L2) and writes the normalised,
// activated output.  The sequence
// interleaves pass 0 of group t with pass 1 of group t - L:
//   * a pass-1 unit depends only on units earlier in the sequence, and every CTA is resident
//     (cooperative launch) and takes its units in sequence order, so each of its waits ends;
//   * with L about two grid-widths of units, the partials are normally complete before a
//     pass-1 unit starts, and the L groups in between (~20 MB) still sit in L2;
//   * units are small and equal, so every CTA gets the same share of the work whatever the
//     number of groups (a CTA per group, or a cluster per group, leaves the last wave ragged).
// Unit k of CTA c is sequence entry c + k * gridDim.x.
//   consumer warps (8 or 16): pass 0 forms sums of clamp(x) - shift and its square about the
//     slice's first value, and max |x|, added over the warps; pass 1 normalises, applies the
//     affine map and SiLU (packed f32x2 arithmetic, and no clamps when max |x| and the affine
//     bound show none can bite), and stores.
//   next warp, lane 0 (producer): bulk-copies the CTA's next units into the ring of stages.
//   publisher warp: a slice's partial from the warps' sums; statistics warp: the group's
//     statistics for pass-1 units (both described at the kernel).
// HBM sees one read and one write of x, plus 16 bytes of partial per slice.
// ---------------------------------------------------------------------------------------
// Slice-unit configuration per element size, measured on B200 at (8,512,128,128) (CUDA
// events, same box): f32 48 KB units in 2 stages with 8 consumer warps, two CTAs per SM
// (106 us; 32 KB x 3: 110, 64 KB x 3 with 16 warps and one CTA per SM: 118); 16-bit 64 KB
// units in 3 stages with 16 consumer warps, one CTA per SM (75 us; 32 KB x 3: 78).  Smaller
// units lose to their per-unit waits (16 KB x 6: 198 / 100 us).
template <int ES>
struct SlCfg;
template <>
struct SlCfg<4> {
  static constexpr int kConsumers = 256, kBytes = 49152, kStages = 2, kMinBlocks = 2;
};
template <>
struct SlCfg<2> {
  static constexpr int kConsumers = 512, kBytes = 65536, kStages = 3, kMinBlocks = 1;
};
template <typename T>
struct SlRoles {
  using C = SlCfg<(int)sizeof(T)>;
  static constexpr int kProducerWarp = C::kConsumers / 32;  // after the consumer warps
  static constexpr int kPublisherWarp = kProducerWarp + 1;
  static constexpr int kStatsWarp = kProducerWarp + 2;
  static constexpr int kThreads = C::kConsumers + 3 * 32;
  static constexpr int kEmptyCount = C::kConsumers / 32 + 1;  // consumer warps, publisher
  static constexpr int kSmem = C::kStages * C::kBytes + 128;
};
inline int64_t sl_unit_bytes(int es) { return es == 4 ? SlCfg<4>::kBytes : SlCfg<2>::kBytes; }
constexpr int kStatSlots = 8;  // pass-1 statistics the statistics warp may prepare ahead

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

// pass-0 partials: published with a release add on the group's counter, read after an
// acquire load of it
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded mbarrier wait that parks the warp (try_wait with a suspend-time hint) instead of
// spinning: the streaming kernel's helper warps wait most of the time, and spinning would
// take issue slots from the consumer warps on the same scheduler.
__device__ __forceinline__ bool sl_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                        int code) {
  const long long t0 = clock64();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
        : "memory");
    if (ok) return true;
    if (abort && *abort) return false;
    if (clock64() - t0 > kWaitBudgetCycles) {
      atomicCAS(&g_watchdog, 0, code);
      if (abort) *abort = 1;
      return false;
    }
  }
}
__device__ __forceinline__ bool sl_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort,
                                             int code) {
  return __all_sync(0xffffffffu, sl_wait(bar, parity, abort, code));
}

// Bounded wait until *ready >= want (set by other CTAs of the same launch).
__device__ __forceinline__ bool wait_ready(const unsigned* ready, unsigned want,
                                           volatile int* abort) {
  if (ld_acquire(ready) >= want) return true;
  const long long t0 = clock64();
  while (true) {
    __nanosleep(64);
    if (ld_acquire(ready) >= want) return true;
    if (*abort) return false;
    if (clock64() - t0 > kWaitBudgetCycles) {
      atomicCAS(&g_watchdog, 0, WD_FLAG_WAIT);
      *abort = 1;
      return false;
    }
  }
}

struct GnSliceParams {
  const void* x;
  const void* gamma;
  const void* beta;
  void* y;
  int64_t C, HW, G, cg;  // channels, H*W, groups, channels per group
  int64_t n;             // elements per group = cg * HW
  int64_t BG;            // batch * groups
  int64_t S, L;          // slices per group; pass-1 lag in groups (1 <= L <= BG)
  unsigned* ready;       // [BG] pass-0 slices finished (zero before the launch)
  float4* part;          // [BG][S] (count, mean, M2, max |x|)
  float eps;
  int act;
};

struct SlUnit {
  int pass;
  uint32_t g, s;
};

// Sequence entry u: L*S pass-0 units of groups [0, L); then per t in [L, BG) the S pass-0
// units of group t followed by the S pass-1 units of group t - L; then the pass-1 units of
// groups [BG - L, BG).  The launcher keeps 2 * BG * S below 2^31, so 32-bit arithmetic
// suffices (a 64-bit division is a long subroutine, and every role decodes every unit).
__device__ __forceinline__ SlUnit sl_unit(const GnSliceParams& p, uint32_t u) {
  const uint32_t S = (uint32_t)p.S, L = (uint32_t)p.L, BG = (uint32_t)p.BG;
  const uint32_t head = L * S, mid = 2 * S * (BG - L);
  SlUnit r;
  if (u < head) {
    r.pass = 0;
    r.g = u / S;
    r.s = u - r.g * S;
  } else if (u < head + mid) {
    const uint32_t v = u - head, t = v / (2 * S), w = v - t * 2 * S;
    r.pass = w < S ? 0 : 1;
    r.g = w < S ? L + t : t;
    r.s = w < S ? w : w - S;
  } else {
    const uint32_t v = u - head - mid, q = v / S;
    r.pass = 1;
    r.g = BG - L + q;
    r.s = v - q * S;
  }
  return r;
}

// grid = resident CTAs (cooperative), SlRoles::kThreads threads, dynamic smem SlRoles::kSmem
// (the ring of stages, + alignment).  x, y contiguous NCHW, HW % VE == 0, 16-B aligned.
//
// Per ring stage st, for the unit k the stage holds (k % kSlStages == st):
//   full[st]       the slice landed (producer's bulk copy)
//   empty[st]      the consumer warps and the publisher are done with it
//   part_full[st]  pass 0: the consumer warps wrote their partials to wpart[st]
// and per statistics slot (the CTA's i-th pass-1 unit uses slot i % kStatSlots):
//   stat_full[i]   the statistics warp wrote the group's stats to gstat[i] (and the channel
//                  factors to gaff[i])
//   stat_empty[i]  the consumer warps have read them
// part_full completes once per pass-0 unit of the stage, so its waiters track the phase
// parity per stage.  The consumers and the publisher arrive on empty[st] for every unit, and
// the producer waits for the stage's previous unit to be released before it starts unit k;
// the statistics warp waits for a slot's previous use to be read before it refills it.  So
// no role can be a whole ring (or slot) cycle ahead of or behind a barrier's phase (a parity
// wait would then match the wrong phase).
template <typename T>
__global__ void __launch_bounds__(SlRoles<T>::kThreads, SlCfg<(int)sizeof(T)>::kMinBlocks)
    gn_slice_kernel(GnSliceParams p) {
  using C = SlCfg<(int)sizeof(T)>;
  using R = SlRoles<T>;
  constexpr int kSlConsumers = C::kConsumers, kSlBytes = C::kBytes, kSlStages = C::kStages;
  constexpr int VE = VecTraits<T>::kElems;
  constexpr int kCWarps = kSlConsumers / 32;
  constexpr int64_t kSv = kSlBytes / 16;  // 16-byte vectors per slice
  constexpr int kIt = (int)(kSv / kSlConsumers);  // vectors per consumer thread per slice
  static_assert(kSv % kSlConsumers == 0, "slice vectors per consumer");
  extern __shared__ uint8_t sl_smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sl_smem_raw) + 127) &
                                             ~uintptr_t(127));
  __shared__ uint64_t full[kSlStages], empty[kSlStages], part_full[kSlStages];
  __shared__ uint64_t stat_full[kStatSlots], stat_empty[kStatSlots];
  // per consumer warp: (sum of x - shift, sum of (x - shift)^2, max |x|, unused)
  __shared__ float4 wpart[kSlStages][kCWarps];
  __shared__ float4 gstat[kStatSlots];  // (mean, rstd, max |x|, no_clamp)
  // (gamma[c] * rstd, beta[c]) of the unit's channel when the slice lies in one channel
  __shared__ float2 gaff[kStatSlots];
  __shared__ int abort_flag_s;
  volatile int* abort_flag = &abort_flag_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t total = (uint32_t)(2 * p.BG * p.S);
  const int64_t nvec = p.n / VE;
  const T* gam = static_cast<const T*>(p.gamma);
  const T* bet = static_cast<const T*>(p.beta);
  const uint32_t vpc = (uint32_t)(p.HW / VE);  // vectors per channel
  // slices start at multiples of kSv vectors: when that divides the channel length, no
  // slice straddles two channels
  const bool one_channel = vpc % (uint32_t)kSv == 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSlStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], R::kEmptyCount);
      mbar_init(&part_full[i], kCWarps);
    }
    for (int i = 0; i < kStatSlots; ++i) {
      mbar_init(&stat_full[i], 1);
      mbar_init(&stat_empty[i], kCWarps);
    }
    abort_flag_s = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == R::kProducerWarp) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t keep = l2_policy(true), drop = l2_policy(false);
      uint32_t k = 0;  // units issued
      for (uint32_t u = blockIdx.x; u < total; u += gridDim.x, ++k) {
        const uint32_t st = k % kSlStages;
        if (k >= kSlStages &&
            !sl_wait(&empty[st], ((k / kSlStages) - 1) & 1, abort_flag, WD_TMA_WAIT))
          break;
        const SlUnit un = sl_unit(p, u);
        const int64_t v0 = un.s * kSv;
        const uint32_t bytes = (uint32_t)((min(nvec, v0 + kSv) - v0) * 16);
        const uint8_t* src =
            reinterpret_cast<const uint8_t*>(static_cast<const T*>(p.x) + un.g * p.n) + v0 * 16;
        mbar_arrive_expect_tx(&full[st], bytes);
        // pass-0 bytes are read again by the group's pass-1 units: keep them in L2
        bulk_load(ring + st * kSlBytes, src, bytes, &full[st], un.pass == 0 ? keep : drop);
      }
      // no copy may still be landing when the CTA exits (the consumers may have left early
      // on an expired wait): wait for the last ones issued (bounded)
      for (uint32_t j = k > kSlStages ? k - kSlStages : 0; j < k; ++j)
        sl_wait(&full[j % kSlStages], (j / kSlStages) & 1, nullptr, WD_TMA_WAIT);
    }
    return;
  }

  if (warp == R::kPublisherWarp) {
    // ------------------------------------------------------------------ publisher
    // pass 0: merge the 8 warp partials in warp order into the slice's partial, release the
    // stage, publish the partial and count it on the group's counter.  Every unit: one
    // arrival on empty[st], after full[st] (so it can never count toward the stage's previous
    // phase).
    uint32_t k = 0, pph = 0;  // pph: per-stage part_full parity
    for (uint32_t u = blockIdx.x; u < total; u += gridDim.x, ++k) {
      const uint32_t st = k % kSlStages;
      if (!sl_wait_warp(&full[st], (k / kSlStages) & 1, abort_flag, WD_CONVERT_WAIT)) break;
      const SlUnit un = sl_unit(p, u);
      if (un.pass == 0) {
        if (!sl_wait_warp(&part_full[st], (pph >> st) & 1, abort_flag, WD_CONVERT_WAIT)) break;
        pph ^= 1u << st;
        if (lane == 0) {
          // the consumer warps' shifted sums, in warp order; the shift is the slice's first
          // element (clamped), as the consumers took it
          float t1 = 0.f, t2 = 0.f, am = 0.f;
          for (int i = 0; i < kCWarps; ++i) {
            const float4 b = wpart[st][i];
            t1 += b.x;
            t2 += b.y;
            am = fmaxf(am, b.z);
          }
          float f0[VE];
          unpack<T>(*reinterpret_cast<const uint4*>(ring + st * kSlBytes), f0);
          mbar_arrive(&empty[st]);  // the stage is no longer read
          const int64_t v0 = (int64_t)un.s * kSv;
          const float cnt = (float)((min(nvec, v0 + kSv) - v0) * VE);
          const float m = t1 / cnt;
          p.part[un.g * p.S + un.s] =
              make_float4(cnt, clamp65k(f0[0]) + m, fmaxf(t2 - t1 * m, 0.f), am);
          red_release_add(p.ready + un.g, 1u);
        }
        __syncwarp();
      } else if (lane == 0) {
        mbar_arrive(&empty[st]);
      }
    }
    return;
  }

  if (warp == R::kStatsWarp) {
    // ------------------------------------------------------------------ statistics
    // pass 1, up to kStatSlots units ahead of the consumers: wait for the group's S partials,
    // merge them (lane j takes partials j, j + 32, ... in order, then a fixed xor tree), and
    // hand (mean, rstd, max |x|, no_clamp) and, for a slice inside one channel,
    // (gamma[c] * rstd, beta[c]) to the consumers through slot i % kStatSlots of the CTA's
    // i-th pass-1 unit.
    float gm = 0.f, bm = 0.f;  // max |gamma|, max |beta| over all channels (for no_clamp)
    for (int64_t c = lane; c < p.C; c += 32) {
      gm = fmaxf(gm, fabsf(to_f32(gam[c])));
      bm = fmaxf(bm, fabsf(to_f32(bet[c])));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
      bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
    }
    uint32_t i = 0;  // pass-1 units handled
    for (uint32_t u = blockIdx.x; u < total; u += gridDim.x) {
      const SlUnit un = sl_unit(p, u);
      if (un.pass != 1) continue;
      const uint32_t slot = i % kStatSlots;
      if (i >= kStatSlots && !sl_wait_warp(&stat_empty[slot], ((i / kStatSlots) - 1) & 1,
                                           abort_flag, WD_CONVERT_WAIT))
        break;
      if (!__all_sync(0xffffffffu, wait_ready(p.ready + un.g, (unsigned)p.S, abort_flag)))
        break;
      const float4* gp = p.part + un.g * p.S;
      Welford t{0.f, 0.f, 0.f};
      float am = 0.f;
      for (int64_t j = lane; j < p.S; j += 32) {
        const float4 q = gp[j];
        t = welford_merge(t, Welford{q.x, q.y, q.z});
        am = fmaxf(am, q.w);
      }
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        Welford b{__shfl_xor_sync(0xffffffffu, t.n, o), __shfl_xor_sync(0xffffffffu, t.mean, o),
                  __shfl_xor_sync(0xffffffffu, t.m2, o)};
        // fixed operand order (lower lane first) so both lanes of a pair agree
        t = (lane & o) ? welford_merge(b, t) : welford_merge(t, b);
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
      }
      if (lane == 0) {
        const float rstd = rsqrtf(t.m2 / t.n + p.eps);
        // no clamp can bite when |x| <= 65000 and |(x - mean) * w + b| <= 65000 for all x, c
        const bool no_clamp = am <= kClamp && (am + fabsf(t.mean)) * gm * rstd + bm <= kClamp;
        gstat[slot] = make_float4(t.mean, rstd, am, no_clamp ? 1.f : 0.f);
        if (one_channel) {
          const uint32_t q = un.s * (uint32_t)kSv / vpc;
          const int64_t c = (int64_t)(un.g % p.G) * p.cg + q;
          gaff[slot] = make_float2(to_f32(gam[c]) * rstd, to_f32(bet[c]));
        }
        mbar_arrive(&stat_full[slot]);  // release: gstat / gaff are visible to the waiters
      }
      __syncwarp();
      ++i;
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  // Waits that expire set the shared abort flag; every later wait then returns false at once
  // and the warps leave the unit loop.
  // kSlConsumers vectors = vstep_q channels + vstep_r vectors
  const uint32_t vstep_q = kSlConsumers / vpc, vstep_r = kSlConsumers % vpc;
  uint32_t k = 0, i1 = 0;  // i1: pass-1 units handled (statistics slot i1 % kStatSlots)
  for (uint32_t u = blockIdx.x; u < total; u += gridDim.x, ++k) {
    const uint32_t st = k % kSlStages, ph = (k / kSlStages) & 1;
    const SlUnit un = sl_unit(p, u);
    const int64_t v0 = un.s * kSv;
    const uint32_t cv = (uint32_t)(min(nvec, v0 + kSv) - v0);
    const uint4* sv = reinterpret_cast<const uint4*>(ring + st * kSlBytes);
    if (un.pass == 0) {
      // ---- pass 0: statistics of clamp(x) and max |x| over the slice.  Sums of x - shift
      // about one value common to the whole slice (its first element), so that the threads'
      // partials combine by plain addition; the publisher turns the slice's sums into
      // (count, mean, M2).
      if (!sl_wait_warp(&full[st], ph, abort_flag, WD_CONVERT_WAIT)) break;
      float f0[VE];
      unpack<T>(sv[0], f0);
      const float shift = clamp65k(f0[0]);
      const uint64_t sh2 = f2(shift, shift);
      uint64_t s1 = f2(0.f, 0.f), s2 = s1;
      float amax = 0.f;
#pragma unroll
      for (int it = 0; it < kIt; ++it) {
        const uint32_t i = threadIdx.x + it * kSlConsumers;
        if (i < cv) {
          float f[VE];
          unpack<T>(sv[i], f);
          float vm = fabsf(f[0]);
#pragma unroll
          for (int e = 1; e < VE; ++e) vm = fmaxf(vm, fabsf(f[e]));
          amax = fmaxf(amax, vm);
          if (vm > kClamp) {  // clamp(x) differs from x only above the bound
#pragma unroll
            for (int e = 0; e < VE; ++e) f[e] = clamp65k(f[e]);
          }
#pragma unroll
          for (int e = 0; e < VE; e += 2) {
            const uint64_t d = f2_sub(f2(f[e], f[e + 1]), sh2);
            s1 = f2_add(s1, d);
            s2 = f2_fma(d, d, s2);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
      float a, b;
      f2_split(s1, a, b);
      float t1 = a + b;
      f2_split(s2, a, b);
      float t2 = a + b;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        t1 += __shfl_xor_sync(0xffffffffu, t1, o);
        t2 += __shfl_xor_sync(0xffffffffu, t2, o);
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      }
      if (lane == 0) {
        wpart[st][warp] = make_float4(t1, t2, amax, 0.f);
        mbar_arrive(&part_full[st]);
      }
      continue;
    }

    // ---- pass 1: normalise, affine, activation, store
    const uint32_t slot = i1 % kStatSlots;
    if (!sl_wait_warp(&stat_full[slot], (i1 / kStatSlots) & 1, abort_flag, WD_CONVERT_WAIT))
      break;
    ++i1;
    const float4 gs = gstat[slot];
    const float2 af = gaff[slot];  // published by the same arrival
    __syncwarp();
    if (lane == 0) mbar_arrive(&stat_empty[slot]);  // the slot may be refilled
    const float mean = gs.x, rstd = gs.y;
    const bool no_clamp = gs.w != 0.f;
    if (!sl_wait_warp(&full[st], ph, abort_flag, WD_CONVERT_WAIT)) break;
    const uint64_t mean2 = f2(mean, mean);
    const bool silu = p.act == SP_ACT_SILU;
    // SiLU as y = h + h * tanh(h) with h = v / 2 (= v * sigmoid(v)): the 1/2 folds into the
    // affine map, exactly (a power of two)
    const float hs = silu ? 0.5f : 1.0f;
    const T* gam_g = gam + (un.g % p.G) * p.cg;  // this group's channels
    const T* bet_g = bet + (un.g % p.G) * p.cg;
    uint4* yv = reinterpret_cast<uint4*>(static_cast<T*>(p.y) + un.g * p.n) + v0;
    // normalise vector i of the slice with channel factors (wc, bc) (w2, b2 = the halved
    // factors for the packed SiLU form) and store it
    auto apply_store = [&](uint32_t i, float wc, float bc, uint64_t w2, uint64_t b2) {
      float f[VE];
      unpack<T>(sv[i], f);
      if constexpr (sizeof(T) == 2) {
        if (no_clamp && silu) {
          // 16-bit output: h = v / 2 rounded to the output type, then tanh and h * t + h on
          // packed 16-bit pairs (one MUFU op per two elements); the rounding of h is below
          // the output's own
          uint32_t w[VE / 2];
#pragma unroll
          for (int e = 0; e < VE; e += 2) {
            float h0, h1;
            f2_split(f2_fma(f2_sub(f2(f[e], f[e + 1]), mean2), w2, b2), h0, h1);
            const uint32_t h16 = cvt2_16<T>(h0, h1);
            w[e / 2] = fma2_16<T>(h16, tanh2_16<T>(h16), h16);
          }
          yv[i] = make_uint4(w[0], w[1], w[2], w[3]);
          return;
        }
      }
      if (no_clamp) {
#pragma unroll
        for (int e = 0; e < VE; e += 2) {
          uint64_t h = f2_fma(f2_sub(f2(f[e], f[e + 1]), mean2), w2, b2);
          if (silu) {
            float h0, h1;
            f2_split(h, h0, h1);
            h = f2_fma(h, f2(tanh_approx(h0), tanh_approx(h1)), h);
          }
          f2_split(h, f[e], f[e + 1]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < VE; ++e) f[e] = apply_act((clamp65k(f[e]) - mean) * wc + bc, p.act);
      }
      yv[i] = pack<T>(f);
    };
    if (one_channel) {
      // the slice lies inside one channel: one (gamma * rstd, beta) for the whole unit,
      // prepared by the statistics warp
      const float wc = af.x, bc = af.y;
      const uint64_t w2 = f2(hs * wc, hs * wc), b2 = f2(hs * bc, hs * bc);
#pragma unroll
      for (int it = 0; it < kIt; ++it) {
        const uint32_t i = threadIdx.x + it * kSlConsumers;
        if (i < cv) apply_store(i, wc, bc, w2, b2);
      }
    } else {
      // channel of the thread's vector v0 + i, tracked as (q, rem) = divmod(v0 + i, vpc) and
      // stepped by kSlConsumers vectors per iteration; gamma, beta reloaded when it changes
      uint32_t q = ((uint32_t)v0 + threadIdx.x) / vpc;
      uint32_t rem = ((uint32_t)v0 + threadIdx.x) - q * vpc;
      uint32_t qc = 0xffffffffu;
      float wc = 0.f, bc = 0.f;
      uint64_t w2 = 0, b2 = 0;
#pragma unroll 2
      for (uint32_t i = threadIdx.x; i < cv; i += kSlConsumers) {
        if (q != qc) {
          qc = q;
          wc = to_f32(__ldg(gam_g + q)) * rstd;
          bc = to_f32(__ldg(bet_g + q));
          w2 = f2(hs * wc, hs * wc);
          b2 = f2(hs * bc, hs * bc);
        }
        apply_store(i, wc, bc, w2, b2);
        rem += vstep_r;
        q += vstep_q;
        if (rem >= vpc) {
          rem -= vpc;
          ++q;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
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
  bool stream_path;  // persistent slice-unit grid (large groups)
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
  // slice units are numbered in 32 bits by the streaming kernel
  const int64_t ub = sl_unit_bytes(16 / vec_elems);
  const int64_t stream_units = 2 * B * G * ((group_bytes + ub - 1) / ub);
  if (contiguous && vec_ok && n < (1LL << 31) && group_bytes >= kStreamMinGroupBytes &&
      stream_units < (1LL << 31)) {
    pl.stream_path = true;
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


// Streaming-path workspace: the [BG] ready counters (padded to 16 bytes), then the [BG][S]
// partials.
int64_t sl_slices(int64_t n, int es) { return (n * es + sl_unit_bytes(es) - 1) / sl_unit_bytes(es); }
size_t sl_ready_bytes(int64_t BG) { return ((size_t)BG * 4 + 15) & ~size_t(15); }
size_t sl_workspace_bytes(int64_t BG, int64_t S) {
  return sl_ready_bytes(BG) + (size_t)BG * (size_t)S * 16;
}

template <typename T>
int launch_slices(GnSliceParams p, void* ws, cudaStream_t stream) {
  auto kern = gn_slice_kernel<T>;
  static unsigned long long attr_set = 0;
  if (first_time_on_device(&attr_set)) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SlRoles<T>::kSmem);
    if (e != cudaSuccess) {
      __atomic_fetch_and(&attr_set, ~(1ull << current_device()), __ATOMIC_ACQ_REL);
      return set_error(SP_ERR_LAUNCH, "groupnorm: kernel attribute failed: %s",
                       cudaGetErrorString(e));
    }
  }
  // resident CTAs per SM, found once per device: the grid is exactly the resident set
  // (cooperative launch), so every CTA a pass-1 unit waits on is running
  static int per_sm[64] = {};
  const int dev = current_device();
  int r = (dev >= 0 && dev < 64) ? __atomic_load_n(&per_sm[dev], __ATOMIC_ACQUIRE) : 0;
  if (r <= 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, kern, SlRoles<T>::kThreads,
                                                      SlRoles<T>::kSmem) !=
            cudaSuccess ||
        r <= 0) {
      cudaGetLastError();
      return set_error(SP_ERR_LAUNCH, "groupnorm: occupancy query failed");
    }
    if (dev >= 0 && dev < 64) __atomic_store_n(&per_sm[dev], r, __ATOMIC_RELEASE);
  }
  const int64_t units = 2 * p.BG * p.S;
  const int64_t grid = std::min<int64_t>((int64_t)r * num_sms(), units);
  // four grid-widths of units between a slice's pass 0 and its pass 1
  p.L = std::min<int64_t>(p.BG, std::max<int64_t>(1, (2 * grid + p.S - 1) / p.S));
  p.ready = static_cast<unsigned*>(ws);
  p.part = reinterpret_cast<float4*>(static_cast<uint8_t*>(ws) + sl_ready_bytes(p.BG));
  cudaError_t e = cudaMemsetAsync(p.ready, 0, (size_t)p.BG * 4, stream);
  if (e != cudaSuccess)
    return set_error(SP_ERR_LAUNCH, "groupnorm: counter reset failed: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(SlRoles<T>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = SlRoles<T>::kSmem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess)
    return set_error(SP_ERR_LAUNCH, "groupnorm slice launch (grid %lld) failed: %s",
                     (long long)grid, cudaGetErrorString(e));
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
  if (pl.stream_path)
    return sp::sl_workspace_bytes(B * groups, sp::sl_slices(C / groups * H * W, es));
  return pl.cluster_path ? 0 : sp::general_workspace_bytes(B, C, H, W, groups);
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
    const int64_t S = sl_slices(n, es);
    const size_t need = sl_workspace_bytes(B * groups, S);
    if (!workspace || workspace_bytes < need)
      return set_error(SP_ERR_WORKSPACE,
                       "groupnorm: this shape takes the streaming path and needs %zu bytes of "
                       "workspace (got %zu)",
                       need, workspace_bytes);
    if (!aligned(workspace, 16)) return set_error(SP_ERR_ALIGN, "groupnorm: workspace misaligned");
    GnSliceParams p{x, gamma, beta, y, C, HW, groups, cg, n, B * groups, S, 1, nullptr, nullptr,
                    eps, act};
    switch (dtype) {
      case SP_F32: return launch_slices<float>(p, workspace, s);
      case SP_F16: return launch_slices<__half>(p, workspace, s);
      default: return launch_slices<__nv_bfloat16>(p, workspace, s);
    }
  }
  if (pl.cluster_path) {
    GnParams p{x, gamma, beta, y, C, HW, groups, cg, n, pl.chunk_vecs, eps, act};
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
