// quant_linear.cu -- y = x . dequant(W)^T (+ bias) with the weight decode fused into the
// mainloop of a tcgen05 GEMM (sm_100a).
//
// Replaces GpuQuantizedLinear::forward (crates/sketchpad-cubecl/src/quantized_matmul.rs:752-766),
// which materialises the whole dequantized matrix and then runs a separate matmul, and
// Fp8Linear::forward (crates/sketchpad-core/src/quantization.rs:601-609).
//
// CTA tile: 256 rows of x (two UMMA M=128 halves) x 256 weight rows (UMMA N), K in steps of
// 64.  Every decoded weight tile feeds both halves, so one decode serves 2*256 FLOPs per weight.
//   warp 0       TMA: x tile (bf16, 128B swizzle), raw 8-bit weight tile and (Q8_0) the
//                k-tile's block scales, RAW_STAGES deep.
//   warp 1       TMEM owner (512 columns: two 128 x 256 f32 accumulators) + MMA issuer.
//   warps 2, 3   idle (the block is sized in whole warpgroups).
//   warps 4..19  decoders: raw 8-bit tile -> bf16 tile in the UMMA K-major 128B-swizzled
//                layout (Q8_0: f16 block scale * int8; FP8: exact e4m3 -> bf16), CVT_STAGES
//                deep (16 warps: two per scheduler, so decode latency overlaps); then the
//                epilogue, each warp one (TMEM lane quarter, M half, column half): TMEM ->
//                per-channel scale, bias [, RoPE] [, gate, residual] -> bf16 -> HBM.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "quant_codec.cuh"
#include "tc.cuh"

namespace sp {
namespace {

constexpr int kQBM = 256, kQHalf = 128, kQBN = 256, kQBK = 64;
constexpr int kQThreads = 640, kQDecoders = 512, kQFirstDecoderWarp = 4;
constexpr int kXBytes = kQBM * kQBK * 2;    // 32 KB
constexpr int kWCvtBytes = kQBN * kQBK * 2; // 32 KB

// W_BF16: plain bf16 weights (the UNet's projections and feed-forward), loaded by TMA straight
// into the UMMA K-major 128B-swizzled layout -- no decode stage; the decoder warps only run the
// epilogue, and each stage holds x and W tiles of 32 KB each.
enum WFormat : int { W_Q8_0 = 0, W_FP8 = 1, W_Q4K = 2, W_Q2K = 3, W_Q3K = 4, W_BF16 = 5 };

// K-quant formats: one 4-bit quant per value (32 bytes per row of a k-tile), f32 factors a, b
// per sub-block of kSub values; w = a * (q - kOff) - b.
// ROWS: weight rows of a CTA's tile.
template <int WF, int ROWS = kQBN>
struct KqFmt {
  static constexpr bool kIsK = WF >= W_Q4K && WF <= W_Q3K;
  enum : int {
    kSub = WF == W_Q4K ? 32 : 16,
    kOff = WF == W_Q3K ? 4 : 0,
    kFactorRows = kQBK / kSub,              // sub-blocks per k-tile
    kQBytes = ROWS * kQBK / 2,              // nibbles (8 KB for 256 rows)
    kFactorBytes = kFactorRows * ROWS * 4,  // one factor array
  };
};

// Paired mode (PAIR): a cluster of two CTAs computes a 512 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256 per instruction, 128 rows from each CTA's x tile).  The
// instruction takes B's 256 columns from both CTAs' shared memory, 128 each, and leaves each
// CTA's 128 rows x all 256 columns in its own TMEM.  So each CTA loads its own 256 x rows as
// in unpaired mode but decodes only 128 of the 256 weight rows: half the decode work and half
// the B-operand shared-memory reads per SM, the stream that limits the unpaired kernel.
//
// Three rings: x tiles (consumed by the MMA), raw 8-bit weights with their scales or factors
// (consumed by the decoders), decoded weights (consumed by the MMA).  The raw-weight ring is
// released by the decoders alone, so weight loads run ahead of the MMA by the whole ring
// instead of waiting for the MMA that shares a stage with them: measured, a shared x + W
// ring made the loop TMA latency -> decode -> MMA -> release the bound (~1,530 SM cycles per
// k-tile against 1,024 of tensor work).
template <bool PAIR>
struct QlGeom {
  static constexpr int kWRows = PAIR ? kQBN / 2 : kQBN;  // weight rows this CTA decodes
  static constexpr int kXSt = PAIR ? 4 : 3;               // x stages
  static constexpr int kWSt = PAIR ? 4 : 3;               // raw-weight stages
  static constexpr int kCvt = PAIR ? 3 : 2;               // decoded-weight stages
  static constexpr int kWRawB = kWRows * kQBK;            // 8-bit weights of a k-tile
  static constexpr int kScB = 2 * kWRows * 2;             // Q8_0: two k-blocks of f16 scales
  static constexpr int kWStage = kWRawB + kScB;           // raw weights, then the scales
  static constexpr int kWCvtB = kWRows * kQBK * 2;        // decoded bf16 weights
  static constexpr int kNumBars = 2 * (kXSt + kWSt + kCvt) + 2;
};

template <bool PAIR>
struct QlSmemT {
  using G = QlGeom<PAIR>;
  static constexpr int kX = 0;
  static constexpr int kWRaw = kX + G::kXSt * kXBytes;
  static constexpr int kWCvt = kWRaw + G::kWSt * G::kWStage;
  static constexpr int kBar = kWCvt + G::kCvt * G::kWCvtB;
  static constexpr int kMisc = kBar + G::kNumBars * 8;
  static constexpr int kAlloc = kMisc + 16 + 1024;
};
using QlSmem = QlSmemT<false>;

// W_BF16: the x ring's stages hold {x tile, bf16 W tile} (3 x 64 KB); no decode
struct QlSmemBf16 {
  static constexpr int kStage = kXBytes + kWCvtBytes;
  static constexpr int kX = 0;
  static constexpr int kW = kXBytes;
  static constexpr int kBar = QlGeom<false>::kXSt * kStage;
  static constexpr int kMisc = kBar + QlGeom<false>::kNumBars * 8;
  static constexpr int kAlloc = kMisc + 16 + 1024;
};

struct QlParams {
  int64_t M, N, K;
  const uint16_t* q8_scale;  // Q8_0: [K/32, N] f16 bits (loaded by TMA)
  const float* fp8_scale;    // FP8: [N] or [1]
  int64_t nscale;
  const float* kq_a;         // K-quants: factors a, b [K/sub, N] (loaded by TMA)
  const float* kq_b;
  const __nv_bfloat16* bias;  // [N] or null
  __nv_bfloat16* y;           // [M, ldy]: columns [0, N) written
  // epilogue y = residual + gate[n] * rope(x.W^T + bias): the DiT blocks' gated residual
  const __nv_bfloat16* gate;      // [N] or null (gate 1)
  const __nv_bfloat16* residual;  // [M, ldy] or null; may alias y
  int64_t ldy;                    // row stride of y and residual (elements, >= N)
  // rotary embedding of the attention projections (rope.rs:145-170) on columns
  // [0, rope_cols): head_dim-wide heads whose (even, odd) column pairs rotate by the angle of
  // position ((m + rope_off) / rope_div) % rope_mod; rope = {cos, sin} per (position, pair)
  const float2* rope;             // [positions, head_dim / 2] or null
  int64_t rope_off, rope_div, rope_mod;
  int rope_cols, rope_half;
  // split-K (grid.y = splits > 1): CTA z sums k-tiles [z * kt_per_split, ...) and writes its
  // raw f32 partial to ws[z][M][N]; a reduce pass sums them in order and runs the epilogue
  float* ws;
  int splits, kt_per_split;
  // GLU epilogue (-1: none): weight rows interleaved as (first-half row j, second-half row j),
  // so columns 2j, 2j+1 of x.W^T + b are (lo, hi) and y[m, j] = lo * gelu(hi) (SP_GLU_GEGLU)
  // or silu(lo) * hi (SP_GLU_SWIGLU); y holds N/2 columns, ldy apart
  int glu;
  // y's element type for the plain / rope epilogue: 0 bf16, 1 f16 (the attention inputs of
  // long-sequence DiTs, where f16's 3 extra mantissa bits shrink the logit error 8x)
  int y_f16;
  // tile raster: grid.x walks tiles_m x tiles_n in groups of `group` tiles along one axis
  // (raster_n 0: groups of m-tiles, m fastest inside a group, so the group's x rows stay in
  // L2 while W streams past them; 1: groups of n-tiles, n fastest, W held and x streamed)
  int tiles_m, tiles_n, group, raster_n;
};

// (m-tile, n-tile) of linear tile t under the grouped raster above
__device__ __forceinline__ void ql_tile_of(const QlParams& p, int t, int& mt, int& nt) {
  const int outer = p.raster_n ? p.tiles_n : p.tiles_m;  // grouped axis
  const int inner = p.raster_n ? p.tiles_m : p.tiles_n;
  const int per_group = p.group * inner;
  const int g = t / per_group;
  const int first = g * p.group;
  const int width = min(outer - first, p.group);
  const int r = t - g * per_group;
  const int a = first + r % width, b = r / width;
  mt = p.raster_n ? b : a;
  nt = p.raster_n ? a : b;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// packed f32x2 operands: two f32 in one 64-bit register pair
__device__ __forceinline__ uint64_t pk2(uint32_t a, uint32_t b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_of(uint64_t v) {
  uint32_t a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(a), "=r"(b) : "l"(v));
  return pack_bf16x2(__uint_as_float(a), __uint_as_float(b));
}
// 4 int8 (one u32) * f32 scale -> 2 x bf16x2 (exact int8 -> f32 via the 2^23 magic number),
// two lanes per packed f32x2 instruction.
__device__ __forceinline__ void q8x4_to_bf16(uint32_t w, float s, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;  // int8 -> biased uint8 (q + 128)
  const uint64_t magic = pk2(0x4B000080u, 0x4B000080u);  // 2^23 + 128
  const uint64_t s2 = pk2(__float_as_uint(s), __float_as_uint(s));
  uint64_t a = pk2(prmt(u, 0x4B000000u, 0x7650), prmt(u, 0x4B000000u, 0x7651));
  uint64_t b = pk2(prmt(u, 0x4B000000u, 0x7652), prmt(u, 0x4B000000u, 0x7653));
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(a) : "l"(a), "l"(magic));
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(b) : "l"(b), "l"(magic));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(a) : "l"(a), "l"(s2));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(b) : "l"(b), "l"(s2));
  lo = bf16x2_of(a);
  hi = bf16x2_of(b);
}

// 8 nibbles (values 0..7 of a group in k order: byte j holds values 2j, 2j+1 in its low and
// high nibble) -> 4 x bf16x2 of a * (q - off) - b, the product and difference each rounded
// in f32 (packed f32x2, no contraction) as the reference's decode computes them.
__device__ __forceinline__ void k4x8_to_bf16(uint32_t w, float a, float b, int off, uint32_t& o0,
                                             uint32_t& o1, uint32_t& o2, uint32_t& o3) {
  const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
  const uint32_t u0 = prmt(lo, hi, 0x5140);  // values 0..3 as bytes
  const uint32_t u1 = prmt(lo, hi, 0x7362);  // values 4..7
  const float m = 8388608.0f + (float)off;   // 2^23 + off: q - off exactly
  const uint64_t magic = pk2(__float_as_uint(m), __float_as_uint(m));
  const uint64_t a2 = pk2(__float_as_uint(a), __float_as_uint(a));
  const uint64_t b2 = pk2(__float_as_uint(b), __float_as_uint(b));
  uint64_t v[4] = {pk2(prmt(u0, 0x4B000000u, 0x7650), prmt(u0, 0x4B000000u, 0x7651)),
                   pk2(prmt(u0, 0x4B000000u, 0x7652), prmt(u0, 0x4B000000u, 0x7653)),
                   pk2(prmt(u1, 0x4B000000u, 0x7650), prmt(u1, 0x4B000000u, 0x7651)),
                   pk2(prmt(u1, 0x4B000000u, 0x7652), prmt(u1, 0x4B000000u, 0x7653))};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(v[i]) : "l"(v[i]), "l"(magic));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(v[i]) : "l"(v[i]), "l"(a2));
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(v[i]) : "l"(v[i]), "l"(b2));
  }
  o0 = bf16x2_of(v[0]);
  o1 = bf16x2_of(v[1]);
  o2 = bf16x2_of(v[2]);
  o3 = bf16x2_of(v[3]);
}

// 4 e4m3 bytes -> 2 x bf16x2, exact: the e4m3 bit pattern is placed in bf16 position
// (exponent bias 7 instead of 127) and multiplied by 2^120; e4m3 subnormals land on bf16
// subnormals and are scaled exactly as well.
__device__ __forceinline__ void e4m3x4_to_bf16(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t a = prmt(w, 0u, 0x4140);  // b0 | b1 << 16
  const uint32_t b = prmt(w, 0u, 0x4342);  // b2 | b3 << 16
  const uint32_t ta = ((a & 0x007F007Fu) << 4) | ((a & 0x00800080u) << 8);
  const uint32_t tb = ((b & 0x007F007Fu) << 4) | ((b & 0x00800080u) << 8);
  const uint32_t k2p120 = 0x7B807B80u;  // bf16x2 {2^120, 2^120}
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(lo) : "r"(ta), "r"(k2p120));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(hi) : "r"(tb), "r"(k2p120));
}

__device__ __forceinline__ float ql_gelu_erf(float g) {
  return 0.5f * g * (1.0f + erff(g * 0.70710678118654752f));
}
// x * sigmoid(x) with an IEEE division, as the reference's silu
__device__ __forceinline__ float ql_silu(float g) { return g / (1.0f + expf(-g)); }

// Eight bf16 values a[n .. n+7] as f32: one 16-byte load when the address allows it (n is a
// multiple of 8 here, so that is when the array itself is 16-byte aligned).
__device__ __forceinline__ void ql_load8(const __nv_bfloat16* a, int64_t n, float (&o)[8]) {
  if ((reinterpret_cast<uintptr_t>(a) & 15) == 0) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(a + n));
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __bfloat162float(h[e]);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __bfloat162float(a[n + e]);
  }
}

// The epilogue of 8 accumulator values with its operands already at hand: bias and gate as f32
// (null: none), the residual's 8 bf16 values (used when p.residual is set).
template <int WF>
__device__ __forceinline__ void ql_finish8_with(const QlParams& p, float (&v)[8], int64_t m,
                                                int64_t n, const float2* rope_row,
                                                const float* bv, const float* gv, uint4 rv) {
  if (p.glu >= 0) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if constexpr (WF == W_FP8) v[e] *= p.fp8_scale[p.nscale == 1 ? 0 : n + e];
      if (bv) v[e] += bv[e];
    }
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o[j] = p.glu == SP_GLU_GEGLU ? v[2 * j] * ql_gelu_erf(v[2 * j + 1])
                                   : ql_silu(v[2 * j]) * v[2 * j + 1];
    *reinterpret_cast<uint2*>(p.y + m * p.ldy + n / 2) =
        make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
    return;
  }
  const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    if constexpr (WF == W_FP8) v[e] *= p.fp8_scale[p.nscale == 1 ? 0 : n + e];
    if (bv) v[e] += bv[e];
  }
  if (rope_row && n < p.rope_cols) {
    // x*cos + rotate_half(x)*sin, rotate_half([x0, x1]) = [-x1, x0]; 8 | head_dim, so the
    // group's 4 pairs sit in one head
    const float2* cs = rope_row + (int)(n % (2 * p.rope_half)) / 2;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = cs[e];
      const float x0 = v[2 * e], x1 = v[2 * e + 1];
      v[2 * e] = x0 * t.x - x1 * t.y;
      v[2 * e + 1] = x1 * t.x + x0 * t.y;
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    if (gv) v[e] *= gv[e];
    if (p.residual) v[e] += __bfloat162float(re[e]);
  }
  *reinterpret_cast<uint4*>(p.y + m * p.ldy + n) =
      p.y_f16 ? make_uint4(pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]),
                           pack_f16x2(v[4], v[5]), pack_f16x2(v[6], v[7]))
              : make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                           pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

// Epilogue of 8 consecutive accumulator values of row m, columns n .. n+7, loading its own
// operands: FP8 per-channel scale, bias, then either the GLU (4 outputs at column n/2) or
// optional RoPE, gate and residual, bf16 (or f16) store.
template <int WF>
__device__ __forceinline__ void ql_finish8(const QlParams& p, float (&v)[8], int64_t m, int64_t n,
                                           const float2* rope_row) {
  float bv[8], gv[8];
  if (p.bias) ql_load8(p.bias, n, bv);
  if (p.gate && p.glu < 0) ql_load8(p.gate, n, gv);
  uint4 rv = make_uint4(0, 0, 0, 0);
  if (p.residual && p.glu < 0) rv = *reinterpret_cast<const uint4*>(p.residual + m * p.ldy + n);
  ql_finish8_with<WF>(p, v, m, n, rope_row, p.bias ? bv : nullptr,
                      p.gate && p.glu < 0 ? gv : nullptr, rv);
}

// Split-K reduce: out[m, n..n+7] = epilogue(sum over z of ws[z][m][n..n+7]), z in order, one
// thread per 8 outputs.
template <int WF>
__global__ void __launch_bounds__(256) ql_splitk_reduce_kernel(const QlParams p) {
  const int64_t groups = p.M * (p.N / 8);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < groups;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / (p.N / 8), n = (i - m * (p.N / 8)) * 8;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int z = 0; z < p.splits; ++z) {
      const float* src = p.ws + ((int64_t)z * p.M + m) * p.N + n;
      const float4 a = *reinterpret_cast<const float4*>(src);
      const float4 b = *reinterpret_cast<const float4*>(src + 4);
      v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
      v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
    }
    const float2* rope_row =
        p.rope ? p.rope + ((m + p.rope_off) / p.rope_div % p.rope_mod) * p.rope_half : nullptr;
    ql_finish8<WF>(p, v, m, n, rope_row);
  }
}

// Shared-memory barrier helpers of the paired mode: a peer CTA's barrier is addressed through
// the cluster window (mapa), arrivals from the peer are released at cluster scope, and the
// leader acquires them at cluster scope.
__device__ __forceinline__ uint32_t ql_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t ql_peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void ql_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void ql_store_remote(uint32_t cluster_addr, int v) {
  asm volatile("st.relaxed.cluster.shared::cluster.s32 [%0], %1;" ::"r"(cluster_addr), "r"(v)
               : "memory");
}
// Bounded wait that acquires at cluster scope (arrivals made by the peer CTA).
__device__ __forceinline__ bool ql_wait_cluster(uint64_t* bar, uint32_t parity,
                                                volatile int* abort, int code) {
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
        atomicCAS(&g_watchdog, 0, code);
        *abort = 1;
        return false;
      }
    }
  }
}
__device__ __forceinline__ void ql_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// tcgen05 forms of the pair (cta_group::2): TMEM allocation by one warp in each CTA, MMA issued
// by the leader, commits arriving on a barrier of either CTA (cluster address)
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void umma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_addr) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          cluster_addr)
      : "memory");
}

template <int WF, bool PAIR>
__global__ void __launch_bounds__(kQThreads, 1)
    qlinear_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                   const __grid_constant__ CUtensorMap tms, const __grid_constant__ CUtensorMap tmb,
                   const QlParams p) {
  static_assert(!(PAIR && WF == W_BF16), "bf16 weights run unpaired");
  using G = QlGeom<PAIR>;
  using L = typename std::conditional<WF == W_BF16, QlSmemBf16, QlSmemT<PAIR>>::type;
  using LQ = QlSmemT<PAIR>;  // stage offsets of the decoded formats
  using KF = KqFmt<WF, G::kWRows>;
  constexpr int kXSt = G::kXSt, kWSt = G::kWSt, kCvtSt = G::kCvt;
  constexpr int kWR = G::kWRows;                    // weight rows this CTA loads and decodes
  constexpr int kDecWarps = kQDecoders / 32;
  // K-quants: a raw stage holds the nibble tile, then factor arrays a and b
  static_assert(KF::kQBytes + 2 * KF::kFactorBytes <= G::kWRawB, "k-quant raw stage");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* x_full = bars;                // x tile (bf16 weights: and the W tile) landed
  uint64_t* x_empty = x_full + kXSt;      // the MMA read it
  uint64_t* w_full = x_empty + kXSt;      // raw weights (+ scales / factors) landed
  uint64_t* w_empty = w_full + kWSt;      // the decoder warps read them
  uint64_t* cvt_full = w_empty + kWSt;    // decoded weights written
  uint64_t* cvt_empty = cvt_full + kCvtSt;  // the MMA read them
  uint64_t* acc_full = cvt_empty + kCvtSt;
  uint64_t* drain = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // pair: rank 0 (the leader) issues the MMAs of both CTAs
  const uint32_t rank = PAIR ? ql_cluster_rank() : 0u;
  const uint32_t peer = rank ^ 1u;
  int mtile, ntile;
  ql_tile_of(p, PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x, mtile, ntile);
  const int m0 = mtile * (PAIR ? 2 * kQBM : kQBM) + (int)rank * kQBM;  // this CTA's x rows
  const int n0 = ntile * kQBN;                                         // the tile's columns
  const int nw0 = n0 + (int)rank * kWR;                                // this CTA's W rows
  // this CTA's k-tiles (all of them without split-K); kt below counts from 0
  const int kbase = (int)blockIdx.y * p.kt_per_split;
  const int ktiles = min((int)(p.K / kQBK) - kbase, p.kt_per_split);
  // an expired wait stops this CTA and, paired, its peer (whose waits would else run out too)
  auto fail = [&]() {
    *abort_flag = 1;
    if constexpr (PAIR) ql_store_remote(ql_peer_addr((const void*)abort_flag, peer), 1);
  };

  constexpr bool kBf16 = WF == W_BF16;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kXSt; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);  // MMA commit
    }
    for (int s = 0; s < kWSt; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], kDecWarps);
    }
    for (int s = 0; s < kCvtSt; ++s) {
      // this CTA's decoder warps; the leader's also takes the peer's forwarded arrival
      mbar_init(&cvt_full[s], PAIR && rank == 0 ? kDecWarps + 1 : kDecWarps);
      mbar_init(&cvt_empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  // paired: the peer's barriers, abort flag and TMEM must exist before either CTA uses them
  if constexpr (PAIR) ql_cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ x producer
    if (lane == 0) {
      tma_prefetch_desc(&tmx);
      tma_prefetch_desc(&tmw);
      if constexpr (WF == W_Q8_0 || KF::kIsK) tma_prefetch_desc(&tms);
      if constexpr (KF::kIsK) tma_prefetch_desc(&tmb);
      constexpr uint32_t kTx = kBf16 ? kXBytes + kWCvtBytes : kXBytes;
      int issued = 0;
      for (int kt = 0; kt < ktiles; ++kt) {
        const int st = kt % kXSt;
        if (kt >= kXSt &&
            !mbar_wait(&x_empty[st], ((kt / kXSt) - 1) & 1, abort_flag, WD_TMA_WAIT)) {
          fail();
          break;
        }
        mbar_arrive_expect_tx(&x_full[st], kTx);
        if constexpr (kBf16) {
          uint8_t* stage = smem + st * QlSmemBf16::kStage;
          tma_load_2d(stage + QlSmemBf16::kX, &tmx, &x_full[st], (kbase + kt) * kQBK, m0);
          tma_load_2d(stage + QlSmemBf16::kW, &tmw, &x_full[st], (kbase + kt) * kQBK, n0);
        } else {
          tma_load_2d(smem + LQ::kX + st * kXBytes, &tmx, &x_full[st], (kbase + kt) * kQBK, m0);
        }
        issued = kt + 1;
      }
      if (*abort_flag)  // let the copies in flight land before the CTA can exit (bounded)
        for (int kt = max(0, issued - kXSt); kt < issued; ++kt)
          mbar_wait(&x_full[kt % kXSt], (kt / kXSt) & 1, nullptr, WD_TMA_WAIT);
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ weight producer
    if (lane == 0 && !kBf16) {
      constexpr uint32_t kTx = KF::kIsK ? KF::kQBytes + 2 * KF::kFactorBytes
                                        : G::kWRawB + (WF == W_Q8_0 ? G::kScB : 0);
      int issued = 0;
      for (int kt = 0; kt < ktiles; ++kt) {
        const int st = kt % kWSt;
        if (kt >= kWSt &&
            !mbar_wait(&w_empty[st], ((kt / kWSt) - 1) & 1, abort_flag, WD_TMA_WAIT)) {
          fail();
          break;
        }
        mbar_arrive_expect_tx(&w_full[st], kTx);
        uint8_t* rw = smem + LQ::kWRaw + st * G::kWStage;
        if constexpr (KF::kIsK) {
          tma_load_2d(rw, &tmw, &w_full[st], (kbase + kt) * (kQBK / 2), nw0);
          tma_load_2d(rw + KF::kQBytes, &tms, &w_full[st], nw0, (kbase + kt) * KF::kFactorRows);
          tma_load_2d(rw + KF::kQBytes + KF::kFactorBytes, &tmb, &w_full[st], nw0,
                      (kbase + kt) * KF::kFactorRows);
        } else {
          tma_load_2d(rw, &tmw, &w_full[st], (kbase + kt) * kQBK, nw0);
          if constexpr (WF == W_Q8_0)
            tma_load_2d(rw + G::kWRawB, &tms, &w_full[st], nw0, (kbase + kt) * (kQBK / 32));
        }
        issued = kt + 1;
      }
      if (*abort_flag)  // let the copies in flight land before the CTA can exit (bounded)
        for (int kt = max(0, issued - kWSt); kt < issued; ++kt)
          mbar_wait(&w_full[kt % kWSt], (kt / kWSt) & 1, nullptr, WD_TMA_WAIT);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA (the leader, paired)
    if (lane == 0 && rank == 0) {
      // paired: M = 256 per instruction (this CTA's 128 rows of a half, then the peer's)
      const uint32_t idesc = make_idesc_f16(PAIR ? 2 * kQHalf : kQHalf, kQBN, 1u, 0, 0);
      bool ok = true;
      for (int kt = 0; kt < ktiles; ++kt) {
        const int xs = kt % kXSt, cs = kt % kCvtSt;
        bool got = mbar_wait(&x_full[xs], (kt / kXSt) & 1, abort_flag, WD_MMA_WAIT);
        // paired: the peer's x tile and decoded stage are forwarded here by its warp 2
        if (got && !kBf16)
          got = PAIR ? ql_wait_cluster(&cvt_full[cs], (kt / kCvtSt) & 1, abort_flag, WD_MMA_WAIT)
                     : mbar_wait(&cvt_full[cs], (kt / kCvtSt) & 1, abort_flag, WD_MMA_WAIT);
        if (!got) {
          fail();
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t xa, wb;
        if constexpr (kBf16) {
          xa = smem_u32(smem + xs * QlSmemBf16::kStage + QlSmemBf16::kX);
          wb = smem_u32(smem + xs * QlSmemBf16::kStage + QlSmemBf16::kW);
        } else {
          xa = smem_u32(smem + LQ::kX + xs * kXBytes);
          wb = smem_u32(smem + LQ::kWCvt + cs * G::kWCvtB);
        }
#pragma unroll
        for (int kk = 0; kk < kQBK / 16; ++kk) {
          const uint64_t b = make_smem_desc(wb + kk * 32, 16, 1024, LAYOUT_SW128);
          const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
          // rows 0..127 and 128..255 of the x tile (16 KB apart, whole swizzle atoms)
          const uint64_t a0 = make_smem_desc(xa + kk * 32, 16, 1024, LAYOUT_SW128);
          const uint64_t a1 = make_smem_desc(xa + kQHalf * 128 + kk * 32, 16, 1024, LAYOUT_SW128);
          if constexpr (PAIR) {
            umma_ss_pair(tmem, a0, b, idesc, acc);
            umma_ss_pair(tmem + kQBN, a1, b, idesc, acc);
          } else {
            umma_ss(tmem, a0, b, idesc, acc);
            umma_ss(tmem + kQBN, a1, b, idesc, acc);
          }
        }
        if constexpr (PAIR) {
          umma_commit_pair(smem_u32(&x_empty[xs]));
          umma_commit_pair(ql_peer_addr(&x_empty[xs], peer));
          umma_commit_pair(smem_u32(&cvt_empty[cs]));
          umma_commit_pair(ql_peer_addr(&cvt_empty[cs], peer));
        } else {
          umma_commit(&x_empty[xs]);
          if constexpr (!kBf16) umma_commit(&cvt_empty[cs]);
        }
      }
      if constexpr (PAIR) {
        if (ok) {
          umma_commit_pair(smem_u32(acc_full));
          umma_commit_pair(ql_peer_addr(acc_full, peer));
        }
        umma_commit_pair(smem_u32(drain));
      } else {
        if (ok) umma_commit(acc_full);
        umma_commit(drain);
      }
      mbar_wait(drain, 0, nullptr, WD_MMA_WAIT);
    }
  } else if (PAIR && warp == 2) {
    // paired, peer only: once this CTA's x tile has landed and its decoder warps have
    // written the stage, tell the leader with ONE cluster-scope release arrival (one per
    // decoder warp would put a cluster-wide fence on every decoder warp's path)
    if (lane == 0 && rank != 0 && !kBf16) {
      const uint32_t leader_cvt_full = ql_peer_addr(cvt_full, 0u);
      for (int kt = 0; kt < ktiles; ++kt) {
        const int xs = kt % kXSt, cs = kt % kCvtSt;
        if (!mbar_wait(&x_full[xs], (kt / kXSt) & 1, abort_flag, WD_CONVERT_WAIT) ||
            !mbar_wait(&cvt_full[cs], (kt / kCvtSt) & 1, abort_flag, WD_CONVERT_WAIT)) {
          fail();
          break;
        }
        ql_arrive_remote(leader_cvt_full + (uint32_t)(cs * 8));
      }
    }
  } else if (warp >= kQFirstDecoderWarp) {
    // ------------------------------------------------------------ decoders
    const int t = threadIdx.x - kQFirstDecoderWarp * 32;  // 0..511
    bool ok = true;
    for (int kt = 0; kt < (kBf16 ? 0 : ktiles); ++kt) {
      const int ws = kt % kWSt, cs = kt % kCvtSt;
      // warp-uniform waits: the warp arrives once per stage, after __syncwarp
      if (!mbar_wait_warp(&w_full[ws], (kt / kWSt) & 1, abort_flag, WD_CONVERT_WAIT) ||
          (kt >= kCvtSt && !mbar_wait_warp(&cvt_empty[cs], ((kt / kCvtSt) - 1) & 1, abort_flag,
                                           WD_CONVERT_WAIT))) {
        fail();
        ok = false;
        break;
      }
      const uint8_t* raw = smem + LQ::kWRaw + ws * G::kWStage;
      const __half* sc = reinterpret_cast<const __half*>(raw + G::kWRawB);
      uint8_t* cvt = smem + LQ::kWCvt + cs * G::kWCvtB;
#pragma unroll 2
      for (int it = 0; it < (kWR * 4) / kQDecoders; ++it) {
        const int task = t + it * kQDecoders;
        const int row = task >> 2, ch = task & 3;  // 16 weights: k = 16*ch .. 16*ch+15
        uint32_t o[8];
        if constexpr (KF::kIsK) {
          // 16 nibbles (8 bytes); rows past N read TMA zero fill: a = b = 0, weights 0
          const uint2 w = *reinterpret_cast<const uint2*>(raw + row * 32 + ch * 8);
          const float* fa = reinterpret_cast<const float*>(raw + KF::kQBytes);
          const int sb = (ch * 16) / KF::kSub;
          const float a = fa[sb * kWR + row];
          const float b = fa[KF::kFactorRows * kWR + sb * kWR + row];
          k4x8_to_bf16(w.x, a, b, KF::kOff, o[0], o[1], o[2], o[3]);
          k4x8_to_bf16(w.y, a, b, KF::kOff, o[4], o[5], o[6], o[7]);
        } else {
          const uint4 w = *reinterpret_cast<const uint4*>(raw + row * 64 + ch * 16);
          if constexpr (WF == W_Q8_0) {
            // rows past N read TMA zero fill: scale 0, weights 0
            const float s = __half2float(sc[(ch >> 1) * kWR + row]);
            q8x4_to_bf16(w.x, s, o[0], o[1]);
            q8x4_to_bf16(w.y, s, o[2], o[3]);
            q8x4_to_bf16(w.z, s, o[4], o[5]);
            q8x4_to_bf16(w.w, s, o[6], o[7]);
          } else {
            e4m3x4_to_bf16(w.x, o[0], o[1]);
            e4m3x4_to_bf16(w.y, o[2], o[3]);
            e4m3x4_to_bf16(w.z, o[4], o[5]);
            e4m3x4_to_bf16(w.w, o[6], o[7]);
          }
        }
        // bf16 row of 64 = eight 16-byte chunks; this task fills chunks 2*ch and 2*ch+1
        uint8_t* rowp = cvt + row * 128;
        *reinterpret_cast<uint4*>(rowp + (((2 * ch) ^ (row & 7)) << 4)) =
            make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(rowp + (((2 * ch + 1) ^ (row & 7)) << 4)) =
            make_uint4(o[4], o[5], o[6], o[7]);
      }
      // every lane's writes -> async proxy, then one arrival per warp
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&w_empty[ws]);
        mbar_arrive(&cvt_full[cs]);  // paired peer: forwarded to the leader by warp 2
      }
    }

    // ------------------------------------------------------------ epilogue
    if (__all_sync(0xffffffffu, ok) && mbar_wait_warp(acc_full, 0, abort_flag, WD_EPILOGUE_WAIT)) {
      tc_fence_after();
      // 16 warps: (lane quarter, M half, column half) each
      const int dw = warp - kQFirstDecoderWarp;
      const int half = (dw >> 2) & 1;
      const int quarter = warp & 3;  // the TMEM lane quarter this warp may access
      const int cbeg = (dw >> 3) * (kQBN / 2);
      const int row = half * kQHalf + quarter * 32 + lane;
      const int64_t m = m0 + row;
      const uint32_t taddr = tmem + half * kQBN + ((uint32_t)(quarter * 32) << 16);
      const float2* rope_row =
          p.rope ? p.rope + ((m + p.rope_off) / p.rope_div % p.rope_mod) * p.rope_half : nullptr;
      for (int c = cbeg; c < cbeg + kQBN / 2; c += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + c, r);
        tmem_wait_ld();
        if (m >= p.M) continue;
        const int64_t nb = n0 + c;
        if (nb >= p.N) continue;
        if (p.splits > 1) {  // raw partial sums; the reduce pass applies the epilogue
          float* wdst = p.ws + ((int64_t)blockIdx.y * p.M + m) * p.N + nb;
#pragma unroll
          for (int g = 0; g < 32; g += 8) {
            if (nb + g >= p.N) break;  // N % 16 == 0, so groups of 8 are whole
            *reinterpret_cast<float4*>(wdst + g) =
                make_float4(__uint_as_float(r[g]), __uint_as_float(r[g + 1]),
                            __uint_as_float(r[g + 2]), __uint_as_float(r[g + 3]));
            *reinterpret_cast<float4*>(wdst + g + 4) =
                make_float4(__uint_as_float(r[g + 4]), __uint_as_float(r[g + 5]),
                            __uint_as_float(r[g + 6]), __uint_as_float(r[g + 7]));
          }
          continue;
        }
#pragma unroll
        for (int g = 0; g < 32; g += 8) {
          if (nb + g >= p.N) break;  // N % 16 == 0, so groups of 8 are whole
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[g + e]);
          ql_finish8<WF>(p, v, m, nb + g, rope_row);
        }
      }
    }
  }

  tc_fence_before();
  // paired: no CTA leaves (or frees TMEM) while the leader's MMAs may still read its shared
  // memory or write its TMEM, or while a peer arrival may still target its barriers
  if constexpr (PAIR) ql_cluster_sync(); else __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem, 512); else tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------------------
// bf16 weights, small products: 128 rows of x x BN weight rows per CTA (the UNet's projection
// and feed-forward GEMMs: K = 320-5120, M = 128-8192, most of them a few GFLOP, where the
// 256 x 256 tiles above leave SMs idle and spend most of a CTA's life filling its pipeline).
// 320 threads: warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 2-9 the epilogue
// (warp w reads TMEM lane quarter w % 4, columns of half (w - 2) / 4); a ring of {x tile 128 x
// 64, W tile BN x 64}, both 128B-swizzled K-major, of 4 / 3 / 2 stages for BN = 64 / 128 /
// 256, so that two CTAs share an SM (96 KB of shared memory each) and one CTA's epilogue
// overlaps the other's loads; the f32 accumulator is BN TMEM columns.  The epilogue is the
// big kernel's (bias, residual, gate, RoPE, GLU, f16 output).
constexpr int kSmThreads = 320;

template <int BN>
struct QlSmallSmem {
  static constexpr int kSt = BN == 256 ? 2 : BN == 128 ? 3 : 4;  // ring stages
  static constexpr int kA = kQBK * 128 * 2;  // 16 KB x tile
  static constexpr int kB = kQBK * BN * 2;   // W tile
  static constexpr int kStage = kA + kB;
  static constexpr int kBar = kSt * kStage;
  static constexpr int kMisc = kBar + (2 * kSt + 1) * 8;
  static constexpr int kAlloc = kMisc + 16 + 1024;
};

template <int BN>
__global__ void __launch_bounds__(kSmThreads, 2)
    qlinear_small_kernel(const __grid_constant__ CUtensorMap tmx,
                         const __grid_constant__ CUtensorMap tmw, const QlParams p) {
  using L = QlSmallSmem<BN>;
  constexpr int kSmSt = L::kSt;
  constexpr uint32_t kCols = BN < 32 ? 32 : BN;  // TMEM allocation: a power of two >= 32
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* empty = full + kSmSt;
  uint64_t* acc_full = empty + kSmSt;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  __shared__ float sbias[BN], sgate[BN];  // the tile's bias and gate columns
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int mtile, ntile;
  ql_tile_of(p, (int)blockIdx.x, mtile, ntile);
  const int m0 = mtile * 128, n0 = ntile * BN;
  const int ktiles = (int)(p.K / kQBK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSmSt; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmx);
      tma_prefetch_desc(&tmw);
      int issued = 0;
      for (int kt = 0; kt < ktiles; ++kt) {
        const int st = kt % kSmSt;
        if (kt >= kSmSt &&
            !mbar_wait(&empty[st], ((kt / kSmSt) - 1) & 1, abort_flag, WD_TMA_WAIT))
          break;
        uint8_t* stage = smem + st * L::kStage;
        mbar_arrive_expect_tx(&full[st], L::kStage);
        tma_load_2d(stage, &tmx, &full[st], kt * kQBK, m0);
        tma_load_2d(stage + L::kA, &tmw, &full[st], kt * kQBK, n0);
        issued = kt + 1;
      }
      // copies still in flight must land before the CTA can exit (bounded)
      for (int kt = max(0, issued - kSmSt); kt < issued; ++kt)
        mbar_wait(&full[kt % kSmSt], (kt / kSmSt) & 1, nullptr, WD_TMA_WAIT);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(128, BN, 1, 0, 0);
      for (int kt = 0; kt < ktiles; ++kt) {
        const int st = kt % kSmSt;
        if (!mbar_wait(&full[st], (kt / kSmSt) & 1, abort_flag, WD_MMA_WAIT)) break;
        tc_fence_after();
        const uint32_t a = smem_u32(smem + st * L::kStage), b = a + L::kA;
#pragma unroll
        for (int kk = 0; kk < kQBK / 16; ++kk)
          umma_ss(tmem, make_smem_desc(a + kk * 32, 16, 1024, LAYOUT_SW128),
                  make_smem_desc(b + kk * 32, 16, 1024, LAYOUT_SW128), idesc,
                  (kt > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[st]);  // the stage is free once these MMAs have read it
      }
      // the accumulator is final once every MMA above has completed (on an early exit the
      // epilogue sees the abort flag instead)
      umma_commit(acc_full);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // The tile's bias and gate go to shared memory while the MMAs run (one element per
    // epilogue thread), and each 32-column step issues its residual loads before it waits for
    // the TMEM load: the epilogue's global-memory latency is paid once per tile and per step,
    // not once per 8 columns.
    const int et = threadIdx.x - 64;  // 0 .. 255
    for (int c = et; c < BN; c += 256) {
      const int64_t n = n0 + c;
      sbias[c] = (p.bias && n < p.N) ? __bfloat162float(p.bias[n]) : 0.f;
      sgate[c] = (p.gate && n < p.N) ? __bfloat162float(p.gate[n]) : 1.f;
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");  // the 8 epilogue warps
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int64_t m = m0 + quarter * 32 + lane;
    const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16);
    const bool res = p.residual && p.glu < 0;
    if (mbar_wait_warp(acc_full, 0, abort_flag, WD_EPILOGUE_WAIT) && !*abort_flag) {
      tc_fence_after();
      const float2* rope_row =
          p.rope ? p.rope + ((m + p.rope_off) / p.rope_div % p.rope_mod) * p.rope_half : nullptr;
      constexpr int kStep = BN / 2 < 32 ? BN / 2 : 32;
#pragma unroll 1
      for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += kStep) {
        uint32_t r[32];
        tmem_ld16(taddr + c, *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
        if constexpr (kStep == 32) tmem_ld16(taddr + c + 16, *reinterpret_cast<uint32_t(*)[16]>(&r[16]));
        const int64_t nb = n0 + c;
        const bool row_ok = m < p.M;
        uint4 rv[kStep / 8];
#pragma unroll
        for (int g = 0; g < kStep / 8; ++g)
          rv[g] = (res && row_ok && nb + 8 * g < p.N)
                      ? *reinterpret_cast<const uint4*>(p.residual + m * p.ldy + nb + 8 * g)
                      : make_uint4(0, 0, 0, 0);
        tmem_wait_ld();
        if (!row_ok) continue;
#pragma unroll
        for (int g = 0; g < kStep / 8; ++g) {
          if (nb + 8 * g >= p.N) break;  // N % 16 == 0: groups of 8 are whole
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[8 * g + e]);
          ql_finish8_with<W_BF16>(p, v, m, nb + 8 * g, rope_row,
                                  p.bias ? &sbias[c + 8 * g] : nullptr,
                                  p.gate ? &sgate[c + 8 * g] : nullptr, rv[g]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// sp_quant_linear_set_pairing: 0 unpaired tiles (default), 1 paired when M > 256
int g_ql_pairing = 0;

// Bytes of one weight row of K values as the kernel reads them (values + scales / factors).
template <int WF>
double ql_w_row_bytes(int64_t K) {
  switch (WF) {
    case W_Q8_0: return K * (1.0 + 2.0 / 32);  // int8 + an f16 scale per 32
    case W_Q4K: return K * (0.5 + 8.0 / 32);   // nibbles + f32 (a, b) per 32
    case W_Q2K:
    case W_Q3K: return K * (0.5 + 8.0 / 16);   // nibbles + f32 (a, b) per 16
    case W_BF16: return K * 2.0;
    default: return (double)K;                 // e4m3
  }
}

#ifndef SP_QL_HOLD_MB
#define SP_QL_HOLD_MB 40
#endif

// Grouped tile raster.  The x row-tiles and W column-tiles a wave of CTAs touches come from
// HBM once if they stay in L2 until their last reader; the plain m-fastest order walks all of x
// for each W column, so a large x (75,600 x 5120 bf16 = 774 MB for a video DiT) is re-read once
// per N tile.  Grouping g tiles of one operand, with the other operand's tiles innermost, holds
// that group (g x tile bytes) in L2 while the other operand streams past it once per group:
//   groups of m-tiles: traffic = X + W * ceil(tiles_m / g)
//   groups of n-tiles: traffic = W + X * ceil(tiles_n / g)
// The orientation with the smaller modelled traffic wins, g as large as the hold budget allows
// (then evened out over the passes it implies).
template <int WF>
void ql_raster(QlParams& q, int tiles_m, int tiles_n, int m_rows) {
  const double hold = SP_QL_HOLD_MB * 1048576.0;
  const double xt = (double)m_rows * q.K * 2, wt = (double)kQBN * ql_w_row_bytes<WF>(q.K);
  const double X = xt * tiles_m, W = wt * tiles_n;
  auto plan = [&](int tiles, double tile_bytes, int& g) {
    g = std::max(1, std::min(tiles, (int)(hold / tile_bytes)));
    const int passes = (tiles + g - 1) / g;
    g = (tiles + passes - 1) / passes;
    return passes;
  };
  int gm, gn;
  const double tm = X + W * plan(tiles_m, xt, gm);
  const double tn = W + X * plan(tiles_n, wt, gn);
  q.tiles_m = tiles_m;
  q.tiles_n = tiles_n;
  q.raster_n = tn < tm ? 1 : 0;
  q.group = q.raster_n ? gn : gm;
}

// Launch of the small-tile bf16 kernel with BN weight rows per CTA.
template <int BN>
int launch_qlinear_small(const void* x, const void* w, const QlParams& p, cudaStream_t s) {
  using L = QlSmallSmem<BN>;
  static_assert(L::kAlloc <= 232448, "small bf16 linear smem budget");
  CUtensorMap mx, mw;
  {
    const uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    const uint64_t strides[1] = {(uint64_t)p.K * 2};
    const uint32_t box[2] = {kQBK, 128};
    if (int rc = encode_tiled(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.N};
    const uint64_t strides[1] = {(uint64_t)p.K * 2};
    const uint32_t box[2] = {kQBK, (uint32_t)BN};
    if (int rc = encode_tiled(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  auto kern = qlinear_small_kernel<BN>;
  static unsigned long long attr_set = 0;
  if (first_time_on_device(&attr_set)) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) {
      __atomic_fetch_and(&attr_set, ~(1ull << current_device()), __ATOMIC_ACQ_REL);
      return set_error(SP_ERR_LAUNCH, "bf16 linear: smem attribute failed: %s",
                       cudaGetErrorString(e));
    }
  }
  QlParams q = p;
  q.ws = nullptr;
  q.splits = 1;
  q.kt_per_split = (int)(p.K / kQBK);
  const int tiles_m = (int)((p.M + 127) / 128), tiles_n = (int)((p.N + BN - 1) / BN);
  ql_raster<W_BF16>(q, tiles_m, tiles_n, 128);
  kern<<<(unsigned)(tiles_m * tiles_n), kSmThreads, L::kAlloc, s>>>(mx, mw, q);
  return check_launch("bf16 linear (small tiles)");
}

// Weight rows per CTA of the small-tile bf16 kernel for this product, or 0 for the 256 x 256
// kernel: products whose 256 x 256 grid fills at least two waves with K >= 2048 keep the big
// tiles; the rest take the widest BN in {256, 128, 64} that divides N and still gives every SM
// a CTA (else 64).
int ql_small_bn(const QlParams& p) {
  const int64_t sms = num_sms();
  const int64_t big = ((p.M + kQBM - 1) / kQBM) * ((p.N + kQBN - 1) / kQBN);
  if (big >= 2 * sms && p.K >= 2048) return 0;
  const int64_t tm = (p.M + 127) / 128;
  for (int bn : {256, 128, 64})
    if (p.N % bn == 0 && tm * (p.N / bn) >= sms) return bn;
  return 64;
}

template <int WF>
int launch_qlinear(const void* x, const void* w8, const QlParams& p, cudaStream_t s) {
  if (!aligned(x, 16) || !aligned(w8, 16) || !aligned(p.y, 16) ||
      (WF == W_Q8_0 && !aligned(p.q8_scale, 16)))
    return set_error(SP_ERR_ALIGN,
                     "quantized linear: x, weights, scales and y must be 16-byte aligned");
  using KF = KqFmt<WF>;
  if (KF::kIsK && (!aligned(p.kq_a, 16) || !aligned(p.kq_b, 16)))
    return set_error(SP_ERR_ALIGN, "quantized linear: k-quant factors must be 16-byte aligned");
  if constexpr (WF == W_BF16) {
    switch (ql_small_bn(p)) {
      case 256: return launch_qlinear_small<256>(x, w8, p, s);
      case 128: return launch_qlinear_small<128>(x, w8, p, s);
      case 64: return launch_qlinear_small<64>(x, w8, p, s);
      default: break;
    }
  }
  // Paired (2-CTA) tiles, when enabled, whenever x has more than one 256-row tile: the
  // pair's CTA count is the unpaired count rounded up to even.
  const bool pair = WF != W_BF16 && p.M > kQBM && __atomic_load_n(&g_ql_pairing, __ATOMIC_RELAXED);
  const uint32_t wrows = pair ? kQBN / 2 : kQBN;  // weight rows per CTA (TMA box height)
  CUtensorMap mx, mw, ms, mb;
  std::memset(&ms, 0, sizeof(ms));
  std::memset(&mb, 0, sizeof(mb));
  {
    const uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.M};
    const uint64_t strides[1] = {(uint64_t)p.K * 2};
    const uint32_t box[2] = {kQBK, kQBM};
    if (int rc = encode_tiled(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  if (KF::kIsK) {
    // nibbles [N, K/2] bytes: a k-tile of 64 values is 32 bytes of each of the CTA's rows
    const uint64_t dims[2] = {(uint64_t)(p.K / 2), (uint64_t)p.N};
    const uint64_t strides[1] = {(uint64_t)(p.K / 2)};
    const uint32_t box[2] = {kQBK / 2, wrows};
    if (int rc = encode_tiled(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w8, dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
    // factors a, b [K/sub, N] f32: one box = the k-tile's sub-blocks x the CTA's rows
    const uint64_t fdims[2] = {(uint64_t)p.N, (uint64_t)(p.K / KF::kSub)};
    const uint64_t fstrides[1] = {(uint64_t)p.N * 4};
    const uint32_t fbox[2] = {wrows, (uint32_t)KF::kFactorRows};
    if (int rc = encode_tiled(&ms, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p.kq_a, fdims, fstrides,
                              fbox, CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
    if (int rc = encode_tiled(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p.kq_b, fdims, fstrides,
                              fbox, CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  } else if (WF == W_BF16) {
    // bf16 W [N, K]: 64 x 256 boxes with the 128B swizzle, the MMA's K-major B layout
    const uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.N};
    const uint64_t strides[1] = {(uint64_t)p.K * 2};
    const uint32_t box[2] = {kQBK, kQBN};
    if (int rc = encode_tiled(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w8, dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  } else {
    const uint64_t dims[2] = {(uint64_t)p.K, (uint64_t)p.N};
    const uint64_t strides[1] = {(uint64_t)p.K};
    const uint32_t box[2] = {kQBK, wrows};
    if (int rc = encode_tiled(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w8, dims, strides, box,
                              CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  }
  if (WF == W_Q8_0) {
    // scales [K/32, N] f16: one box = the 2 k-blocks of a k-tile x the CTA's rows
    const uint64_t dims[2] = {(uint64_t)p.N, (uint64_t)(p.K / 32)};
    const uint64_t strides[1] = {(uint64_t)p.N * 2};
    const uint32_t box[2] = {wrows, kQBK / 32};
    if (int rc = encode_tiled(&ms, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, p.q8_scale, dims, strides,
                              box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  }
  static_assert(QlSmem::kAlloc <= 232448 && QlSmemT<true>::kAlloc <= 232448 &&
                    QlSmemBf16::kAlloc <= 232448,
                "quantized linear smem budget");
  constexpr int kSmem1 = WF == W_BF16 ? QlSmemBf16::kAlloc : QlSmem::kAlloc;
  constexpr int kSmem2 = QlSmemT<true>::kAlloc;
  auto kern1 = qlinear_kernel<WF, false>;
  auto kern2 = qlinear_kernel<WF, WF != W_BF16>;  // (bf16 weights never pair)
  static unsigned long long attr_set[2] = {0, 0};
  if (first_time_on_device(&attr_set[pair])) {
    cudaError_t e = pair ? cudaFuncSetAttribute(kern2, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                kSmem2)
                         : cudaFuncSetAttribute(kern1, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                kSmem1);
    if (e != cudaSuccess) {
      __atomic_fetch_and(&attr_set[pair], ~(1ull << current_device()), __ATOMIC_ACQ_REL);
      return set_error(SP_ERR_LAUNCH, "quantized linear: smem attribute failed: %s", cudaGetErrorString(e));
    }
  }
  // a paired tile is 512 x rows (two CTAs of 256), an unpaired one 256
  const int m_rows = pair ? 2 * kQBM : kQBM, cta_per_tile = pair ? 2 : 1;
  const int tiles_m = (int)((p.M + m_rows - 1) / m_rows), tiles_n = (int)((p.N + kQBN - 1) / kQBN);
  // Split-K when the tile grid leaves most SMs idle (the text-stream and modulation GEMMs of
  // the DiT blocks): each split's CTAs write f32 partials to stream-ordered scratch, and one
  // reduce pass sums them in a fixed order and runs the epilogue.  Scratch that cannot be had
  // means no split.
  QlParams q = p;
  const int ktotal = (int)(p.K / kQBK), tiles = tiles_m * tiles_n, sms = num_sms();
  const int units = tiles * cta_per_tile;  // CTAs per split
  int splits = 1;
  if (2 * units <= sms && ktotal >= 8) {
    splits = std::min(std::min(8, sms / units), ktotal / 4);
  } else if (ktotal >= 128) {
    // long K with a badly quantised last wave (e.g. 192 tiles on 148 SMs: 65 % busy): split
    // 2-4 ways when that fills the waves better; the f32 partials (S x M x N x 4 bytes, written
    // and read once) cost little next to K >= 8192 of MMA work
    auto eff = [&](int sp) {
      const int ctas = units * sp;
      return (double)ctas / ((double)((ctas + sms - 1) / sms) * sms);
    };
    double best = eff(1);
    for (int sp = 2; sp <= 4; ++sp)
      if (eff(sp) > best + 0.1) {
        best = eff(sp);
        splits = sp;
      }
  }
  // no stream-ordered scratch inside a CUDA-graph capture (a captured pool allocation would
  // tie the graph to this pool): one split there
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (splits > 1 && (cudaStreamIsCapturing(s, &cap) != cudaSuccess ||
                     cap != cudaStreamCaptureStatusNone)) {
    cudaGetLastError();
    splits = 1;
  }
  void* ws = nullptr;
  if (splits > 1) {
    q.kt_per_split = (ktotal + splits - 1) / splits;
    splits = (ktotal + q.kt_per_split - 1) / q.kt_per_split;  // no empty split
    const size_t bytes = (size_t)splits * (size_t)p.M * (size_t)p.N * sizeof(float);
    cudaMemPool_t pool = scratch_pool();
    if (!pool || cudaMallocFromPoolAsync(&ws, bytes, pool, s) != cudaSuccess) {
      cudaGetLastError();
      ws = nullptr;
      splits = 1;
      q.kt_per_split = ktotal;
    }
  }
  q.ws = static_cast<float*>(ws);
  q.splits = splits;
  ql_raster<WF>(q, tiles_m, tiles_n, m_rows);
  if (pair) {
    // clusters of two consecutive CTAs along x: CTA 2t is tile t's leader, 2t + 1 its peer
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)units, (unsigned)splits, 1);
    cfg.blockDim = dim3(kQThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmem2;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern2, mx, mw, ms, mb, q);
    if (e != cudaSuccess)
      return set_error(SP_ERR_LAUNCH, "quantized linear: paired launch failed: %s",
                       cudaGetErrorString(e));
  } else {
    dim3 grid((unsigned)units, (unsigned)splits);
    kern1<<<grid, kQThreads, kSmem1, s>>>(mx, mw, ms, mb, q);
  }
  if (splits > 1) {
    const int64_t groups = p.M * (p.N / 8);
    const unsigned rblocks = (unsigned)std::min<int64_t>((groups + 255) / 256, 8LL * sms);
    ql_splitk_reduce_kernel<WF><<<rblocks, 256, 0, s>>>(q);
    const cudaError_t e = cudaFreeAsync(ws, s);
    if (e != cudaSuccess) return set_error(SP_ERR_LAUNCH, "quantized linear: scratch free failed");
  }
  return check_launch("quantized linear");
}

int check_ql_shape(int64_t M, int64_t N, int64_t K, int dtype) {
  if (M <= 0 || N <= 0 || K <= 0) return set_error(SP_ERR_INVALID_ARG, "quantized linear: bad shape");
  if (K % kQBK) return set_error(SP_ERR_SHAPE, "quantized linear: K=%lld must be a multiple of 64", (long long)K);
  if (N % 16) return set_error(SP_ERR_SHAPE, "quantized linear: N=%lld must be a multiple of 16", (long long)N);
  if (dtype != SP_BF16) return set_error(SP_ERR_DTYPE, "quantized linear: activations must be bf16");
  if (M > 65535LL * kQBM || N > 65535LL * kQBN || K > (1LL << 31))
    return set_error(SP_ERR_SHAPE, "quantized linear: shape too large");
  return SP_OK;
}

}  // namespace
}  // namespace sp

namespace sp {
namespace {
// Shared argument checks and launch for every quantized-linear entry point.
struct QlEpilogue {
  const void* gate = nullptr;
  const void* residual = nullptr;
  int64_t ldy = 0;  // 0: N
  const float* rope = nullptr;
  int64_t rope_positions = 0, rope_cols = 0, head_dim = 0, pos_off = 0, pos_div = 1, pos_mod = 1;
  int glu = -1;
  bool out_dtype_free = false;  // the rope / strided-output entries: y may be bf16 or f16
};

template <int WF>
int ql_entry(const char* what, const void* x, const void* w, const void* q8_scale,
             const float* fp8_scale, int64_t nscale, const void* bias, void* y, int64_t M,
             int64_t N, int64_t K, int dtype, const QlEpilogue& e, void* stream,
             const float* kq_a = nullptr, const float* kq_b = nullptr) {
  clear_error();
  const bool have_scales = WF == W_Q8_0 ? q8_scale != nullptr
                           : WF == W_FP8 ? fp8_scale != nullptr
                           : WF == W_BF16 ? true
                                          : (kq_a != nullptr && kq_b != nullptr);
  if (!x || !w || !have_scales || !y)
    return set_error(SP_ERR_INVALID_ARG, "%s: null pointer", what);
  if (KqFmt<WF>::kIsK && K % 256)
    return set_error(SP_ERR_SHAPE, "%s: K=%lld must be a multiple of 256 (k-quant super-blocks)",
                     what, (long long)K);
  if (WF == W_FP8 && nscale != 1 && nscale != N)
    return set_error(SP_ERR_SHAPE, "%s: scale count %lld must be 1 or N", what, (long long)nscale);
  const bool y_f16 = e.out_dtype_free && dtype == SP_F16;
  if (int rc = check_ql_shape(M, N, K, y_f16 ? SP_BF16 : dtype)) return rc;
  if (e.glu >= 0 && (e.glu > SP_GLU_SWIGLU || e.gate || e.residual || e.rope))
    return set_error(SP_ERR_INVALID_ARG, "%s: the GLU epilogue takes no gate, residual or rope",
                     what);
  const int64_t out_cols = e.glu >= 0 ? N / 2 : N;
  const int64_t ldy = e.ldy ? e.ldy : out_cols;
  if (ldy < out_cols || ldy % 8)
    return set_error(SP_ERR_SHAPE, "%s: row stride %lld must be >= N and a multiple of 8", what,
                     (long long)ldy);
  if (e.residual && !aligned(e.residual, 16))
    return set_error(SP_ERR_ALIGN, "%s: residual must be 16-byte aligned", what);
  if (e.rope) {
    if (e.head_dim <= 0 || e.head_dim % 8 || e.rope_cols <= 0 || e.rope_cols % e.head_dim ||
        e.rope_cols > N)
      return set_error(SP_ERR_SHAPE, "%s: rope needs 8 | head_dim, head_dim | rope_cols <= N",
                       what);
    if (e.pos_div < 1 || e.pos_mod < 1 || e.pos_off < 0 || e.pos_mod > e.rope_positions)
      return set_error(SP_ERR_INVALID_ARG,
                       "%s: rope positions need div, mod >= 1, offset >= 0, mod <= table rows",
                       what);
    if (!aligned(e.rope, 8)) return set_error(SP_ERR_ALIGN, "%s: rope table must be 8-byte aligned", what);
  }
  if (int rc = require_sm100()) return rc;
  QlParams p{M, N, K, static_cast<const uint16_t*>(q8_scale), fp8_scale, nscale, kq_a, kq_b,
             static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(y),
             static_cast<const __nv_bfloat16*>(e.gate), static_cast<const __nv_bfloat16*>(e.residual),
             ldy, reinterpret_cast<const float2*>(e.rope), e.pos_off, e.pos_div, e.pos_mod,
             (int)e.rope_cols, (int)(e.head_dim / 2), nullptr, 1, (int)(K / kQBK), e.glu,
             y_f16 ? 1 : 0};
  return launch_qlinear<WF>(x, w, p, static_cast<cudaStream_t>(stream));
}

QlEpilogue gated(const void* gate, const void* residual) {
  QlEpilogue e;
  e.gate = gate;
  e.residual = residual;
  return e;
}

QlEpilogue roped(int64_t ldy, const float* rope, int64_t positions, int64_t cols, int64_t hd,
                 int64_t off, int64_t div, int64_t mod) {
  QlEpilogue e;
  e.ldy = ldy;
  e.rope = rope;
  e.rope_positions = positions;
  e.rope_cols = cols;
  e.head_dim = hd;
  e.pos_off = off;
  e.pos_div = div;
  e.pos_mod = mod;
  e.out_dtype_free = true;
  return e;
}
}  // namespace
}  // namespace sp

extern "C" {

int sp_q8_0_linear(const void* x, const void* q, const void* scale, const void* bias, void* y, int64_t M,
                   int64_t N, int64_t K, int dtype, void* stream) {
  return sp::ql_entry<sp::W_Q8_0>("q8_0 linear", x, q, scale, nullptr, 0, bias, y, M, N, K, dtype,
                                  sp::QlEpilogue{}, stream);
}

int sp_q8_0_linear_gated(const void* x, const void* q, const void* scale, const void* bias,
                         const void* gate, const void* residual, void* y, int64_t M, int64_t N,
                         int64_t K, int dtype, void* stream) {
  return sp::ql_entry<sp::W_Q8_0>("q8_0 linear", x, q, scale, nullptr, 0, bias, y, M, N, K, dtype,
                                  sp::gated(gate, residual), stream);
}

int sp_q8_0_linear_rope(const void* x, const void* q, const void* scale, const void* bias, void* y,
                        int64_t ldy, int64_t M, int64_t N, int64_t K, const float* rope_cos_sin,
                        int64_t rope_positions, int64_t rope_cols, int64_t head_dim,
                        int64_t pos_offset, int64_t pos_div, int64_t pos_mod, int dtype,
                        void* stream) {
  return sp::ql_entry<sp::W_Q8_0>(
      "q8_0 linear", x, q, scale, nullptr, 0, bias, y, M, N, K, dtype,
      sp::roped(ldy, rope_cos_sin, rope_positions, rope_cols, head_dim, pos_offset, pos_div,
                pos_mod),
      stream);
}

int sp_kquant_linear(int fmt, const void* x, const void* qpack, const float* a, const float* b,
                     const void* bias, void* y, int64_t M, int64_t N, int64_t K, int dtype,
                     void* stream) {
  using namespace sp;
  switch (fmt) {
    case SP_QK_Q4_K:
      return ql_entry<W_Q4K>("q4_k linear", x, qpack, nullptr, nullptr, 0, bias, y, M, N, K,
                             dtype, QlEpilogue{}, stream, a, b);
    case SP_QK_Q2_K:
      return ql_entry<W_Q2K>("q2_k linear", x, qpack, nullptr, nullptr, 0, bias, y, M, N, K,
                             dtype, QlEpilogue{}, stream, a, b);
    case SP_QK_Q3_K:
      return ql_entry<W_Q3K>("q3_k linear", x, qpack, nullptr, nullptr, 0, bias, y, M, N, K,
                             dtype, QlEpilogue{}, stream, a, b);
    default:
      clear_error();
      return set_error(SP_ERR_DTYPE, "k-quant linear: unknown format %d", fmt);
  }
}

int sp_q8_0_linear_glu(const void* x, const void* q, const void* scale, const void* bias, void* y,
                       int64_t M, int64_t N, int64_t K, int glu_kind, int dtype, void* stream) {
  sp::QlEpilogue e;
  e.glu = glu_kind < 0 ? SP_GLU_SWIGLU + 1 : glu_kind;  // negative kinds are rejected
  return sp::ql_entry<sp::W_Q8_0>("q8_0 linear", x, q, scale, nullptr, 0, bias, y, M, N, K, dtype,
                                  e, stream);
}

int sp_quant_linear_set_pairing(int mode) {
  sp::clear_error();
  if (mode != 0 && mode != 1)
    return sp::set_error(SP_ERR_INVALID_ARG, "quantized linear pairing: mode must be 0 or 1");
  return __atomic_exchange_n(&sp::g_ql_pairing, mode, __ATOMIC_RELAXED);
}

int sp_fp8_linear_glu(const void* x, const void* w_e4m3, const float* scale, int64_t nscale,
                      const void* bias, void* y, int64_t M, int64_t N, int64_t K, int glu_kind,
                      int dtype, void* stream) {
  sp::QlEpilogue e;
  e.glu = glu_kind < 0 ? SP_GLU_SWIGLU + 1 : glu_kind;
  return sp::ql_entry<sp::W_FP8>("fp8 linear", x, w_e4m3, nullptr, scale, nscale, bias, y, M, N, K,
                                 dtype, e, stream);
}

int sp_fp8_linear(const void* x, const void* w_e4m3, const float* scale, int64_t nscale, const void* bias,
                  void* y, int64_t M, int64_t N, int64_t K, int dtype, void* stream) {
  return sp::ql_entry<sp::W_FP8>("fp8 linear", x, w_e4m3, nullptr, scale, nscale, bias, y, M, N, K,
                                 dtype, sp::QlEpilogue{}, stream);
}

int sp_fp8_linear_gated(const void* x, const void* w_e4m3, const float* scale, int64_t nscale,
                        const void* bias, const void* gate, const void* residual, void* y,
                        int64_t M, int64_t N, int64_t K, int dtype, void* stream) {
  return sp::ql_entry<sp::W_FP8>("fp8 linear", x, w_e4m3, nullptr, scale, nscale, bias, y, M, N, K,
                                 dtype, sp::gated(gate, residual), stream);
}

int sp_fp8_linear_rope(const void* x, const void* w_e4m3, const float* scale, int64_t nscale,
                       const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                       const float* rope_cos_sin, int64_t rope_positions, int64_t rope_cols,
                       int64_t head_dim, int64_t pos_offset, int64_t pos_div, int64_t pos_mod,
                       int dtype, void* stream) {
  return sp::ql_entry<sp::W_FP8>(
      "fp8 linear", x, w_e4m3, nullptr, scale, nscale, bias, y, M, N, K, dtype,
      sp::roped(ldy, rope_cos_sin, rope_positions, rope_cols, head_dim, pos_offset, pos_div,
                pos_mod),
      stream);
}

int sp_bf16_linear(const void* x, const void* w, const void* bias, void* y, int64_t M, int64_t N,
                   int64_t K, int dtype, void* stream) {
  return sp::ql_entry<sp::W_BF16>("bf16 linear", x, w, nullptr, nullptr, 0, bias, y, M, N, K,
                                  dtype, sp::QlEpilogue{}, stream);
}

int sp_bf16_linear_gated(const void* x, const void* w, const void* bias, const void* gate,
                         const void* residual, void* y, int64_t M, int64_t N, int64_t K,
                         int dtype, void* stream) {
  return sp::ql_entry<sp::W_BF16>("bf16 linear", x, w, nullptr, nullptr, 0, bias, y, M, N, K,
                                  dtype, sp::gated(gate, residual), stream);
}

int sp_bf16_linear_glu(const void* x, const void* w, const void* bias, void* y, int64_t M,
                       int64_t N, int64_t K, int glu_kind, int dtype, void* stream) {
  sp::QlEpilogue e;
  e.glu = glu_kind < 0 ? SP_GLU_SWIGLU + 1 : glu_kind;
  return sp::ql_entry<sp::W_BF16>("bf16 linear", x, w, nullptr, nullptr, 0, bias, y, M, N, K,
                                  dtype, e, stream);
}

}  // extern "C"
