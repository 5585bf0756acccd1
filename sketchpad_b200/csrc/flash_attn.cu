// flash_attn.cu -- flash-attention forward for sm_100a: TMA-fed tcgen05 UMMA with TMEM
// accumulators and an online softmax.
//
// Computes out = softmax(Q K^T * scale [+ mask] [causal]) V with f32 accumulation, the
// operation of sketchpad_cubecl::flash_attention (crates/sketchpad-cubecl/src/attention.rs:97-178)
// and of the CPU attention it must match (crates/sketchpad-unet/src/blocks.rs:370-410).
//
// One CTA = one 128-query tile of one (batch, head).  Warp roles (192 threads):
//   warp 0      TMA producer: Q once, then K/V tiles of 128 keys through a STAGES-deep ring.
//   warp 1      TMEM owner + MMA issuer (one elected lane):
//                 S[j%2] = Q K_j^T         (M=128, N=128, K=D padded to 16)
//                 O     += P_{j-1} V_{j-1} (M=128, N=Dv padded to 64, K=128)
//   warps 2..5  softmax + epilogue, one query row per thread (= one TMEM lane):
//                 tcgen05.ld S row -> mask -> exp2 -> P (16-bit) into shared memory in the
//                 UMMA K-major 128B-swizzled layout; O is rescaled in TMEM only when the row
//                 max grows by more than 2^8 (exact: P and l always use the same reference).
// TMEM: S0 = cols [0,128), S1 = [128,256), O = [256, 256+DvPad).
// Tiles in shared memory are 128 rows x 64 elements (128 B) boxes with the 128B swizzle, the
// canonical K-major layout for Q, K and P and the MN-major layout for V.
#include "common.cuh"
#include "tc.cuh"

namespace sp {
namespace {

constexpr int kBM = 128;            // queries per CTA
constexpr int kBN = 128;            // keys per KV tile
constexpr int kBox = 16384;         // bytes of one 128 x 64 16-bit box
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS0 = 0, kTmemS1 = 128, kTmemO = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when max grows > 2^8

struct FaParams {
  int64_t Sq, Skv, H;
  int D, Dv;
  int dqk_pad;          // D rounded up to the UMMA K step (16)
  int dv_pad;           // Dv rounded up to 64 (whole MN-major swizzle atoms)
  int n_kv_tiles;       // tiles of kBN keys (before causal trimming)
  float scale_log2;     // softmax scale * log2(e)
  float inv_scale;      // 1 / softmax scale (additive masks are applied to raw scores)
  int causal;
  const float* mask;
  int64_t mask_stride;
  void* out;
  int64_t os0, os1, os2;  // output element strides (b, h, s); innermost is 1
  int out_dtype;
  int in_f16;  // 1 if inputs are f16 (P is then f16 too), 0 for bf16
};

template <int NBQ, int NBV, int STAGES>
struct FaSmem {
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + NBQ * kBox;
  static constexpr int kV = kK + STAGES * NBQ * kBox;
  static constexpr int kP = kV + STAGES * NBV * kBox;  // two P buffers of 128 x 128 (2 boxes)
  static constexpr int kBar = kP + 4 * kBox;
  // barriers: q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], s_free[2],
  // p_full[2], o_done[2], drain
  static constexpr int kNumBars = 1 + 4 * STAGES + 2 + 2 + 2 + 2 + 1;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;  // tmem base + abort flag
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-B alignment of the base
};

__device__ __forceinline__ uint32_t float_bits(float f) { return __float_as_uint(f); }

template <int NBQ, int NBV, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, const FaParams p) {
  using L = FaSmem<NBQ, NBV, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + STAGES;
  uint64_t* v_full = k_empty + STAGES;
  uint64_t* v_empty = v_full + STAGES;
  uint64_t* s_full = v_empty + STAGES;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * kBM;

  // KV tiles this query tile needs (causal: keys <= last query of the tile).
  int n_tiles = p.n_kv_tiles;
  if (p.causal) {
    const int last_q = min((int)p.Sq - 1, q0 + kBM - 1);
    n_tiles = min(n_tiles, last_q / kBN + 1);
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 128);
      mbar_init(&p_full[s], 128);
      mbar_init(&o_done[s], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      mbar_arrive_expect_tx(q_full, NBQ * kBox);
      for (int blk = 0; blk < NBQ; ++blk)
        tma_load_4d(smem + L::kQ + blk * kBox, &tmq, q_full, blk * 64, q0, h, b);
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (j >= STAGES && !mbar_wait(&k_empty[st], ph ^ 1, abort_flag, WD_TMA_WAIT)) break;
        mbar_arrive_expect_tx(&k_full[st], NBQ * kBox);
        for (int blk = 0; blk < NBQ; ++blk)
          tma_load_4d(smem + L::kK + (st * NBQ + blk) * kBox, &tmk, &k_full[st], blk * 64,
                      j * kBN, h, b);
        issued_k = j + 1;
        if (j >= STAGES && !mbar_wait(&v_empty[st], ph ^ 1, abort_flag, WD_TMA_WAIT)) break;
        mbar_arrive_expect_tx(&v_full[st], NBV * kBox);
        for (int blk = 0; blk < NBV; ++blk)
          tma_load_4d(smem + L::kV + (st * NBV + blk) * kBox, &tmv, &v_full[st], blk * 64,
                      j * kBN, h, b);
        issued_v = j + 1;
      }
      if (*abort_flag) {
        // Let every copy still in flight land before the CTA can exit (bounded).
        mbar_wait(q_full, 0, nullptr, WD_TMA_WAIT);
        for (int j = max(0, issued_k - STAGES); j < issued_k; ++j)
          mbar_wait(&k_full[j % STAGES], (j / STAGES) & 1, nullptr, WD_TMA_WAIT);
        for (int j = max(0, issued_v - STAGES); j < issued_v; ++j)
          mbar_wait(&v_full[j % STAGES], (j / STAGES) & 1, nullptr, WD_TMA_WAIT);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t ab = p.in_f16 ? 0u : 1u;
      const uint32_t idesc_qk = make_idesc_f16(kBM, kBN, ab, 0, 0);
      const uint32_t idesc_pv = make_idesc_f16(kBM, (uint32_t)p.dv_pad, ab, 0, 1);
      const uint32_t q_base = smem_u32(smem + L::kQ);
      const uint32_t p_base = smem_u32(smem + L::kP);
      const int qk_steps = p.dqk_pad / 16;
      bool ok = mbar_wait(q_full, 0, abort_flag, WD_MMA_WAIT);
      tc_fence_after();

      // O += P_i V_i, P_i in shared buffer i % 2
      auto issue_pv = [&](int i) -> bool {
        const int st = i % STAGES;
        if (!mbar_wait(&v_full[st], (i / STAGES) & 1, abort_flag, WD_MMA_WAIT)) return false;
        if (!mbar_wait(&p_full[i & 1], (i >> 1) & 1, abort_flag, WD_MMA_WAIT)) return false;
        tc_fence_after();
        const uint32_t v_base = smem_u32(smem + L::kV + st * NBV * kBox);
        const uint32_t pb = p_base + (i & 1) * 2 * kBox;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // A = P (K-major, 2 boxes of 64 keys), B = V (MN-major: keys x Dv, Dv contiguous)
          const uint64_t a = make_smem_desc(pb + (kk >> 2) * kBox + (kk & 3) * 32, 16, 1024,
                                            LAYOUT_SW128);
          const uint64_t bd = make_smem_desc(v_base + kk * 16 * 128, kBox, 1024, LAYOUT_SW128);
          umma_ss(tmem + kTmemO, a, bd, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&v_empty[st]);
        umma_commit(&o_done[i & 1]);
        return true;
      };

      for (int j = 0; ok && j < n_tiles; ++j) {
        const int st = j % STAGES;
        const int sb = j & 1;
        if (!mbar_wait(&k_full[st], (j / STAGES) & 1, abort_flag, WD_MMA_WAIT)) break;
        if (j >= 2 && !mbar_wait(&s_free[sb], ((j >> 1) - 1) & 1, abort_flag, WD_MMA_WAIT)) break;
        tc_fence_after();
        const uint32_t k_base = smem_u32(smem + L::kK + st * NBQ * kBox);
        const uint32_t s_col = sb ? kTmemS1 : kTmemS0;
        for (int kk = 0; kk < qk_steps; ++kk) {
          const uint32_t off = (kk >> 2) * kBox + (kk & 3) * 32;
          const uint64_t a = make_smem_desc(q_base + off, 16, 1024, LAYOUT_SW128);
          const uint64_t bd = make_smem_desc(k_base + off, 16, 1024, LAYOUT_SW128);
          umma_ss(tmem + s_col, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[st]);
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && !*abort_flag && n_tiles > 0) issue_pv(n_tiles - 1);
      // Drain: every MMA issued above has completed once this commit arrives.
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, WD_MMA_WAIT);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const int qi = q0 + row;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;  // running max in log2 units, running row sum
    bool ok = true;

    for (int j = 0; j < n_tiles; ++j) {
      const int sb = j & 1;
      if (!mbar_wait_warp(&s_full[sb], (j >> 1) & 1, abort_flag, WD_SOFTMAX_WAIT)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // S row: four 32-column loads in flight, one wait
      float s[kBN];
      {
        const uint32_t s_addr = lane_addr + (sb ? kTmemS1 : kTmemS0);
        uint32_t r0[32], r1[32], r2[32], r3[32];
        tmem_ld32(s_addr + 0, r0);
        tmem_ld32(s_addr + 32, r1);
        tmem_ld32(s_addr + 64, r2);
        tmem_ld32(s_addr + 96, r3);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          s[t] = __uint_as_float(r0[t]);
          s[32 + t] = __uint_as_float(r1[t]);
          s[64 + t] = __uint_as_float(r2[t]);
          s[96 + t] = __uint_as_float(r3[t]);
        }
      }
      tc_fence_before();
      mbar_arrive(&s_free[sb]);  // S buffer may be overwritten by QK_{j+2}

      // Masks act on raw scores: x_log2 = (s + mask / scale) * scale * log2(e).
      const int kv0 = j * kBN;
      const bool need_mask = p.mask != nullptr || (kv0 + kBN > p.Skv) ||
                             (p.causal && kv0 + kBN - 1 > q0);
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          const int kv = kv0 + c;
          const bool valid = kv < p.Skv && !(p.causal && kv > qi);
          float x = s[c];
          if (p.mask && valid && qi < p.Sq) x += p.mask[(int64_t)qi * p.mask_stride + kv] * p.inv_scale;
          s[c] = valid ? x : -INFINITY;
        }
      }
      float mx0 = s[0], mx1 = s[1], mx2 = s[2], mx3 = s[3];
#pragma unroll
      for (int c = 4; c < kBN; c += 4) {
        mx0 = fmaxf(mx0, s[c]);
        mx1 = fmaxf(mx1, s[c + 1]);
        mx2 = fmaxf(mx2, s[c + 2]);
        mx3 = fmaxf(mx3, s[c + 3]);
      }
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
      const float m_tile = mx == -INFINITY ? -INFINITY : mx * sl2;
      const float m_new = fmaxf(m_run, m_tile);
      bool rescale = false;
      float m_use = m_run;
      if (m_run == -INFINITY) {
        m_use = m_new;  // nothing accumulated yet (O and l are zero)
      } else if (m_new > m_run + kRescaleThreshold) {
        rescale = true;
        m_use = m_new;
      }
      const float m_ref = m_use == -INFINITY ? 0.f : m_use;  // fully masked so far: p = 0

      // P buffer j % 2 was last read by PV_{j-2}
      if (j >= 2 && !mbar_wait_warp(&o_done[sb], ((j - 2) >> 1) & 1, abort_flag, WD_SOFTMAX_WAIT)) {
        ok = false;
        break;
      }
      // tcgen05.ld/st are warp-collective: the whole warp rescales if any of its rows must,
      // rows that need no rescale use alpha = 1.  O must hold PV_{j-1} first.
      if (__any_sync(0xffffffffu, rescale)) {
        if (j >= 1 &&
            !mbar_wait_warp(&o_done[sb ^ 1], ((j - 1) >> 1) & 1, abort_flag, WD_SOFTMAX_WAIT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float alpha = rescale ? ex2_approx(m_run - m_ref) : 1.0f;
        l_run *= alpha;
        for (int c = 0; c < p.dv_pad; c += 16) {
          uint32_t r[16];
          tmem_ld16(lane_addr + kTmemO + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 16; ++t) r[t] = float_bits(__uint_as_float(r[t]) * alpha);
          tmem_st16(lane_addr + kTmemO + c, r);
        }
        tmem_wait_st();
      }
      m_run = m_use;

      // exp2, row sum, 16-bit P into shared memory (UMMA K-major SW128: box c8/8,
      // 16-byte chunk (c8 % 8) ^ (row % 8))
      uint8_t* p_smem = smem + L::kP + sb * 2 * kBox;
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < kBN / 8; ++c8) {
        uint32_t pk[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float e0 = ex2_approx(fmaf(s[c8 * 8 + 2 * t], sl2, -m_ref));
          const float e1 = ex2_approx(fmaf(s[c8 * 8 + 2 * t + 1], sl2, -m_ref));
          rs0 += e0;
          rs1 += e1;
          pk[t] = p.in_f16 ? pack_f16x2(e0, e1) : pack_bf16x2(e0, e1);
        }
        const uint32_t off = (c8 >> 3) * kBox + row * 128 + (((c8 & 7) ^ (row & 7)) << 4);
        *reinterpret_cast<uint4*>(p_smem + off) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      l_run += rs0 + rs1;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }

    // ---- epilogue: O / l -> global
    const int last = n_tiles - 1;
    if (ok && n_tiles > 0 &&
        mbar_wait_warp(&o_done[last & 1], (last >> 1) & 1, abort_flag, WD_EPILOGUE_WAIT)) {
      tc_fence_after();
      const float inv_l = l_run > 0.f ? 1.0f / l_run : 0.f;
      const bool row_ok = qi < p.Sq;
      const int64_t obase = (int64_t)b * p.os0 + (int64_t)h * p.os1 + (int64_t)qi * p.os2;
      for (int c = 0; c < p.dv_pad; c += 16) {
        uint32_t r[16];
        tmem_ld16(lane_addr + kTmemO + c, r);
        tmem_wait_ld();
        if (!row_ok || c >= p.Dv) continue;
        float o[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) o[t] = __uint_as_float(r[t]) * inv_l;
        const int ncol = min(16, p.Dv - c);  // multiple of 8
        if (p.out_dtype == SP_F32) {
          float* dst = static_cast<float*>(p.out) + obase + c;
          for (int t = 0; t < ncol; t += 4)
            *reinterpret_cast<float4*>(dst + t) = make_float4(o[t], o[t + 1], o[t + 2], o[t + 3]);
        } else {
          uint16_t* dst = static_cast<uint16_t*>(p.out) + obase + c;
          for (int t = 0; t < ncol; t += 8) {
            uint4 u;
            if (p.out_dtype == SP_BF16) {
              u = make_uint4(pack_bf16x2(o[t], o[t + 1]), pack_bf16x2(o[t + 2], o[t + 3]),
                             pack_bf16x2(o[t + 4], o[t + 5]), pack_bf16x2(o[t + 6], o[t + 7]));
            } else {
              u = make_uint4(pack_f16x2(o[t], o[t + 1]), pack_f16x2(o[t + 2], o[t + 3]),
                             pack_f16x2(o[t + 4], o[t + 5]), pack_f16x2(o[t + 6], o[t + 7]));
            }
            *reinterpret_cast<uint4*>(dst + t) = u;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int make_qkv_map(CUtensorMap* m, const void* base, int in_f16, int64_t S, int64_t H, int64_t B,
                 int D, const int64_t st[4], const char* name) {
  (void)in_f16;
  if (st[3] != 1) return set_error(SP_ERR_ALIGN, "flash_attn: %s innermost stride must be 1", name);
  for (int i = 0; i < 3; ++i)
    if ((st[i] * 2) % 16 != 0)
      return set_error(SP_ERR_ALIGN, "flash_attn: %s stride[%d]=%lld is not a multiple of 8 "
                       "elements", name, i, (long long)st[i]);
  if (!aligned(base, 16)) return set_error(SP_ERR_ALIGN, "flash_attn: %s not 16-byte aligned", name);
  const uint64_t dims[4] = {(uint64_t)D, (uint64_t)S, (uint64_t)H, (uint64_t)B};
  const uint64_t strides[3] = {(uint64_t)st[2] * 2, (uint64_t)st[1] * 2, (uint64_t)st[0] * 2};
  const uint32_t box[4] = {64, (uint32_t)kBM, 1, 1};
  return encode_tiled(m, in_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                      4, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int NBQ, int NBV, int STAGES>
int launch_fa(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
              const FaParams& p, int64_t B, cudaStream_t s) {
  using L = FaSmem<NBQ, NBV, STAGES>;
  auto kern = fa_fwd_kernel<NBQ, NBV, STAGES>;
  static_assert(L::kAlloc <= 232448, "flash_attn smem budget");
  static unsigned long long attr_set = 0;
  if (first_time_on_device(&attr_set)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
    if (e != cudaSuccess) {
      __atomic_fetch_and(&attr_set, ~(1ull << current_device()), __ATOMIC_ACQ_REL);
      return set_error(SP_ERR_LAUNCH, "flash_attn: smem attribute failed: %s", cudaGetErrorString(e));
    }
  }
  dim3 grid((unsigned)((p.Sq + kBM - 1) / kBM), (unsigned)p.H, (unsigned)B);
  kern<<<grid, kThreads, L::kAlloc, s>>>(mq, mk, mv, p);
  return check_launch("flash_attn");
}

}  // namespace
}  // namespace sp

extern "C" int sp_flash_attn_fwd(const void* q, const void* k, const void* v, const float* mask,
                                 int64_t mask_row_stride, void* out, int64_t B, int64_t H,
                                 int64_t Sq, int64_t Skv, int64_t D, int64_t Dv,
                                 const int64_t q_strides[4], const int64_t k_strides[4],
                                 const int64_t v_strides[4], const int64_t o_strides[4],
                                 int dtype_in, int dtype_out, int causal, float scale,
                                 void* stream) {
  using namespace sp;
  clear_error();
  if (!q || !k || !v || !out || !q_strides || !k_strides || !v_strides || !o_strides)
    return set_error(SP_ERR_INVALID_ARG, "flash_attn: null pointer argument");
  if (B <= 0 || H <= 0 || Sq <= 0 || Skv <= 0 || D <= 0 || Dv <= 0)
    return set_error(SP_ERR_INVALID_ARG, "flash_attn: non-positive dimension");
  if (D % 8 || Dv % 8 || D > 128 || Dv > 128)
    return set_error(SP_ERR_SHAPE, "flash_attn: head dims must be multiples of 8 in [8,128] "
                     "(D=%lld, Dv=%lld)", (long long)D, (long long)Dv);
  if (dtype_in != SP_BF16 && dtype_in != SP_F16)
    return set_error(SP_ERR_DTYPE, "flash_attn: inputs must be bf16 or f16");
  if (dtype_out != SP_BF16 && dtype_out != SP_F16 && dtype_out != SP_F32)
    return set_error(SP_ERR_DTYPE, "flash_attn: unknown output dtype %d", dtype_out);
  if (Sq > (1LL << 30) || Skv > (1LL << 30) || H > 65535 || B > 65535)
    return set_error(SP_ERR_SHAPE, "flash_attn: dimension too large");
  if (o_strides[3] != 1) return set_error(SP_ERR_ALIGN, "flash_attn: output innermost stride must be 1");
  const int oes = dtype_size(dtype_out);
  for (int i = 0; i < 3; ++i)
    if ((o_strides[i] * oes) % 16)
      return set_error(SP_ERR_ALIGN, "flash_attn: output stride[%d] not a multiple of 16 bytes", i);
  if (!aligned(out, 16)) return set_error(SP_ERR_ALIGN, "flash_attn: output not 16-byte aligned");
  if (mask && mask_row_stride < Skv)
    return set_error(SP_ERR_SHAPE, "flash_attn: mask row stride smaller than Skv");
  if (int rc = require_sm100()) return rc;

  const int in_f16 = dtype_in == SP_F16;
  CUtensorMap mq, mk, mv;
  if (int rc = make_qkv_map(&mq, q, in_f16, Sq, H, B, (int)D, q_strides, "q")) return rc;
  if (int rc = make_qkv_map(&mk, k, in_f16, Skv, H, B, (int)D, k_strides, "k")) return rc;
  if (int rc = make_qkv_map(&mv, v, in_f16, Skv, H, B, (int)Dv, v_strides, "v")) return rc;

  FaParams p{};
  p.Sq = Sq;
  p.Skv = Skv;
  p.H = H;
  p.D = (int)D;
  p.Dv = (int)Dv;
  p.dqk_pad = (int)((D + 15) / 16 * 16);
  // V is an MN-major operand; its 128B-swizzle atoms are 64 elements wide, so the PV
  // product runs on whole atoms (Dv 40 -> N 64; the extra columns are TMA zero fill).
  p.dv_pad = (int)((Dv + 63) / 64 * 64);
  p.n_kv_tiles = (int)((Skv + kBN - 1) / kBN);
  const float sc = scale > 0.f ? scale : 1.0f / sqrtf((float)D);
  p.scale_log2 = sc * kLog2e;
  p.inv_scale = 1.0f / sc;
  p.causal = causal ? 1 : 0;
  p.mask = mask;
  p.mask_stride = mask_row_stride;
  p.out = out;
  p.os0 = o_strides[0];
  p.os1 = o_strides[1];
  p.os2 = o_strides[2];
  p.out_dtype = dtype_out;
  p.in_f16 = in_f16;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool qk2 = D > 64, v2 = Dv > 64;
  if (!qk2 && !v2) return launch_fa<1, 1, 3>(mq, mk, mv, p, B, s);  // 176 KB smem
  if (qk2 && v2) return launch_fa<2, 2, 2>(mq, mk, mv, p, B, s);     // 224 KB smem
  if (qk2) return launch_fa<2, 1, 2>(mq, mk, mv, p, B, s);
  return launch_fa<1, 2, 2>(mq, mk, mv, p, B, s);
}
