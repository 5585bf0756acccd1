// flash_attn.cu -- flash-attention forward for sm_100a: TMA-fed tcgen05 UMMA with TMEM
// accumulators and an online softmax.
//
// Computes out = softmax(Q K^T * scale [+ mask] [causal]) V with f32 accumulation, the
// operation of sketchpad_cubecl::flash_attention (crates/sketchpad-cubecl/src/attention.rs:97-178)
// and of the CPU attention it must match (crates/sketchpad-unet/src/blocks.rs:370-410).
//
// One CTA = two 128-query tiles (T0, T1) of one (batch, head); 384 threads = 3 warpgroups:
//   warps 0..3  softmax + epilogue of T0, warps 4..7 of T1
//   warp 8      TMA producer: both Q tiles once, then K/V tiles of 128 keys (STAGES ring).
//   warp 9      TMEM owner + MMA issuer (one elected lane), per key tile j:
//                 S_t = Q_t K_j^T   (M=128, N=128, K=D padded to 16; f32 in TMEM)
//                 O_t += P_t V_j    (M=128, N=Dv padded to 64, K=128; P_t read from TMEM)
//               so the tensor core works on one tile while the other tile's softmax runs.
//               Dv > 64 (P aliases S): S_0(0) S_1(0) | PV_0(j) S_0(j+1) PV_1(j) S_1(j+1) | ...
//               Dv <= 64 (P has its own columns): S_t(j+1) is issued as soon as the softmax
//               has loaded S_t(j) into registers (s_free barrier), then PV_0(j), PV_1(j).
//   softmax:    one query row per thread (= TMEM lane): tcgen05.ld S, mask, exp2, write P
//               (16-bit, 2 per column) back to
//               TMEM with tcgen05.st; O is rescaled in TMEM only when the row max grows by
//               more than 2^8 (P and the row sum always share one reference maximum).
// TMEM per tile t (base 256*t): Dv <= 64: S [0,128) P [128,192) O [192,256);
//                              Dv  > 64: S and P share [0,128) (P in [0,64)), O [128,256).
// A commit makes its mbarrier wait for every earlier tcgen05 op of the issuing thread.  When
// P aliases S, S_t(j) is issued after PV_t(j-1), so once S_t(j) is ready P_t may be rewritten
// and O_t rescaled without further waits (and the tensor core executes a thread's MMAs in
// issue order).  With the early-S schedule the softmax instead waits for PV_t(j-1)
// (o_done) after computing its exponentials, just before it rescales O_t and writes P_t.
// Q, K, V tiles in shared memory are 128 rows x 64 elements (128 B) boxes with the 128B
// swizzle: the canonical K-major layout for Q and K, MN-major for V.
#include <type_traits>

#include "common.cuh"
#include "tc.cuh"

namespace sp {
namespace {

constexpr int kBM = 128;            // queries per tile (two tiles per CTA)
constexpr int kBN = 128;            // keys per KV tile
constexpr int kBox = 16384;         // bytes of one 128 x 64 16-bit box
// Three whole warpgroups: registers are reserved per warpgroup, so 320 threads would cost
// as much as 384; warps 10 and 11 have no role.  168 registers per thread.
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;
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
  int single;  // 1: one query tile per CTA (grids that would leave SMs idle), 0: two
  // bounded waits: budget of each mbarrier wait in SM cycles; a tile index >= 0 here is
  // never loaded (sp_flash_attn_fwd_wait_test), so the waits for it expire and the CTA
  // takes its abort path
  long long wait_budget;
  int skip_kv_tile;
};

template <int NBQ, int NBV, int STAGES>
struct FaSmem {
  static constexpr int kQ = 0;                                // two tiles x NBQ boxes
  static constexpr int kK = kQ + 2 * NBQ * kBox;
  static constexpr int kV = kK + STAGES * NBQ * kBox;
  static constexpr int kBar = kV + STAGES * NBV * kBox;
  // barriers: q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_full[2],
  // o_done[2], s_free[2], drain
  static constexpr int kNumBars = 1 + 4 * STAGES + 2 + 2 + 2 + 2 + 1;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16;  // tmem base + abort flag
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-B alignment of the base
};

__device__ __forceinline__ uint32_t float_bits(float f) { return __float_as_uint(f); }

// TMEM column offsets inside one tile's 256 columns
template <int NBV>
struct FaTmem {
  static constexpr uint32_t kS = 0;
  static constexpr uint32_t kP = NBV == 1 ? 128 : 0;   // Dv > 64: P overwrites S
  static constexpr uint32_t kO = NBV == 1 ? 192 : 128;
};

template <int NBQ, int NBV, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, const FaParams p) {
  using L = FaSmem<NBQ, NBV, STAGES>;
  using TM = FaTmem<NBV>;
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
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* s_free = o_done + 2;
  uint64_t* drain = s_free + 2;
  // Dv <= 64: P has its own TMEM columns, so S_t(j+1) is issued as soon as the softmax has
  // loaded S_t(j) (s_free) instead of after PV_t(j): the MMA round trip leaves the softmax's
  // critical path, and the softmax waits for PV_t(j-1) (o_done) only before writing P.
  constexpr bool kEarlyQK = NBV == 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  // query tiles of this CTA: two, or one when the grid of tile pairs would leave SMs idle
  const int ntq = p.single ? 1 : 2;
  const int q0 = qt * ntq * kBM;

  // KV tiles this pair of query tiles needs (causal: keys <= last query of tile 1).
  int n_tiles = p.n_kv_tiles;
  if (p.causal) {
    const int last_q = min((int)p.Sq - 1, q0 + ntq * kBM - 1);
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
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 128);
      mbar_init(&o_done[t], 1);
      mbar_init(&s_free[t], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      mbar_arrive_expect_tx(q_full, ntq * NBQ * kBox);
      for (int t = 0; t < ntq; ++t)
        for (int blk = 0; blk < NBQ; ++blk)
          tma_load_4d(smem + L::kQ + (t * NBQ + blk) * kBox, &tmq, q_full, blk * 64, q0 + t * kBM,
                      h, b);
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (j >= STAGES && !mbar_wait(&k_empty[st], ph ^ 1, abort_flag, WD_TMA_WAIT, p.wait_budget)) break;
        if (j == p.skip_kv_tile) continue;  // test hook: this tile's barriers never complete
        mbar_arrive_expect_tx(&k_full[st], NBQ * kBox);
        for (int blk = 0; blk < NBQ; ++blk)
          tma_load_4d(smem + L::kK + (st * NBQ + blk) * kBox, &tmk, &k_full[st], blk * 64,
                      j * kBN, h, b);
        issued_k = j + 1;
        if (j >= STAGES && !mbar_wait(&v_empty[st], ph ^ 1, abort_flag, WD_TMA_WAIT, p.wait_budget)) break;
        mbar_arrive_expect_tx(&v_full[st], NBV * kBox);
        for (int blk = 0; blk < NBV; ++blk)
          tma_load_4d(smem + L::kV + (st * NBV + blk) * kBox, &tmv, &v_full[st], blk * 64,
                      j * kBN, h, b);
        issued_v = j + 1;
      }
      if (*abort_flag) {
        // Let every copy still in flight land before the CTA can exit (bounded).
        mbar_wait(q_full, 0, nullptr, WD_TMA_WAIT, p.wait_budget);
        for (int j = max(0, issued_k - STAGES); j < issued_k; ++j)
          mbar_wait(&k_full[j % STAGES], (j / STAGES) & 1, nullptr, WD_TMA_WAIT, p.wait_budget);
        for (int j = max(0, issued_v - STAGES); j < issued_v; ++j)
          mbar_wait(&v_full[j % STAGES], (j / STAGES) & 1, nullptr, WD_TMA_WAIT, p.wait_budget);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t ab = p.in_f16 ? 0u : 1u;
      const uint32_t idesc_qk = make_idesc_f16(kBM, kBN, ab, 0, 0);
      const uint32_t idesc_pv = make_idesc_f16(kBM, (uint32_t)p.dv_pad, ab, 0, 1);
      const uint32_t q_base = smem_u32(smem + L::kQ);
      const int qk_steps = p.dqk_pad / 16;

      // S_t = Q_t K_j^T
      auto issue_qk = [&](int t, int j) {
        const uint32_t k_base = smem_u32(smem + L::kK + (j % STAGES) * NBQ * kBox);
        const uint32_t qb = q_base + t * NBQ * kBox;
        for (int kk = 0; kk < qk_steps; ++kk) {
          const uint32_t off = (kk >> 2) * kBox + (kk & 3) * 32;
          const uint64_t a = make_smem_desc(qb + off, 16, 1024, LAYOUT_SW128);
          const uint64_t bd = make_smem_desc(k_base + off, 16, 1024, LAYOUT_SW128);
          umma_ss(tmem + t * 256 + TM::kS, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      // O_t += P_t V_j, P_t from TMEM (8 columns per 16 keys)
      auto issue_pv = [&](int t, int j) {
        const uint32_t v_base = smem_u32(smem + L::kV + (j % STAGES) * NBV * kBox);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t bd = make_smem_desc(v_base + kk * 16 * 128, kBox, 1024, LAYOUT_SW128);
          umma_ts(tmem + t * 256 + TM::kO, tmem + t * 256 + TM::kP + kk * 8, bd, idesc_pv,
                  (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&o_done[t]);
      };

      bool ok = mbar_wait(q_full, 0, abort_flag, WD_MMA_WAIT, p.wait_budget) &&
                (n_tiles == 0 || mbar_wait(&k_full[0], 0, abort_flag, WD_MMA_WAIT, p.wait_budget));
      tc_fence_after();
      if (ok && n_tiles > 0) {
        issue_qk(0, 0);
        if (ntq == 2) issue_qk(1, 0);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int st = j % STAGES;
        const bool more = j + 1 < n_tiles;
        const int st1 = (j + 1) % STAGES;
        if constexpr (kEarlyQK) {
          if (more) {
            if (!mbar_wait(&k_full[st1], ((j + 1) / STAGES) & 1, abort_flag, WD_MMA_WAIT, p.wait_budget)) break;
            if (!mbar_wait(&s_free[0], j & 1, abort_flag, WD_MMA_WAIT, p.wait_budget)) break;
            tc_fence_after();
            issue_qk(0, j + 1);
            if (ntq == 2) {
              if (!mbar_wait(&s_free[1], j & 1, abort_flag, WD_MMA_WAIT, p.wait_budget)) break;
              tc_fence_after();
              issue_qk(1, j + 1);
            }
            umma_commit(&k_empty[st1]);
          }
          if (!mbar_wait(&v_full[st], (j / STAGES) & 1, abort_flag, WD_MMA_WAIT, p.wait_budget)) break;
          if (!mbar_wait(&p_full[0], j & 1, abort_flag, WD_MMA_WAIT, p.wait_budget)) break;
          tc_fence_after();
          issue_pv(0, j);
          if (ntq == 2) {
            if (!mbar_wait(&p_full[1], j & 1, abort_flag, WD_MMA_WAIT, p.wait_budget)) break;
            tc_fence_after();
            issue_pv(1, j);
          }
          umma_commit(&v_empty[st]);
          continue;
        }
        if (!mbar_wait(&v_full[st], (j / STAGES) & 1, abort_flag, WD_MMA_WAIT, p.wait_budget)) break;
        if (!mbar_wait(&p_full[0], j & 1, abort_flag, WD_MMA_WAIT, p.wait_budget)) break;
        tc_fence_after();
        issue_pv(0, j);
        if (more) {
          if (!mbar_wait(&k_full[st1], ((j + 1) / STAGES) & 1, abort_flag, WD_MMA_WAIT, p.wait_budget)) break;
          tc_fence_after();
          issue_qk(0, j + 1);
        }
        if (ntq == 2) {
          if (!mbar_wait(&p_full[1], j & 1, abort_flag, WD_MMA_WAIT, p.wait_budget)) break;
          tc_fence_after();
          issue_pv(1, j);
        }
        umma_commit(&v_empty[st]);
        if (more) {
          if (ntq == 2) issue_qk(1, j + 1);
          umma_commit(&k_empty[st1]);
        }
      }
      // Drain: every MMA issued above has completed once this commit arrives.
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, WD_MMA_WAIT, p.wait_budget);
    }
  } else if (warp < 4 * ntq) {
    // ------------------------------------------------------------------ softmax + epilogue
    const int t = warp >> 2;       // query tile of this warpgroup
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const int qi = q0 + t * kBM + row;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16) + t * 256;
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;  // running max in log2 units, running row sum
    bool ok = true;

    for (int j = 0; j < n_tiles; ++j) {
      if (!mbar_wait_warp(&s_full[t], j & 1, abort_flag, WD_SOFTMAX_WAIT, p.wait_budget)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // Masks act on raw scores: x_log2 = (s + mask / scale) * scale * log2(e).
      const int kv0 = j * kBN;
      const bool need_mask = p.mask != nullptr || (kv0 + kBN > p.Skv) ||
                             (p.causal && kv0 + kBN - 1 > q0 + t * kBM);
      // the whole S row: four 32-column loads in flight, one wait; masked tiles (tail keys,
      // causal, additive mask) are rewritten in place on a separate, rarely taken path
      uint32_t r[4][32];
#pragma unroll
      for (int q = 0; q < 4; ++q) tmem_ld32(lane_addr + TM::kS + q * 32, r[q]);
      tmem_wait_ld();
      if constexpr (kEarlyQK) {
        tc_fence_before();
        mbar_arrive(&s_free[t]);  // S_t may now be overwritten by S_t(j+1)
      }
      if (need_mask) {
        if (p.mask == nullptr && !p.causal) {
          // only the key tail: columns at and past Skv - kv0 get -inf
          const int lim = (int)p.Skv - kv0;
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (q * 32 + c >= lim) r[q][c] = float_bits(-INFINITY);
        } else {
          // tail keys and causal positions -> -inf; the additive mask is applied in raw units
          // (x_log2 = (s + mask / scale) * scale * log2 e)
          const int lim = (int)p.Skv - kv0;
          const int clim = p.causal ? qi - kv0 + 1 : lim;  // causal: keys <= qi
          const float* mrow =
              (p.mask && qi < p.Sq) ? p.mask + (int64_t)qi * p.mask_stride + kv0 : nullptr;
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const int col = q * 32 + c;
              const bool valid = col < lim && col < clim;
              float x = __uint_as_float(r[q][c]);
              if (mrow && valid) x += mrow[col] * p.inv_scale;
              r[q][c] = float_bits(valid ? x : -INFINITY);
            }
        }
      }
      float mx;
      {
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int c = 0; c < 32; ++c) m4[c & 3] = fmaxf(m4[c & 3], __uint_as_float(r[q][c]));
        mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      }
      const float m_tile = mx == -INFINITY ? -INFINITY : __fmul_rn(mx, sl2);
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

      // tcgen05.ld/st are warp-collective: the whole warp rescales O if any of its rows
      // must (alpha = 1 for the others).  O must already hold PV_t(j-1).
      auto rescale_o = [&]() {
        if (__any_sync(0xffffffffu, rescale)) {
          const float alpha = rescale ? ex2_approx(m_run - m_ref) : 1.0f;
          l_run *= alpha;
          for (int c = 0; c < p.dv_pad; c += 16) {
            uint32_t ro[16];
            tmem_ld16(lane_addr + TM::kO + c, ro);
            tmem_wait_ld();
#pragma unroll
            for (int u = 0; u < 16; ++u) ro[u] = float_bits(__uint_as_float(ro[u]) * alpha);
            tmem_st16(lane_addr + TM::kO + c, ro);
          }
        }
      };
      // Aliased layout: S_t(j)'s commit followed PV_t(j-1), so O is final here.
      if constexpr (!kEarlyQK) rescale_o();

      // exp2 (MUFU), row sum, 16-bit P (column c holds keys 2c, 2c+1); -inf scores of
      // masked tiles give exactly 0.  x = s * scale - m_ref is one fused multiply-add while
      // m_ref is the ROUNDED product max * scale, so the row maximum's x is off by up to half
      // an ulp of m_ref either way: harmless for ordinary logits, but past |m_ref| ~ 2^24 that
      // is more than 1 -- with logits of 1e11 and up (activations in the millions) ex2
      // overflows to inf or the maximum's P underflows to 0.  Warps with such a reference
      // form x = fl(s * scale) - m_ref from separately rounded operations: exactly 0 for the
      // maximum (rounded like m_ref), <= 0 for every other key.
      float rs0 = 0.f, rs1 = 0.f;
      uint32_t pk[4][16];
      auto exps = [&](auto exact) {
        constexpr bool kExact = decltype(exact)::value;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            float x0, x1;
            if constexpr (kExact) {
              x0 = __fsub_rn(__fmul_rn(__uint_as_float(r[q][2 * u]), sl2), m_ref);
              x1 = __fsub_rn(__fmul_rn(__uint_as_float(r[q][2 * u + 1]), sl2), m_ref);
            } else {
              x0 = fmaf(__uint_as_float(r[q][2 * u]), sl2, -m_ref);
              x1 = fmaf(__uint_as_float(r[q][2 * u + 1]), sl2, -m_ref);
            }
            const float e0 = ex2_approx(x0), e1 = ex2_approx(x1);
            rs0 += e0;
            rs1 += e1;
            pk[q][u] = p.in_f16 ? pack_f16x2(e0, e1) : pack_bf16x2(e0, e1);
          }
          if constexpr (!kEarlyQK) tmem_st16(lane_addr + TM::kP + q * 16, pk[q]);
        }
      };
      if (__any_sync(0xffffffffu, fabsf(m_ref) > 1.0e6f))
        exps(std::true_type{});
      else
        exps(std::false_type{});
      if constexpr (kEarlyQK) {
        // PV_t(j-1) must be done before P_t is rewritten and O rescaled
        if (j >= 1 && !mbar_wait_warp(&o_done[t], (j - 1) & 1, abort_flag, WD_SOFTMAX_WAIT, p.wait_budget)) {
          ok = false;
          break;
        }
        tc_fence_after();
        rescale_o();
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_st16(lane_addr + TM::kP + q * 16, pk[q]);
      }
      m_run = m_use;
      l_run += rs0 + rs1;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }

    // ---- epilogue: O / l -> global
    const int last = n_tiles - 1;
    if (ok && n_tiles > 0 &&
        mbar_wait_warp(&o_done[t], last & 1, abort_flag, WD_EPILOGUE_WAIT, p.wait_budget)) {
      tc_fence_after();
      const float inv_l = l_run > 0.f ? 1.0f / l_run : 0.f;
      const bool row_ok = qi < p.Sq;
      const int64_t obase = (int64_t)b * p.os0 + (int64_t)h * p.os1 + (int64_t)qi * p.os2;
      for (int c = 0; c < p.dv_pad; c += 16) {
        uint32_t r[16];
        tmem_ld16(lane_addr + TM::kO + c, r);
        tmem_wait_ld();
        if (!row_ok || c >= p.Dv) continue;
        float o[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) o[u] = __uint_as_float(r[u]) * inv_l;
        const int ncol = min(16, p.Dv - c);  // multiple of 8
        if (p.out_dtype == SP_F32) {
          float* dst = static_cast<float*>(p.out) + obase + c;
          for (int u = 0; u < ncol; u += 4)
            *reinterpret_cast<float4*>(dst + u) = make_float4(o[u], o[u + 1], o[u + 2], o[u + 3]);
        } else {
          uint16_t* dst = static_cast<uint16_t*>(p.out) + obase + c;
          for (int u = 0; u < ncol; u += 8) {
            uint4 w;
            if (p.out_dtype == SP_BF16) {
              w = make_uint4(pack_bf16x2(o[u], o[u + 1]), pack_bf16x2(o[u + 2], o[u + 3]),
                             pack_bf16x2(o[u + 4], o[u + 5]), pack_bf16x2(o[u + 6], o[u + 7]));
            } else {
              w = make_uint4(pack_f16x2(o[u], o[u + 1]), pack_f16x2(o[u + 2], o[u + 3]),
                             pack_f16x2(o[u + 4], o[u + 5]), pack_f16x2(o[u + 6], o[u + 7]));
            }
            *reinterpret_cast<uint4*>(dst + u) = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
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
    cudaFuncAttributes fa{};
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess || fa.maxThreadsPerBlock < kThreads) {
      __atomic_fetch_and(&attr_set, ~(1ull << current_device()), __ATOMIC_ACQ_REL);
      return set_error(SP_ERR_LAUNCH,
                       "flash_attn: kernel cannot launch %d threads (%s; regs/thread %d, max threads "
                       "%d, dynamic smem %d of %d)",
                       kThreads, cudaGetErrorString(e), fa.numRegs, fa.maxThreadsPerBlock, L::kAlloc,
                       fa.maxDynamicSharedSizeBytes);
    }
  }
  const int tiles = p.single ? 1 : 2;
  dim3 grid((unsigned)((p.Sq + tiles * kBM - 1) / (tiles * kBM)), (unsigned)p.H, (unsigned)B);
  kern<<<grid, kThreads, L::kAlloc, s>>>(mq, mk, mv, p);
  return check_launch("flash_attn");
}

}  // namespace
}  // namespace sp

namespace sp {
namespace {

// ---------------------------------------------------------------------------------------
// Short sequences (Sq, Skv <= 32, D = Dv in {64, 128}, no mask, not causal): one warp per
// (batch, head).  Wan's temporal attention runs 144,000 such problems of 21 tokens, where
// 128-row tensor-core tiles would be 84 % padding and per-CTA setup dominates.  The warp
// works on 32-row tiles with mma.sync m16n8k16 (f32 accumulate), the softmax in exp2 with
// the scale folded in, as the tiled kernel does.
// ---------------------------------------------------------------------------------------
constexpr int kShortWarps = 4;
constexpr int kShortMax = 32;

struct ShortArgs {
  int64_t BH, H, Sq, Skv;
  int64_t qs0, qs1, qs2, ks0, ks1, ks2, vs0, vs1, vs2, os0, os1, os2;
  float scale_log2;
  int out_dtype;
};

// The warp's Q, K and V rows are copied to shared memory by cp.async (rows past Sq / Skv
// zero filled), S = Q K^T is formed as 16 x 8 tiles over K = DH with ldmatrix fragments,
// P = softmax(S) stays in registers as the A operand of O = P V (the S accumulator layout is
// the A fragment layout of the next product), and V's B fragments come from its row-major
// rows by ldmatrix.trans.  The bf16/f16 output is staged in the Q rows of the finished tile
// and written back as 16-byte rows.  Padded keys get -inf before the softmax.
// Fragment layouts (PTX mma.m16n8k16, g = lane / 4, t = lane % 4): A a0 = A[g][2t..2t+1],
// a1 = A[g+8][2t..], a2 = A[g][2t+8..], a3 = A[g+8][2t+8..]; B b0 = B[2t..2t+1][g],
// b1 = B[2t+8..2t+9][g]; C c0,c1 = C[g][2t..2t+1], c2,c3 = C[g+8][2t..2t+1].
constexpr int kSmRow = 8;  // padding elements per shared row: 8 rows of a fragment hit 32 banks

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// 16-byte global -> shared copy; src_bytes = 0 writes 16 zero bytes and reads nothing
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (std::is_same<T, __half>::value) return pack_f16x2(lo, hi);
  else return pack_bf16x2(lo, hi);
}

template <int OUT>
__device__ __forceinline__ uint32_t pack_out2(float lo, float hi) {
  if constexpr (OUT == SP_F16) return pack_f16x2(lo, hi);
  else return pack_bf16x2(lo, hi);
}

template <typename T, int DH, int OUT>
__global__ void __launch_bounds__(kShortWarps * 32) attn_short_mma_kernel(const T* __restrict__ q,
                                                                          const T* __restrict__ k,
                                                                          const T* __restrict__ v,
                                                                          void* out, ShortArgs a) {
  constexpr int RS = DH + kSmRow;  // row stride of the Q / K / V rows in shared memory (elements)
  constexpr int kChunks = DH / 8;  // 16-byte chunks per row
  constexpr int kRowsBytes = kShortMax * RS * 2;
  extern __shared__ uint4 sh_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t pb = (int64_t)blockIdx.x * kShortWarps + warp;
  if (pb >= a.BH) return;  // warp-uniform
  T* sq = reinterpret_cast<T*>(sh_raw) + (int64_t)warp * 3 * kShortMax * RS;
  const uint32_t sq_a = (uint32_t)__cvta_generic_to_shared(sq);
  const uint32_t sk_a = sq_a + kRowsBytes, sv_a = sk_a + kRowsBytes;
  const int64_t b = pb / a.H, h = pb - b * a.H;
  const T* qp = q + b * a.qs0 + h * a.qs1;
  const T* kp = k + b * a.ks0 + h * a.ks1;
  const T* vp = v + b * a.vs0 + h * a.vs1;
  const int Sq = (int)a.Sq, Skv = (int)a.Skv;
#pragma unroll 4
  for (int e = lane; e < kShortMax * kChunks; e += 32) {
    const int r = e / kChunks, c = e - r * kChunks;
    const uint32_t so = (uint32_t)(r * RS + c * 8) * 2;
    const bool rq = r < Sq, rkv = r < Skv;
    cp_async16(sq_a + so, rq ? qp + r * a.qs2 + c * 8 : qp, rq ? 16 : 0);
    cp_async16(sk_a + so, rkv ? kp + r * a.ks2 + c * 8 : kp, rkv ? 16 : 0);
    cp_async16(sv_a + so, rkv ? vp + r * a.vs2 + c * 8 : vp, rkv ? 16 : 0);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncwarp();
  // ldmatrix lane addressing: lane l supplies row (l & 7) of matrix (l >> 3)
  const int mi = lane >> 3, rr = lane & 7;
  const bool kv_hi = Skv > 16;  // keys 16..31 present (second S tile pair, second PV k-step)
  for (int mt = 0; mt < 2; ++mt) {
    if (mt * 16 >= Sq) break;
    float sacc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) sacc[nt][i] = 0.f;
    // S = Q K^T: rows 16mt .. 16mt+15, keys 0..31 (the upper 16 only when present)
#pragma unroll
    for (int ks = 0; ks < DH / 16; ++ks) {
      uint32_t af[4], kb[4];
      ldsm_x4(af, sq_a + (uint32_t)((mt * 16 + (mi & 1) * 8 + rr) * RS + ks * 16 + (mi >> 1) * 8) * 2);
      ldsm_x4(kb, sk_a + (uint32_t)(((mi >> 1) * 8 + rr) * RS + ks * 16 + (mi & 1) * 8) * 2);
      mma16816<T>(sacc[0], af, kb[0], kb[1]);
      mma16816<T>(sacc[1], af, kb[2], kb[3]);
      if (kv_hi) {
        ldsm_x4(kb, sk_a + (uint32_t)((16 + (mi >> 1) * 8 + rr) * RS + ks * 16 + (mi & 1) * 8) * 2);
        mma16816<T>(sacc[2], af, kb[0], kb[1]);
        mma16816<T>(sacc[3], af, kb[2], kb[3]);
      }
    }
    // softmax over keys for rows g and g+8 of the tile; the 4 lanes of a row hold 8 keys each
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int key = nt * 8 + 2 * t + (i & 1);
        const float x = key < Skv ? sacc[nt][i] * a.scale_log2 : -INFINITY;
        sacc[nt][i] = x;
        if (i < 2) mx0 = fmaxf(mx0, x);
        else mx1 = fmaxf(mx1, x);
      }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    float l0 = 0.f, l1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float pe = ex2_approx(sacc[nt][i] - (i < 2 ? mx0 : mx1));
        sacc[nt][i] = pe;
        if (i < 2) l0 += pe;
        else l1 += pe;
      }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    // P as A fragments: k-step kk covers keys 16kk .. 16kk+15 = S tiles 2kk, 2kk+1
    uint32_t pf[2][4];
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      pf[kk][0] = pack2<T>(sacc[2 * kk][0], sacc[2 * kk][1]);
      pf[kk][1] = pack2<T>(sacc[2 * kk][2], sacc[2 * kk][3]);
      pf[kk][2] = pack2<T>(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
      pf[kk][3] = pack2<T>(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
    }
    const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
    const int r0 = mt * 16 + g, r1 = r0 + 8;
    __syncwarp();  // every lane's Q fragments of this tile are read: its rows take the output
    // O = P V, 16 output columns (two 8-column tiles) per step
#pragma unroll 2
    for (int np = 0; np < DH / 16; ++np) {
      float oa[4] = {0.f, 0.f, 0.f, 0.f}, ob[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t vb[4];
      ldsm_x4_trans(vb, sv_a + (uint32_t)(((mi & 1) * 8 + rr) * RS + np * 16 + (mi >> 1) * 8) * 2);
      mma16816<T>(oa, pf[0], vb[0], vb[1]);
      mma16816<T>(ob, pf[0], vb[2], vb[3]);
      if (kv_hi) {
        ldsm_x4_trans(vb, sv_a + (uint32_t)((16 + (mi & 1) * 8 + rr) * RS + np * 16 + (mi >> 1) * 8) * 2);
        mma16816<T>(oa, pf[1], vb[0], vb[1]);
        mma16816<T>(ob, pf[1], vb[2], vb[3]);
      }
      const int col = np * 16 + 2 * t;
      if constexpr (OUT == SP_F32) {
        float* o = static_cast<float*>(out) + b * a.os0 + h * a.os1 + col;
        if (r0 < Sq) {
          *reinterpret_cast<float2*>(o + (int64_t)r0 * a.os2) = make_float2(oa[0] * inv0, oa[1] * inv0);
          *reinterpret_cast<float2*>(o + (int64_t)r0 * a.os2 + 8) = make_float2(ob[0] * inv0, ob[1] * inv0);
        }
        if (r1 < Sq) {
          *reinterpret_cast<float2*>(o + (int64_t)r1 * a.os2) = make_float2(oa[2] * inv1, oa[3] * inv1);
          *reinterpret_cast<float2*>(o + (int64_t)r1 * a.os2 + 8) = make_float2(ob[2] * inv1, ob[3] * inv1);
        }
      } else {
        uint32_t* s0 = reinterpret_cast<uint32_t*>(sq + r0 * RS + col);
        uint32_t* s1 = reinterpret_cast<uint32_t*>(sq + r1 * RS + col);
        s0[0] = pack_out2<OUT>(oa[0] * inv0, oa[1] * inv0);
        s0[4] = pack_out2<OUT>(ob[0] * inv0, ob[1] * inv0);
        s1[0] = pack_out2<OUT>(oa[2] * inv1, oa[3] * inv1);
        s1[4] = pack_out2<OUT>(ob[2] * inv1, ob[3] * inv1);
      }
    }
  }
  if constexpr (OUT != SP_F32) {
    __syncwarp();
    uint16_t* o = static_cast<uint16_t*>(out) + b * a.os0 + h * a.os1;
    for (int e = lane; e < Sq * kChunks; e += 32) {
      const int r = e / kChunks, c = e - r * kChunks;
      *reinterpret_cast<uint4*>(o + r * a.os2 + c * 8) =
          *reinterpret_cast<const uint4*>(sq + r * RS + c * 8);
    }
  }
}

template <typename T, int DH, int OUT>
int launch_attn_short_mma(const void* q, const void* k, const void* v, void* out,
                          const ShortArgs& a, cudaStream_t s) {
  auto kern = attn_short_mma_kernel<T, DH, OUT>;
  const int smem = kShortWarps * 3 * kShortMax * (DH + kSmRow) * (int)sizeof(T);
  static unsigned long long attr_set = 0;
  if (smem > 48 * 1024 && first_time_on_device(&attr_set)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      __atomic_fetch_and(&attr_set, ~(1ull << current_device()), __ATOMIC_ACQ_REL);
      return set_error(SP_ERR_LAUNCH, "flash_attn: short-sequence smem attribute: %s",
                       cudaGetErrorString(e));
    }
  }
  const unsigned grid = (unsigned)((a.BH + kShortWarps - 1) / kShortWarps);
  kern<<<grid, kShortWarps * 32, smem, s>>>(static_cast<const T*>(q), static_cast<const T*>(k),
                                            static_cast<const T*>(v), out, a);
  return check_launch("flash_attn short (mma)");
}

template <typename T, int DH>
int launch_attn_short_out(const void* q, const void* k, const void* v, void* out,
                          const ShortArgs& a, cudaStream_t s) {
  switch (a.out_dtype) {
    case SP_F32: return launch_attn_short_mma<T, DH, SP_F32>(q, k, v, out, a, s);
    case SP_F16: return launch_attn_short_mma<T, DH, SP_F16>(q, k, v, out, a, s);
    default: return launch_attn_short_mma<T, DH, SP_BF16>(q, k, v, out, a, s);
  }
}


}  // namespace
}  // namespace sp

namespace sp {
namespace {
int flash_attn_impl(const void* q, const void* k, const void* v, const float* mask,
                    int64_t mask_row_stride, void* out, int64_t B, int64_t H, int64_t Sq,
                    int64_t Skv, int64_t D, int64_t Dv, const int64_t q_strides[4],
                    const int64_t k_strides[4], const int64_t v_strides[4],
                    const int64_t o_strides[4], int dtype_in, int dtype_out, int causal,
                    float scale, void* stream, long long wait_budget, int skip_kv_tile) {
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const float sc0 = scale > 0.f ? scale : 1.0f / sqrtf((float)D);
  if (!mask && !causal && Sq <= kShortMax && Skv <= kShortMax && D == Dv && (D == 64 || D == 128) &&
      q_strides[3] == 1 && k_strides[3] == 1 && v_strides[3] == 1 && aligned(q, 16) &&
      aligned(k, 16) && aligned(v, 16) && q_strides[0] % 8 == 0 && q_strides[1] % 8 == 0 &&
      q_strides[2] % 8 == 0 && k_strides[0] % 8 == 0 && k_strides[1] % 8 == 0 &&
      k_strides[2] % 8 == 0 && v_strides[0] % 8 == 0 && v_strides[1] % 8 == 0 &&
      v_strides[2] % 8 == 0) {
    const ShortArgs a{B * H, H, Sq, Skv,
                      q_strides[0], q_strides[1], q_strides[2],
                      k_strides[0], k_strides[1], k_strides[2],
                      v_strides[0], v_strides[1], v_strides[2],
                      o_strides[0], o_strides[1], o_strides[2], sc0 * kLog2e, dtype_out};
    if (in_f16)
      return D == 64 ? launch_attn_short_out<__half, 64>(q, k, v, out, a, s)
                     : launch_attn_short_out<__half, 128>(q, k, v, out, a, s);
    return D == 64 ? launch_attn_short_out<__nv_bfloat16, 64>(q, k, v, out, a, s)
                   : launch_attn_short_out<__nv_bfloat16, 128>(q, k, v, out, a, s);
  }
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
  // one query tile per CTA when the grid of tile pairs would not cover the SMs
  p.single = (Sq + 2 * kBM - 1) / (2 * kBM) * H * B < num_sms() ? 1 : 0;
  p.wait_budget = wait_budget;
  p.skip_kv_tile = skip_kv_tile;
  const bool qk2 = D > 64, v2 = Dv > 64;
  if (!qk2 && !v2) return launch_fa<1, 1, 4>(mq, mk, mv, p, B, s);  // 160 KB smem
  if (qk2 && v2) return launch_fa<2, 2, 2>(mq, mk, mv, p, B, s);     // 192 KB smem
  if (qk2) return launch_fa<2, 1, 3>(mq, mk, mv, p, B, s);           // 208 KB smem
  return launch_fa<1, 2, 3>(mq, mk, mv, p, B, s);                    // 176 KB smem
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
  sp::clear_error();
  return sp::flash_attn_impl(q, k, v, mask, mask_row_stride, out, B, H, Sq, Skv, D, Dv,
                             q_strides, k_strides, v_strides, o_strides, dtype_in, dtype_out,
                             causal, scale, stream, sp::kWaitBudgetCycles, -1);
}

extern "C" int sp_flash_attn_fwd_wait_test(const void* q, const void* k, const void* v, void* out,
                                           int64_t B, int64_t H, int64_t S, int64_t D,
                                           int skip_kv_tile, int64_t wait_budget_cycles,
                                           void* stream) {
  sp::clear_error();
  if (S <= sp::kShortMax || skip_kv_tile < 0 || skip_kv_tile >= (S + sp::kBN - 1) / sp::kBN ||
      wait_budget_cycles < 1000000 || wait_budget_cycles > sp::kWaitBudgetCycles)
    return sp::set_error(SP_ERR_INVALID_ARG,
                         "wait test: needs S > %d, a key tile index in range and a budget in "
                         "[1e6, %lld] cycles", sp::kShortMax, (long long)sp::kWaitBudgetCycles);
  const int64_t st[4] = {H * S * D, S * D, D, 1};
  return sp::flash_attn_impl(q, k, v, nullptr, 0, out, B, H, S, S, D, D, st, st, st, st, SP_BF16,
                             SP_BF16, 0, 0.f, stream, wait_budget_cycles, skip_kv_tile);
}
