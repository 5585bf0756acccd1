/*
 * sketchpad_b200.h -- C ABI of the B200-native (sm_100a) diffusion-denoiser kernels.
 *
 * Drop-in boundary for the GPU operator surface of rhi-zone/sketchpad
 * (crates/sketchpad-cubecl): fused flash attention, fused GroupNorm(+SiLU), Q8_0 and FP8
 * quantized linears.  Conventions shared by every entry point:
 *   - all pointers are device pointers unless the name ends in _host;
 *   - every launch is asynchronous on `stream` (a cudaStream_t; NULL = legacy default);
 *   - outputs are allocated by the caller (the reference allocates them inside the op and
 *     hands them to the caller; here the caller owns both sides);
 *   - the return value is a status code (SP_OK = 0, negative = error) and the library never
 *     aborts; sp_last_error() returns a message for the calling thread's last failure;
 *   - strides are in ELEMENTS, dimension order as in the reference tensor's shape.
 */
#ifndef SKETCHPAD_B200_H
#define SKETCHPAD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SP_ABI_VERSION 1

typedef enum sp_status {
  SP_OK = 0,
  SP_ERR_INVALID_ARG = -1, /* null pointer, non-positive size, bad enum */
  SP_ERR_SHAPE = -2,       /* inconsistent or unsupported shape (e.g. C % groups != 0) */
  SP_ERR_DTYPE = -3,       /* dtype combination not supported */
  SP_ERR_ALIGN = -4,       /* pointer/stride alignment the kernel cannot use */
  SP_ERR_LAUNCH = -5,      /* CUDA launch / driver call failed */
  SP_ERR_WORKSPACE = -6,   /* workspace missing or too small */
  SP_ERR_DEVICE = -7,      /* device is not sm_100 */
  SP_ERR_COMM = -8         /* NCCL missing or failed, or a communication deadline passed */
} sp_status;

typedef enum sp_dtype { SP_F32 = 0, SP_F16 = 1, SP_BF16 = 2 } sp_dtype;

typedef enum sp_act { SP_ACT_NONE = 0, SP_ACT_SILU = 1 } sp_act;

/* Library ABI version (SP_ABI_VERSION). */
int sp_abi_version(void);
/* Message describing the calling thread's most recent failed call ("" if none). */
const char* sp_last_error(void);
/* Reads and clears the device watchdog word of the current device: 0 when no bounded
 * device-side wait has expired since the last call, else the code of the first expiry.
 * Synchronizes `stream`. */
int sp_watchdog_read_and_clear(void* stream, int* code_out);

/* ------------------------------------------------------------------------------------
 * Flash attention forward.
 * Replaces sketchpad_cubecl::flash_attention / flash_attention_masked
 *   (crates/sketchpad-cubecl/src/attention.rs:97, :119, impl :130-178).
 * out = softmax(Q K^T * scale [+ mask] [causal]) V with an f32 accumulator.
 *   q [B,H,Sq,D], k [B,H,Skv,D], v [B,H,Skv,Dv], out [B,H,Sq,Dv], any element strides
 *   whose innermost stride is 1 and whose other strides are multiples of 8 elements.
 *   dtype_in: SP_BF16 or SP_F16 (q, k, v share it); dtype_out: SP_BF16, SP_F16 or SP_F32.
 *   D, Dv: multiples of 8 in [8, 128].
 *   mask: NULL or an additive f32 mask [Sq, Skv] (row stride mask_row_stride), shared by
 *         every batch and head (the reference's Tensor<B,2> mask).
 *   causal: key j > query i is excluded (FlashAttentionOptions::causal, :40-68).
 *   scale <= 0 selects 1/sqrt(D).
 * ------------------------------------------------------------------------------------ */
int sp_flash_attn_fwd(const void* q, const void* k, const void* v, const float* mask,
                      int64_t mask_row_stride, void* out, int64_t B, int64_t H, int64_t Sq,
                      int64_t Skv, int64_t D, int64_t Dv, const int64_t q_strides[4],
                      const int64_t k_strides[4], const int64_t v_strides[4],
                      const int64_t o_strides[4], int dtype_in, int dtype_out, int causal,
                      float scale, void* stream);

/* Failure-handling check (no reference counterpart): sp_flash_attn_fwd on contiguous bf16
 * q, k, v, out [B,H,S,D] (S > 32) whose TMA producer never loads key/value tile
 * `skip_kv_tile`, with every bounded device wait given `wait_budget_cycles` (>= 1e6 SM
 * cycles) instead of the ~2 s default.  The waits for the missing tile run out, the kernel
 * records the code in the device watchdog word (sp_watchdog_read_and_clear), lets its copies
 * in flight land, frees its tensor memory and returns; out is left unspecified.  Lets a test
 * make a device wait expire without faulting or hanging the GPU and check that the context
 * stays usable. */
int sp_flash_attn_fwd_wait_test(const void* q, const void* k, const void* v, void* out, int64_t B,
                                int64_t H, int64_t S, int64_t D, int skip_kv_tile,
                                int64_t wait_budget_cycles, void* stream);

/* ------------------------------------------------------------------------------------
 * GroupNorm (+ SiLU), single pass over HBM.
 * Replaces sketchpad_cubecl::groupnorm_silu / groupnorm
 *   (crates/sketchpad-cubecl/src/groupnorm_silu.rs:232, :323; GroupNormSiLuOptions :22-46)
 * with the semantics of the CPU path crates/sketchpad-core/src/groupnorm.rs:62-102
 * (clamp +-65000, f32 statistics, biased variance, clamp after the affine).
 *   x [B,C,H,W] with element strides x_strides (NULL = contiguous NCHW).  y [B,C,H,W] is
 *   written channels-last (strides C*H*W, 1, W*C, C) when x is dense channels-last -- the
 *   layout sm_100 implicit-GEMM convolutions use -- and contiguous NCHW otherwise.
 *   gamma, beta [C]; x, y, gamma, beta all of `dtype` (SP_F32, SP_F16, SP_BF16).
 *   act: SP_ACT_SILU (groupnorm_silu) or SP_ACT_NONE (groupnorm).
 *   Returns SP_ERR_SHAPE when C % groups != 0 (the reference panics there).
 * workspace: NCHW groups of 256 KB and more take the streaming path, which keeps per-slice
 *   statistics in device workspace (16 bytes per 32 KB slice plus 4 bytes per group, zeroed
 *   by the call itself); channels-last and other strided inputs use two-kernel paths that
 *   need workspace too.  sp_groupnorm_act_workspace_size() returns its size, or 0 when x and
 *   y are 16-byte aligned and the single-pass on-chip NCHW path applies (workspace may then
 *   be NULL).  Workspace must be 16-byte aligned and not in use by another call in flight.
 * ------------------------------------------------------------------------------------ */
size_t sp_groupnorm_act_workspace_size(int64_t B, int64_t C, int64_t H, int64_t W,
                                       const int64_t x_strides[4], int64_t groups, int dtype);
int sp_groupnorm_act(const void* x, const void* gamma, const void* beta, void* y, int64_t B,
                     int64_t C, int64_t H, int64_t W, const int64_t x_strides[4], int64_t groups,
                     float eps, int act, int dtype, void* workspace, size_t workspace_bytes,
                     void* stream);
/* The element strides sp_groupnorm_act writes y with for this x: channels-last when x is
 * dense channels-last (dimensions of size 1 ignored, C == 1 counts as NCHW), else contiguous
 * NCHW.  Callers that allocate y (the reference allocates it inside groupnorm_silu,
 * groupnorm_silu.rs:287) use this to label it.  SP_ERR_INVALID_ARG on non-positive sizes. */
int sp_groupnorm_act_output_strides(int64_t B, int64_t C, int64_t H, int64_t W,
                                    const int64_t x_strides[4], int64_t y_strides[4]);

/* GroupNorm (+ SiLU) of x + x_add[b, c]: the ResBlock's time-embedding add (h + temb[:, :,
 * None, None]) followed by its second GroupNorm(+SiLU), as ResBlockCubeCL::forward does in two
 * steps (crates/sketchpad-unet/src/cubecl.rs:115-124; CPU: ResBlock::forward,
 * crates/sketchpad-unet/src/blocks.rs:123-150), in one pass over x.  x_add is [B, C] in the
 * same dtype (contiguous); the sum is formed in f32 and never stored.  x must be dense
 * channels-last (NHWC) -- the layout the UNet keeps -- otherwise SP_ERR_SHAPE.  Workspace:
 * sp_groupnorm_act_workspace_size() for the same arguments. */
int sp_groupnorm_add_act(const void* x, const void* x_add, const void* gamma, const void* beta,
                         void* y, int64_t B, int64_t C, int64_t H, int64_t W,
                         const int64_t x_strides[4], int64_t groups, float eps, int act,
                         int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* GroupNorm (+ SiLU) that allocates nothing.  No counterpart in the reference: it exists
 * for callers that cannot hand the library device memory -- hosts whose allocator must not
 * be used while they run, or FFI hosts holding raw device pointers without access to a CUDA
 * allocator.  Same semantics and arguments as sp_groupnorm_act minus the workspace; it
 * always runs the two-pass kernels, keeping their per-chunk statistics in a fixed array
 * inside the library (sp_groupnorm_act_noalloc_max_scratch_bytes() bytes, 256 KB, held on
 * every device that loads the library until exit).  Shapes needing more are rejected with
 * SP_ERR_WORKSPACE (the limit is batch x groups x ceil(C/groups*H*W / 16384) <= 21845).
 * The first call on a device looks up the array's device address and must come before any
 * stream capture on that device.  Calls sharing a device share the array, so calls that can
 * overlap on the GPU race. */
size_t sp_groupnorm_act_noalloc_max_scratch_bytes(void);
int sp_groupnorm_act_noalloc(const void* x, const void* gamma, const void* beta, void* y,
                             int64_t B, int64_t C, int64_t H, int64_t W,
                             const int64_t x_strides[4], int64_t groups, float eps, int act,
                             int dtype, void* stream);

/* Gated-linear-unit gate of a feed-forward, one pass over the stacked [rows, 2F] hidden:
 *   SP_GLU_GEGLU:  y = x[:, :F] * gelu(x[:, F:])  (erf GELU; UNet FeedForward::forward,
 *                  crates/sketchpad-unet/src/blocks.rs:446-458)
 *   SP_GLU_SWIGLU: y = silu(x[:, :F]) * x[:, F:]  (SwiGluFfn::forward,
 *                  crates/sketchpad-core/src/glu.rs:91-96; WanExpert::forward,
 *                  crates/sketchpad-dit/src/wan.rs:330-337)
 * Row strides in elements (x >= 2F, y >= F); F and both strides multiples of the 16-byte
 * vector; x, y 16-byte aligned; f32 arithmetic for every dtype. */
typedef enum sp_glu_kind { SP_GLU_GEGLU = 0, SP_GLU_SWIGLU = 1 } sp_glu_kind;
int sp_glu_gate(const void* x, void* y, int64_t rows, int64_t F, int64_t x_row_stride,
                int64_t y_row_stride, int kind, int dtype, void* stream);

/* out[p, c] = y[p, c] + bias[c] (+ r[p, c]) over channels-last [rows, C] activations: a
 * convolution's bias together with the ResBlock residual add (ResBlock::forward,
 * crates/sketchpad-unet/src/blocks.rs:123-150, conv2(h) + skip(x)), one pass.  r may be NULL
 * (bias only) and may alias out.  C a multiple of the 16-byte vector; all pointers 16-byte
 * aligned; f32 arithmetic. */
int sp_add_bias_residual(const void* y, const void* r, const void* bias, void* out, int64_t rows,
                         int64_t C, int dtype, void* stream);

/* ------------------------------------------------------------------------------------
 * Q8_0 (GGUF) weights.
 * A Q8_0 row of in_f values is in_f/32 blocks of 34 bytes: f16 LE scale + 32 int8.
 * The GPU layout is planar: q [out_f, in_f] int8 and scale [in_f/32, out_f] f16 bits
 * (k-block-major: scale[kb][n] belongs to q[n][32*kb .. 32*kb+31]); the repack is
 * lossless, so decode stays bit-exact.
 * ------------------------------------------------------------------------------------ */
/* Host repack of GGUF bytes (replaces the upload in GpuQuantizedLinear::from_bytes,
 * crates/sketchpad-cubecl/src/quantized_matmul.rs:670-702). */
int sp_q8_0_repack_host(const uint8_t* gguf_host, size_t nbytes, int64_t out_f, int64_t in_f,
                        int8_t* q_host, uint16_t* scale_host);
/* Device repack of GGUF bytes already in device memory. */
int sp_q8_0_repack(const void* gguf, size_t nbytes, int64_t out_f, int64_t in_f, void* q,
                   void* scale, void* stream);
/* Dequantize to [out_f, in_f] (replaces dequantize_q8_0, quantized_matmul.rs:376-408 and
 * GpuQuantizedLinear::dequantize :705).  out_dtype SP_F32 gives f32(scale)*q exactly as
 * crates/sketchpad-convert/src/gguf.rs:643-656 does (subnormal scales included). */
int sp_q8_0_dequant(const void* q, const void* scale, int64_t out_f, int64_t in_f, void* out,
                    int out_dtype, void* stream);
/* ------------------------------------------------------------------------------------
 * GGUF K-quants (GpuQuantType::{Q4K, Q2K, Q3K}, quantized_matmul.rs:33-43): the CPU decode of
 * crates/sketchpad-convert/src/gguf.rs:737-871 is the semantics (f16 d/dmin with subnormals).
 * The format id is the GGML type id.  Repacked layout: qpack [N, K/2] bytes (value k of a row
 * in the low nibble of byte k/2 for even k, high nibble for odd k; one 4-bit unsigned quant
 * per value) and f32 factors a, b [K/sub, N] (k-block-major; sub = 32 for Q4_K, 16 for
 * Q2_K/Q3_K): w[n, k] = a * (q - off) - b, off = 4 for Q3_K (b = 0), else 0, exactly the
 * reference's f32 value.  K must be a multiple of 256.
 * ------------------------------------------------------------------------------------ */
typedef enum sp_kquant_format { SP_QK_Q2_K = 10, SP_QK_Q3_K = 11, SP_QK_Q4_K = 12 } sp_kquant_format;
/* Host repack of nbytes of row-major GGUF super-blocks (out_f rows of in_f/256 blocks):
 * qpack_host [out_f * in_f/2], a_host and b_host [in_f/sub * out_f]. */
int sp_kquant_repack_host(int fmt, const uint8_t* gguf_host, size_t nbytes, int64_t out_f,
                          int64_t in_f, uint8_t* qpack_host, float* a_host, float* b_host);
/* Dequantize to [out_f, in_f] of out_dtype (replaces dequantize_q4k / dequantize_q2k /
 * dequantize_q3k, quantized_matmul.rs:410-520); SP_F32 is bit-exact with the CPU decode. */
int sp_kquant_dequant(int fmt, const void* qpack, const float* a, const float* b, int64_t out_f,
                      int64_t in_f, void* out, int out_dtype, void* stream);
/* y[M,N] = x[M,K] . dequant(W)[N,K]^T (+ bias[N]), the K-quant decode inside the GEMM
 * mainloop (GpuQuantizedLinear::forward for Q4K/Q2K/Q3K, quantized_matmul.rs:752-766).
 * x, y, bias bf16; qpack/a/b as above. */
int sp_kquant_linear(int fmt, const void* x, const void* qpack, const float* a, const float* b,
                     const void* bias, void* y, int64_t M, int64_t N, int64_t K, int dtype,
                     void* stream);

/* Tile mode of the quantized linears (Q8_0, FP8, K-quants; no reference counterpart), for the
 * whole process: 0 (default) = one CTA per 256 x 256 tile; 1 = two-CTA clusters per 512 x 256
 * tile (tcgen05.mma.cta_group::2) whenever M > 256, which halves each SM's decode work and
 * weight-operand shared-memory reads.  Both give bit-identical results; on B200 the paired
 * mode measured no faster, because the mainloop is bound by TMA latency, so it stays opt-in.
 * Returns the previous mode; SP_ERR_INVALID_ARG for another value. */
int sp_quant_linear_set_pairing(int mode);

/* y[M,N] = x[M,K] . dequant(W)[N,K]^T (+ bias[N]); the dequantization happens inside the
 * GEMM mainloop (replaces GpuQuantizedLinear::forward, quantized_matmul.rs:752-766).
 * x, y, bias: SP_BF16.  K % 64 == 0, N % 16 == 0.  bias may be NULL.  x, q, scale and y
 * must be 16-byte aligned. */
int sp_q8_0_linear(const void* x, const void* q, const void* scale, const void* bias, void* y,
                   int64_t M, int64_t N, int64_t K, int dtype, void* stream);
/* sp_q8_0_linear with a gated-residual epilogue: y = residual + gate[n] * (x.W^T + bias[n]).
 * The DiT blocks' `x + gate * attn(...)` / `x + gate * ffn(...)` (crates/sketchpad-dit/src/
 * flux.rs:450-517, :573-607) and Wan's ungated residuals (wan.rs:489-573, gate NULL) without
 * the two element-wise passes.  gate [N] or NULL, residual [M, N] or NULL (may equal y);
 * bf16; residual 16-byte aligned. */
int sp_q8_0_linear_gated(const void* x, const void* q, const void* scale, const void* bias,
                         const void* gate, const void* residual, void* y, int64_t M, int64_t N,
                         int64_t K, int dtype, void* stream);

/* y[M,N] = x[M,K] . W[N,K]^T (+ bias[N]) with plain bf16 weights on the same tcgen05 GEMM
 * (TMA loads the weight tiles straight into the MMA layout; no decode): the UNet's attention
 * projections, proj_in / proj_out and feed-forward (crates/sketchpad-unet/src/blocks.rs
 * :213-231, :292-305, :446-458), which the reference runs as burn Linear matmuls.  x, W,
 * bias, y bf16; K % 64 == 0, N % 16 == 0; 16-byte aligned.  _gated: y = residual + gate[n] *
 * (x.W^T + bias[n]) (gate and residual may be NULL; residual may equal y: the UNet's
 * in-place residual accumulation).  _glu: W's rows interleaved (first-half row j,
 * second-half row j), y [M, N/2] = lo * gelu(hi) (SP_GLU_GEGLU, the UNet feed-forward) or
 * silu(lo) * hi (SP_GLU_SWIGLU). */
int sp_bf16_linear(const void* x, const void* w, const void* bias, void* y, int64_t M, int64_t N,
                   int64_t K, int dtype, void* stream);
int sp_bf16_linear_gated(const void* x, const void* w, const void* bias, const void* gate,
                         const void* residual, void* y, int64_t M, int64_t N, int64_t K,
                         int dtype, void* stream);
int sp_bf16_linear_glu(const void* x, const void* w, const void* bias, void* y, int64_t M,
                       int64_t N, int64_t K, int glu_kind, int dtype, void* stream);

/* ------------------------------------------------------------------------------------
 * FP8 (e4m3) weights with f32 scales (per output channel, or one per tensor).
 * The reference simulates FP8 in f32 (crates/sketchpad-core/src/quantization.rs:422-615);
 * here the weights are real e4m3 bytes.
 * ------------------------------------------------------------------------------------ */
/* quantize_fp8 with the E4M3 config (quantization.rs:495-577): w f32 [N,K] ->
 * e4m3 bytes [N,K] + scale (N floats per channel, else 1).  Rounds like
 * quantize_fp8_scalar (:451-492) -- nearest, ties away from zero -- for every value the
 * e4m3 grid can hold; scaled magnitudes below 2^-6 go to the nearest e4m3 subnormal. */
typedef enum sp_fp8_scale_mode {
  SP_FP8_PER_TENSOR = 0,  /* scale[0] = max|w| / 448 (1 if w == 0), computed here */
  SP_FP8_PER_CHANNEL = 1, /* scale[n] = max|w[n,:]| / 448, computed here */
  SP_FP8_GIVEN_SCALE = 2  /* scale[0] supplied by the caller (Fp8Config::with_scale) */
} sp_fp8_scale_mode;
int sp_fp8_quantize(const float* w, int64_t N, int64_t K, int scale_mode, void* w_e4m3,
                    float* scale, void* stream);
/* Fp8Tensor::dequantize (quantization.rs:435-447): out[n,k] = e4m3(w[n,k]) * scale[n or 0]. */
int sp_fp8_dequant(const void* w_e4m3, const float* scale, int64_t nscale, int64_t N, int64_t K,
                   void* out, int out_dtype, void* stream);
/* Fp8Linear::forward (quantization.rs:601-609): y = x . dequant(W)^T + bias with the e4m3
 * decode in the GEMM mainloop and the scale in the epilogue.  x, y, bias: SP_BF16.
 * K % 64 == 0, N % 16 == 0. */
int sp_fp8_linear(const void* x, const void* w_e4m3, const float* scale, int64_t nscale,
                  const void* bias, void* y, int64_t M, int64_t N, int64_t K, int dtype,
                  void* stream);
/* sp_fp8_linear with the gated-residual epilogue of sp_q8_0_linear_gated. */
int sp_fp8_linear_gated(const void* x, const void* w_e4m3, const float* scale, int64_t nscale,
                        const void* bias, const void* gate, const void* residual, void* y,
                        int64_t M, int64_t N, int64_t K, int dtype, void* stream);
/* The feed-forward gate in the GEMM epilogue: W's rows interleaved as (first-half row j,
 * second-half row j) of the stacked [2F, K] gate/up (or value/gate) weight, so the GEMM's
 * columns 2j, 2j+1 are (lo, hi) and y[M, N/2] (row stride N/2) gets lo * gelu(hi)
 * (SP_GLU_GEGLU, crates/sketchpad-unet/src/blocks.rs:446-458) or silu(lo) * hi
 * (SP_GLU_SWIGLU, crates/sketchpad-core/src/glu.rs:91-96; crates/sketchpad-dit/src/wan.rs:
 * 330-337) from the f32 accumulators — no [M, 2F] intermediate in HBM. */
int sp_q8_0_linear_glu(const void* x, const void* q, const void* scale, const void* bias, void* y,
                       int64_t M, int64_t N, int64_t K, int glu_kind, int dtype, void* stream);
int sp_fp8_linear_glu(const void* x, const void* w_e4m3, const float* scale, int64_t nscale,
                      const void* bias, void* y, int64_t M, int64_t N, int64_t K, int glu_kind,
                      int dtype, void* stream);
/* The attention projection GEMM of the DiT blocks with its rotary embedding done in the
 * epilogue, written into a strided output:
 *   y[m, n] (row stride ldy >= N, ldy % 8 == 0) = rope(x . W^T + bias)[m, n]
 * where columns [0, rope_cols) form head_dim-wide heads (8 | head_dim, head_dim | rope_cols)
 * whose (even, odd) column pairs (x0, x1) become (x0 c - x1 s, x1 c + x0 s), the RoPE of
 * crates/sketchpad-dit/src/rope.rs:145-170 applied to q and k after FluxAttention's qkv
 * projection (crates/sketchpad-dit/src/flux.rs:330-352) and WanAttention's to_qkv
 * (crates/sketchpad-dit/src/wan.rs:371-390).  (c, s) = rope_cos_sin[pos * head_dim/2 + pair]
 * as f32 pairs, pos = ((m + pos_offset) / pos_div) % pos_mod, pos_mod <= rope_positions
 * (the table's rows).  rope_cos_sin may be NULL (no rotation: a plain strided-output GEMM,
 * used to write the cross stream's k/v next to the self stream's in one buffer).  x and
 * bias are bf16; dtype is y's type, SP_BF16 or SP_F16 (f16 attention inputs: 3 more
 * mantissa bits for q and k, for activations inside f16's range). */
int sp_q8_0_linear_rope(const void* x, const void* q, const void* scale, const void* bias, void* y,
                        int64_t ldy, int64_t M, int64_t N, int64_t K, const float* rope_cos_sin,
                        int64_t rope_positions, int64_t rope_cols, int64_t head_dim,
                        int64_t pos_offset, int64_t pos_div, int64_t pos_mod, int dtype,
                        void* stream);
/* sp_fp8_linear with the strided-output RoPE epilogue of sp_q8_0_linear_rope. */
int sp_fp8_linear_rope(const void* x, const void* w_e4m3, const float* scale, int64_t nscale,
                       const void* bias, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                       const float* rope_cos_sin, int64_t rope_positions, int64_t rope_cols,
                       int64_t head_dim, int64_t pos_offset, int64_t pos_div, int64_t pos_mod,
                       int dtype, void* stream);

/* ------------------------------------------------------------------------------------
 * LayerNorm over the last dimension (crates/sketchpad-core/src/layernorm.rs:63-73), which
 * uses burn's unbiased (n-1) variance; unbiased = 0 gives the biased form.
 * x, y [rows, n] contiguous; gamma, beta [n]; all of `dtype`.
 * ------------------------------------------------------------------------------------ */
int sp_layernorm(const void* x, const void* gamma, const void* beta, void* y, int64_t rows,
                 int64_t n, float eps, int unbiased, int dtype, void* stream);
/* LayerNorm of x + x_add[column] (x_add: n values, the same dtype; the sum is rounded to the
 * dtype as a separate element-wise add would round it, then normalised).  Lets a caller carry
 * a residual stream whose per-channel bias is added only where it is read -- the UNet
 * transformer accumulates its projection biases that way (BasicTransformerBlock residuals,
 * crates/sketchpad-unet/src/blocks.rs:292-305). */
int sp_layernorm_add(const void* x, const void* x_add, const void* gamma, const void* beta,
                     void* y, int64_t rows, int64_t n, float eps, int unbiased, int dtype,
                     void* stream);
/* The DiT blocks' modulated norm: y = LN(x) * (1 + scale[g]) + shift[g] with LN = LayerNorm::new
 * (gamma 1, beta 0), g = row / rows_per_group, and group g's scale / shift vectors starting
 * g * mod_stride elements after `scale` / `shift` (so both may point into the modulation
 * GEMM's output [batch, k, n]).  Replaces the norm + `(ones_like(scale) + scale) * x + shift`
 * of FluxDoubleBlock / FluxSingleBlock (crates/sketchpad-dit/src/flux.rs:479-481, 504-506,
 * 597-599) and WanBlock (crates/sketchpad-dit/src/wan.rs:541-542, 549-550, 564-565,
 * 569-570).  A null scale reads as 0 and a null shift as 0 (plain LayerNorm::new); computed
 * in f32 and rounded once. */
int sp_layernorm_modulate(const void* x, const void* scale, const void* shift, void* y,
                          int64_t rows, int64_t n, int64_t rows_per_group, int64_t mod_stride,
                          float eps, int unbiased, int dtype, void* stream);

/* ------------------------------------------------------------------------------------
 * Denoising-loop latent update fused with classifier-free guidance (one pass over the
 * latent).  eps = eps_uncond + (eps_cond - eps_uncond) * guidance (apply_guidance,
 * crates/sketchpad-samplers/src/ddim.rs:158-164); eps_cond NULL means eps = eps_uncond.
 * x, eps_*, noise, out: n elements of `dtype`, f32 arithmetic in the reference's order;
 * out may be x.  The scalars are the host values of the reference's step.
 * ------------------------------------------------------------------------------------ */
/* DdimSampler::step (ddim.rs:72-133): out = (x - eps*sqrt_one_minus_at)/sqrt_at * sqrt_at_prev
 * + dir_xt * eps (+ noise * sigma when noise is non-NULL, eta > 0). */
int sp_cfg_ddim_step(const void* x, const void* eps_uncond, const void* eps_cond, const void* noise,
                     void* out, int64_t n, float guidance, float sqrt_one_minus_at, float sqrt_at,
                     float sqrt_at_prev, float dir_xt, float sigma, int dtype, void* stream);
/* DpmPlusPlusSampler::step (crates/sketchpad-samplers/src/dpm.rs:101-171): denoised = x - eps
 * * sigma; out = x * sigma_ratio + d * one_minus_exp_neg_h with d = denoised (first order) or
 * denoised * one_plus_coeff - prev_denoised * coeff (second order).  prev_denoised (f32, n;
 * may be NULL for a first-order-only call) receives this step's denoised. */
int sp_cfg_dpmpp_2m_step(const void* x, const void* eps_uncond, const void* eps_cond,
                         float* prev_denoised, void* out, int64_t n, float guidance, float sigma,
                         float sigma_ratio, float one_minus_exp_neg_h, float one_plus_coeff,
                         float coeff, int second_order, int dtype, void* stream);

/* ------------------------------------------------------------------------------------
 * Sequence-parallel (Ulysses) exchange of the long-video DiT, over NCCL.
 * The reference runs Wan::forward on one device (crates/sketchpad-dit/src/wan.rs:720-757,
 * blocks :489-573) and has no collectives; splitting its 75,600 tokens over P GPUs needs an
 * all-to-all around each self-attention ([S/P tokens, H heads] <-> [S tokens, H/P heads]).
 * NCCL is loaded at run time (libnccl.so.2; the copy already in the process, if any).
 *
 * Communicators are NON-BLOCKING (ncclConfig_t.blocking = 0): every call below returns once
 * its work is enqueued, polling ncclCommGetAsyncError against a host deadline of timeout_s
 * seconds; on an NCCL error or an expired deadline the communicator is aborted
 * (ncclCommAbort: its kernels and proxy threads stop) and SP_ERR_COMM is returned, so a rank
 * that never joins or stops answering ends the others' calls with an error, not a hang.
 * ------------------------------------------------------------------------------------ */
/* Size of an NCCL unique id (128 bytes) and a fresh one, made by one rank and passed to the
 * others by any host channel. */
size_t sp_nccl_unique_id_bytes(void);
int sp_nccl_unique_id(void* id_out, size_t id_bytes);
/* Joins rank `rank` of `nranks` to the communicator named by `id` on the current device. */
int sp_nccl_comm_init(void** comm_out, int nranks, int rank, const void* id, double timeout_s);
/* The communicator's asynchronous state (an ncclResult_t: 0 success, 7 in progress). */
int sp_nccl_comm_poll(void* comm, int* nccl_status_out);
/* Waits until `stream` has finished (cudaStreamQuery) while polling the communicator; aborts
 * it and returns SP_ERR_COMM on an NCCL error or when timeout_s passes first. */
int sp_nccl_wait(void* comm, void* stream, double timeout_s);
int sp_nccl_comm_abort(void* comm);
/* Finalizes (bounded by timeout_s, abort on expiry) and frees the communicator. */
int sp_nccl_comm_destroy(void* comm, double timeout_s);
/* All-to-all of P equal chunks: chunk p of `send` (count elements of dtype) goes to rank p,
 * chunk p of `recv` comes from rank p; the rank's own chunk is a device copy.  send and recv
 * hold P * count elements and must not alias.  For Ulysses, chunk p of the send buffer holds
 * this rank's tokens for head group p, and the receive buffer is then [P ranks' tokens] x
 * [this rank's heads] in global token order. */
int sp_ulysses_a2a(const void* send, void* recv, int64_t count, int dtype, void* comm,
                   void* stream, double timeout_s);
/* All-gather of count elements per rank (the Wan velocity's token shards). */
int sp_nccl_all_gather(const void* send, void* recv, int64_t count, int dtype, void* comm,
                       void* stream, double timeout_s);

/* ------------------------------------------------------------------------------------
 * Weight files (host only, no GPU): GGUF v3 as crates/sketchpad-convert/src/gguf.rs:351-470
 * reads it (version 3 only, tensor data at the header end rounded up to 32 bytes, shapes
 * reversed to row-major) and safetensors as crates/sketchpad-convert/src/loader.rs:60-90
 * reads it (8-byte header length, JSON header, data_offsets after it), with F8_E4M3 /
 * F8_E5M2 tensors accepted as well.  The file is memory-mapped read-only; tensor bytes are
 * returned as pointers into the map, valid until sp_model_close.  GGUF Q8_0 / Q2_K / Q3_K /
 * Q4_K bytes go to sp_q8_0_repack_host / sp_kquant_repack_host unchanged.
 * ------------------------------------------------------------------------------------ */
typedef enum sp_container { SP_CONTAINER_GGUF = 1, SP_CONTAINER_SAFETENSORS = 2 } sp_container;
/* Tensor element types: the sp_dtype values, then the other safetensors dtypes, then GGUF's
 * block-quantized types as SP_T_GGML_BASE + the ggml type id (Q8_0 = 108, Q2_K = 110, Q3_K =
 * 111, Q4_K = 112, ...). */
typedef enum sp_tensor_type {
  SP_T_F32 = 0, SP_T_F16 = 1, SP_T_BF16 = 2, SP_T_F8_E4M3 = 3, SP_T_F8_E5M2 = 4, SP_T_F64 = 5,
  SP_T_I8 = 6, SP_T_U8 = 7, SP_T_I16 = 8, SP_T_I32 = 9, SP_T_I64 = 10, SP_T_BOOL = 11,
  SP_T_GGML_BASE = 100
} sp_tensor_type;
/* Opens a GGUF (by its magic) or safetensors file; SP_ERR_INVALID_ARG / SP_ERR_DTYPE /
 * SP_ERR_SHAPE on a malformed file, an unknown type or offsets outside the file. */
int sp_model_open(const char* path, void** file_out);
int sp_model_close(void* file);
int sp_model_info(void* file, int* container_out, int64_t* tensor_count_out,
                  int64_t* meta_count_out);
int sp_model_meta_key(void* file, int64_t index, char* name_out, size_t name_cap);
/* Name, sp_tensor_type, rank and row-major dims (up to 8, unused entries 0) and byte size of
 * tensor `index` (file order). */
int sp_model_tensor_info(void* file, int64_t index, char* name_out, size_t name_cap,
                         int* type_out, int* ndims_out, int64_t dims_out[8],
                         uint64_t* nbytes_out);
int sp_model_find(void* file, const char* name, int64_t* index_out);
int sp_model_tensor_data(void* file, int64_t index, const uint8_t** data_out);

#ifdef __cplusplus
}
#endif

#endif /* SKETCHPAD_B200_H */
