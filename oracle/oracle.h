/*
 * oracle.h -- CPU restatement of the reference's fp32 (Burn ndarray) semantics for the
 * diffusion-denoiser hot path of rhi-zone/sketchpad.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the cpu_baseline /
 * reference legs of bench.py load this library, and only as the checker or the timed CPU
 * baseline.  The product path (sketchpad_b200) never links or calls it.
 *
 * Parity status:
 *   - Q8_0 decode / Q8_0 matmul: pinned to the reference's golden vectors
 *     (crates/sketchpad-convert/src/gguf.rs:5390-5412, :5541-5562;
 *      crates/sketchpad-llm/src/quantized.rs:516-552).
 *   - FP8 scalar rounding: pinned to crates/sketchpad-core/src/quantization.rs:793-812.
 *   - GroupNorm(+SiLU), attention, LayerNorm, conv/linear: the reference has no golden
 *     vectors for these (its tests compare random tensors against a differently-defined
 *     helper), so they are pinned only to hand-computed known answers of the reference
 *     formulas -- "parity unpinned" against reference-produced outputs.
 *
 * All tensors are contiguous row-major fp32 unless stated.  Every function returns 0 on
 * success and a negative value on invalid arguments.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Thread count used by the OpenMP loops (0 = library default). Returns the count in use. */
int or_set_threads(int n);
int or_get_threads(void);

/* IEEE binary16 -> binary32 including subnormals/inf/nan (the `half` crate 2.7.1 `to_f32`,
 * used by crates/sketchpad-convert/src/gguf.rs:638-641). */
void or_f16_to_f32(const uint16_t* h, float* f, int64_t n);
/* binary32 -> binary16, round-to-nearest-even (the `half` crate `from_f32`). */
void or_f32_to_f16(const float* f, uint16_t* h, int64_t n);

/* GroupNorm (+ optional SiLU), crates/sketchpad-core/src/groupnorm.rs:62-102 and
 * crates/sketchpad-core/src/silu.rs:5-7.  x,y: [B,C,H,W]; gamma,beta: [C].
 * act: 0 = none, 1 = silu. */
int or_groupnorm_act(const float* x, const float* gamma, const float* beta, float* y,
                     int64_t B, int64_t C, int64_t H, int64_t W, int64_t G, float eps, int act);
/* The same for f16 (dtype 1) / bf16 (dtype 2) tensors: the normalised value is cast back
 * to the tensor dtype before the affine, and the affine, clamp and SiLU run as tensor ops in
 * that dtype (groupnorm.rs:88-99), each rounded.  dtype 0 is or_groupnorm_act. */
int or_groupnorm_act_dtype(const float* x, const float* gamma, const float* beta, float* y,
                           int64_t B, int64_t C, int64_t H, int64_t W, int64_t G, float eps,
                           int act, int dtype);

/* Attention over [BH, S, D] contiguous heads.
 * variant 0: crates/sketchpad-unet/src/blocks.rs:393-401 (scores = QK^T * d^-1/2, explicit
 *            max-subtracted exp, divide by sum, then @V);
 * variant 1: crates/sketchpad-core/src/attention.rs:4-27 (q,k each * d^-1/4, + mask, softmax).
 * mask: optional additive [Sq,Skv]; causal: key j > query i is excluded.
 * scale: <= 0 selects the reference default 1/sqrt(D). */
int or_attention(const float* q, const float* k, const float* v, const float* mask, float* out,
                 int64_t BH, int64_t Sq, int64_t Skv, int64_t D, int64_t Dv, int causal,
                 float scale, int variant);

/* Q8_0 block decode, crates/sketchpad-convert/src/gguf.rs:643-656.
 * data: nblocks * 34 bytes (f16 LE scale + 32 int8); out: nblocks*32 floats. */
int or_q8_0_dequantize(const uint8_t* data, int64_t nblocks, float* out);
// K-quant super-blocks (fmt = GGML type id: 10 Q2_K, 11 Q3_K, 12 Q4_K) -> 256 f32 values each.
int or_kquant_dequantize(int fmt, const uint8_t* data, int64_t nblocks, float* out);
/* Q8_0 row-dequant matmul, crates/sketchpad-llm/src/quantized.rs:70-92 / :421-446:
 * y[M,N] = x[M,K] . W[N,K]^T, each dot a sequential f32 sum (Rust Iterator::sum). */
int or_q8_0_matmul(const uint8_t* data, int64_t N, int64_t K, const float* x, int64_t M,
                   float* y);

/* FP8 simulation, crates/sketchpad-core/src/quantization.rs.
 * format: 0 = E4M3, 1 = E5M2. */
float or_fp8_quantize_scalar(float v, int format);                     /* :451-492 */
/* quantize_fp8 (:495-577). scale_out holds rows floats if per_channel else 1.
 * explicit_scale is used only for per-tensor mode when has_explicit_scale != 0. */
int or_fp8_quantize(const float* w, int64_t rows, int64_t cols, int format, int per_channel,
                    int has_explicit_scale, float explicit_scale, float* data_out,
                    float* scale_out);
/* Fp8Tensor::dequantize (:435-447): out = data * scale[row] (nscale == rows) or * scale[0]. */
int or_fp8_dequantize(const float* data, const float* scale, int64_t nscale, int64_t rows,
                      int64_t cols, float* out);

/* y[M,N] = x[M,K] @ W^T + b with W given as [N,K] (Fp8Linear::forward :601-609, the
 * dequantized-weight GEMMs).  b may be NULL. */
int or_linear_nt(const float* x, const float* w_nk, const float* b, float* y, int64_t M,
                 int64_t K, int64_t N);
/* burn nn::Linear: y[M,N] = x[M,K] @ W[K,N] + b (weight stored [in,out]). */
int or_linear_kn(const float* x, const float* w_kn, const float* b, float* y, int64_t M,
                 int64_t K, int64_t N);

/* LayerNorm over the last dim with the UNBIASED variance (burn `var`),
 * crates/sketchpad-core/src/layernorm.rs:63-73. x,y: [rows, n]. */
int or_layernorm(const float* x, const float* gamma, const float* beta, float* y,
                 int64_t rows, int64_t n, float eps);

/* Elementwise activations: 0 = silu (x*sigmoid(x)), 1 = gelu (erf form), 2 = sigmoid. */
int or_activation(const float* x, float* y, int64_t n, int kind);

/* conv2d NCHW, weight [Cout, Cin, kh, kw], bias [Cout] or NULL, symmetric padding. */
int or_conv2d(const float* x, const float* w, const float* b, float* y, int64_t B, int64_t Cin,
              int64_t H, int64_t W, int64_t Cout, int64_t kh, int64_t kw, int64_t stride,
              int64_t pad);

#ifdef __cplusplus
}
#endif
