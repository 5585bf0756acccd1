// sketchpad_b200.hpp -- C++ host mirror of the reference's GPU operator surface for the
// diffusion-denoiser hot path, over the C ABI of sketchpad_b200.h.
//
// The reference's host side is Rust (crates/sketchpad-cubecl); this header gives compiled
// callers the same operators with the same names, argument meaning and error behaviour:
//   flash_attention / flash_attention_masked + FlashAttentionOptions
//       crates/sketchpad-cubecl/src/attention.rs:40-68, :97, :119 (Err(AttentionSetupError)
//       -> throws AttentionSetupError)
//   groupnorm_silu / groupnorm + GroupNormSiLuOptions
//       crates/sketchpad-cubecl/src/groupnorm_silu.rs:22-46, :232, :323 (the reference
//       panics on C % groups != 0 -> throws std::invalid_argument)
//   dequantize_q8_0 / GpuQuantizedLinear::{from_bytes, forward, dequantize}
//       crates/sketchpad-cubecl/src/quantized_matmul.rs:376-408, :655-767
//   quantize_fp8 / Fp8Tensor::dequantize / Fp8Linear::forward
//       crates/sketchpad-core/src/quantization.rs:435-447, :495-577, :601-609
//   layer_norm (LayerNorm::forward, crates/sketchpad-core/src/layernorm.rs:63-73)
// Like the reference, each operator allocates its output on the device and hands it to the
// caller (Tensor owns the memory).  Every launch is asynchronous on the given stream.
// Link with libsketchpad_b200.so and the CUDA runtime.
#ifndef SKETCHPAD_B200_HPP
#define SKETCHPAD_B200_HPP

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "sketchpad_b200.h"

namespace sketchpad_b200 {

enum class DType : int { F32 = SP_F32, F16 = SP_F16, BF16 = SP_BF16 };

inline size_t dtype_size(DType d) { return d == DType::F32 ? 4 : 2; }

// A failed library call: the status code and the library's message.
class SketchpadError : public std::runtime_error {
 public:
  SketchpadError(int status, const std::string& what) : std::runtime_error(what), status_(status) {}
  int status() const { return status_; }

 private:
  int status_;
};

// Where the reference returns Err(AttentionSetupError) (attention.rs:97-104).
class AttentionSetupError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

inline void check(int rc) {
  if (rc != SP_OK) throw SketchpadError(rc, sp_last_error());
}

// Device memory owned by a Tensor (cudaMalloc / cudaFree).
class DeviceBuffer {
 public:
  explicit DeviceBuffer(size_t bytes) : bytes_(bytes) {
    if (bytes && cudaMalloc(&ptr_, bytes) != cudaSuccess) {
      cudaGetLastError();
      throw SketchpadError(SP_ERR_LAUNCH, "cudaMalloc of " + std::to_string(bytes) + " bytes failed");
    }
  }
  ~DeviceBuffer() {
    if (ptr_) cudaFree(ptr_);
  }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  void* get() const { return ptr_; }
  size_t bytes() const { return bytes_; }

 private:
  void* ptr_ = nullptr;
  size_t bytes_ = 0;
};

// A strided view of device memory: shape in the reference's dimension order, strides in
// elements.
struct TensorView {
  void* data = nullptr;
  DType dtype = DType::BF16;
  std::vector<int64_t> shape, strides;

  static TensorView contiguous(void* data, DType dtype, std::vector<int64_t> shape) {
    TensorView t{data, dtype, std::move(shape), {}};
    t.strides.assign(t.shape.size(), 1);
    for (int i = (int)t.shape.size() - 2; i >= 0; --i) t.strides[i] = t.strides[i + 1] * t.shape[i + 1];
    return t;
  }
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t s : shape) n *= s;
    return n;
  }
  size_t rank() const { return shape.size(); }
  bool is_contiguous() const {
    if (strides.size() != shape.size()) return false;
    int64_t want = 1;
    for (int i = (int)shape.size() - 1; i >= 0; --i) {
      if (shape[i] > 1 && strides[i] != want) return false;
      want *= shape[i];
    }
    return true;
  }
};

// A tensor that owns its device memory (what the reference's operators return).
struct Tensor {
  std::shared_ptr<DeviceBuffer> buffer;
  TensorView view;
  const TensorView& operator*() const { return view; }
  const TensorView* operator->() const { return &view; }
};

inline Tensor empty(DType dtype, std::vector<int64_t> shape) {
  TensorView v = TensorView::contiguous(nullptr, dtype, std::move(shape));
  auto buf = std::make_shared<DeviceBuffer>((size_t)v.numel() * dtype_size(dtype));
  v.data = buf->get();
  return Tensor{std::move(buf), std::move(v)};
}

// ------------------------------------------------------------------------------------------
// Flash attention (attention.rs:40-178)
// ------------------------------------------------------------------------------------------
struct FlashAttentionOptions {
  std::optional<DType> out_dtype;  // none: the query dtype
  bool causal = false;
  static FlashAttentionOptions new_causal() { return FlashAttentionOptions{std::nullopt, true}; }
  FlashAttentionOptions with_dtype(DType d) const { return FlashAttentionOptions{d, causal}; }
  FlashAttentionOptions with_causal(bool c) const { return FlashAttentionOptions{out_dtype, c}; }
};

namespace detail {
inline void strides4(const TensorView& t, int64_t out[4]) {
  for (int i = 0; i < 4; ++i) out[i] = t.strides[i];
}

// A hand-built view must carry one stride per dimension before any stride is read.
inline bool well_formed(const TensorView& t) { return t.strides.size() == t.shape.size(); }

// Argument and layout problems are setup errors (AttentionSetupError in the reference);
// launch failures and a missing sm_100 device keep their status as SketchpadError.
inline bool is_setup_status(int rc) {
  return rc == SP_ERR_INVALID_ARG || rc == SP_ERR_SHAPE || rc == SP_ERR_DTYPE || rc == SP_ERR_ALIGN;
}

inline Tensor flash(const TensorView& q, const TensorView& k, const TensorView& v,
                    const TensorView* mask, const FlashAttentionOptions& opts,
                    std::optional<float> scale, cudaStream_t stream) {
  if (q.rank() != 4 || k.rank() != 4 || v.rank() != 4)
    throw AttentionSetupError("query, key and value must be [batch, heads, seq, dim]");
  if (!well_formed(q) || !well_formed(k) || !well_formed(v) || (mask && !well_formed(*mask)))
    throw AttentionSetupError("every view needs one stride per dimension");
  const int64_t B = q.shape[0], H = q.shape[1], Sq = q.shape[2], D = q.shape[3];
  const int64_t Skv = k.shape[2], Dv = v.shape[3];
  if (k.shape[0] != B || k.shape[1] != H || k.shape[3] != D || v.shape[0] != B ||
      v.shape[1] != H || v.shape[2] != Skv)
    throw AttentionSetupError("query, key and value shapes do not match");
  if (q.dtype != k.dtype || q.dtype != v.dtype)
    throw AttentionSetupError("query, key and value must share one dtype");
  if (q.dtype == DType::F32)
    throw AttentionSetupError("the kernel reads bf16 or f16 query, key and value");
  const float* m = nullptr;
  int64_t mstride = 0;
  if (mask) {
    if (mask->rank() != 2 || mask->shape[0] != Sq || mask->shape[1] != Skv ||
        mask->dtype != DType::F32 || mask->strides[1] != 1)
      throw AttentionSetupError("mask must be an f32 [seq_q, seq_k] tensor with unit column stride");
    m = static_cast<const float*>(mask->data);
    mstride = mask->strides[0];
  }
  const DType od = opts.out_dtype.value_or(q.dtype);
  Tensor out = empty(od, {B, H, Sq, Dv});
  int64_t qs[4], ks[4], vs[4], os[4];
  strides4(q, qs);
  strides4(k, ks);
  strides4(v, vs);
  strides4(out.view, os);
  const int rc = sp_flash_attn_fwd(q.data, k.data, v.data, m, mstride, out.view.data, B, H, Sq, Skv,
                                   D, Dv, qs, ks, vs, os, (int)q.dtype, (int)od,
                                   opts.causal ? 1 : 0, scale.value_or(0.f), stream);
  if (rc != SP_OK) {
    if (is_setup_status(rc)) throw AttentionSetupError(sp_last_error());
    check(rc);
  }
  return out;
}
}  // namespace detail

// softmax(Q K^T / sqrt(d) [causal]) V -> [batch, heads, seq_q, val_dim] (attention.rs:97).
inline Tensor flash_attention(const TensorView& q, const TensorView& k, const TensorView& v,
                              const FlashAttentionOptions& opts = {},
                              std::optional<float> scale = std::nullopt,
                              cudaStream_t stream = nullptr) {
  return detail::flash(q, k, v, nullptr, opts, scale, stream);
}

// The same with an additive f32 [seq_q, seq_k] mask (attention.rs:119).
inline Tensor flash_attention_masked(const TensorView& q, const TensorView& k,
                                     const TensorView& v, const TensorView& mask,
                                     const FlashAttentionOptions& opts = {},
                                     std::optional<float> scale = std::nullopt,
                                     cudaStream_t stream = nullptr) {
  return detail::flash(q, k, v, &mask, opts, scale, stream);
}

// ------------------------------------------------------------------------------------------
// GroupNorm (+ SiLU) (groupnorm_silu.rs:22-46, :232, :323)
// ------------------------------------------------------------------------------------------
struct GroupNormSiLuOptions {
  int64_t num_groups = 32;
  float eps = 1e-5f;
};

namespace detail {
inline Tensor groupnorm_act(const TensorView& x, const TensorView& weight, const TensorView& bias,
                            const GroupNormSiLuOptions& opts, int act, cudaStream_t stream) {
  if (x.rank() != 4) throw std::invalid_argument("groupnorm: input must be [batch, channels, h, w]");
  if (!well_formed(x)) throw std::invalid_argument("groupnorm: input needs one stride per dimension");
  const int64_t B = x.shape[0], C = x.shape[1], H = x.shape[2], W = x.shape[3];
  if (opts.num_groups <= 0 || C % opts.num_groups != 0)
    throw std::invalid_argument("groupnorm: channels must be divisible by num_groups");
  if (weight.numel() != C || bias.numel() != C || weight.dtype != x.dtype || bias.dtype != x.dtype)
    throw std::invalid_argument("groupnorm: weight and bias must be [channels] of the input dtype");
  int64_t xs[4], ys[4];
  strides4(x, xs);
  // y follows x as the library decides it (dense channels-last stays channels-last, size-1
  // dimensions ignored; anything else becomes NCHW): ask the library, do not guess
  check(sp_groupnorm_act_output_strides(B, C, H, W, xs, ys));
  Tensor y = empty(x.dtype, {B, C, H, W});
  y.view.strides = {ys[0], ys[1], ys[2], ys[3]};
  const size_t ws_bytes =
      sp_groupnorm_act_workspace_size(B, C, H, W, xs, opts.num_groups, (int)x.dtype);
  void* ws = nullptr;  // stream-ordered: allocated and freed on `stream`
  if (ws_bytes && cudaMallocAsync(&ws, ws_bytes, stream) != cudaSuccess) {
    cudaGetLastError();
    throw SketchpadError(SP_ERR_LAUNCH, "groupnorm: workspace allocation failed");
  }
  const int rc = sp_groupnorm_act(x.data, weight.data, bias.data, y.view.data, B, C, H, W, xs,
                                  opts.num_groups, opts.eps, act, (int)x.dtype, ws, ws_bytes,
                                  stream);
  if (ws) cudaFreeAsync(ws, stream);
  check(rc);
  return y;
}
}  // namespace detail

// GroupNorm followed by SiLU (groupnorm_silu.rs:232).
inline Tensor groupnorm_silu(const TensorView& x, const TensorView& weight,
                             const TensorView& bias, const GroupNormSiLuOptions& opts = {},
                             cudaStream_t stream = nullptr) {
  return detail::groupnorm_act(x, weight, bias, opts, SP_ACT_SILU, stream);
}

// GroupNorm alone (groupnorm_silu.rs:323).
inline Tensor groupnorm(const TensorView& x, const TensorView& weight, const TensorView& bias,
                        const GroupNormSiLuOptions& opts = {}, cudaStream_t stream = nullptr) {
  return detail::groupnorm_act(x, weight, bias, opts, SP_ACT_NONE, stream);
}

// ------------------------------------------------------------------------------------------
// LayerNorm (crates/sketchpad-core/src/layernorm.rs:63-73: burn's unbiased variance)
// ------------------------------------------------------------------------------------------
inline Tensor layer_norm(const TensorView& x, const TensorView& gamma, const TensorView& beta,
                         float eps = 1e-5f, bool unbiased = true, cudaStream_t stream = nullptr) {
  if (x.rank() < 1 || !x.is_contiguous())
    throw std::invalid_argument("layer_norm: x must be a contiguous [..., n] tensor");
  const int64_t n = x.shape.back();
  if (gamma.numel() != n || beta.numel() != n || gamma.dtype != x.dtype || beta.dtype != x.dtype)
    throw std::invalid_argument("layer_norm: gamma and beta must be [n] of the input dtype");
  Tensor y = empty(x.dtype, x.shape);
  check(sp_layernorm(x.data, gamma.data, beta.data, y.view.data, x.numel() / n, n, eps,
                     unbiased ? 1 : 0, (int)x.dtype, stream));
  return y;
}

// ------------------------------------------------------------------------------------------
// Q8_0 quantized linear (quantized_matmul.rs:376-408, :655-767)
// ------------------------------------------------------------------------------------------
class GpuQuantizedLinear {
 public:
  // GpuQuantizedLinear::from_bytes for Q8_0: GGUF bytes on the host ([out_f rows of in_f/32
  // blocks of 34 bytes]), repacked losslessly into the planar device layout.  bias: [out_f]
  // bf16 on the device, or none.  The upload runs on `stream` and is complete when this
  // returns, so kernels later queued on any stream (non-blocking ones included) see it.
  static GpuQuantizedLinear from_bytes(const uint8_t* gguf, size_t nbytes, int64_t out_f,
                                       int64_t in_f, std::optional<TensorView> bias = std::nullopt,
                                       cudaStream_t stream = nullptr) {
    if (out_f <= 0 || in_f <= 0 || in_f % 32 != 0)
      throw std::invalid_argument("Q8_0: in_features must be a positive multiple of 32");
    if (nbytes != (size_t)(out_f * (in_f / 32) * 34))
      throw std::invalid_argument("Q8_0: byte count does not match [out_f, in_f]");
    if (bias && (bias->numel() != out_f || bias->dtype != DType::BF16))
      throw std::invalid_argument("Q8_0: bias must be [out_features] bf16");
    std::vector<int8_t> q((size_t)(out_f * in_f));
    std::vector<uint16_t> sc((size_t)(out_f * (in_f / 32)));
    check(sp_q8_0_repack_host(gguf, nbytes, out_f, in_f, q.data(), sc.data()));
    GpuQuantizedLinear l;
    l.out_f_ = out_f;
    l.in_f_ = in_f;
    l.q_ = std::make_shared<DeviceBuffer>(q.size());
    l.scale_ = std::make_shared<DeviceBuffer>(sc.size() * 2);
    // pageable sources: wait for the copies before q / sc go out of scope (a plain
    // cudaMemcpy may return before its DMA lands, unordered with non-blocking streams)
    if (cudaMemcpyAsync(l.q_->get(), q.data(), q.size(), cudaMemcpyHostToDevice, stream) !=
            cudaSuccess ||
        cudaMemcpyAsync(l.scale_->get(), sc.data(), sc.size() * 2, cudaMemcpyHostToDevice,
                        stream) != cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess) {
      cudaGetLastError();
      throw SketchpadError(SP_ERR_LAUNCH, "Q8_0: weight upload failed");
    }
    l.bias_ = bias;
    return l;
  }

  // y[..., out_f] = x[..., in_f] . dequant(W)^T + bias, the dequantization inside the GEMM
  // (GpuQuantizedLinear::forward, :752-766).  x: bf16, contiguous.
  Tensor forward(const TensorView& x, cudaStream_t stream = nullptr) const {
    if (x.rank() < 1 || x.shape.back() != in_f_ || x.dtype != DType::BF16 || !x.is_contiguous())
      throw std::invalid_argument("Q8_0 forward: x must be contiguous bf16 [..., in_features]");
    std::vector<int64_t> shape = x.shape;
    shape.back() = out_f_;
    Tensor y = empty(DType::BF16, shape);
    check(sp_q8_0_linear(x.data, q_->get(), scale_->get(), bias_ ? bias_->data : nullptr,
                         y.view.data, x.numel() / in_f_, out_f_, in_f_, SP_BF16, stream));
    return y;
  }

  // GpuQuantizedLinear::dequantize (:705): [out_f, in_f] of out_dtype, bit-exact for f32.
  Tensor dequantize(DType out_dtype = DType::F32, cudaStream_t stream = nullptr) const {
    Tensor w = empty(out_dtype, {out_f_, in_f_});
    check(sp_q8_0_dequant(q_->get(), scale_->get(), out_f_, in_f_, w.view.data, (int)out_dtype,
                          stream));
    return w;
  }

  int64_t out_features() const { return out_f_; }
  int64_t in_features() const { return in_f_; }

 private:
  GpuQuantizedLinear() = default;
  int64_t out_f_ = 0, in_f_ = 0;
  std::shared_ptr<DeviceBuffer> q_, scale_;
  std::optional<TensorView> bias_;
};

// dequantize_q8_0 (:376-408): GGUF bytes on the host -> [out_f, in_f] of out_dtype.
inline Tensor dequantize_q8_0(const uint8_t* gguf, size_t nbytes, int64_t out_f, int64_t in_f,
                              DType out_dtype = DType::F32, cudaStream_t stream = nullptr) {
  return GpuQuantizedLinear::from_bytes(gguf, nbytes, out_f, in_f, std::nullopt, stream)
      .dequantize(out_dtype, stream);
}

// ------------------------------------------------------------------------------------------
// FP8 e4m3 weights (quantization.rs:422-615)
// ------------------------------------------------------------------------------------------
struct Fp8Tensor {
  std::shared_ptr<DeviceBuffer> bytes;  // [N, K] e4m3
  std::shared_ptr<DeviceBuffer> scale;  // N floats per channel, else 1
  int64_t N = 0, K = 0, nscale = 1;

  // Fp8Tensor::dequantize (:435-447).
  Tensor dequantize(DType out_dtype = DType::F32, cudaStream_t stream = nullptr) const {
    Tensor w = empty(out_dtype, {N, K});
    check(sp_fp8_dequant(bytes->get(), static_cast<const float*>(scale->get()), nscale, N, K,
                         w.view.data, (int)out_dtype, stream));
    return w;
  }
};

// quantize_fp8 with the E4M3 config (:495-577): w f32 [N, K] on the device.
inline Fp8Tensor quantize_fp8(const TensorView& w, bool per_channel = true,
                              std::optional<float> given_scale = std::nullopt,
                              cudaStream_t stream = nullptr) {
  if (w.rank() != 2 || w.dtype != DType::F32 || !w.is_contiguous())
    throw std::invalid_argument("quantize_fp8: weights must be contiguous f32 [out, in]");
  Fp8Tensor t;
  t.N = w.shape[0];
  t.K = w.shape[1];
  t.nscale = (per_channel && !given_scale) ? t.N : 1;
  t.bytes = std::make_shared<DeviceBuffer>((size_t)(t.N * t.K));
  t.scale = std::make_shared<DeviceBuffer>((size_t)t.nscale * sizeof(float));
  int mode = per_channel ? SP_FP8_PER_CHANNEL : SP_FP8_PER_TENSOR;
  if (given_scale) {
    mode = SP_FP8_GIVEN_SCALE;
    // ordered on `stream` ahead of sp_fp8_quantize; synchronised because the source is a
    // host value that does not outlive this call
    if (cudaMemcpyAsync(t.scale->get(), &*given_scale, sizeof(float), cudaMemcpyHostToDevice,
                        stream) != cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess) {
      cudaGetLastError();
      throw SketchpadError(SP_ERR_LAUNCH, "quantize_fp8: scale upload failed");
    }
  }
  check(sp_fp8_quantize(static_cast<const float*>(w.data), t.N, t.K, mode, t.bytes->get(),
                        static_cast<float*>(t.scale->get()), stream));
  return t;
}

// Fp8Linear::forward (:601-609): y = x . dequant(W)^T + bias, e4m3 decode in the GEMM.
class Fp8Linear {
 public:
  Fp8Linear(Fp8Tensor weight, std::optional<TensorView> bias = std::nullopt)
      : w_(std::move(weight)), bias_(bias) {
    if (bias_ && (bias_->numel() != w_.N || bias_->dtype != DType::BF16))
      throw std::invalid_argument("Fp8Linear: bias must be [out_features] bf16");
  }
  Tensor forward(const TensorView& x, cudaStream_t stream = nullptr) const {
    if (x.rank() < 1 || x.shape.back() != w_.K || x.dtype != DType::BF16 || !x.is_contiguous())
      throw std::invalid_argument("Fp8Linear forward: x must be contiguous bf16 [..., in_features]");
    std::vector<int64_t> shape = x.shape;
    shape.back() = w_.N;
    Tensor y = empty(DType::BF16, shape);
    check(sp_fp8_linear(x.data, w_.bytes->get(), static_cast<const float*>(w_.scale->get()),
                        w_.nscale, bias_ ? bias_->data : nullptr, y.view.data,
                        x.numel() / w_.K, w_.N, w_.K, SP_BF16, stream));
    return y;
  }

 private:
  Fp8Tensor w_;
  std::optional<TensorView> bias_;
};

}  // namespace sketchpad_b200

#endif  // SKETCHPAD_B200_HPP
