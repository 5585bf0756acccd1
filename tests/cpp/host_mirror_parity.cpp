// Runs the C++ host mirror (include/sketchpad_b200.hpp) on seeded inputs and writes every
// input and output to the file named by argv[1] as raw little-endian arrays, in this order:
//   attention   q, k, v (bf16 bits [1,2,200,64], [1,2,77,64] x2), out (f32 [1,2,200,64])
//   groupnorm   x (f32 [2,64,16,16]), gamma, beta (f32 [64]), y (f32, NCHW)
//   Q8_0 linear GGUF bytes (128 rows x 256), x (bf16 bits [64,256]), y (bf16 bits [64,128])
//   LayerNorm   x (f32 [64,320]), gamma, beta (f32 [320]), y (f32)
//   FP8 linear  w (f32 [128,256], quantized per channel), x (bf16 bits [64,256]),
//               y (bf16 bits [64,128])
//   groupnorm   channels-last x [1,64,16,16] whose batch stride is not H*W*C (any stride
//               is valid for a size-1 batch): x, gamma, beta (f32), y (f32) -- x and y
//               gathered to NCHW order through each tensor's own strides
// The test compares the outputs with the CPU oracle.  Needs a B200.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "sketchpad_b200.hpp"

namespace sp = sketchpad_b200;

static uint64_t g_state = 0x9E3779B97F4A7C15ull;
static float uniform() {  // [0, 1)
  g_state = g_state * 6364136223846793005ull + 1442695040888963407ull;
  return (float)((g_state >> 40) & 0xFFFFFF) / 16777216.0f;
}
static float normal() {
  const float u1 = uniform() + 1e-7f, u2 = uniform();
  return std::sqrt(-2.0f * std::log(u1)) * std::cos(6.2831853f * u2);
}
static uint16_t to_bf16_bits(float f) {  // round to nearest even (finite inputs)
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

template <typename T>
static void upload(void* dst, const std::vector<T>& src) {
  if (cudaMemcpy(dst, src.data(), src.size() * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess)
    throw std::runtime_error("upload failed");
}
template <typename T>
static std::vector<T> download(const sp::Tensor& t) {
  std::vector<T> h((size_t)t.view.numel());
  if (cudaMemcpy(h.data(), t.view.data, h.size() * sizeof(T), cudaMemcpyDeviceToHost) != cudaSuccess)
    throw std::runtime_error("download failed");
  return h;
}
// the elements of a 4-D tensor in NCHW order, read through its strides
static std::vector<float> gather_nchw(const sp::Tensor& t, const std::vector<float>& mem) {
  const auto& sh = t.view.shape;
  const auto& st = t.view.strides;
  std::vector<float> out;
  for (int64_t a = 0; a < sh[0]; ++a)
    for (int64_t b = 0; b < sh[1]; ++b)
      for (int64_t c = 0; c < sh[2]; ++c)
        for (int64_t d = 0; d < sh[3]; ++d)
          out.push_back(mem[(size_t)(a * st[0] + b * st[1] + c * st[2] + d * st[3])]);
  return out;
}
template <typename T>
static void put(FILE* f, const std::vector<T>& v) {
  std::fwrite(v.data(), sizeof(T), v.size(), f);
}

int main(int argc, char** argv) {
  if (argc != 2) return 2;
  FILE* f = std::fopen(argv[1], "wb");
  if (!f) return 2;
  try {
    // ---- attention: bf16 in, f32 out, 77 keys (a key tail)
    std::vector<uint16_t> hq(1 * 2 * 200 * 64), hk(1 * 2 * 77 * 64), hv(1 * 2 * 77 * 64);
    for (auto* a : {&hq, &hk, &hv})
      for (auto& e : *a) e = to_bf16_bits(normal());
    sp::Tensor q = sp::empty(sp::DType::BF16, {1, 2, 200, 64});
    sp::Tensor k = sp::empty(sp::DType::BF16, {1, 2, 77, 64});
    sp::Tensor v = sp::empty(sp::DType::BF16, {1, 2, 77, 64});
    upload(q.view.data, hq);
    upload(k.view.data, hk);
    upload(v.view.data, hv);
    sp::Tensor o = sp::flash_attention(q.view, k.view, v.view,
                                       sp::FlashAttentionOptions{}.with_dtype(sp::DType::F32));
    put(f, hq);
    put(f, hk);
    put(f, hv);
    put(f, download<float>(o));

    // ---- GroupNorm + SiLU, f32 NCHW, 32 groups
    std::vector<float> hx(2 * 64 * 16 * 16), hg(64), hb(64);
    for (auto& e : hx) e = normal() * 3.f + 0.5f;
    for (auto& e : hg) e = 1.f + 0.1f * normal();
    for (auto& e : hb) e = 0.1f * normal();
    sp::Tensor x = sp::empty(sp::DType::F32, {2, 64, 16, 16});
    sp::Tensor g = sp::empty(sp::DType::F32, {64});
    sp::Tensor b = sp::empty(sp::DType::F32, {64});
    upload(x.view.data, hx);
    upload(g.view.data, hg);
    upload(b.view.data, hb);
    sp::Tensor y = sp::groupnorm_silu(x.view, g.view, b.view);
    put(f, hx);
    put(f, hg);
    put(f, hb);
    put(f, download<float>(y));

    // ---- Q8_0 linear: 128 x 256 weights from GGUF bytes, no bias
    const int N = 128, K = 256, M = 64;
    std::vector<uint8_t> gguf((size_t)N * (K / 32) * 34);
    for (size_t blk = 0; blk < gguf.size() / 34; ++blk) {
      const uint16_t scale = 0x1C00 + (uint16_t)(uniform() * 512);  // f16 in [2^-8, 2^-7)
      gguf[blk * 34] = (uint8_t)(scale & 0xFF);
      gguf[blk * 34 + 1] = (uint8_t)(scale >> 8);
      for (int i = 0; i < 32; ++i) gguf[blk * 34 + 2 + i] = (uint8_t)(int8_t)(uniform() * 254.f - 127.f);
    }
    std::vector<uint16_t> hxq((size_t)M * K);
    for (auto& e : hxq) e = to_bf16_bits(normal());
    sp::GpuQuantizedLinear lin = sp::GpuQuantizedLinear::from_bytes(gguf.data(), gguf.size(), N, K);
    sp::Tensor xq = sp::empty(sp::DType::BF16, {M, K});
    upload(xq.view.data, hxq);
    sp::Tensor yq = lin.forward(xq.view);
    put(f, gguf);
    put(f, hxq);
    put(f, download<uint16_t>(yq));

    // ---- LayerNorm, f32 [64, 320], unbiased variance
    std::vector<float> hl(64 * 320), hlg(320), hlb(320);
    for (auto& e : hl) e = normal() * 2.f + 0.3f;
    for (auto& e : hlg) e = 1.f + 0.1f * normal();
    for (auto& e : hlb) e = 0.1f * normal();
    sp::Tensor lx = sp::empty(sp::DType::F32, {64, 320});
    sp::Tensor lg = sp::empty(sp::DType::F32, {320});
    sp::Tensor lb = sp::empty(sp::DType::F32, {320});
    upload(lx.view.data, hl);
    upload(lg.view.data, hlg);
    upload(lb.view.data, hlb);
    sp::Tensor ly = sp::layer_norm(lx.view, lg.view, lb.view);
    put(f, hl);
    put(f, hlg);
    put(f, hlb);
    put(f, download<float>(ly));

    // ---- FP8 e4m3 linear, per-channel scales
    std::vector<float> hw((size_t)N * K);
    for (auto& e : hw) e = 0.05f * normal();
    sp::Tensor w = sp::empty(sp::DType::F32, {N, K});
    upload(w.view.data, hw);
    sp::Fp8Linear fp8(sp::quantize_fp8(w.view));
    sp::Tensor yf = fp8.forward(xq.view);
    put(f, hw);
    put(f, hxq);
    put(f, download<uint16_t>(yf));

    // ---- GroupNorm + SiLU, channels-last B = 1 with an unusual batch stride: the library
    // writes y channels-last (size-1 dimensions do not decide the layout) and the mirror
    // must label y with the strides the library used
    {
      const int64_t C = 64, H = 16, W = 16;
      std::vector<float> mem((size_t)(C * H * W));
      for (auto& e : mem) e = normal() * 3.f + 0.5f;
      sp::Tensor xb = sp::empty(sp::DType::F32, {1, C, H, W});
      upload(xb.view.data, mem);
      xb.view.strides = {7 * C * H * W + 3, 1, W * C, C};  // channels-last, odd batch stride
      std::vector<float> g2(C), b2(C);
      for (auto& e : g2) e = 1.f + 0.1f * normal();
      for (auto& e : b2) e = 0.1f * normal();
      sp::Tensor gg = sp::empty(sp::DType::F32, {C});
      sp::Tensor bb = sp::empty(sp::DType::F32, {C});
      upload(gg.view.data, g2);
      upload(bb.view.data, b2);
      sp::Tensor yb = sp::groupnorm_silu(xb.view, gg.view, bb.view);
      put(f, gather_nchw(xb, mem));
      put(f, g2);
      put(f, b2);
      put(f, gather_nchw(yb, download<float>(yb)));
    }
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    std::fclose(f);
    return 1;
  }
  std::fclose(f);
  std::printf("ok\n");
  return 0;
}
