// Setup errors of the C++ host mirror (include/sketchpad_b200.hpp): each case must throw the
// exception type the reference's operator reports with, before any device call -- so this
// program runs on a machine without a GPU.  Prints "ok" and exits 0 when every case holds.
#include <cstdio>
#include <vector>

#include "sketchpad_b200.hpp"

namespace sp = sketchpad_b200;

template <typename E, typename F>
static bool throws(const char* what, F&& f) {
  try {
    f();
  } catch (const E&) {
    return true;
  } catch (...) {
    std::printf("FAIL %s: wrong exception type\n", what);
    return false;
  }
  std::printf("FAIL %s: no exception\n", what);
  return false;
}

int main() {
  bool ok = sp_abi_version() == SP_ABI_VERSION;
  const auto bf = sp::DType::BF16;
  const sp::TensorView q = sp::TensorView::contiguous(nullptr, bf, {2, 4, 64, 64});
  const sp::TensorView k = sp::TensorView::contiguous(nullptr, bf, {2, 4, 77, 64});
  const sp::TensorView v = sp::TensorView::contiguous(nullptr, bf, {2, 4, 77, 64});
  const sp::TensorView q3 = sp::TensorView::contiguous(nullptr, bf, {2, 64, 64});
  const sp::TensorView kbad = sp::TensorView::contiguous(nullptr, bf, {2, 4, 77, 32});
  const sp::TensorView qf = sp::TensorView::contiguous(nullptr, sp::DType::F32, {2, 4, 64, 64});
  const sp::TensorView mask = sp::TensorView::contiguous(nullptr, sp::DType::F32, {64, 76});
  ok &= throws<sp::AttentionSetupError>("rank-3 query", [&] { sp::flash_attention(q3, k, v); });
  ok &= throws<sp::AttentionSetupError>("key head dim", [&] { sp::flash_attention(q, kbad, v); });
  ok &= throws<sp::AttentionSetupError>("value length", [&] { sp::flash_attention(q, k, q); });
  ok &= throws<sp::AttentionSetupError>("f32 inputs", [&] { sp::flash_attention(qf, qf, qf); });
  ok &= throws<sp::AttentionSetupError>("mask shape",
                                        [&] { sp::flash_attention_masked(q, k, v, mask); });

  const sp::TensorView x = sp::TensorView::contiguous(nullptr, bf, {2, 320, 8, 8});
  const sp::TensorView w = sp::TensorView::contiguous(nullptr, bf, {320});
  ok &= throws<std::invalid_argument>("groups do not divide channels", [&] {
    sp::groupnorm_silu(x, w, w, sp::GroupNormSiLuOptions{30, 1e-5f});
  });
  ok &= throws<std::invalid_argument>("rank-3 groupnorm input", [&] { sp::groupnorm(q3, w, w); });
  const sp::TensorView w_short = sp::TensorView::contiguous(nullptr, bf, {160});
  ok &= throws<std::invalid_argument>("groupnorm weight length",
                                      [&] { sp::groupnorm_silu(x, w_short, w_short); });

  ok &= throws<std::invalid_argument>("layer_norm gamma length", [&] {
    sp::layer_norm(sp::TensorView::contiguous(nullptr, bf, {8, 320}), w_short, w_short);
  });

  std::vector<uint8_t> bytes(34 * 4);
  ok &= throws<std::invalid_argument>("Q8_0 in_features not a multiple of 32", [&] {
    sp::GpuQuantizedLinear::from_bytes(bytes.data(), bytes.size(), 4, 48);
  });
  ok &= throws<std::invalid_argument>("Q8_0 byte count", [&] {
    sp::GpuQuantizedLinear::from_bytes(bytes.data(), bytes.size(), 4, 64);
  });
  ok &= throws<std::invalid_argument>("FP8 weights rank", [&] {
    sp::quantize_fp8(sp::TensorView::contiguous(nullptr, sp::DType::F32, {64}));
  });
  ok &= throws<std::invalid_argument>("FP8 weights dtype", [&] {
    sp::quantize_fp8(sp::TensorView::contiguous(nullptr, bf, {64, 64}));
  });
  // a hand-built view with fewer strides than dimensions is a setup error, not a read past
  // the end of the stride vector
  sp::TensorView qshort = q;
  qshort.strides.resize(2);
  ok &= throws<sp::AttentionSetupError>("short query strides",
                                        [&] { sp::flash_attention(qshort, k, v); });
  sp::TensorView xshort = x;
  xshort.strides.clear();
  ok &= throws<std::invalid_argument>("missing groupnorm strides", [&] { sp::groupnorm_silu(xshort, w, w); });

  // the output layout comes from the library: channels-last with B == 1 stays channels-last
  // whatever the batch stride; C == 1 and NCHW inputs give NCHW
  {
    int64_t ys[4];
    const int64_t nhwc_b1[4] = {12345, 1, 16 * 64, 64};
    ok &= sp_groupnorm_act_output_strides(1, 64, 16, 16, nhwc_b1, ys) == SP_OK && ys[1] == 1 &&
          ys[3] == 64 && ys[2] == 16 * 64;
    const int64_t nchw[4] = {64 * 256, 256, 16, 1};
    ok &= sp_groupnorm_act_output_strides(2, 64, 16, 16, nchw, ys) == SP_OK && ys[3] == 1 &&
          ys[1] == 256;
    ok &= sp_groupnorm_act_output_strides(2, 64, 16, 16, nullptr, ys) == SP_OK && ys[3] == 1;
    ok &= sp_groupnorm_act_output_strides(0, 64, 16, 16, nullptr, ys) == SP_ERR_INVALID_ARG;
    if (!ok) std::printf("FAIL groupnorm output strides\n");
  }
  if (!ok) return 1;
  std::printf("ok\n");
  return 0;
}
