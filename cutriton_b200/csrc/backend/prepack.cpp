// Registered constant transforms (see prepack.h).

#include "prepack.h"

#include <cstring>
#include <functional>
#include <unordered_map>

namespace cutriton {
namespace {

using Transform = std::function<Status(const TensorDesc&, const void*, TensorDesc*, std::vector<std::uint8_t>*)>;

// [K, N] -> [N, K] for any element size: turns a row-major GEMM weight into
// the K-major operand layout the tensor-core kernels read with TMA.
Status Transpose2d(const TensorDesc& in, const void* data, TensorDesc* out, std::vector<std::uint8_t>* bytes) {
  if (in.shape.size() != 2) return Status::ShapeError("transpose_2d expects a rank-2 constant");
  const std::size_t rows = static_cast<std::size_t>(in.shape[0]);
  const std::size_t cols = static_cast<std::size_t>(in.shape[1]);
  const std::size_t elem = ElementSize(in.dtype);
  *out = in;
  out->shape = {in.shape[1], in.shape[0]};
  out->layout = "";
  bytes->assign(rows * cols * elem, 0);
  const auto* src = static_cast<const std::uint8_t*>(data);
  for (std::size_t r = 0; r < rows; ++r) {
    for (std::size_t c = 0; c < cols; ++c) {
      std::memcpy(bytes->data() + (c * rows + r) * elem, src + (r * cols + c) * elem, elem);
    }
  }
  return Status::OK();
}

// TF32 split of an FP32 value: hi keeps sign, exponent and the top 10
// mantissa bits (exactly representable in TF32); lo = x - hi is exact in FP32.
inline void SplitTf32(float x, float* hi, float* lo) {
  std::uint32_t bits;
  std::memcpy(&bits, &x, sizeof bits);
  bits &= 0xFFFFE000u;
  std::memcpy(hi, &bits, sizeof bits);
  *lo = x - *hi;
}

// OIHW fp32 weights -> [2][O][Kpad] (hi plane, then lo plane), the
// implicit-GEMM A operand of the tensor-core convolution: K-major with
// k = (r * S + s) * Ip + i, channels fastest. Ip = I when I % 32 == 0 (a
// 32-wide k block is one filter tap of 32 channels), else I rounded up to a
// multiple of 4 with zero weights (every 4-wide, 16-byte k chunk is then 4
// channels of one tap). The k axis is zero-padded to a multiple of 32 so
// every k block is a whole 128-byte TMA row.
Status ConvWeightSplit(const TensorDesc& in, const void* data, TensorDesc* out,
                       std::vector<std::uint8_t>* bytes) {
  if (in.shape.size() != 4 || in.dtype != DataType::kFloat32) {
    return Status::ShapeError("conv_w_tf32x2_okpad expects an OIHW float32 constant");
  }
  const int64_t O = in.shape[0], I0 = in.shape[1], R = in.shape[2], S = in.shape[3];
  const int64_t Ip = I0 % 32 == 0 ? I0 : (I0 + 3) / 4 * 4;
  const int64_t K = Ip * R * S;
  const int64_t Kpad = (K + 31) / 32 * 32;
  const std::size_t plane = static_cast<std::size_t>(O * Kpad);
  *out = TensorDesc({2, O, Kpad}, DataType::kFloat32, in.device_type, in.device_id, "");
  bytes->assign(2 * plane * sizeof(float), 0);
  const auto* w = static_cast<const float*>(data);
  auto* dst = reinterpret_cast<float*>(bytes->data());
  for (int64_t o = 0; o < O; ++o)
    for (int64_t i = 0; i < I0; ++i)
      for (int64_t r = 0; r < R; ++r)
        for (int64_t s = 0; s < S; ++s) {
          float hi, lo;
          SplitTf32(w[((o * I0 + i) * R + r) * S + s], &hi, &lo);
          const std::size_t at = static_cast<std::size_t>(o * Kpad + (r * S + s) * Ip + i);
          dst[at] = hi;
          dst[plane + at] = lo;
        }
  return Status::OK();
}

// OIHW fp32 weights -> [2][O][Kpad] (hi, lo) with the k order of the
// TMEM-operand convolution. When I % 32 == 0 the k blocks walk the filter
// taps inside each 32-channel block: k = ((i / 32) * R * S + r * S + s) * 32
// + i % 32, so consecutive k blocks of one pixel tile re-read the same 32
// input channel planes (shifted by one tap) and hit in L1. Other channel
// counts keep the tap-major order of conv_w_tf32x2_okpad.
Status ConvWeightSplitChannelBlocks(const TensorDesc& in, const void* data, TensorDesc* out,
                                    std::vector<std::uint8_t>* bytes) {
  if (in.shape.size() != 4 || in.dtype != DataType::kFloat32) {
    return Status::ShapeError("conv_w_tf32x2_cb expects an OIHW float32 constant");
  }
  const int64_t I0 = in.shape[1];
  if (I0 % 32 != 0) return ConvWeightSplit(in, data, out, bytes);
  const int64_t O = in.shape[0], R = in.shape[2], S = in.shape[3];
  const int64_t Kpad = I0 * R * S;  // already a multiple of 32
  const std::size_t plane = static_cast<std::size_t>(O * Kpad);
  *out = TensorDesc({2, O, Kpad}, DataType::kFloat32, in.device_type, in.device_id, "");
  bytes->assign(2 * plane * sizeof(float), 0);
  const auto* w = static_cast<const float*>(data);
  auto* dst = reinterpret_cast<float*>(bytes->data());
  for (int64_t o = 0; o < O; ++o)
    for (int64_t i = 0; i < I0; ++i)
      for (int64_t r = 0; r < R; ++r)
        for (int64_t s = 0; s < S; ++s) {
          float hi, lo;
          SplitTf32(w[((o * I0 + i) * R + r) * S + s], &hi, &lo);
          const int64_t k = ((i / 32) * R * S + r * S + s) * 32 + i % 32;
          const std::size_t at = static_cast<std::size_t>(o * Kpad + k);
          dst[at] = hi;
          dst[plane + at] = lo;
        }
  return Status::OK();
}

// [K, N] fp32 GEMM weights -> [2][N][K] (hi, lo) K-major TF32 split.
Status GemmWeightSplit(const TensorDesc& in, const void* data, TensorDesc* out,
                       std::vector<std::uint8_t>* bytes) {
  if (in.shape.size() != 2 || in.dtype != DataType::kFloat32) {
    return Status::ShapeError("gemm_w_tf32x2_nk expects a rank-2 float32 constant");
  }
  const int64_t K = in.shape[0], N = in.shape[1];
  const std::size_t plane = static_cast<std::size_t>(K * N);
  *out = TensorDesc({2, N, K}, DataType::kFloat32, in.device_type, in.device_id, "");
  bytes->assign(2 * plane * sizeof(float), 0);
  const auto* w = static_cast<const float*>(data);
  auto* dst = reinterpret_cast<float*>(bytes->data());
  for (int64_t k = 0; k < K; ++k)
    for (int64_t n = 0; n < N; ++n) {
      float hi, lo;
      SplitTf32(w[k * N + n], &hi, &lo);
      dst[n * K + k] = hi;
      dst[plane + n * K + k] = lo;
    }
  return Status::OK();
}

const std::unordered_map<std::string, Transform>& Registry() {
  static const std::unordered_map<std::string, Transform> table = {
      {"transpose_2d", Transpose2d},
      {"conv_w_tf32x2_okpad", ConvWeightSplit},
      {"conv_w_tf32x2_cb", ConvWeightSplitChannelBlocks},
      {"gemm_w_tf32x2_nk", GemmWeightSplit},
  };
  return table;
}

}  // namespace

std::string PrepackedName(const std::string& constant, const std::string& prepack) {
  return constant + "::" + prepack;
}

bool IsKnownPrepack(const std::string& prepack) { return Registry().count(prepack) != 0; }

Status RunPrepack(const std::string& prepack, const TensorDesc& desc, const void* data,
                  TensorDesc* out_desc, std::vector<std::uint8_t>* out_bytes) {
  const auto it = Registry().find(prepack);
  if (it == Registry().end()) return Status::NotFound("unknown prepack transform: " + prepack);
  return it->second(desc, data, out_desc, out_bytes);
}

}  // namespace cutriton
