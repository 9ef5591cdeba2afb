#pragma once
// welvet/weights.hpp -- the reference's FormatNone weight store (include/welvet/weights.hpp:12-51):
// the same fields with the same meaning, so that a caller that fills or reads a store (a layer's
// `weights`) works unchanged. Quantization, export and SGD run on the GPU (bit-exact with the
// reference codec and WeightStore::apply_sgd); the reference store's host matvec helpers are
// not part of this library's path and are not declared.

#include <cstddef>
#include <cstdint>
#include <vector>

#include "welvet/dtype.hpp"
#include "welvet/status.hpp"

namespace welvet {

enum class QuantFormat : int32_t {
  None = 0,
};

struct WELVET_CXX_API WeightStore {
  DType dtype = DType::Float32;
  QuantFormat format = QuantFormat::None;
  int rows = 0;
  int cols = 0;
  std::vector<float> f32;       // Float32 payload
  std::vector<uint8_t> native;  // FP8 / FP4 / Int8 payload, reference layout
  float scale = 1.0f;
  std::vector<double> bias;

  // rows x cols from float32 values (zeros when init_or_null is null), quantized to `dt`.
  static Status make(int rows, int cols, DType dt, const float* init_or_null, WeightStore* out);
  static Status make_f32(int rows, int cols, const float* init_or_null, WeightStore* out) {
    return make(rows, cols, DType::Float32, init_or_null, out);
  }
  // Decoded float32 weights [rows * cols] (src/weights/store.cpp export_f32).
  Status export_f32(float* dst) const;
  // w <- float(double(w) - lr * dW[i]) in the native storage, re-encoded
  // (src/core/native_codec.cpp:1080-1133, Go weights.ApplySGD). dW has rows * cols values.
  Status apply_sgd(const double* dW, double lr);
};

} // namespace welvet
