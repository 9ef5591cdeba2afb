#pragma once
// welvet/tensor.hpp -- the reference's host tensor (include/welvet/tensor.hpp): a shape and
// row-major float data.

#include <cstddef>
#include <cstdint>
#include <vector>

#ifndef WELVET_CXX_API
#define WELVET_CXX_API __attribute__((visibility("default")))
#endif

namespace welvet {

struct WELVET_CXX_API TensorF32 {
  std::vector<int64_t> shape;
  std::vector<float> data;

  static TensorF32 zeros(int64_t a, int64_t b);
  std::size_t numel() const { return data.size(); }
};

} // namespace welvet
