#pragma once
// welvet/activate.hpp -- activation ids of the reference (include/welvet/activate.hpp:8-17).

#include <cstdint>

namespace welvet {

enum class Activation : int32_t {
  Linear = -1,
  ReLU = 0,
  Silu = 1,
  GELU = 2,
  Tanh = 3,
  Sigmoid = 4,
  LeakyReLU = 5,
  ReLU2 = 6,
};

} // namespace welvet
