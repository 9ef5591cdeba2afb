#pragma once
// welvet/swiglu.hpp -- the reference's SwiGLU layer C++ API (include/welvet/swiglu.hpp:9-31) over
// libwelvet_b200. forward runs the library's fused cell (Gate and Up in one kernel with the
// product in its epilogue, then Down), mounted lazily from the three layers' stores and kept in
// Gate's device state until one of the three is invalidated.

#include "welvet/dense.hpp"
#include "welvet/dtype.hpp"
#include "welvet/status.hpp"
#include "welvet/tensor.hpp"

namespace welvet::swiglu {

struct Config {
  int input_dim = 0;
  int intermediate_dim = 0;
};

WELVET_CXX_API Status validate(const Config& cfg);

// Llama-style ~8/3 intermediate, rounded to a multiple of 8.
WELVET_CXX_API Config default_ffn(int d_model);

struct Layer {
  Config cfg{};
  dense::Layer Gate, Up, Down;
};

WELVET_CXX_API Status new_configured(const Config& cfg, DType dt, const float* gate_init, const float* up_init,
                                     const float* down_init, Layer* out);

// pre = h = SiLU(Gate(x)) * Up(x); post = Down(h). input [batch, in] or [batch, seq, in].
WELVET_CXX_API Status forward(Layer& layer, const TensorF32& input, TensorF32* pre, TensorF32* post);

} // namespace welvet::swiglu
