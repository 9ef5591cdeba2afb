// train.hpp -- one Dense training step on the GPU (train.cpp).
#pragma once

#include "dense.hpp"

namespace wb {

// The reference's welvet_dense_normalbp_f32 (src/interop/c_abi.cpp:119-184): build the layer
// from W_init (quantized on the GPU), forward x, take gy from grad_or_target (use_target:
// MSE against it, *loss set), backward to dX / dW, SGD with lr when lr != 0, and W_after as the
// store's decoded weights. Host buffers in and out; the same argument checks and status codes.
Status dense_normalbp(int batch, int in, int out, int act, int32_t dtype, const float* W_init, const double* bias,
                      size_t bias_len, const float* x, const float* grad_or_target, bool use_target, double lr,
                      float* pre, float* post, float* dX, float* dW, float* W_after, double* loss);

} // namespace wb
