#pragma once
// welvet/dense.hpp -- the reference's Dense layer C++ API (include/welvet/dense.hpp:13-76) over
// libwelvet_b200: the same Layer fields and move semantics, new_layer, forward_f32, the NormalBP
// backward family and SGD with the same signatures, shape checks and messages
// (src/layers/dense/dense.cpp:58-209). The device
// mirror is mounted lazily, as in the reference: on the first forward, after
// invalidate_gpu(), and when the batch changes.

#include "welvet/activate.hpp"
#include "welvet/cuda/matvec.hpp"
#include "welvet/dtype.hpp"
#include "welvet/status.hpp"
#include "welvet/tensor.hpp"
#include "welvet/weights.hpp"

namespace welvet::dense {

struct WELVET_CXX_API Layer {
  int input_height = 0;
  int output_height = 0;
  Activation activation = Activation::Linear;
  WeightStore weights;

  mutable cuda::ResidentDense gpu{};
  mutable bool gpu_valid = false;
  mutable int gpu_batch = -1;

  Layer() = default;
  Layer(const Layer&) = delete;
  Layer& operator=(const Layer&) = delete;
  Layer(Layer&& o) noexcept
      : input_height(o.input_height), output_height(o.output_height), activation(o.activation),
        weights(static_cast<WeightStore&&>(o.weights)), gpu(o.gpu), gpu_valid(o.gpu_valid), gpu_batch(o.gpu_batch) {
    o.gpu = {};
    o.gpu_valid = false;
    o.gpu_batch = -1;
  }
  Layer& operator=(Layer&& o) noexcept {
    if (this == &o) return *this;
    cuda::resident_release(&gpu);
    input_height = o.input_height;
    output_height = o.output_height;
    activation = o.activation;
    weights = static_cast<WeightStore&&>(o.weights);
    gpu = o.gpu;
    gpu_valid = o.gpu_valid;
    gpu_batch = o.gpu_batch;
    o.gpu = {};
    o.gpu_valid = false;
    o.gpu_batch = -1;
    return *this;
  }
  ~Layer() { cuda::resident_release(&gpu); }

  void invalidate_gpu() const { gpu_valid = false; }
};

WELVET_CXX_API Status new_layer(int in_h, int out_h, Activation act, DType dt, const float* init_or_null,
                                Layer* layer);

WELVET_CXX_API bool dtype_supported_cuda_forward(DType dt);

// FormatNone Dense forward on the GPU: input [batch, in] -> pre, post [batch, out].
WELVET_CXX_API Status forward_f32(const Layer& layer, const TensorF32& input, TensorF32* pre, TensorF32* post);

// Dense NormalBP backward on the GPU: grad_in = W^T (grad_out * act'(pre)) [batch, in],
// grad_w = sum over the batch of the outer products [out, in] (src/layers/dense/dense.cpp:88-120).
WELVET_CXX_API Status backward_f32(const Layer& layer, const TensorF32& grad_out, const TensorF32& input,
                                   const TensorF32& pre, TensorF32* grad_in, TensorF32* grad_w);
// gx = W^T gy with no act' (gy resampled to batch * out values first; dense.cpp:141-166).
WELVET_CXX_API Status linear_grad_in(const Layer& layer, const TensorF32& gy, const TensorF32& input,
                                     TensorF32* gx);
// dW only (gy resampled as above; pre zeros when short; dense.cpp:168-190).
WELVET_CXX_API Status grad_w_only(const Layer& layer, const TensorF32& gy, const TensorF32& input,
                                  const TensorF32& pre, TensorF32* dw);
// W <- W - lr * dW on the store (on the GPU), then invalidate_gpu() (dense.cpp:192-209).
WELVET_CXX_API Status apply_grad_sgd(Layer* layer, const TensorF32& dW, double lr);
// (Re)mounts the layer's device mirror for `batch` rows from its store.
WELVET_CXX_API Status sync_gpu_from_weights(const Layer& layer, int batch);

} // namespace welvet::dense
