// backward.hpp -- Dense NormalBP backward, SGD on FormatNone stores and MSE on the GPU
// (backward.cu).
#pragma once

#include "dense.hpp"

namespace wb {

// Over a mounted layer (its packed device mirror), for `batch` rows (device pointers):
// d_pre = float(gy * act'(pre)) (linear: gy), gx = float(W^T d_pre) [batch][cols] (fp64,
// sequential over rows), dW [rows][cols] (per-batch float accumulation). Bit-exact with the
// reference's CUDA backward (src/cuda/kernels.cu:83-128) up to CUDA's exp / tanh in act'.
Status dense_backward_device(const DeviceDense& d, int batch, const float* gy, const float* x, const float* pre,
                             bool linear, float* d_pre, float* gx, float* dW, cudaStream_t st);
// WeightStore::apply_sgd on a device copy of the store's payload (native bytes; Float32: the
// float payload) of n elements, dW float [n]: decode, float(double(v) - lr * dW), encode.
Status apply_sgd_native(DType dt, void* payload_dev, int64_t n, float scale, const float* dW_dev, double lr,
                        cudaStream_t st);
Status apply_sgd_native(DType dt, void* payload_dev, int64_t n, float scale, const double* dW_dev, double lr,
                        cudaStream_t st);
// MSE of pred against target (n floats): grad = float(2 / n * (pred - target)), *loss_dev.
Status mse_device(const float* pred, const float* target, int64_t n, float* grad, double* loss_dev, cudaStream_t st);

} // namespace wb
