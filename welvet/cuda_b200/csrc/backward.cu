// backward.cu -- Dense NormalBP backward, SGD on the packed store and the MSE loss, on the GPU.
//
// Replaces the reference's training leaf of one Dense layer (src/interop/c_abi.cpp:119-184:
// forward, MSE from a target or a given gradient, backward, optional SGD, export):
//   act' / MatVec^T / outer    src/cuda/kernels.cu:48-128 and resident_backward (:917-1000)
//   SGD on FormatNone stores   src/weights/native_codec.cpp:1080-1133 (weight_at :513-568,
//                              set_weight_at :774-830)
//   MSE and its gradient       src/runtime/training.cpp:44-69
// The reference decodes the store to an fp64 mirror on the host and runs one thread per
// output element with a sequential fp64 loop; here W^T d reads the packed device mirror (the
// same codes, decoded with the reference's values in registers). Every product is of two
// floats or of a 4-bit/8-bit code value and a float, exact in fp64, and the sums keep the
// reference's order (sequential over rows for W^T d, over the batch for dW, per-batch float
// rounding in dW as the reference), so dX and dW equal the reference's bit for bit; the SGD
// re-encodes every element with the bit-exact codecs, as set_weight_at does.
#include "backward.hpp"

#include "codec.cuh"

namespace wb {

namespace {

// src/cuda/kernels.cu:48-81 (activate_deriv_dev), CUDA's double exp / tanh as the reference.
__device__ double activate_deriv(int act, double x) {
  switch (act) {
  case -1: return 1.0;
  case 0: return x > 0.0 ? 1.0 : 0.0;
  case 6: return x > 0.0 ? 2.0 * x : 0.0;
  case 5: return x > 0.0 ? 1.0 : 0.01;
  case 1: {
    const double sig = 1.0 / (1.0 + exp(-x));
    return sig * (1.0 + x * (1.0 - sig));
  }
  case 2: {
    constexpr double k = 0.7978845608028654;
    const double u = k * (x + 0.044715 * x * x * x);
    const double th = tanh(u);
    const double du = k * (1.0 + 3.0 * 0.044715 * x * x);
    return 0.5 * (1.0 + th) + 0.5 * x * (1.0 - th * th) * du;
  }
  case 3: {
    const double t = tanh(x);
    return 1.0 - t * t;
  }
  case 4: {
    const double s = 1.0 / (1.0 + exp(-x));
    return s * (1.0 - s);
  }
  default: return 1.0;
  }
}

// d_pre = float(double(gy) * act'(double(pre))), or gy for the linear walk.
__global__ void k_bwd_dpre(const float* __restrict__ gy, const float* __restrict__ pre, float* __restrict__ d_pre,
                           int act, int linear, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    d_pre[i] = linear ? gy[i] : static_cast<float>(static_cast<double>(gy[i]) *
                                                   activate_deriv(act, static_cast<double>(pre[i])));
}

// The reference value of element i of mirror row `row` (canonical codes decode as the
// original ones: FP8 subnormals and E4M3 0x7f/0xff were mapped to codes of the same value).
template <int kDt>
__device__ __forceinline__ double mirror_value(const uint8_t* __restrict__ row, int i, float scale) {
  if constexpr (kDt == 1) return static_cast<double>(reinterpret_cast<const float*>(row)[i]);
  else if constexpr (kDt == 16) return static_cast<double>(dec_fp4_ref((row[i >> 1] >> ((i & 1) * 4)) & 0xF));
  else if constexpr (kDt == 4) return static_cast<double>(dec_e4m3_ref(row[i]));
  else if constexpr (kDt == 5) return static_cast<double>(dec_e5m2_ref(row[i]));
  else return static_cast<double>(static_cast<float>(static_cast<int8_t>(row[i])) * scale);
}

// gx[b, i] = float(sum_o W[o, i] * double(d_pre[b, o])), o in order. One thread per (b, i):
// consecutive threads read consecutive codes of one mirror row.
template <int kDt>
__global__ void k_matvect(const uint8_t* __restrict__ W, int64_t row_stride, float scale,
                          const float* __restrict__ d_pre, float* __restrict__ gx, int rows, int cols) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (i >= cols) return;
  const float* dp = d_pre + static_cast<int64_t>(b) * rows;
  double sum = 0.0;
  for (int o = 0; o < rows; ++o)
    sum += mirror_value<kDt>(W + static_cast<int64_t>(o) * row_stride, i, scale) * static_cast<double>(dp[o]);
  gx[static_cast<int64_t>(b) * cols + i] = static_cast<float>(sum);
}

// dW[o, i]: over the batch in order, acc = float(double(acc) + double(d_pre[b, o]) * double(x[b, i])).
__global__ void k_outer(const float* __restrict__ d_pre, const float* __restrict__ x, float* __restrict__ dW,
                        int batch, int rows, int cols) {
  const int64_t n = static_cast<int64_t>(rows) * cols;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int o = static_cast<int>(t / cols);
    const int i = static_cast<int>(t - static_cast<int64_t>(o) * cols);
    float acc = 0.0f;
    for (int b = 0; b < batch; ++b)
      acc = static_cast<float>(static_cast<double>(acc) +
                               static_cast<double>(d_pre[static_cast<int64_t>(b) * rows + o]) *
                                   static_cast<double>(x[static_cast<int64_t>(b) * cols + i]));
    dW[t] = acc;
  }
}

// One element of the SGD: decode (reference values), next = float(double(v) - lr * dW), encode.
template <int kDt>
__device__ __forceinline__ uint32_t sgd_code(uint32_t code, double dw, double lr, float scale) {
  float v;
  if constexpr (kDt == 16) v = dec_fp4_ref(code);
  else if constexpr (kDt == 4) v = dec_e4m3_ref(code);
  else if constexpr (kDt == 5) v = dec_e5m2_ref(code);
  else v = static_cast<float>(static_cast<int8_t>(code)) * scale;
  const float next = static_cast<float>(static_cast<double>(v) - lr * dw);
  if constexpr (kDt == 16) return enc_fp4(next) & 0xF;
  else if constexpr (kDt == 4) return enc_e4m3(next);
  else if constexpr (kDt == 5) return enc_e5m2(next);
  else {
    double q = round(static_cast<double>(next / scale));  // float division, then round half away
    q = q < -128.0 ? -128.0 : (q > 127.0 ? 127.0 : q);
    return static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(q)));
  }
}

// One thread per payload byte (FP4: both nibbles of the byte). dW float (a backward's output)
// or double (WeightStore::apply_sgd's own argument type); either is widened to double.
template <int kDt, typename TW>
__global__ void k_sgd_native(uint8_t* __restrict__ native, int64_t n, const TW* __restrict__ dW, double lr,
                             float scale) {
  const int64_t bytes = kDt == 16 ? (n + 1) / 2 : n;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < bytes;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t byte = native[t];
    if constexpr (kDt == 16) {
      uint32_t lo = byte & 0xF, hi = byte >> 4;
      lo = sgd_code<16>(lo, dW[2 * t], lr, scale);
      if (2 * t + 1 < n) hi = sgd_code<16>(hi, dW[2 * t + 1], lr, scale);
      native[t] = static_cast<uint8_t>(lo | (hi << 4));
    } else {
      native[t] = static_cast<uint8_t>(sgd_code<kDt>(byte, dW[t], lr, scale));
    }
  }
}

template <typename TW>
__global__ void k_sgd_f32(float* __restrict__ w, int64_t n, const TW* __restrict__ dW, double lr) {
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x)
    w[t] -= static_cast<float>(lr * static_cast<double>(dW[t]));
}

// MSE: grad = float(2 / n * (pred - target)); the loss sum in a fixed order (each thread a
// strided run, then a tree over the block): deterministic, in another order than the
// reference's sequential sum.
constexpr int kMseThreads = 1024;
__global__ void __launch_bounds__(kMseThreads) k_mse(const float* __restrict__ pred, const float* __restrict__ target,
                                                     float* __restrict__ grad, int64_t n, double* __restrict__ loss) {
  __shared__ double part[kMseThreads];
  const double sc = 2.0 / static_cast<double>(n);
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += kMseThreads) {
    const double d = static_cast<double>(pred[i]) - static_cast<double>(target[i]);
    s += d * d;
    grad[i] = static_cast<float>(sc * d);
  }
  part[threadIdx.x] = s;
  __syncthreads();
  for (int w = kMseThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) *loss = part[0] / static_cast<double>(n);
}

unsigned grid_for(int64_t n) {
  int64_t b = (n + 255) / 256;
  if (b > 148 * 32) b = 148 * 32;
  return static_cast<unsigned>(b < 1 ? 1 : b);
}

} // namespace

Status dense_backward_device(const DeviceDense& d, int batch, const float* gy, const float* x, const float* pre,
                             bool linear, float* d_pre, float* gx, float* dW, cudaStream_t st) {
  if (batch <= 0 || !gy || !x || (!pre && !linear) || !d_pre || !gx || !dW || !d.W)
    return Status::Invalid("dense backward: null arguments");
  const int64_t ny = static_cast<int64_t>(batch) * d.rows;
  k_bwd_dpre<<<grid_for(ny), 256, 0, st>>>(gy, pre, d_pre, d.act, linear ? 1 : 0, ny);
  WB_CUDA(cudaGetLastError());
  const dim3 g(static_cast<unsigned>((d.cols + 255) / 256), static_cast<unsigned>(batch));
  switch (d.dtype) {
  case DType::Float32: k_matvect<1><<<g, 256, 0, st>>>(d.W, d.row_stride, d.scale, d_pre, gx, d.rows, d.cols); break;
  case DType::FP4: k_matvect<16><<<g, 256, 0, st>>>(d.W, d.row_stride, d.scale, d_pre, gx, d.rows, d.cols); break;
  case DType::FP8E4M3: k_matvect<4><<<g, 256, 0, st>>>(d.W, d.row_stride, d.scale, d_pre, gx, d.rows, d.cols); break;
  case DType::FP8E5M2: k_matvect<5><<<g, 256, 0, st>>>(d.W, d.row_stride, d.scale, d_pre, gx, d.rows, d.cols); break;
  case DType::Int8: k_matvect<9><<<g, 256, 0, st>>>(d.W, d.row_stride, d.scale, d_pre, gx, d.rows, d.cols); break;
  default: return Status::Unsupported("dense backward: dtype");
  }
  WB_CUDA(cudaGetLastError());
  k_outer<<<grid_for(static_cast<int64_t>(d.rows) * d.cols), 256, 0, st>>>(d_pre, x, dW, batch, d.rows, d.cols);
  return cuda_status(cudaGetLastError(), "dense backward launch");
}

namespace {

template <typename TW>
Status launch_sgd(DType dt, void* payload_dev, int64_t n, float scale, const TW* dW_dev, double lr,
                  cudaStream_t st) {
  if (!payload_dev || !dW_dev || n <= 0) return Status::Invalid("sgd: null arguments");
  const float s = scale == 0.0f ? 1.0f : scale;  // weight_at / set_weight_at treat 0 as 1
  auto* raw = static_cast<uint8_t*>(payload_dev);
  const int64_t units = dt == DType::FP4 ? (n + 1) / 2 : n;
  switch (dt) {
  case DType::Float32: k_sgd_f32<TW><<<grid_for(n), 256, 0, st>>>(static_cast<float*>(payload_dev), n, dW_dev, lr); break;
  case DType::FP4: k_sgd_native<16, TW><<<grid_for(units), 256, 0, st>>>(raw, n, dW_dev, lr, s); break;
  case DType::FP8E4M3: k_sgd_native<4, TW><<<grid_for(units), 256, 0, st>>>(raw, n, dW_dev, lr, s); break;
  case DType::FP8E5M2: k_sgd_native<5, TW><<<grid_for(units), 256, 0, st>>>(raw, n, dW_dev, lr, s); break;
  case DType::Int8: k_sgd_native<9, TW><<<grid_for(units), 256, 0, st>>>(raw, n, dW_dev, lr, s); break;
  default: return Status::Unsupported("sgd: dtype");
  }
  return cuda_status(cudaGetLastError(), "sgd launch");
}

} // namespace

Status apply_sgd_native(DType dt, void* payload_dev, int64_t n, float scale, const float* dW_dev, double lr,
                        cudaStream_t st) {
  return launch_sgd(dt, payload_dev, n, scale, dW_dev, lr, st);
}

Status apply_sgd_native(DType dt, void* payload_dev, int64_t n, float scale, const double* dW_dev, double lr,
                        cudaStream_t st) {
  return launch_sgd(dt, payload_dev, n, scale, dW_dev, lr, st);
}

Status mse_device(const float* pred, const float* target, int64_t n, float* grad, double* loss_dev, cudaStream_t st) {
  if (!pred || !target || !grad || !loss_dev || n <= 0) return Status::Invalid("training: MSE shape");
  k_mse<<<1, kMseThreads, 0, st>>>(pred, target, grad, n, loss_dev);
  return cuda_status(cudaGetLastError(), "mse launch");
}

} // namespace wb
