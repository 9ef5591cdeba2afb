// common.hpp -- status, dtype and activation vocabulary shared by the library.
//
// The numeric values are ABI facts of welvet.cuda and are kept identical:
//   StatusCode   include/welvet/status.hpp:8-14   (welvet_status.code in welvet_c.h:26-29)
//   DType        include/welvet/dtype.hpp:9-44
//   Activation   include/welvet/activate.hpp:8-17
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

namespace wb {

enum class StatusCode : int32_t { Ok = 0, InvalidArgument = 1, Unsupported = 2, Gap = 3, Internal = 4 };

struct Status {
  StatusCode code = StatusCode::Ok;
  std::string message;
  static Status Ok() { return {}; }
  static Status Err(StatusCode c, std::string m) { return Status{c, std::move(m)}; }
  static Status Invalid(std::string m) { return Err(StatusCode::InvalidArgument, std::move(m)); }
  static Status Unsupported(std::string m) { return Err(StatusCode::Unsupported, std::move(m)); }
  static Status Internal(std::string m) { return Err(StatusCode::Internal, std::move(m)); }
  bool ok() const { return code == StatusCode::Ok; }
  explicit operator bool() const { return ok(); }
};

enum class DType : int32_t {
  Float32 = 1,
  FP8E4M3 = 4,
  FP8E5M2 = 5,
  Int8 = 9,
  FP4 = 16,
};

// The storage types this library serves on the GPU. Every other welvet DType id is
// rejected with StatusCode::Unsupported (never a host fallback).
inline bool dtype_on_path(int32_t id) {
  return id == 1 || id == 4 || id == 5 || id == 9 || id == 16;
}

inline const char* dtype_name(int32_t id) {
  switch (id) {
  case 1: return "float32";
  case 4: return "fp8e4m3";
  case 5: return "fp8e5m2";
  case 9: return "int8";
  case 16: return "fp4";
  default: return "unsupported";
  }
}

// Bytes of a FormatNone native payload of n elements (src/weights/native_codec.cpp:193-262);
// Float32 keeps a float payload of 4 bytes per element.
inline int64_t native_bytes(DType dt, int64_t n) {
  switch (dt) {
  case DType::FP4: return (n + 1) / 2;
  case DType::Float32: return n * 4;
  default: return n;
  }
}

// Bytes of one weight row in the device mirror before padding.
inline int64_t row_bytes(DType dt, int64_t cols) {
  switch (dt) {
  case DType::FP4: return (cols + 1) / 2;
  case DType::Float32: return cols * 4;
  default: return cols;
  }
}

enum class Activation : int32_t {
  Linear = -1, ReLU = 0, Silu = 1, GELU = 2, Tanh = 3, Sigmoid = 4, LeakyReLU = 5, ReLU2 = 6,
};

inline bool activation_valid(int32_t a) { return a >= -1 && a <= 6; }

inline Status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return Status::Ok();
  return Status::Internal(std::string(what) + ": " + cudaGetErrorString(e));
}

#define WB_TRY(expr)                      \
  do {                                    \
    ::wb::Status _st = (expr);            \
    if (!_st.ok()) return _st;            \
  } while (0)

#define WB_CUDA(call) WB_TRY(::wb::cuda_status((call), #call))

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// Further destinations of a layer's post, besides the local one: a column-sharded layer
// (sharded.hpp) writes its slice of the output straight into the other ranks' gathered
// buffers over NVLink peer memory. Each pointer has the local post's layout ([M][ld_out],
// offset to the shard's first column). n = 0: the layer writes only its own outputs.
constexpr int kMaxPeerOut = 7;
struct PeerOut {
  int n = 0;
  float* post[kMaxPeerOut] = {};
};

// An RMSNorm layer run as the prologue of the projection that consumes it (the reference's
// norm_forward_f64 with center = 0, src/cuda/kernels.cu:172-204): x is the norm's input,
// pre = x / sqrt(mean(x^2) + eps) and post = pre * gamma ([M][cols], the norm layer's outputs)
// are written by the launch's first kernel, and the GEMM multiplies post. gamma == nullptr:
// no prologue.
struct SplitNorm {
  const double* gamma = nullptr;  // [cols], the store's decoded gamma widened to fp64
  double eps = 0.0;
  float* pre = nullptr;
  float* post = nullptr;
};

} // namespace wb
