// gemv.hpp -- fused dequant GEMV for small batches (the batch-1 hot path).
#pragma once

#include "common.hpp"

namespace wb {

// One Dense forward y = W x over the device mirror (see codec.hpp: rows padded to
// row_stride bytes, canonical codes). x rows must be zero-padded to x_stride floats with
// x_stride >= (row_stride/16) * elements-per-16-bytes and 16-byte aligned.
struct GemvArgs {
  DType dtype = DType::FP4;
  const uint8_t* W = nullptr;   // mirror [rows][row_stride]
  const uint8_t* W2 = nullptr;  // SwiGLU: Up mirror (same shape); nullptr for a plain Dense
  int64_t row_stride = 0;       // bytes, multiple of 16
  int rows = 0;                 // out
  int cols = 0;                 // in
  float scale = 1.0f;           // Int8 per-tensor scale of W
  float scale2 = 1.0f;          // Int8 per-tensor scale of W2
  const float* x = nullptr;     // [batch][x_stride]
  int64_t x_stride = 0;
  int batch = 1;
  float* pre = nullptr;         // [batch][ld_out]  (SwiGLU: h)
  float* post = nullptr;        // [batch][ld_out]  (unused for SwiGLU)
  int64_t ld_out = 0;
  const double* bias = nullptr; // f64 [bias_len]; applies to rows o < bias_len
  int bias_len = 0;
  int act = -1;
  bool exact = false;           // fp64 products and accumulation (small layers)
  PeerOut peers;                // further destinations of post (column-sharded layers)
};

// Elements covered by 16 bytes of the mirror.
inline int elems_per_16B(DType dt) {
  switch (dt) {
  case DType::FP4: return 32;
  case DType::Float32: return 4;
  default: return 16;
  }
}

// Launches on `st`. With pdl=true the launch may overlap the previous kernel in the stream
// (programmatic dependent launch): the kernel only prefetches its weights into L2 before
// griddepcontrol.wait and reads x / writes outputs after it.
Status launch_gemv(const GemvArgs& a, cudaStream_t st, bool pdl);

// Copies `rows` rows of `cols` floats from src (leading dimension src_ld, any memory the device
// can read, mapped pinned host memory included) into dst (leading dimension dst_ld); the pad
// columns of dst are left as they are. The kernel releases its dependents at once, so a
// following launch made with pdl=true starts streaming its weights while x is in flight.
Status launch_stage_rows(float* dst, int64_t dst_ld, const float* src, int64_t src_ld, int cols, int rows,
                         cudaStream_t st);

} // namespace wb
