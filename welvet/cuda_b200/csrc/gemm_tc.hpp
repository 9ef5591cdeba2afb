// gemm_tc.hpp -- batched dequant GEMM on the 5th-generation tensor cores (tcgen05 / TMEM).
#pragma once

#include "common.hpp"

#include <cuda_fp16.h>

namespace wb {

// y[t][o] = sum_k W[o][k] x[t][k] for t < M tokens, over the packed device mirror.
//
// Numerics: x is split per token into `xsplit` f16 planes after scaling by a power of two
// (x * 2^e = p0 + p1 + p2); FP8/FP4/Int8 weights are exact in f16, so each product is exact
// and the tensor core accumulates in fp32. xsplit = 3 carries all 24 bits of every x
// element (only fp32 accumulation error remains); 2 carries 22 bits, 1 carries 11 bits.
struct GemmArgs {
  DType dtype = DType::FP4;
  const uint8_t* W = nullptr;   // mirror [rows][row_stride]
  const uint8_t* Wg = nullptr;  // GEMM mirror (build_gemm_mirror); required by the default kernel
  int64_t row_stride = 0;
  int rows = 0;                 // out
  int cols = 0;                 // in (K)
  float scale = 1.0f;           // Int8 per-tensor scale
  const float* x = nullptr;     // [M][x_ld]
  int64_t x_ld = 0;
  int M = 0;
  float* pre = nullptr;         // [M][ld_out]
  float* post = nullptr;        // [M][ld_out] (may equal pre when act is Linear and no bias)
  int64_t ld_out = 0;
  const double* bias = nullptr;
  int bias_len = 0;
  int act = -1;
  int xsplit = 3;
  // scratch (device): see gemm_scratch_bytes
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  int max_tb = 0;               // tokens per token block at most (0: the plan's own; k_gemm_tm)
  int* err = nullptr;           // device error word (0 = ok), may be nullptr
  // SwiGLU Gate/Up pair (k_gemm_tm only): Wg is a pair mirror (rows 2i = Gate row i,
  // 2i+1 = Up row i, rows = 2 x intermediate) and the epilogue writes
  // h[t][i] = SiLU(gate)·up with the reference's rounding (src/cuda/kernels.cu:296-305)
  // instead of pre/post; `scale` / `scale2` are Gate's / Up's Int8 scales.
  bool pair = false;
  float scale2 = 1.0f;
  float* h = nullptr;           // [M][ld_h]
  int64_t ld_h = 0;
  // Further destinations of post (column-sharded layers, peer memory): same layout as post.
  PeerOut peers;
  // The launch's first kernel (k_split_x) as a programmatic dependent of the kernel before it
  // on the stream (it waits for that kernel's completion before reading x). The launch's own
  // kernels always chain this way: k_split_x -> the GEMM -> the split-K / tail reduce, each
  // releasing its dependent at once and waiting for its predecessor before any global access.
  bool pdl = false;
  SplitNorm norm;
};

// Token tile (B rows per plane) used for M tokens; the MMA N is xsplit * tile.
int gemm_token_tile(int M, int xsplit);
// Bytes of scratch a launch with these sizes needs (planes, per-token scales, split-K partials;
// with `tail`, room for the K slices of a last partial wave's tiles, which the launch uses
// when the scratch it is given holds them).
size_t gemm_scratch_bytes(int M, int cols, int rows, int xsplit, bool tail = true, int max_tb = 0);

// The TMEM kernel's launch plan as numbers (see welvet_b200_gemm_plan): writes the first n of
// them to out and returns how many there are.
int gemm_plan_values(int M, int cols, int rows, int xsplit, DType dt, int max_tb, int64_t* out, int n);

bool gemm_supported(DType dt);

// The GEMM mirror: the row-major mirror cut into tiles of 128 rows x 64 k, each stored as one
// contiguous block ([rows/128][K/64][128][bytes of 64 codes]) so that a pipeline stage is
// one bulk copy, with the 16-byte chunks of row r at chunk ^ swizzle(r) (the 32-byte
// swizzle for FP4 rows, 64-byte for 8-bit rows) so that one thread per row reads shared
// memory without bank conflicts. Rows and k past the layer are zero.
size_t gemm_mirror_bytes(DType dt, int rows, int cols);
Status build_gemm_mirror(DType dt, const uint8_t* W, int rows, int64_t row_stride, int cols, uint8_t* Wg,
                         cudaStream_t st);
// The pair mirror of a SwiGLU cell (gemm_mirror_bytes(dt, 2 * inter, cols) bytes) from the
// row-major mirrors of Gate and Up (same geometry).
Status build_gemm_pair_mirror(DType dt, const uint8_t* Wgate, const uint8_t* Wup, int inter, int64_t row_stride,
                              int cols, uint8_t* Wg, cudaStream_t st);
// Whether launches use the TMEM kernel (the pair mode needs it): false only when
// WELVET_B200_GEMM=smem selects the shared-memory variant.
bool gemm_uses_tmem();

Status launch_gemm_tc(const GemmArgs& a, cudaStream_t st);

// The same launch with its scratch in a fixed static device array instead of a.scratch:
// makes no allocation of any kind. Rejects (status 1) a launch whose scratch would exceed
// gemm_static_scratch_bytes(). The first call on a device looks up the array's device
// address (again after the device's context was re-created) and should come before any
// stream capture. Calls that overlap on one GPU race.
Status launch_gemm_tc_static(const GemmArgs& a, cudaStream_t st);
size_t gemm_static_scratch_bytes();

} // namespace wb
