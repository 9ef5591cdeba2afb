// cells.hpp -- SwiGLU, MHA and RMSNorm cells built from the Dense mirror.
//
// Reference interfaces mirrored:
//   swiglu::Layer / new_configured / forward   include/welvet/swiglu.hpp:20-31
//   mha::Config / validate / Layer / forward   include/welvet/mha.hpp:40-84
//   rmsnorm forward                            src/layers/rmsnorm/rmsnorm.cpp:60-113
#pragma once

#include "cell_kernels.hpp"
#include "dense.hpp"

namespace wb {

// A weight matrix as a cell mount reads it: float32 values (host or device) quantized at
// mount, or reference-layout native bytes with their scale (a stored model's store section,
// src/interop/model_session.cpp:135-153).
struct WeightSrc {
  const float* f32 = nullptr;
  bool f32_on_device = false;
  const uint8_t* native = nullptr;
  size_t native_len = 0;
  float scale = 1.0f;
};
Status mount_dense_src(int device, int rows, int cols, DType dt, int act, const WeightSrc& w,
                       const double* bias, size_t bias_len, WeightStore* store, DeviceDense* dev,
                       cudaStream_t st);

struct SwigluCell {
  int device = 0;
  int in = 0, inter = 0;
  WeightStore sg, su, sd;
  DeviceDense gate, up, down;  // Linear, no bias (src/layers/swiglu/swiglu.cpp:74-82)
  // work buffers for `bs` rows
  int bs = 0;
  float* x_pad = nullptr;  // [bs][gate.x_stride]
  float* h_pad = nullptr;  // [bs][down.x_stride] (padding stays zero)
  float* g_buf = nullptr;  // [bs][inter] gate output (tensor-core GEMM path, unfused)
  float* u_buf = nullptr;  // [bs][inter] up output
  DenseIO io_gate, io_up, io_down;  // per-projection staging and scratch
  // Gate/Up pair mirror for the batched path: one tcgen05 GEMM over 2 x inter interleaved
  // rows whose epilogue writes h (gemm_tc.hpp, GemmArgs::pair); built at mount when the
  // layers take the tensor-core path.
  uint8_t* Wg_pair = nullptr;
  void* pair_scratch = nullptr;  // that GEMM's scratch for `bs` rows
  size_t pair_scratch_bytes = 0;
  void release_work();
  ~SwigluCell();
};

Status swiglu_mount(int device, int in, int inter, DType dt, const float* G, const float* U, const float* D,
                    bool w_is_device, SwigluCell* c, cudaStream_t st);
// The same from weight sources Gate, Up, Down.
Status swiglu_mount_src(int device, int in, int inter, DType dt, const WeightSrc (&w)[3], SwigluCell* c,
                        cudaStream_t st);
Status swiglu_reserve(SwigluCell* c, int bs, cudaStream_t st);
// x [bs][in] (device) -> h [bs][inter] (the reference's pre) and y [bs][in] (post).
// h may be nullptr (h stays in the cell's padded work buffer).
// `norm` (may be nullptr): an RMSNorm of width in in front (x is its input; see forward_device).
Status swiglu_forward_device(SwigluCell* c, int bs, const float* x, float* h, float* y, cudaStream_t st,
                             bool pdl, const SplitNorm* norm = nullptr);

struct MhaConfig {
  int d_model = 0, num_heads = 0, num_kv_heads = 0, head_dim = 0, max_seq_len = 0;
  int mask = 1, pos = 0, softmax = 0, window = 0, prefix_len = 0, window_causal = 1;
  double rope_theta = 10000.0, scale_override = 0.0;
};

// src/layers/mha/mha.cpp:57-85 (defaults and divisibility checks).
Status mha_validate(MhaConfig* cfg);

struct MhaCell {
  int device = 0;
  MhaConfig cfg;
  WeightStore sq, sk, sv, so;
  DeviceDense q, k, v, o;
  int bs = 0;
  float *x_pad = nullptr, *qb = nullptr, *kb = nullptr, *vb = nullptr, *attn = nullptr, *attn_pad = nullptr;
  double *Qr = nullptr, *Kr = nullptr, *Vd = nullptr;
  DenseIO io_q, io_k, io_v, io_o;  // per-projection staging and scratch
  void release_work();
  ~MhaCell() { release_work(); }
};

Status mha_mount(int device, const MhaConfig& cfg, DType dt, const float* Q, const float* K, const float* V,
                 const float* O, bool w_is_device, MhaCell* c, cudaStream_t st);
// The same from weight sources Q, K, V, O.
Status mha_mount_src(int device, const MhaConfig& cfg, DType dt, const WeightSrc (&w)[4], MhaCell* c,
                     cudaStream_t st);
Status mha_reserve(MhaCell* c, int bs, cudaStream_t st);
// x [batch*seq][d_model] (device) -> attn [bs][q_dim] (pre) and y [bs][d_model] (post).
Status mha_forward_device(MhaCell* c, int batch, int seq, const float* x, float* attn, float* y,
                          cudaStream_t st, const SplitNorm* norm = nullptr);

// gamma f32 [dim] quantized with `dt` then decoded to f64 as the reference's gamma store.
Status rmsnorm_gamma(int device, int dim, DType dt, const float* gamma, double** gamma64_dev, cudaStream_t st);
// The same from a weight source (host float32 or native bytes).
Status rmsnorm_gamma_src(int device, int dim, DType dt, const WeightSrc& w, double** gamma64_dev, cudaStream_t st);

} // namespace wb
