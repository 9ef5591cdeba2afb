// cell_kernels.hpp -- RMSNorm, MHA attention core and SwiGLU product launchers.
#pragma once

#include "common.hpp"

namespace wb {

// Attention configuration after the reference's mha::validate (src/layers/mha/mha.cpp:57-85).
struct AttnParams {
  int batch = 1, seq = 1;
  int num_heads = 1, num_kv = 1, head_dim = 1;
  int max_seq_len = 512;
  int mask = 1;          // MaskKind: 1 causal, 2 bidirectional, 3 sliding window, 4 prefix LM
  int pos_kind = 0;      // PosKind: 0 RoPE, 1 none, 2 ALiBi, 3 RoPE+ALiBi
  int softmax_kind = 0;  // 0 standard, 1 sigmoid
  int window = 0, prefix_len = 0, window_causal = 1;
  double rope_theta = 10000.0;
  double scale_override = 0.0;
};

Status launch_rmsnorm(const float* x, const double* gamma, float* pre, float* post, int n_tok, int dim,
                      double eps, cudaStream_t st);

// q [bs][q_dim], k/v [bs][kv_dim] float32 projections -> out [bs][q_dim]. Qr/Kr/Vd are f64
// work buffers of bs*q_dim, bs*kv_dim, bs*kv_dim elements.
Status launch_mha_attention(const float* q, const float* k, const float* v, double* Qr, double* Kr,
                            double* Vd, float* out, const AttnParams& p, cudaStream_t st);

Status launch_swiglu_product(const float* g, const float* u, float* h, int64_t n, cudaStream_t st);

} // namespace wb
