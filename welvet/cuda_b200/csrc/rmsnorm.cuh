// rmsnorm.cuh -- the per-row arithmetic of the reference RMSNorm (src/cuda/kernels.cu:172-204,
// norm_forward_f64 with center = 0: pre = x / sqrt(mean(x^2) + eps) in fp64, post = pre * gamma),
// shared by the standalone kernel (cell_kernels.cu) and the prologue of the projection GEMM
// (gemm_tc.cu k_split_x), so that both write the same bits.
#pragma once

#include <cuda_runtime.h>

namespace wb {

// Threads per row in both kernels: the sum-of-squares order below depends on it.
constexpr int kNormThreads = 512;

// Sum of x^2 over one row in fp64, one block of kNormThreads per row, in a fixed order: thread j
// adds the 4-element chunks j, j + 512, ... (elements in order; `load4(k)` returns elements
// k..k+3 with zeros past the row), each warp sums its threads by a butterfly, and every thread
// adds the 16 warp sums in warp order. `dim` <= 0 gives 0 (a padding row). s_part holds
// kNormThreads / 32 doubles of shared memory; every thread of the block must call this.
template <class Load4>
__device__ __forceinline__ double rms_block_ss(Load4 load4, int dim, double* s_part) {
  const int tid = threadIdx.x;
  double ss = 0.0;
  for (int k = 4 * tid; k < dim; k += 4 * kNormThreads) {
    const float4 v = load4(k);
    const double a = v.x, b = v.y, c = v.z, d = v.w;
    ss += a * a;
    ss += b * b;
    ss += c * c;
    ss += d * d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) s_part[tid >> 5] = ss;
  __syncthreads();
  double tot = s_part[0];
#pragma unroll
  for (int w = 1; w < kNormThreads / 32; ++w) tot += s_part[w];
  return tot;
}

__device__ __forceinline__ double rms_inv(double ss, int dim, double eps) {
  return 1.0 / sqrt(ss / static_cast<double>(dim) + eps);
}

// Elements k..k+3 of one row (v = x[k..k+3], zeros past dim): pre = x * inv and post = pre *
// gamma in fp64, each rounded once to float. With `store`, the elements below dim go to
// pre_row / post_row (one 16-byte store each when `vec_out` and all four are inside). Returns
// post (zeros past dim).
__device__ __forceinline__ float4 rms_apply4(float4 v, int k, int dim, double inv, const double* gamma,
                                             float* pre_row, float* post_row, bool store, bool vec_out) {
  float4 p, q;
  float* pv = &p.x;
  float* qv = &q.x;
  const float* xv = &v.x;
  if (k + 3 < dim) {
    // gamma + k is 32-byte aligned (k is a multiple of 4, gamma comes from cudaMalloc)
    const double2 g01 = *reinterpret_cast<const double2*>(gamma + k);
    const double2 g23 = *reinterpret_cast<const double2*>(gamma + k + 2);
    const double g[4] = {g01.x, g01.y, g23.x, g23.y};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const double xh = static_cast<double>(xv[j]) * inv;
      pv[j] = static_cast<float>(xh);
      qv[j] = static_cast<float>(xh * g[j]);
    }
    if (store) {
      if (vec_out) {
        *reinterpret_cast<float4*>(pre_row + k) = p;
        *reinterpret_cast<float4*>(post_row + k) = q;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          pre_row[k + j] = pv[j];
          post_row[k + j] = qv[j];
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      pv[j] = 0.0f;
      qv[j] = 0.0f;
      if (k + j < dim) {
        const double xh = static_cast<double>(xv[j]) * inv;
        pv[j] = static_cast<float>(xh);
        qv[j] = static_cast<float>(xh * gamma[k + j]);
        if (store) {
          pre_row[k + j] = pv[j];
          post_row[k + j] = qv[j];
        }
      }
    }
  }
  return q;
}

} // namespace wb
