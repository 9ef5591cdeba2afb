// gemv.cu -- fused dequant-GEMV over resident FP8/FP4/Int8/Float32 weights (sm_100a).
//
// Replaces the reference's dense_matvec_f64_batch + dense_bias_act pair
// (src/cuda/kernels.cu:130-161), which reads a host-decoded fp64 copy of W (8 B/weight)
// with one thread per output. Here the GPU streams the packed codes (0.5 B/weight FP4,
// 1 B/weight FP8/Int8) once, decodes in registers and fuses bias/activation (or the SwiGLU
// product, src/cuda/kernels.cu:296-305) into the epilogue.
//
// Work split: a warp owns kRows consecutive output rows; its lanes stride the row in 16-byte
// vectors (coalesced 512 B per warp-load, ld.global.nc.L1::no_allocate). Each vector's
// products are accumulated in fp32 (16 or 32 products), then added to an fp64 accumulator;
// lanes are combined with an fp64 butterfly. Error vs the reference's sequential fp64 sum:
// at most ~2^-21 * sum_k |W x| before the final rounding to float (exact fp32 products for
// FP8/FP4, whose values carry <= 4 significant bits).
//
// Programmatic dependent launch: the weights of this layer do not depend on the previous
// kernel, so thread 0 prefetches the CTA's first rows into L2 (cp.async.bulk.prefetch.L2)
// before griddepcontrol.wait; x is read and outputs are written only after the wait.
#include "gemv.hpp"
#include "codec.cuh"

namespace wb {
namespace {

constexpr int kWarps = 8;   // warps per CTA
constexpr int kRows = 4;    // rows per warp group
constexpr int kUnroll = 2;  // 16-byte vectors in flight per lane per row

__device__ __forceinline__ uint4 ld_stream(const uint8_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int j) {
  return j == 0 ? v.x : (j == 1 ? v.y : (j == 2 ? v.z : v.w));
}

template <int kDt>
struct Geo {
  static constexpr int EPW = kDt == 16 ? 8 : 4;     // elements per 32-bit word
  static constexpr int EPV = kDt == 16 ? 32 : (kDt == 1 ? 4 : 16);  // per 16 bytes
};

template <int kDt>
__device__ __forceinline__ void decode_word(uint32_t w, float* f) {
  if constexpr (kDt == 16) dec_fp4x8(w, f);
  else if constexpr (kDt == 4) dec_e4m3x4(w, f);
  else if constexpr (kDt == 5) dec_e5m2x4(w, f);
  else dec_i8x4(w, f);
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Products of one 16-byte weight vector (per row) with the matching x slice, accumulated in
// fp32 into part[r][b].
template <int kDt, int kB>
__device__ __forceinline__ void dot_vector(const uint4 (&wv)[kRows], const float* __restrict__ xv,
                                           int64_t xs, float (&part)[kRows][kB]) {
  if constexpr (kDt == 1) {
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      const float4 xq = ld_dep4(xv + b * xs);
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        float p = part[r][b];
        p = fmaf(__uint_as_float(wv[r].x), xq.x, p);
        p = fmaf(__uint_as_float(wv[r].y), xq.y, p);
        p = fmaf(__uint_as_float(wv[r].z), xq.z, p);
        p = fmaf(__uint_as_float(wv[r].w), xq.w, p);
        part[r][b] = p;
      }
    }
  } else {
    constexpr int EPW = Geo<kDt>::EPW;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float wf[kRows][EPW];
#pragma unroll
      for (int r = 0; r < kRows; ++r) decode_word<kDt>(word_of(wv[r], j), wf[r]);
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        float x[EPW];
        const float* xp = xv + b * xs + j * EPW;
#pragma unroll
        for (int q = 0; q < EPW / 4; ++q) {
          const float4 t = ld_dep4(xp + 4 * q);
          x[4 * q + 0] = t.x; x[4 * q + 1] = t.y; x[4 * q + 2] = t.z; x[4 * q + 3] = t.w;
        }
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          float p = part[r][b];
#pragma unroll
          for (int e = 0; e < EPW; ++e) p = fmaf(wf[r][e], x[e], p);
          part[r][b] = p;
        }
      }
    }
  }
}

// Exact variant: every product is formed and accumulated in fp64 (products of the decoded
// weight and x are exact in fp64), in increasing k within a lane; Int8 weights are
// dequantized first as the reference does, float(q) * scale in fp32
// (src/weights/native_codec.cpp:565-568). Used for small, latency-bound layers.
template <int kDt, int kB>
__device__ __forceinline__ void dot_vector_exact(const uint4 (&wv)[kRows], const float* __restrict__ xv,
                                                 int64_t xs, float wscale, double (&acc)[kRows][kB]) {
  if constexpr (kDt == 1) {
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      const float4 xq = ld_dep4(xv + b * xs);
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        double p = acc[r][b];
        p = fma(static_cast<double>(__uint_as_float(wv[r].x)), static_cast<double>(xq.x), p);
        p = fma(static_cast<double>(__uint_as_float(wv[r].y)), static_cast<double>(xq.y), p);
        p = fma(static_cast<double>(__uint_as_float(wv[r].z)), static_cast<double>(xq.z), p);
        p = fma(static_cast<double>(__uint_as_float(wv[r].w)), static_cast<double>(xq.w), p);
        acc[r][b] = p;
      }
    }
  } else {
    constexpr int EPW = Geo<kDt>::EPW;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float wf[kRows][EPW];
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        decode_word<kDt>(word_of(wv[r], j), wf[r]);
        if (kDt == 9) {
#pragma unroll
          for (int e = 0; e < EPW; ++e) wf[r][e] = __fmul_rn(wf[r][e], wscale);
        }
      }
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        float x[EPW];
        const float* xp = xv + b * xs + j * EPW;
#pragma unroll
        for (int q = 0; q < EPW / 4; ++q) {
          const float4 t = ld_dep4(xp + 4 * q);
          x[4 * q + 0] = t.x; x[4 * q + 1] = t.y; x[4 * q + 2] = t.z; x[4 * q + 3] = t.w;
        }
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          double p = acc[r][b];
#pragma unroll
          for (int e = 0; e < EPW; ++e) p = fma(static_cast<double>(wf[r][e]), static_cast<double>(x[e]), p);
          acc[r][b] = p;
        }
      }
    }
  }
}

template <int kDt, int kB, bool kDual, bool kExact>
__global__ void __launch_bounds__(kWarps * 32) k_gemv(const GemvArgs a) {
  constexpr int EPV = Geo<kDt>::EPV;
  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t nvec = a.row_stride >> 4;
  const int ngroups = (a.rows + kRows - 1) / kRows;

  if (threadIdx.x == 0) {
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kWarps * kRows;
    if (r0 < a.rows) {
      int64_t nr = a.rows - r0;
      if (nr > kWarps * kRows) nr = kWarps * kRows;
      int64_t bytes = nr * a.row_stride;
      if (bytes > (1 << 20)) bytes = 1 << 20;
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.W + r0 * a.row_stride),
                   "r"(static_cast<uint32_t>(bytes))
                   : "memory");
      if (kDual)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.W2 + r0 * a.row_stride),
                     "r"(static_cast<uint32_t>(bytes))
                     : "memory");
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");

  for (int g = blockIdx.x * kWarps + warp; g < ngroups; g += gridDim.x * kWarps) {
    const int r0 = g * kRows;
    const uint8_t* wrow[kRows];
    const uint8_t* wrow2[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const int row = min(r0 + r, a.rows - 1);
      wrow[r] = a.W + static_cast<int64_t>(row) * a.row_stride;
      wrow2[r] = kDual ? a.W2 + static_cast<int64_t>(row) * a.row_stride : nullptr;
    }
    double acc[kRows][kB];
    double acc2[kRows][kB];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int b = 0; b < kB; ++b) acc[r][b] = acc2[r][b] = 0.0;

    for (int64_t v0 = lane; v0 < nvec; v0 += 32 * kUnroll) {
      uint4 wv[kUnroll][kRows];
      uint4 wv2[kUnroll][kRows];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t v = v0 + 32 * u;
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          wv[u][r] = v < nvec ? ld_stream(wrow[r] + v * 16) : make_uint4(0, 0, 0, 0);
          if (kDual) wv2[u][r] = v < nvec ? ld_stream(wrow2[r] + v * 16) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t v = v0 + 32 * u;
        if (v < nvec) {
          const float* xv = a.x + v * EPV;
          if constexpr (kExact) {
            dot_vector_exact<kDt, kB>(wv[u], xv, a.x_stride, a.scale, acc);
            if (kDual) dot_vector_exact<kDt, kB>(wv2[u], xv, a.x_stride, a.scale2, acc2);
          } else {
            float part[kRows][kB];
#pragma unroll
            for (int r = 0; r < kRows; ++r)
#pragma unroll
              for (int b = 0; b < kB; ++b) part[r][b] = 0.0f;
            dot_vector<kDt, kB>(wv[u], xv, a.x_stride, part);
#pragma unroll
            for (int r = 0; r < kRows; ++r)
#pragma unroll
              for (int b = 0; b < kB; ++b) acc[r][b] += static_cast<double>(part[r][b]);
            if (kDual) {
#pragma unroll
              for (int r = 0; r < kRows; ++r)
#pragma unroll
                for (int b = 0; b < kB; ++b) part[r][b] = 0.0f;
              dot_vector<kDt, kB>(wv2[u], xv, a.x_stride, part);
#pragma unroll
              for (int r = 0; r < kRows; ++r)
#pragma unroll
                for (int b = 0; b < kB; ++b) acc2[r][b] += static_cast<double>(part[r][b]);
            }
          }
        }
      }
    }

#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        acc[r][b] = warp_sum(acc[r][b]);
        if (kDual) acc2[r][b] = warp_sum(acc2[r][b]);
      }

#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        const int o = r0 + r;
        if (lane == r * kB + b && o < a.rows) {
          const int64_t idx = static_cast<int64_t>(b) * a.ld_out + o;
          double sum = acc[r][b];
          if (kDt == 9 && !kExact) sum *= static_cast<double>(a.scale);
          if (!kDual) {
            // src/cuda/kernels.cu:141-160: pre = float(sum); v = double(pre) (+ bias, then
            // pre = float(v)); post = float(act(v)).
            float pre = static_cast<float>(sum);
            double v = static_cast<double>(pre);
            if (a.bias != nullptr && o < a.bias_len) {
              v += a.bias[o];
              pre = static_cast<float>(v);
            }
            a.pre[idx] = pre;
            const float post = static_cast<float>(activate(a.act, v));
            a.post[idx] = post;
#pragma unroll
            for (int i = 0; i < kMaxPeerOut; ++i)  // static indices: the parameter stays in registers
              if (i < a.peers.n) a.peers.post[i][idx] = post;
          } else {
            double up = acc2[r][b];
            if (kDt == 9 && !kExact) up *= static_cast<double>(a.scale2);
            // Gate/Up are Linear without bias: gate_pre = float(sum), up_post = float(sum);
            // h = float(double(float(SiLU(double(gate_pre)))) * double(up_post)).
            const float gate_pre = static_cast<float>(sum);
            const float up_post = static_cast<float>(up);
            const float g = static_cast<float>(activate(1, static_cast<double>(gate_pre)));
            a.pre[idx] = static_cast<float>(static_cast<double>(g) * static_cast<double>(up_post));
          }
        }
      }
  }
}

template <int kDt, int kB, bool kDual, bool kExact>
Status launch_t(const GemvArgs& a, cudaStream_t st, bool pdl) {
  const int ngroups = (a.rows + kRows - 1) / kRows;
  int grid = (ngroups + kWarps - 1) / kWarps;
  if (grid > 148 * 64) grid = 148 * 64;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, k_gemv<kDt, kB, kDual, kExact>, a), "gemv launch");
}

template <int kDt, bool kDual, bool kExact>
Status launch_e(const GemvArgs& a, cudaStream_t st, bool pdl) {
  switch (a.batch) {
  case 1: return launch_t<kDt, 1, kDual, kExact>(a, st, pdl);
  case 2: return launch_t<kDt, 2, kDual, kExact>(a, st, pdl);
  case 3: return launch_t<kDt, 3, kDual, kExact>(a, st, pdl);
  case 4: return launch_t<kDt, 4, kDual, kExact>(a, st, pdl);
  default: return Status::Internal("gemv: batch chunk must be 1..4");
  }
}

template <int kDt, bool kDual>
Status launch_b(const GemvArgs& a, cudaStream_t st, bool pdl) {
  return a.exact ? launch_e<kDt, kDual, true>(a, st, pdl) : launch_e<kDt, kDual, false>(a, st, pdl);
}

template <bool kDual>
Status launch_d(const GemvArgs& a, cudaStream_t st, bool pdl) {
  switch (a.dtype) {
  case DType::FP4: return launch_b<16, kDual>(a, st, pdl);
  case DType::FP8E4M3: return launch_b<4, kDual>(a, st, pdl);
  case DType::FP8E5M2: return launch_b<5, kDual>(a, st, pdl);
  case DType::Int8: return launch_b<9, kDual>(a, st, pdl);
  case DType::Float32: return launch_b<1, kDual>(a, st, pdl);
  }
  return Status::Unsupported("gemv: dtype");
}

} // namespace

namespace {
__global__ void __launch_bounds__(256) k_stage_rows(float* __restrict__ dst, int64_t dst_ld,
                                                    const float* __restrict__ src, int64_t src_ld, int cols,
                                                    int rows, bool vec) {
  asm volatile("griddepcontrol.launch_dependents;");
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (vec) {  // 16-byte rows: cols, both leading dimensions and both bases multiples of 4 floats
    const int c4 = cols >> 2;
    const int64_t n = static_cast<int64_t>(rows) * c4;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
      const int64_t r = i / c4, c = (i - r * c4) << 2;
      *reinterpret_cast<float4*>(dst + r * dst_ld + c) = *reinterpret_cast<const float4*>(src + r * src_ld + c);
    }
  } else {
    const int64_t n = static_cast<int64_t>(rows) * cols;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
      const int64_t r = i / cols, c = i - r * cols;
      dst[r * dst_ld + c] = src[r * src_ld + c];
    }
  }
}
} // namespace

Status launch_stage_rows(float* dst, int64_t dst_ld, const float* src, int64_t src_ld, int cols, int rows,
                         cudaStream_t st) {
  if (!dst || !src || cols <= 0 || rows <= 0 || dst_ld < cols || src_ld < cols)
    return Status::Invalid("stage rows: bad arguments");
  const bool vec = (cols & 3) == 0 && (dst_ld & 3) == 0 && (src_ld & 3) == 0 &&
                   ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0;
  const int64_t units = static_cast<int64_t>(rows) * (vec ? cols / 4 : cols);
  int64_t blocks = (units + 255) / 256;
  if (blocks > 4 * 148) blocks = 4 * 148;
  k_stage_rows<<<static_cast<int>(blocks), 256, 0, st>>>(dst, dst_ld, src, src_ld, cols, rows, vec);
  return cuda_status(cudaGetLastError(), "stage rows launch");
}

Status launch_gemv(const GemvArgs& a, cudaStream_t st, bool pdl) {
  if (a.rows <= 0 || a.cols <= 0 || a.batch <= 0) return Status::Invalid("gemv: bad dims");
  if (a.row_stride % 16 != 0) return Status::Internal("gemv: row stride must be a multiple of 16");
  if (a.x_stride % 4 != 0 || (reinterpret_cast<uintptr_t>(a.x) & 15) != 0)
    return Status::Internal("gemv: x must be 16-byte aligned with a stride that is a multiple of 4");
  if (a.x_stride < (a.row_stride / 16) * elems_per_16B(a.dtype))
    return Status::Internal("gemv: x stride shorter than the padded row");
  // Batches above 4 run in chunks of up to 4 columns (each chunk re-streams W).
  for (int b0 = 0; b0 < a.batch; b0 += 4) {
    GemvArgs c = a;
    c.batch = a.batch - b0 < 4 ? a.batch - b0 : 4;
    c.x = a.x + static_cast<int64_t>(b0) * a.x_stride;
    c.pre = a.pre + static_cast<int64_t>(b0) * a.ld_out;
    c.post = a.post ? a.post + static_cast<int64_t>(b0) * a.ld_out : nullptr;
    WB_TRY(a.W2 ? launch_d<true>(c, st, pdl) : launch_d<false>(c, st, pdl));
  }
  return Status::Ok();
}

} // namespace wb
