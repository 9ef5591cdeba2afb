// codec.cu -- sm_100a codec kernels: FormatNone encode (bit exact with the reference),
// the device mirror build (row padding + canonical codes), reference-semantics decode,
// and the exhaustive-encode digest used by the parity tests.
//
// Reference behaviour restated: src/weights/native_codec.cpp:174-262 (pack_native for
// FP8E4M3/FP8E5M2/FP4/Int8; FP4 low nibble = even flat index; Int8 s = absmax/127 with
// s == 0 -> 1), :513-568 (weight_at), src/core/float_codecs.cpp:57-200.
#include "codec.hpp"
#include "codec.cuh"

namespace wb {
namespace {

constexpr int kThreads = 256;

inline int grid_for(int64_t n, int per_thread = 1) {
  int64_t blocks = (n + static_cast<int64_t>(kThreads) * per_thread - 1) /
                   (static_cast<int64_t>(kThreads) * per_thread);
  if (blocks < 1) blocks = 1;
  if (blocks > 148 * 32) blocks = 148 * 32;
  return static_cast<int>(blocks);
}

// E4M3 / E5M2: one code per element.
template <int kCodec>
__global__ void k_encode_fp8(const float* __restrict__ w, int64_t n, uint8_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    out[i] = kCodec == 0 ? enc_e4m3(w[i]) : enc_e5m2(w[i]);
  }
}

// FP4: one output byte per thread, low nibble = even flat index; an odd tail byte keeps a
// zero high nibble (the reference zero-fills before packing).
__global__ void k_encode_fp4(const float* __restrict__ w, int64_t n, uint8_t* __restrict__ out) {
  const int64_t nb = (n + 1) / 2;
  for (int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; j < nb;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint32_t b = enc_fp4(w[2 * j]) & 0xF;
    if (2 * j + 1 < n) b |= static_cast<uint32_t>(enc_fp4(w[2 * j + 1]) & 0xF) << 4;
    out[j] = static_cast<uint8_t>(b);
  }
}

// max |w| over non-NaN elements ('a > m' never admits a NaN). Non-negative floats order
// like their bit patterns, so an integer atomicMax on the bits is exact and order-free.
__global__ void k_absmax(const float* __restrict__ w, int64_t n, unsigned int* __restrict__ out_bits) {
  float m = 0.0f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float a = fabsf(w[i]);
    if (a > m) m = a;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, m, o);
    if (t > m) m = t;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(out_bits, __float_as_uint(m));
}

// Int8 codes with s = absmax / 127 (s == 0 -> 1); thread 0 of block 0 also stores s.
__global__ void k_encode_i8(const float* __restrict__ w, int64_t n,
                            const unsigned int* __restrict__ absmax_bits, uint8_t* __restrict__ out,
                            float* __restrict__ scale_out) {
  float s = __fdiv_rn(__uint_as_float(*absmax_bits), 127.0f);
  if (s == 0.0f) s = 1.0f;
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = s;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    out[i] = enc_i8(w[i], s);
  }
}

__global__ void k_set_scale_one(float* scale_out) { *scale_out = 1.0f; }

// Device mirror: row o occupies [o*row_stride, (o+1)*row_stride), codes canonical, pad = 0.
// One thread per mirror byte (per 4-byte word for Float32).
template <int kDt>
__global__ void k_build_mirror(const uint8_t* __restrict__ native, int64_t rows, int64_t cols,
                               int64_t row_stride, uint8_t* __restrict__ mirror) {
  const int64_t total = kDt == 1 ? rows * (row_stride / 4) : rows * row_stride;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (kDt == 1) {  // Float32
      const int64_t words = row_stride / 4;
      const int64_t o = t / words, k = t - o * words;
      const float* src = reinterpret_cast<const float*>(native);
      reinterpret_cast<float*>(mirror)[t] = k < cols ? src[o * cols + k] : 0.0f;
      continue;
    }
    const int64_t o = t / row_stride, j = t - o * row_stride;
    uint32_t b = 0;
    if (kDt == 16) {  // FP4: nibble-realign each row (rows start mid-byte when cols is odd)
      const int64_t k0 = 2 * j;
      if (k0 < cols) {
        const int64_t f0 = o * cols + k0;
        b = (native[f0 >> 1] >> ((f0 & 1) * 4)) & 0xF;
        if (k0 + 1 < cols) {
          const int64_t f1 = f0 + 1;
          b |= ((native[f1 >> 1] >> ((f1 & 1) * 4)) & 0xF) << 4;
        }
      }
    } else if (j < cols) {
      const uint32_t c = native[o * cols + j];
      b = kDt == 4 ? canon_e4m3(c) : (kDt == 5 ? canon_e5m2(c) : c);
    }
    mirror[t] = static_cast<uint8_t>(b);
  }
}

// Reference-semantics decode (weight_at) of n elements to float.
__global__ void k_decode_ref(int dt, const uint8_t* __restrict__ native, int64_t n, float scale,
                             float* __restrict__ out) {
  if (scale == 0.0f) scale = 1.0f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v;
    switch (dt) {
    case 4: v = dec_e4m3_ref(native[i]); break;
    case 5: v = dec_e5m2_ref(native[i]); break;
    case 16: v = dec_fp4_ref((native[i >> 1] >> ((i & 1) * 4)) & 0xF); break;
    case 9: v = static_cast<float>(static_cast<int8_t>(native[i])) * scale; break;
    default: v = reinterpret_cast<const float*>(native)[i]; break;
    }
    out[i] = v;
  }
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// sum over bit patterns i in [start, start+count) of mix64((i << 8) | encode(i)).
__global__ void k_encode_digest(int codec, uint64_t start, uint64_t count,
                                unsigned long long* __restrict__ out) {
  uint64_t s = 0;
  for (uint64_t t = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; t < count;
       t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t i = start + t;
    const float f = __uint_as_float(static_cast<uint32_t>(i));
    const uint32_t c = codec == 0 ? enc_e4m3(f) : (codec == 1 ? enc_e5m2(f) : enc_fp4(f));
    s += mix64((i << 8) | c);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(out, static_cast<unsigned long long>(s));
}

// Decode every code through the hot-path vector decoders (after canonicalisation), so the
// tests can check the hardware converters' lane order and values against the reference.
//   FP4: out[512] for the 256 bytes (low nibble first)   FP8/Int8: out[256]
__global__ void k_selftest_decode(int dt, float* __restrict__ out) {
  const uint32_t t = threadIdx.x;  // 64 threads, 4 bytes each
  uint32_t w = 0;
  for (int i = 0; i < 4; ++i) {
    uint32_t c = 4 * t + i;
    if (dt == 4) c = canon_e4m3(c);
    if (dt == 5) c = canon_e5m2(c);
    w |= c << (8 * i);
  }
  float f[8];
  if (dt == 16) {
    dec_fp4x8(w, f);
    for (int i = 0; i < 8; ++i) out[8 * t + i] = f[i];
  } else {
    if (dt == 4) dec_e4m3x4(w, f);
    else if (dt == 5) dec_e5m2x4(w, f);
    else dec_i8x4(w, f);
    for (int i = 0; i < 4; ++i) out[4 * t + i] = f[i];
  }
}

} // namespace

Status encode_native(DType dt, const float* w, int64_t n, uint8_t* native, float* scale_dev,
                     unsigned int* absmax_scratch, cudaStream_t st) {
  if (n <= 0) return Status::Invalid("encode: empty");
  switch (dt) {
  case DType::FP8E4M3:
    k_encode_fp8<0><<<grid_for(n, 4), kThreads, 0, st>>>(w, n, native);
    break;
  case DType::FP8E5M2:
    k_encode_fp8<1><<<grid_for(n, 4), kThreads, 0, st>>>(w, n, native);
    break;
  case DType::FP4:
    k_encode_fp4<<<grid_for((n + 1) / 2, 2), kThreads, 0, st>>>(w, n, native);
    break;
  case DType::Int8:
    WB_CUDA(cudaMemsetAsync(absmax_scratch, 0, sizeof(unsigned int), st));
    k_absmax<<<grid_for(n, 8), kThreads, 0, st>>>(w, n, absmax_scratch);
    WB_CUDA(cudaGetLastError());
    k_encode_i8<<<grid_for(n, 4), kThreads, 0, st>>>(w, n, absmax_scratch, native, scale_dev);
    WB_CUDA(cudaGetLastError());
    return Status::Ok();
  case DType::Float32:
    WB_CUDA(cudaMemcpyAsync(native, w, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToDevice, st));
    break;
  default:
    return Status::Unsupported("encode: dtype not on the quantized Dense path");
  }
  WB_CUDA(cudaGetLastError());
  k_set_scale_one<<<1, 1, 0, st>>>(scale_dev);
  return cuda_status(cudaGetLastError(), "encode launch");
}

Status build_mirror(DType dt, const uint8_t* native, int64_t rows, int64_t cols, int64_t row_stride,
                    uint8_t* mirror, cudaStream_t st) {
  const int64_t total = dt == DType::Float32 ? rows * (row_stride / 4) : rows * row_stride;
  const int g = grid_for(total, 4);
  switch (dt) {
  case DType::Float32: k_build_mirror<1><<<g, kThreads, 0, st>>>(native, rows, cols, row_stride, mirror); break;
  case DType::FP8E4M3: k_build_mirror<4><<<g, kThreads, 0, st>>>(native, rows, cols, row_stride, mirror); break;
  case DType::FP8E5M2: k_build_mirror<5><<<g, kThreads, 0, st>>>(native, rows, cols, row_stride, mirror); break;
  case DType::Int8: k_build_mirror<9><<<g, kThreads, 0, st>>>(native, rows, cols, row_stride, mirror); break;
  case DType::FP4: k_build_mirror<16><<<g, kThreads, 0, st>>>(native, rows, cols, row_stride, mirror); break;
  default: return Status::Unsupported("mirror: dtype");
  }
  return cuda_status(cudaGetLastError(), "mirror launch");
}

Status decode_ref(DType dt, const uint8_t* native, int64_t n, float scale, float* out, cudaStream_t st) {
  k_decode_ref<<<grid_for(n, 4), kThreads, 0, st>>>(static_cast<int>(dt), native, n, scale, out);
  return cuda_status(cudaGetLastError(), "decode launch");
}

Status encode_digest(int codec, uint64_t start, uint64_t count, unsigned long long* out_dev,
                     cudaStream_t st) {
  if (codec < 0 || codec > 2) return Status::Invalid("digest: codec must be 0 (e4m3), 1 (e5m2) or 2 (fp4)");
  WB_CUDA(cudaMemsetAsync(out_dev, 0, sizeof(unsigned long long), st));
  k_encode_digest<<<148 * 16, kThreads, 0, st>>>(codec, start, count, out_dev);
  return cuda_status(cudaGetLastError(), "digest launch");
}

Status selftest_decode(DType dt, float* out, cudaStream_t st) {
  k_selftest_decode<<<1, 64, 0, st>>>(static_cast<int>(dt), out);
  return cuda_status(cudaGetLastError(), "selftest launch");
}

} // namespace wb
