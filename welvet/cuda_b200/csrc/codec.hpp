// codec.hpp -- host launchers of the codec kernels (codec.cu).
#pragma once

#include "common.hpp"

namespace wb {

// FormatNone encode of n float32 weights on the device into reference-layout native bytes
// (FP8: 1 B/elt; FP4: (n+1)/2 B, low nibble = even flat index; Int8: 1 B/elt) and the
// per-tensor scale (1 for FP8/FP4, absmax/127 for Int8). Float32 copies the payload.
// absmax_scratch: one device uint (Int8 only).
Status encode_native(DType dt, const float* w_dev, int64_t n, uint8_t* native_dev, float* scale_dev,
                     unsigned int* absmax_scratch, cudaStream_t st);

// Device mirror from reference-layout bytes: rows padded to row_stride bytes (multiple of
// 16), FP4 rows nibble-realigned, FP8 codes canonicalised, padding = code 0.
Status build_mirror(DType dt, const uint8_t* native_dev, int64_t rows, int64_t cols,
                    int64_t row_stride, uint8_t* mirror_dev, cudaStream_t st);

// Reference-semantics decode (weight_at) of n elements to float32.
Status decode_ref(DType dt, const uint8_t* native_dev, int64_t n, float scale, float* out_dev,
                  cudaStream_t st);

// Exhaustive-encode digest over float32 bit patterns [start, start+count).
Status encode_digest(int codec, uint64_t start, uint64_t count, unsigned long long* out_dev,
                     cudaStream_t st);

// All codes through the GEMV vector decoders (FP4: 512 floats, others 256).
Status selftest_decode(DType dt, float* out_dev, cudaStream_t st);

} // namespace wb
