// codec.cuh -- device-side FormatNone codecs for the quantized Dense path.
//
// Encoders are bit-for-bit restatements of the reference's host codecs as integer/fp32
// device code (no cvt.satfinite / __nv_fp8 conversions: those round to nearest-even and
// saturate differently):
//   E4M3  src/core/float_codecs.cpp:57-97    E5M2  :119-158    FP4 (E2M1)  :184-198
// Reference-semantics decoders (:99-117, :160-181, :200) are used for exports and tests.
//
// The GEMV/GEMM kernels decode with the hardware e2m1/e4m3/e5m2 -> f16x2 converters. Those
// agree with the reference decode on every code once the device mirror has been
// canonicalised (canon_e4m3 / canon_e5m2): the reference decodes FP8 subnormal codes to a
// signed zero (float_codecs.cpp:106-111, :167-172) and E4M3 0x7f/0xff to +-448 (:112-114),
// where the hardware would produce subnormals and NaN.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace wb {

__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// ---------------------------------------------------------------- loads after griddepcontrol.wait
//
// A kernel launched as a programmatic dependent starts while the kernel before it still runs
// and reads that kernel's outputs (x, prepared fragments) only after griddepcontrol.wait. The
// read-only __ldg path tells the compiler the data never changes during the kernel, so it may
// move such loads above the wait; these loads are volatile asm, kept in program order after it.
__device__ __forceinline__ float ld_dep(const float* p) {
  float v;
  asm volatile("ld.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ld_dep4(const float* p) {  // 16-byte aligned
  float4 v;
  asm volatile("ld.global.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_dep4u(const void* p) {  // 16-byte aligned
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// ---------------------------------------------------------------- encoders (bit exact)

__device__ __forceinline__ uint8_t enc_e4m3(float f) {
  if (f == 0.0f || isnan(f)) return 0;
  uint32_t sign = 0;
  if (f < 0.0f) { sign = 0x80; f = -f; }
  if (f > 448.0f) return static_cast<uint8_t>(sign | 0x7e);
  const uint32_t bits = f2u(f);
  const int ex = static_cast<int>((bits >> 23) & 0xff) - 127;
  uint32_t mant = bits & 0x7fffff;
  int e = ex + 7;
  if (e <= 0) {
    if (e < -2) return static_cast<uint8_t>(sign);
    mant |= 0x800000;
    const uint32_t m = mant >> static_cast<unsigned>(21 - e);  // 1 - e + 20
    return static_cast<uint8_t>(sign | (m & 0x7));
  }
  if (e >= 15) return static_cast<uint8_t>(sign | 0x7e);
  uint32_t m = (mant >> 20) & 0x7;
  if (mant & 0x80000) {  // half-up on the first dropped bit
    if (++m == 8) {
      m = 0;
      if (++e >= 15) return static_cast<uint8_t>(sign | 0x7e);
    }
  }
  return static_cast<uint8_t>(sign | (static_cast<uint32_t>(e) << 3) | m);
}

__device__ __forceinline__ uint8_t enc_e5m2(float f) {
  if (isnan(f)) return 0x7e;
  uint32_t sign = 0;
  if (f < 0.0f || signbit(f)) {
    sign = 0x80;
    if (f < 0.0f) f = -f;
  }
  if (isinf(f)) return static_cast<uint8_t>(sign | 0x7c);
  if (f == 0.0f) return static_cast<uint8_t>(sign);
  const uint32_t bits = f2u(f);
  const int ex = static_cast<int>((bits >> 23) & 0xff) - 127;
  const uint32_t mant = bits & 0x7fffff;
  int e = ex + 15;
  if (e <= 0) return static_cast<uint8_t>(sign);
  if (e >= 31) return static_cast<uint8_t>(sign | 0x7c);
  uint32_t m = (mant >> 21) & 0x3;
  if (mant & 0x100000) {
    if (++m == 4) {
      m = 0;
      if (++e >= 31) return static_cast<uint8_t>(sign | 0x7c);
    }
  }
  return static_cast<uint8_t>(sign | (static_cast<uint32_t>(e) << 2) | m);
}

// Nearest of the 16 E2M1 values by |f - v| evaluated in float, strict '<' (ties keep the
// lower code); NaN/Inf never beat FLT_MAX and give code 0.
__device__ __forceinline__ uint8_t enc_fp4(float f) {
  const float v[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                       -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};
  uint32_t best = 0;
  float best_err = 3.402823466e+38f;
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    const float e = fabsf(__fsub_rn(f, v[c]));
    if (e < best_err) {
      best_err = e;
      best = static_cast<uint32_t>(c);
    }
  }
  return static_cast<uint8_t>(best);
}

// Int8 quantisation of one weight with the per-tensor scale s
// (src/weights/native_codec.cpp:252-262): q = clamp(roundf(w / s), -128, 127). A NaN
// quotient converts to 0, as the reference's x86-64 build stores.
__device__ __forceinline__ uint8_t enc_i8(float w, float s) {
  const float r = roundf(__fdiv_rn(w, s));
  double d = static_cast<double>(r);
  if (d < -128.0) d = -128.0;
  if (d > 127.0) d = 127.0;
  const int q = isnan(r) ? 0 : static_cast<int>(d);
  return static_cast<uint8_t>(static_cast<int8_t>(q));
}

// ---------------------------------------------------------------- reference decoders

__device__ __forceinline__ float dec_e4m3_ref(uint32_t b) {
  const uint32_t sign = (b & 0x80) ? 0x80000000u : 0u;
  const uint32_t e = (b >> 3) & 0xf, m = b & 0x7;
  if (e == 0) return u2f(sign);  // subnormal codes: (+-0) * m / 8 / 64 = +-0
  if (e == 15 && m == 7) return u2f(sign | 0x43e00000u);  // +-448
  return u2f(sign | ((e - 7 + 127) << 23) | (m << 20));
}

__device__ __forceinline__ float dec_e5m2_ref(uint32_t b) {
  const uint32_t sign = (b & 0x80) ? 0x80000000u : 0u;
  const uint32_t e = (b >> 2) & 0x1f, m = b & 0x3;
  if (e == 0) return u2f(sign);
  if (e == 31) return u2f(sign | (m == 0 ? 0x7f800000u : 0x7fc00000u));
  return u2f(sign | ((e - 15 + 127) << 23) | (m << 21));
}

__device__ __forceinline__ float dec_fp4_ref(uint32_t c) {
  // E2M1 magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}; bit 3 is the sign (code 8 = -0).
  const uint32_t mag = c & 7;
  const uint32_t e = mag >> 1, m = mag & 1;
  uint32_t bits;
  if (e == 0) bits = m ? 0x3f000000u : 0u;
  else bits = ((e + 126) << 23) | (m << 22);
  return u2f(bits | ((c & 8) ? 0x80000000u : 0u));
}

// ---------------------------------------------------------------- canonical device codes

// Map reference codes onto codes whose hardware decode equals the reference decode.
__device__ __forceinline__ uint8_t canon_e4m3(uint32_t b) {
  if ((b & 0x78) == 0) return static_cast<uint8_t>(b & 0x80);     // subnormal -> signed zero
  if ((b & 0x7f) == 0x7f) return static_cast<uint8_t>(b & 0xfe);  // 0x7f/0xff -> +-448
  return static_cast<uint8_t>(b);
}

__device__ __forceinline__ uint8_t canon_e5m2(uint32_t b) {
  if ((b & 0x7c) == 0) return static_cast<uint8_t>(b & 0x80);     // subnormal -> signed zero
  return static_cast<uint8_t>(b);
}

// ---------------------------------------------------------------- vector decoders (hot path)

// 8 E2M1 codes (low nibble first) -> 8 floats, via the hardware e2m1x2 -> f16x2 converter.
__device__ __forceinline__ void dec_fp4x8(uint32_t w, float* f) {
  uint32_t h0, h1, h2, h3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
      : "r"(w));
  float2 a = __half22float2(*reinterpret_cast<__half2*>(&h0));
  float2 b = __half22float2(*reinterpret_cast<__half2*>(&h1));
  float2 c = __half22float2(*reinterpret_cast<__half2*>(&h2));
  float2 d = __half22float2(*reinterpret_cast<__half2*>(&h3));
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

// 4 canonical E4M3 codes (lowest byte first) -> 4 floats.
__device__ __forceinline__ void dec_e4m3x4(uint32_t w, float* f) {
  uint32_t h0, h1;
  asm("{\n\t.reg .b16 lo, hi;\n\t"
      "mov.b32 {lo, hi}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, lo;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, hi;\n\t}"
      : "=r"(h0), "=r"(h1)
      : "r"(w));
  float2 a = __half22float2(*reinterpret_cast<__half2*>(&h0));
  float2 b = __half22float2(*reinterpret_cast<__half2*>(&h1));
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}

// 4 canonical E5M2 codes -> 4 floats.
__device__ __forceinline__ void dec_e5m2x4(uint32_t w, float* f) {
  uint32_t h0, h1;
  asm("{\n\t.reg .b16 lo, hi;\n\t"
      "mov.b32 {lo, hi}, %2;\n\t"
      "cvt.rn.f16x2.e5m2x2 %0, lo;\n\t"
      "cvt.rn.f16x2.e5m2x2 %1, hi;\n\t}"
      : "=r"(h0), "=r"(h1)
      : "r"(w));
  float2 a = __half22float2(*reinterpret_cast<__half2*>(&h0));
  float2 b = __half22float2(*reinterpret_cast<__half2*>(&h1));
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}

// 4 int8 codes -> 4 exact floats: byte ^ 0x80 placed in the mantissa of 2^23, minus 2^23+128.
__device__ __forceinline__ void dec_i8x4(uint32_t w, float* f) {
  const uint32_t u = w ^ 0x80808080u;
  f[0] = u2f(__byte_perm(u, 0x4b000000u, 0x7440)) - 8388736.0f;
  f[1] = u2f(__byte_perm(u, 0x4b000000u, 0x7441)) - 8388736.0f;
  f[2] = u2f(__byte_perm(u, 0x4b000000u, 0x7442)) - 8388736.0f;
  f[3] = u2f(__byte_perm(u, 0x4b000000u, 0x7443)) - 8388736.0f;
}

// The transcendental activations, out of line: inlined into unrolled epilogues they made the
// code of a 16-output step large enough to stall on instruction fetch.
static __device__ __noinline__ double activate_transcendental(int act, double x) {
  switch (act) {
  case 1: return x / (1.0 + exp(-x));
  case 2: {
    const double k = 0.7978845608028654;
    return 0.5 * x * (1.0 + tanh(k * (x + 0.044715 * x * x * x)));
  }
  case 3: return tanh(x);
  case 4: return 1.0 / (1.0 + exp(-x));
  default: return x;
  }
}

// Activation in float64 (the reference's activate_dev, src/cuda/kernels.cu:22-46), calling
// CUDA's double exp/tanh exactly as the reference does.
__device__ __forceinline__ double activate(int act, double x) {
  switch (act) {
  case -1: return x;
  case 0: return x < 0.0 ? 0.0 : x;
  case 6: return x < 0.0 ? 0.0 : x * x;
  case 5: return x < 0.0 ? 0.01 * x : x;
  default: return activate_transcendental(act, x);
  }
}

} // namespace wb
