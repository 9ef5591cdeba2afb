/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C CPU restatement of welvet.cuda's quantized-weight Dense forward path, used
 * as the parity checker by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference arm. Nothing in the product library links, loads or calls this file.
 *
 * Every function cites the reference file:line it restates (paths relative to the
 * welvet.cuda project root). Floating-point expressions are written in the same order
 * and precision as the reference and this file is compiled with -ffp-contract=off and
 * without -ffast-math, as the reference host code is (CMakeLists.txt:102-110).
 *
 * Pinning: tests/test_oracle.py checks every function here against the reference's own
 * codec compiled from its sources (oracle/_ref, built by oracle/Makefile) and against the
 * committed fixtures in tests/golden/ (generated from that same reference build).
 */
#include <math.h>
#include <float.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

#define OR_EXPORT __attribute__((visibility("default")))

/* DType ids (include/welvet/dtype.hpp:9-44) */
enum { OR_FLOAT32 = 1, OR_FP8E4M3 = 4, OR_FP8E5M2 = 5, OR_INT8 = 9, OR_FP4 = 16 };

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ---------------------------------------------------------------- codecs */

/* src/core/float_codecs.cpp:57-97 -- E4M3 encode: half-up on mantissa bit 19, truncated
 * subnormals, |x| < 2^-9 -> signed zero, NaN and +-0 -> 0x00, exponent >= 15 saturates to
 * 0x7e (448). */
OR_EXPORT uint8_t or_e4m3_encode(float f) {
  if (f == 0.0f || isnan(f)) return 0;
  uint8_t sign = 0;
  if (f < 0) { sign = 0x80; f = -f; }
  if (f > 448.0f) return (uint8_t)(sign | 0x7e);
  const uint32_t bits = f2u(f);
  const int exp = (int)((bits >> 23) & 0xff) - 127;
  uint32_t mant = bits & 0x7fffff;
  int e = exp + 7;
  if (e <= 0) {
    if (e < -2) return sign;
    mant |= 0x800000;
    const unsigned shift = (unsigned)(1 - e + 20);
    const uint32_t m = mant >> shift;
    return (uint8_t)(sign | (m & 0x7));
  }
  if (e >= 15) return (uint8_t)(sign | 0x7e);
  uint32_t m = (mant >> 20) & 0x7;
  if (mant & 0x80000) {
    m++;
    if (m == 8) {
      m = 0;
      e++;
      if (e >= 15) return (uint8_t)(sign | 0x7e);
    }
  }
  return (uint8_t)(sign | (e << 3) | m);
}

/* src/core/float_codecs.cpp:99-117 -- E4M3 decode. Subnormal codes compute
 * (signed zero) * m / 8 / 64 and therefore decode to a signed zero; 0x7f/0xff -> +-448. */
OR_EXPORT float or_e4m3_decode(uint8_t b) {
  const uint32_t sign = (b & 0x80) ? 0x80000000u : 0u;
  const int e = (b >> 3) & 0xf;
  const int m = b & 0x7;
  if (e == 0) {
    if (m == 0) return u2f(sign);
    return u2f(sign) * (float)m / 8.0f / 64.0f;
  }
  if (e == 15 && m == 7) return u2f(sign | f2u(448.0f));
  const uint32_t fexp = (uint32_t)(e - 7 + 127);
  return u2f(sign | (fexp << 23) | ((uint32_t)m << 20));
}

/* src/core/float_codecs.cpp:119-158 -- E5M2 encode: NaN -> 0x7e, +-Inf -> 0x7c|sign,
 * -0 keeps its sign, subnormal results flush to signed zero, half-up rounding. */
OR_EXPORT uint8_t or_e5m2_encode(float f) {
  if (isnan(f)) return 0x7e;
  uint8_t sign = 0;
  if (f < 0 || signbit(f)) {
    sign = 0x80;
    if (f < 0) f = -f;
  }
  if (isinf(f)) return (uint8_t)(sign | 0x7c);
  if (f == 0.0f) return sign;
  const uint32_t bits = f2u(f);
  const int exp = (int)((bits >> 23) & 0xff) - 127;
  const uint32_t mant = bits & 0x7fffff;
  int e = exp + 15;
  if (e <= 0) return sign;
  if (e >= 31) return (uint8_t)(sign | 0x7c);
  uint32_t m = (mant >> 21) & 0x3;
  if (mant & 0x100000) {
    m++;
    if (m == 4) {
      m = 0;
      e++;
      if (e >= 31) return (uint8_t)(sign | 0x7c);
    }
  }
  return (uint8_t)(sign | (e << 2) | m);
}

/* src/core/float_codecs.cpp:160-181 -- E5M2 decode (subnormal codes -> signed zero,
 * e == 31: m == 0 -> +-Inf, else a quiet NaN carrying the sign). */
OR_EXPORT float or_e5m2_decode(uint8_t b) {
  const uint32_t sign = (b & 0x80) ? 0x80000000u : 0u;
  const int e = (b >> 2) & 0x1f;
  const int m = b & 0x3;
  if (e == 0) {
    if (m == 0) return u2f(sign);
    return u2f(sign) * (float)m / 4.0f / 16384.0f;
  }
  if (e == 31) {
    if (m == 0) return u2f(sign | 0x7f800000u);
    return u2f(sign | 0x7fc00000u);
  }
  const uint32_t fexp = (uint32_t)(e - 15 + 127);
  return u2f(sign | (fexp << 23) | ((uint32_t)m << 21));
}

/* src/core/float_codecs.cpp:183-185 -- the 16 E2M1 values, code 8 is -0. */
static const float kFp4[16] = {0, 0.5f, 1, 1.5f, 2, 3, 4, 6, -0.0f, -0.5f, -1, -1.5f, -2, -3, -4, -6};

/* src/core/float_codecs.cpp:187-198 -- nearest of the 16 values by |f - v| computed in
 * float, strict '<' so ties keep the lower index; NaN and +-Inf never beat FLT_MAX and so
 * map to code 0, as do values so large that f - v rounds to f for every v. */
OR_EXPORT uint8_t or_fp4_encode(float f) {
  uint8_t best = 0;
  float best_err = FLT_MAX;
  for (int c = 0; c < 16; ++c) {
    const float e = fabsf(f - kFp4[c]);
    if (e < best_err) {
      best_err = e;
      best = (uint8_t)c;
    }
  }
  return best;
}

/* src/core/float_codecs.cpp:200 */
OR_EXPORT float or_fp4_decode(uint8_t code) { return kFp4[code & 0xf]; }

/* ---------------------------------------------------------------- packing */

/* src/weights/native_codec.cpp:21-28 (abs_max: NaN never wins the '>' test). */
static float abs_max(const float* w, int64_t n) {
  float m = 0;
  for (int64_t i = 0; i < n; ++i) {
    const float a = fabsf(w[i]);
    if (a > m) m = a;
  }
  return m;
}

/* src/weights/native_codec.cpp:38-42 */
static double clamp_i(double v, double lo, double hi) {
  if (v < lo) return lo;
  if (v > hi) return hi;
  return v;
}

/* Packed byte count of a FormatNone store (native_codec.cpp:193-262). */
OR_EXPORT int64_t or_native_bytes(int dtype, int64_t n) {
  switch (dtype) {
  case OR_FP8E4M3: case OR_FP8E5M2: case OR_INT8: return n;
  case OR_FP4: return (n + 1) / 2;
  default: return -1;
  }
}

/* src/weights/native_codec.cpp:174-177 (scale = 1 for every dtype first), :193-211 (FP8,
 * FP4: low nibble = even flat index), :252-262 (Int8: s = absmax/127, q = clamp(round(w/s)))
 * Returns 0 on success, -1 for a dtype outside the quantized Dense path. */
OR_EXPORT int or_pack(int dtype, const float* w, int64_t n, uint8_t* out, float* scale) {
  *scale = 1;
  switch (dtype) {
  case OR_FP8E4M3:
    for (int64_t i = 0; i < n; ++i) out[i] = or_e4m3_encode(w[i]);
    return 0;
  case OR_FP8E5M2:
    for (int64_t i = 0; i < n; ++i) out[i] = or_e5m2_encode(w[i]);
    return 0;
  case OR_FP4:
    memset(out, 0, (size_t)((n + 1) / 2));
    for (int64_t i = 0; i < n; ++i) {
      const uint8_t code = or_fp4_encode(w[i]) & 0xF;
      if (i % 2 == 0) out[i / 2] = code;
      else out[i / 2] |= (uint8_t)(code << 4);
    }
    return 0;
  case OR_INT8: {
    float s = abs_max(w, n) / 127.0f;
    if (s == 0) s = 1;
    for (int64_t i = 0; i < n; ++i) {
      const double r = clamp_i((double)roundf(w[i] / s), -128, 127);
      /* A NaN weight gives NaN here; the reference's static_cast<int> of NaN yields
       * INT_MIN on x86-64 (cvttsd2si), whose low byte is 0x00. Both that and the GPU's
       * saturating conversion store code 0. */
      const int q = isnan(r) ? 0 : (int)r;
      out[i] = (uint8_t)(int8_t)q;
    }
    *scale = s;
    return 0;
  }
  default:
    return -1;
  }
}

/* src/weights/native_codec.cpp:513-568 (weight_at: scale 0 -> 1; FP8/FP4 ignore scale;
 * Int8 dequantizes in float: float(q) * scale) and :1043-1078 (decode_row_f64 widens the
 * float result to double). Decodes `count` elements starting at flat index `start`. */
OR_EXPORT int or_decode_f64(int dtype, const uint8_t* raw, float scale, int64_t start,
                            int64_t count, double* dst) {
  if (scale == 0) scale = 1;
  for (int64_t j = 0; j < count; ++j) {
    const int64_t i = start + j;
    float v;
    switch (dtype) {
    case OR_FP8E4M3: v = or_e4m3_decode(raw[i]); break;
    case OR_FP8E5M2: v = or_e5m2_decode(raw[i]); break;
    case OR_FP4: {
      const uint8_t code = (i % 2 == 0) ? (raw[i / 2] & 0xF) : (raw[i / 2] >> 4);
      v = or_fp4_decode(code);
      break;
    }
    case OR_INT8: v = (float)(int8_t)raw[i] * scale; break;
    default: return -1;
    }
    dst[j] = (double)v;
  }
  return 0;
}

/* ---------------------------------------------------------------- Dense forward */

/* src/cuda/kernels.cu:22-46 (activate_dev). The reference calls CUDA's double exp/tanh;
 * this oracle calls the host libm ones. */
OR_EXPORT double or_activate(int act, double x) {
  switch (act) {
  case -1: return x;
  case 0: return x < 0.0 ? 0.0 : x;
  case 6: return x < 0.0 ? 0.0 : x * x;
  case 5: return x < 0.0 ? 0.01 * x : x;
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

typedef struct {
  int dtype;           /* 0: W64 given; else a packed store */
  const double* W64;   /* [out][in] */
  const uint8_t* raw;  /* packed store */
  const float* wf32;   /* Float32 store */
  float scale;
  int batch, in, out, act;
  const double* bias;
  int bias_len;
  const float* x;
  float* pre;
  float* post;
  double* y64;   /* optional [batch][out]: the f64 sum before any rounding */
  double* sabs;  /* optional [batch][out]: sum_k |W[o,k] * x[b,k]| */
  int o_begin, o_end;
} dense_job;

/* One output row: src/cuda/kernels.cu:130-145 (y = float(sum_k W64[o,k] * double(x[b,k])),
 * sequential k) followed by :147-161 (v = double(pre); bias only for o < bias_len, in which
 * case pre is rewritten as float(v); post = float(act(v))). The weight row is decoded first,
 * as dense session mount does (src/layers/dense/session.cpp:21-32). */
static void* dense_rows(void* arg) {
  dense_job* j = (dense_job*)arg;
  const int in = j->in;
  double* row = NULL;
  if (j->dtype != 0) row = (double*)malloc(sizeof(double) * (size_t)in);
  for (int o = j->o_begin; o < j->o_end; ++o) {
    const double* w;
    if (j->dtype == 0) {
      w = j->W64 + (size_t)o * (size_t)in;
    } else if (j->dtype == OR_FLOAT32) {
      for (int k = 0; k < in; ++k) row[k] = (double)j->wf32[(size_t)o * in + k];
      w = row;
    } else {
      or_decode_f64(j->dtype, j->raw, j->scale, (int64_t)o * in, in, row);
      w = row;
    }
    for (int b = 0; b < j->batch; ++b) {
      const float* xb = j->x + (size_t)b * (size_t)in;
      double sum = 0.0;
      double sa = 0.0;
      for (int k = 0; k < in; ++k) {
        sum += w[k] * (double)xb[k];
        if (j->sabs) sa += fabs(w[k] * (double)xb[k]);
      }
      const size_t idx = (size_t)b * (size_t)j->out + (size_t)o;
      if (j->y64) j->y64[idx] = sum;
      if (j->sabs) j->sabs[idx] = sa;
      float pre = (float)sum;
      double v = (double)pre;
      if (j->bias && o < j->bias_len) {
        v += j->bias[o];
        pre = (float)v;
      }
      j->pre[idx] = pre;
      j->post[idx] = (float)or_activate(j->act, v);
    }
  }
  free(row);
  return NULL;
}

static void run_dense(dense_job* proto, int threads) {
  if (threads < 1) threads = 1;
  if (threads > proto->out) threads = proto->out;
  if (threads <= 1) {
    proto->o_begin = 0;
    proto->o_end = proto->out;
    dense_rows(proto);
    return;
  }
  pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  dense_job* jobs = (dense_job*)malloc(sizeof(dense_job) * (size_t)threads);
  for (int t = 0; t < threads; ++t) {
    jobs[t] = *proto;
    jobs[t].o_begin = (int)((int64_t)proto->out * t / threads);
    jobs[t].o_end = (int)((int64_t)proto->out * (t + 1) / threads);
    pthread_create(&tid[t], NULL, dense_rows, &jobs[t]);
  }
  for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
  free(jobs);
  free(tid);
}

/* Dense forward from a decoded f64 matrix (the reference's resident mirror, A7/A8/A9). */
OR_EXPORT void or_dense_forward_f64w(int batch, int in, int out, int act, const double* W64,
                                     const double* bias, int bias_len, const float* x,
                                     float* pre, float* post, double* y64, double* sabs,
                                     int threads) {
  dense_job j;
  memset(&j, 0, sizeof(j));
  j.dtype = 0; j.W64 = W64;
  j.batch = batch; j.in = in; j.out = out; j.act = act;
  j.bias = bias; j.bias_len = bias_len; j.x = x; j.pre = pre; j.post = post;
  j.y64 = y64; j.sabs = sabs;
  run_dense(&j, threads);
}

/* Dense forward from a packed store: decode each row (weight_at) then the fp64 loop. This
 * is the host loop timed as the CPU baseline: rows are split across `threads` threads and
 * every row is computed exactly as in the single-thread case. For dtype Float32 `raw` is
 * the float32 payload. */
OR_EXPORT void or_dense_forward_native(int dtype, const uint8_t* raw, float scale, int batch,
                                       int in, int out, int act, const double* bias,
                                       int bias_len, const float* x, float* pre, float* post,
                                       double* y64, double* sabs, int threads) {
  dense_job j;
  memset(&j, 0, sizeof(j));
  j.dtype = dtype;
  if (dtype == OR_FLOAT32) j.wf32 = (const float*)raw; else j.raw = raw;
  j.scale = scale;
  j.batch = batch; j.in = in; j.out = out; j.act = act;
  j.bias = bias; j.bias_len = bias_len; j.x = x; j.pre = pre; j.post = post;
  j.y64 = y64; j.sabs = sabs;
  run_dense(&j, threads);
}

/* src/cuda/kernels.cu:296-305 -- h = float(double(float(SiLU(double(g)))) * double(up)). */
OR_EXPORT void or_swiglu_product(const float* gate_pre, const float* up_post, float* h,
                                 int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const double silu = or_activate(1, (double)gate_pre[i]);
    const float g_f = (float)silu;
    h[i] = (float)((double)g_f * (double)up_post[i]);
  }
}

/* ---------------------------------------------------------------- exhaustive digests */

/* splitmix64 finaliser (Steele, Lea, Flood 2014) -- the digest's per-element hash. */
static uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* Codec ids for the digest: 0 = E4M3 encode, 1 = E5M2 encode, 2 = FP4 encode. */
static uint8_t encode_one(int codec, uint32_t bits) {
  const float f = u2f(bits);
  switch (codec) {
  case 0: return or_e4m3_encode(f);
  case 1: return or_e5m2_encode(f);
  default: return or_fp4_encode(f);
  }
}

typedef struct {
  int codec;
  uint64_t start, count;
  uint64_t sum;
} digest_job;

static void* digest_rows(void* arg) {
  digest_job* j = (digest_job*)arg;
  uint64_t s = 0;
  for (uint64_t i = j->start; i < j->start + j->count; ++i) {
    const uint8_t c = encode_one(j->codec, (uint32_t)i);
    s += mix64((i << 8) | c);
  }
  j->sum = s;
  return NULL;
}

/* digest(codec, start, count) = sum over bit patterns i in [start, start+count) of
 * mix64((i << 8) | encode(i)) modulo 2^64. The sum is order-free, so the GPU computes
 * the same value with any reduction order. */
OR_EXPORT uint64_t or_encode_digest(int codec, uint64_t start, uint64_t count, int threads) {
  if (threads < 1) threads = 1;
  pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  digest_job* jobs = (digest_job*)malloc(sizeof(digest_job) * (size_t)threads);
  for (int t = 0; t < threads; ++t) {
    const uint64_t b = start + count * (uint64_t)t / (uint64_t)threads;
    const uint64_t e = start + count * (uint64_t)(t + 1) / (uint64_t)threads;
    jobs[t].codec = codec; jobs[t].start = b; jobs[t].count = e - b; jobs[t].sum = 0;
    pthread_create(&tid[t], NULL, digest_rows, &jobs[t]);
  }
  uint64_t s = 0;
  for (int t = 0; t < threads; ++t) { pthread_join(tid[t], NULL); s += jobs[t].sum; }
  free(jobs);
  free(tid);
  return s;
}

/* ---------------------------------------------------------------- Dense backward + SGD */

/* src/cuda/kernels.cu:48-81 (activate_deriv_dev); host libm exp/tanh as or_activate. */
OR_EXPORT double or_activate_deriv(int act, double x) {
  switch (act) {
  case -1: return 1.0;
  case 0: return x > 0.0 ? 1.0 : 0.0;
  case 6: return x > 0.0 ? 2.0 * x : 0.0;
  case 5: return x > 0.0 ? 1.0 : 0.01;
  case 1: {
    const double sig = 1.0 / (1.0 + exp(-x));
    return sig * (1.0 + x * (1.0 - sig));
  }
  case 2: {
    const double k = 0.7978845608028654;
    const double u = k * (x + 0.044715 * x * x * x);
    const double th = tanh(u);
    const double du = k * (1.0 + 3.0 * 0.044715 * x * x);
    return 0.5 * (1.0 + th) + 0.5 * x * (1.0 - th * th) * du;
  }
  case 3: {
    const double t = tanh(x);
    return 1.0 - t * t;
  }
  case 4: {
    const double s = 1.0 / (1.0 + exp(-x));
    return s * (1.0 - s);
  }
  default: return 1.0;
  }
}

/* Dense NormalBP backward, src/cuda/kernels.cu:83-128 with resident_backward (:917-1000):
 *   d_pre[b,o] = float(double(gy[b,o]) * act'(double(pre[b,o])))       (linear: d_pre = gy)
 *   gx[b,i]    = float(sum_o W64[o,i] * double(d_pre[b,o]))             sequential o
 *   dW[o,i]    = acc over b: acc = float(double(acc) + double(d_pre[b,o]) * double(x[b,i]))
 * W64 is the store decoded as weight_at does (FP8 / FP4 table value, Int8 float(q) * scale,
 * Float32 the payload). Products are of two floats, exact in double, so the order of
 * multiply and add does not change the sums. */
OR_EXPORT int or_dense_backward(int dtype, const uint8_t* raw, float scale, int batch, int in, int out,
                                int act, int linear, const float* gy, const float* x, const float* pre,
                                float* d_pre, float* gx, float* dW) {
  const int64_t n = (int64_t)out * in;
  double* W = (double*)malloc(sizeof(double) * (size_t)n);
  if (!W) return 1;
  if (dtype == OR_FLOAT32) {
    const float* wf = (const float*)raw;
    for (int64_t i = 0; i < n; ++i) W[i] = (double)wf[i];
  } else if (or_decode_f64(dtype, raw, scale, 0, n, W) != 0) {
    free(W);
    return 1;
  }
  for (int64_t i = 0; i < (int64_t)batch * out; ++i)
    d_pre[i] = linear ? gy[i] : (float)((double)gy[i] * or_activate_deriv(act, (double)pre[i]));
  for (int b = 0; b < batch; ++b)
    for (int i = 0; i < in; ++i) {
      double sum = 0.0;
      for (int o = 0; o < out; ++o) sum += W[(size_t)o * in + i] * (double)d_pre[(size_t)b * out + o];
      gx[(size_t)b * in + i] = (float)sum;
    }
  for (int o = 0; o < out; ++o)
    for (int i = 0; i < in; ++i) {
      float acc = 0.0f;
      for (int b = 0; b < batch; ++b)
        acc = (float)((double)acc + (double)d_pre[(size_t)b * out + o] * (double)x[(size_t)b * in + i]);
      dW[(size_t)o * in + i] = acc;
    }
  free(W);
  return 0;
}

/* WeightStore::apply_sgd for the FormatNone types of this path,
 * src/weights/native_codec.cpp:1080-1133 with weight_at (:513-568) and set_weight_at
 * (:774-830): every element is decoded, updated in float (next = float(double(v) - lr * dW)),
 * and encoded again with the same codec (FP8 / FP4: the float codecs, so codes that decode to
 * the same value may change, e.g. FP8 subnormal codes become signed zeros; Int8:
 * q = clamp(round(double(next / scale)), -128, 127) with the stored scale, 1 when it is 0);
 * Float32: w -= float(lr * dW). `raw` is updated in place (Float32: the float payload). */
OR_EXPORT int or_apply_sgd(int dtype, uint8_t* raw, float scale, int64_t n, const double* dW, double lr) {
  const float s = scale == 0.0f ? 1.0f : scale;
  if (dtype == OR_FLOAT32) {
    float* wf = (float*)raw;
    for (int64_t i = 0; i < n; ++i) wf[i] -= (float)(lr * dW[i]);
    return 0;
  }
  for (int64_t i = 0; i < n; ++i) {
    float v;
    switch (dtype) {
    case OR_FP8E4M3: v = or_e4m3_decode(raw[i]); break;
    case OR_FP8E5M2: v = or_e5m2_decode(raw[i]); break;
    case OR_FP4: v = or_fp4_decode((uint8_t)((raw[i >> 1] >> ((i & 1) * 4)) & 0xF)); break;
    case OR_INT8: v = (float)(int8_t)raw[i] * s; break;
    default: return 1;
    }
    const float next = (float)((double)v - lr * dW[i]);
    switch (dtype) {
    case OR_FP8E4M3: raw[i] = or_e4m3_encode(next); break;
    case OR_FP8E5M2: raw[i] = or_e5m2_encode(next); break;
    case OR_FP4: {
      const uint8_t c = (uint8_t)(or_fp4_encode(next) & 0xF);
      const int sh = (int)(i & 1) * 4;
      raw[i >> 1] = (uint8_t)((raw[i >> 1] & ~(0xF << sh)) | (c << sh));
      break;
    }
    case OR_INT8: {
      double q = round((double)(next / s));
      if (q < -128.0) q = -128.0;
      if (q > 127.0) q = 127.0;
      raw[i] = (uint8_t)(int8_t)q;
      break;
    }
    }
  }
  return 0;
}

/* src/runtime/training.cpp:44-69: loss = sum (pred - target)^2 / n (sequential, f64);
 * grad = float(2 / n * (pred - target)). */
OR_EXPORT double or_mse(const float* pred, const float* target, int64_t n, float* grad) {
  double sum = 0.0;
  const double sc = 2.0 / (double)n;
  for (int64_t i = 0; i < n; ++i) {
    const double d = (double)pred[i] - (double)target[i];
    sum += d * d;
    if (grad) grad[i] = (float)(sc * d);
  }
  return sum / (double)n;
}
