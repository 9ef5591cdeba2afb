// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Thin extern "C" wrappers over the welvet.cuda reference's own C++ API, linked by
// oracle/Makefile with the reference sources (compiled where they lie, never copied) into
// oracle/_ref/libwelvet_ref.so. Used only to pin the C oracle (oracle.c) against the
// reference itself, to generate tests/golden/ fixtures, and to time the reference's own
// CUDA Dense kernels on the GPU box beside the product.
//
// Reference entry points wrapped:
//   codec        include/welvet/float_codecs.hpp:9-20 (src/core/float_codecs.cpp:57-200)
//   store        include/welvet/weights.hpp:18-51   (WeightStore::make / decode_row_f64)
//   dense        include/welvet/dense_session.hpp:10-17 (session_mount/execute/release)
//                include/welvet/dense.hpp:53-59 (new_layer / forward_f32)
//   swiglu       include/welvet/swiglu.hpp:26-31   mha  include/welvet/mha.hpp:78-84
#include "welvet/dense.hpp"
#include "welvet/dense_session.hpp"
#include "welvet/float_codecs.hpp"
#include "welvet/mha.hpp"
#include "welvet/swiglu.hpp"
#include "welvet/weights.hpp"

#include <cstring>
#include <thread>
#include <vector>

namespace {

uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint8_t encode_one(int codec, uint32_t bits) {
  float f;
  std::memcpy(&f, &bits, 4);
  switch (codec) {
  case 0: return welvet::float32_to_fp8e4m3(f);
  case 1: return welvet::float32_to_fp8e5m2(f);
  default: return welvet::float32_to_fp4(f);
  }
}

int fill_msg(const welvet::Status& st, char* msg, int cap) {
  if (msg && cap > 0) {
    std::strncpy(msg, st.message.c_str(), static_cast<size_t>(cap - 1));
    msg[cap - 1] = 0;
  }
  return static_cast<int>(st.code);
}

} // namespace

extern "C" {

uint8_t ref_e4m3_encode(float f) { return welvet::float32_to_fp8e4m3(f); }
float ref_e4m3_decode(uint8_t b) { return welvet::fp8e4m3_to_float32(b); }
uint8_t ref_e5m2_encode(float f) { return welvet::float32_to_fp8e5m2(f); }
float ref_e5m2_decode(uint8_t b) { return welvet::fp8e5m2_to_float32(b); }
uint8_t ref_fp4_encode(float f) { return welvet::float32_to_fp4(f); }
float ref_fp4_decode(uint8_t c) { return welvet::fp4_to_float32(c); }

// Same digest definition as oracle.c:or_encode_digest, over the reference codec.
uint64_t ref_encode_digest(int codec, uint64_t start, uint64_t count, int threads) {
  if (threads < 1) threads = 1;
  std::vector<uint64_t> sums(static_cast<size_t>(threads), 0);
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    const uint64_t b = start + count * static_cast<uint64_t>(t) / static_cast<uint64_t>(threads);
    const uint64_t e = start + count * static_cast<uint64_t>(t + 1) / static_cast<uint64_t>(threads);
    pool.emplace_back([=, &sums] {
      uint64_t s = 0;
      for (uint64_t i = b; i < e; ++i) s += mix64((i << 8) | encode_one(codec, static_cast<uint32_t>(i)));
      sums[static_cast<size_t>(t)] = s;
    });
  }
  uint64_t s = 0;
  for (int t = 0; t < threads; ++t) {
    pool[static_cast<size_t>(t)].join();
    s += sums[static_cast<size_t>(t)];
  }
  return s;
}

// WeightStore::make(rows, cols, dtype, w) -> native bytes + scale (Float32 -> f32 payload).
int ref_store_make(int rows, int cols, int dtype, const float* w, uint8_t* native_out,
                   size_t cap, size_t* native_len, float* scale, char* msg, int msg_cap) {
  welvet::WeightStore s;
  auto st = welvet::WeightStore::make(rows, cols, static_cast<welvet::DType>(dtype), w, &s);
  if (!st) return fill_msg(st, msg, msg_cap);
  const uint8_t* src = s.native.data();
  size_t len = s.native.size();
  if (s.dtype == welvet::DType::Float32) {
    src = reinterpret_cast<const uint8_t*>(s.f32.data());
    len = s.f32.size() * sizeof(float);
  }
  *native_len = len;
  *scale = s.scale;
  if (len > cap) return 1;
  std::memcpy(native_out, src, len);
  return 0;
}

// WeightStore{dtype, rows, cols, native, scale}.decode_row_f64(row) for every row.
int ref_store_decode(int rows, int cols, int dtype, const uint8_t* native, size_t native_len,
                     float scale, double* out, char* msg, int msg_cap) {
  welvet::WeightStore s;
  s.dtype = static_cast<welvet::DType>(dtype);
  s.rows = rows;
  s.cols = cols;
  s.scale = scale;
  if (s.dtype == welvet::DType::Float32) {
    s.f32.assign(reinterpret_cast<const float*>(native),
                 reinterpret_cast<const float*>(native) + native_len / sizeof(float));
  } else {
    s.native.assign(native, native + native_len);
  }
  for (int r = 0; r < rows; ++r) {
    auto st = s.decode_row_f64(r, out + static_cast<size_t>(r) * static_cast<size_t>(cols));
    if (!st) return fill_msg(st, msg, msg_cap);
  }
  return 0;
}

// WeightStore{dtype, rows, cols, native, scale}.apply_sgd(dW, lr) (src/weights/native_codec.cpp:
// 1080-1133); the updated payload is written back over `native`.
int ref_store_apply_sgd(int rows, int cols, int dtype, uint8_t* native, size_t native_len, float scale,
                        const double* dW, double lr, char* msg, int msg_cap) {
  welvet::WeightStore s;
  s.dtype = static_cast<welvet::DType>(dtype);
  s.rows = rows;
  s.cols = cols;
  s.scale = scale;
  if (s.dtype == welvet::DType::Float32) {
    s.f32.assign(reinterpret_cast<const float*>(native), reinterpret_cast<const float*>(native) + native_len / 4);
  } else {
    s.native.assign(native, native + native_len);
  }
  auto st = s.apply_sgd(dW, lr);
  if (!st) return fill_msg(st, msg, msg_cap);
  if (s.dtype == welvet::DType::Float32) std::memcpy(native, s.f32.data(), native_len);
  else std::memcpy(native, s.native.data(), native_len);
  return 0;
}

// The steps of the reference's welvet_dense_normalbp_f32 (src/interop/c_abi.cpp:119-184) on
// its own layer API and CUDA kernels: new_layer, forward_f32, MSE and its gradient
// (src/runtime/training.cpp:44-69, restated here because that file is not in this build),
// backward_f32, apply_grad_sgd when lr != 0, export_f32.
int ref_dense_normalbp(int batch, int in, int out, int act, int dtype, const float* W, const double* bias,
                       size_t bias_len, const float* x, const float* grad_or_target, int use_target, double lr,
                       float* pre, float* post, float* dX, float* dW, float* W_after, double* loss, char* msg,
                       int msg_cap) {
  welvet::dense::Layer layer;
  auto st = welvet::dense::new_layer(in, out, static_cast<welvet::Activation>(act),
                                     static_cast<welvet::DType>(dtype), W, &layer);
  if (!st) return fill_msg(st, msg, msg_cap);
  if (bias && bias_len > 0) layer.weights.bias.assign(bias, bias + bias_len);
  welvet::TensorF32 input;
  input.shape = {batch, in};
  input.data.assign(x, x + static_cast<size_t>(batch) * in);
  welvet::TensorF32 p, q;
  st = welvet::dense::forward_f32(layer, input, &p, &q);
  if (!st) return fill_msg(st, msg, msg_cap);
  welvet::TensorF32 gy;
  gy.shape = {batch, out};
  gy.data.assign(grad_or_target, grad_or_target + static_cast<size_t>(batch) * out);
  *loss = 0.0;
  if (use_target) {
    double sum = 0.0;
    const double sc = 2.0 / static_cast<double>(q.data.size());
    for (size_t i = 0; i < q.data.size(); ++i) {
      const double d = static_cast<double>(q.data[i]) - static_cast<double>(gy.data[i]);
      sum += d * d;
      gy.data[i] = static_cast<float>(sc * d);
    }
    *loss = sum / static_cast<double>(q.data.size());
  }
  welvet::TensorF32 dx_t, dw_t;
  st = welvet::dense::backward_f32(layer, gy, input, p, &dx_t, &dw_t);
  if (!st) return fill_msg(st, msg, msg_cap);
  if (lr != 0.0) {
    st = welvet::dense::apply_grad_sgd(&layer, dw_t, lr);
    if (!st) return fill_msg(st, msg, msg_cap);
  }
  st = layer.weights.export_f32(W_after);
  if (!st) return fill_msg(st, msg, msg_cap);
  std::memcpy(pre, p.data.data(), p.data.size() * sizeof(float));
  std::memcpy(post, q.data.data(), q.data.size() * sizeof(float));
  std::memcpy(dX, dx_t.data.data(), dx_t.data.size() * sizeof(float));
  std::memcpy(dW, dw_t.data.data(), dw_t.data.size() * sizeof(float));
  return 0;
}

// Reference resident Dense session (GPU): host decode -> fp64 mirror -> dense_matvec_f64_batch.
int ref_dense_mount(int batch, int in, int out, int act, int dtype, const float* W,
                    const double* bias, size_t bias_len, void** sess, char* msg, int msg_cap) {
  welvet::dense::Session* s = nullptr;
  auto st = welvet::dense::session_mount(batch, in, out, static_cast<welvet::Activation>(act),
                                         static_cast<welvet::DType>(dtype), W, bias, bias_len, &s);
  if (!st) return fill_msg(st, msg, msg_cap);
  *sess = s;
  return 0;
}

int ref_dense_execute(void* sess, const float* x, float* pre, float* post, char* msg,
                      int msg_cap) {
  auto st = welvet::dense::session_execute(static_cast<welvet::dense::Session*>(sess), x, pre, post);
  return st ? 0 : fill_msg(st, msg, msg_cap);
}

void ref_dense_release(void* sess) {
  welvet::dense::session_release(static_cast<welvet::dense::Session*>(sess));
}

// swiglu::new_configured + forward, the path of the reference's welvet_swiglu_forward_f32.
int ref_swiglu_forward(int batch, int seq, int input_dim, int inter, int dtype, const float* G,
                       const float* U, const float* D, const float* x, float* pre, float* post,
                       char* msg, int msg_cap) {
  welvet::swiglu::Config cfg;
  cfg.input_dim = input_dim;
  cfg.intermediate_dim = inter;
  welvet::swiglu::Layer layer;
  auto st = welvet::swiglu::new_configured(cfg, static_cast<welvet::DType>(dtype), G, U, D, &layer);
  if (!st) return fill_msg(st, msg, msg_cap);
  welvet::TensorF32 input;
  if (seq == 1) input.shape = {batch, input_dim};
  else input.shape = {batch, seq, input_dim};
  input.data.assign(x, x + static_cast<size_t>(batch) * seq * input_dim);
  welvet::TensorF32 p, q;
  st = welvet::swiglu::forward(layer, input, &p, &q);
  if (!st) return fill_msg(st, msg, msg_cap);
  std::memcpy(pre, p.data.data(), p.data.size() * sizeof(float));
  std::memcpy(post, q.data.data(), q.data.size() * sizeof(float));
  return 0;
}

// mha::new_configured + forward (ModeSelf), the path of welvet_mha_forward_f32.
int ref_mha_forward(int batch, int seq, int d_model, int num_heads, int num_kv_heads,
                    int head_dim, int max_seq_len, int mask, int pos, int dtype, const float* Q,
                    const float* K, const float* V, const float* O, const float* x, float* pre,
                    float* post, char* msg, int msg_cap) {
  welvet::mha::Config cfg;
  cfg.d_model = d_model;
  cfg.num_heads = num_heads;
  cfg.num_kv_heads = num_kv_heads;
  cfg.head_dim = head_dim;
  cfg.max_seq_len = max_seq_len;
  cfg.mask = static_cast<welvet::mha::MaskKind>(mask);
  cfg.pos = static_cast<welvet::mha::PosKind>(pos);
  cfg.mode = welvet::mha::AttnMode::Self;
  cfg.causal = (cfg.mask == welvet::mha::MaskKind::Causal);
  welvet::mha::Layer layer;
  auto st = welvet::mha::new_configured(cfg, static_cast<welvet::DType>(dtype), Q, K, V, O, &layer);
  if (!st) return fill_msg(st, msg, msg_cap);
  welvet::TensorF32 input;
  input.shape = {batch, seq, d_model};
  input.data.assign(x, x + static_cast<size_t>(batch) * seq * d_model);
  welvet::TensorF32 p, q;
  st = welvet::mha::forward(layer, input, &p, &q);
  if (!st) return fill_msg(st, msg, msg_cap);
  std::memcpy(pre, p.data.data(), p.data.size() * sizeof(float));
  std::memcpy(post, q.data.data(), q.data.size() * sizeof(float));
  return 0;
}

} // extern "C"
