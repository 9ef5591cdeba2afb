// A caller of the reference's C++ layer API, written against its signatures
// (include/welvet/dense.hpp:59, swiglu.hpp:31, mha.hpp:82 of the reference) and built against
// this repository's include/ and libwelvet_b200.so. tests/test_cxx_api.py compiles and links it
// (CPU) and, on a GPU, calls the extern "C" wrappers below through ctypes.
#include "welvet/dense.hpp"
#include "welvet/mha.hpp"
#include "welvet/swiglu.hpp"

#include <cstring>
#include <vector>

using welvet::Status;
using welvet::TensorF32;

// The three entry points with exactly the reference's types.
static Status (*const kDenseForward)(const welvet::dense::Layer&, const TensorF32&, TensorF32*, TensorF32*) =
    &welvet::dense::forward_f32;
static Status (*const kSwigluForward)(welvet::swiglu::Layer&, const TensorF32&, TensorF32*, TensorF32*) =
    &welvet::swiglu::forward;
static Status (*const kMhaForward)(welvet::mha::Layer&, const TensorF32&, TensorF32*, TensorF32*) =
    &welvet::mha::forward;

// The training entry points (reference include/welvet/dense.hpp:62-74, weights.hpp:36-44).
static Status (*const kDenseBackward)(const welvet::dense::Layer&, const TensorF32&, const TensorF32&,
                                      const TensorF32&, TensorF32*, TensorF32*) = &welvet::dense::backward_f32;
static Status (*const kLinearGradIn)(const welvet::dense::Layer&, const TensorF32&, const TensorF32&, TensorF32*) =
    &welvet::dense::linear_grad_in;
static Status (*const kGradWOnly)(const welvet::dense::Layer&, const TensorF32&, const TensorF32&,
                                  const TensorF32&, TensorF32*) = &welvet::dense::grad_w_only;
static Status (*const kApplyGradSgd)(welvet::dense::Layer*, const TensorF32&, double) = &welvet::dense::apply_grad_sgd;

static int fail(const Status& st, char* msg) {
  if (msg) std::strncpy(msg, st.message.c_str(), 255);
  return static_cast<int>(st.code);
}

static TensorF32 tensor(std::vector<int64_t> shape, const float* p, size_t n) {
  TensorF32 t;
  t.shape = std::move(shape);
  t.data.assign(p, p + n);
  return t;
}

extern "C" {

// Two forwards of one Dense layer: x1 [b1][in], then (after the weights are replaced by W2 and
// the layer invalidated) x2 [b2][in] -- a new batch and new weights, both remounted lazily.
int run_dense(int in, int out, int act, int dtype, const float* W1, const float* W2, const double* bias, int bias_len,
              int b1, const float* x1, int b2, const float* x2, float* pre1, float* post1, float* pre2, float* post2,
              char* msg) {
  welvet::dense::Layer L;
  Status st = welvet::dense::new_layer(in, out, static_cast<welvet::Activation>(act), static_cast<welvet::DType>(dtype),
                                       W1, &L);
  if (!st) return fail(st, msg);
  L.weights.bias.assign(bias, bias + bias_len);
  TensorF32 pre, post;
  st = kDenseForward(L, tensor({b1, in}, x1, static_cast<size_t>(b1) * in), &pre, &post);
  if (!st) return fail(st, msg);
  std::memcpy(pre1, pre.data.data(), pre.data.size() * 4);
  std::memcpy(post1, post.data.data(), post.data.size() * 4);
  welvet::WeightStore W;
  st = welvet::WeightStore::make(out, in, static_cast<welvet::DType>(dtype), W2, &W);
  if (!st) return fail(st, msg);
  W.bias = L.weights.bias;
  L.weights = std::move(W);
  L.invalidate_gpu();
  st = kDenseForward(L, tensor({b2, in}, x2, static_cast<size_t>(b2) * in), &pre, &post);
  if (!st) return fail(st, msg);
  std::memcpy(pre2, pre.data.data(), pre.data.size() * 4);
  std::memcpy(post2, post.data.data(), post.data.size() * 4);
  // a shape error comes back as the reference's status
  TensorF32 bad = tensor({1, in + 1}, x1, static_cast<size_t>(in + 1));
  st = kDenseForward(L, bad, &pre, &post);
  return st.code == welvet::StatusCode::InvalidArgument ? 0 : 99;
}

// The steps of the reference's welvet_dense_normalbp_f32 on the C++ API (given output
// gradient, no MSE): forward, backward_f32, apply_grad_sgd when lr != 0, export_f32; plus
// linear_grad_in and grad_w_only on the updated layer, and a second forward after the SGD.
int run_dense_train(int in, int out, int act, int dtype, const float* W, int batch, const float* x, const float* gy,
                    double lr, float* pre, float* post, float* dX, float* dW, float* W_after, float* gx_lin,
                    float* dw_only, float* post_after, char* msg) {
  welvet::dense::Layer L;
  Status st = welvet::dense::new_layer(in, out, static_cast<welvet::Activation>(act), static_cast<welvet::DType>(dtype),
                                       W, &L);
  if (!st) return fail(st, msg);
  const TensorF32 input = tensor({batch, in}, x, static_cast<size_t>(batch) * in);
  const TensorF32 g = tensor({batch, out}, gy, static_cast<size_t>(batch) * out);
  TensorF32 p, q, gx, gw;
  st = kDenseForward(L, input, &p, &q);
  if (!st) return fail(st, msg);
  st = kDenseBackward(L, g, input, p, &gx, &gw);
  if (!st) return fail(st, msg);
  if (lr != 0.0) {
    st = kApplyGradSgd(&L, gw, lr);
    if (!st) return fail(st, msg);
    if (L.gpu_valid) return 98;  // the SGD invalidates the device mirror
  }
  st = L.weights.export_f32(W_after);
  if (!st) return fail(st, msg);
  std::memcpy(pre, p.data.data(), p.data.size() * 4);
  std::memcpy(post, q.data.data(), q.data.size() * 4);
  std::memcpy(dX, gx.data.data(), gx.data.size() * 4);
  std::memcpy(dW, gw.data.data(), gw.data.size() * 4);
  TensorF32 lin, only, p2, q2;
  st = kLinearGradIn(L, g, input, &lin);
  if (!st) return fail(st, msg);
  st = kGradWOnly(L, g, input, p, &only);
  if (!st) return fail(st, msg);
  st = kDenseForward(L, input, &p2, &q2);
  if (!st) return fail(st, msg);
  std::memcpy(gx_lin, lin.data.data(), lin.data.size() * 4);
  std::memcpy(dw_only, only.data.data(), only.data.size() * 4);
  std::memcpy(post_after, q2.data.data(), q2.data.size() * 4);
  TensorF32 bad = tensor({batch, out + 1}, gy, static_cast<size_t>(batch) * out);
  st = kDenseBackward(L, bad, input, p, &gx, &gw);
  return st.code == welvet::StatusCode::InvalidArgument ? 0 : 97;
}

int run_swiglu(int batch, int seq, int in, int inter, int dtype, const float* G, const float* U, const float* D,
               const float* x, float* pre, float* post, char* msg) {
  welvet::swiglu::Layer L;
  Status st = welvet::swiglu::new_configured({in, inter}, static_cast<welvet::DType>(dtype), G, U, D, &L);
  if (!st) return fail(st, msg);
  TensorF32 p, q;
  const size_t n = static_cast<size_t>(batch) * seq * in;
  for (int call = 0; call < 2; ++call) {  // the second call reuses the mounted cell
    st = kSwigluForward(L, seq == 1 ? tensor({batch, in}, x, n) : tensor({batch, seq, in}, x, n), &p, &q);
    if (!st) return fail(st, msg);
  }
  std::memcpy(pre, p.data.data(), p.data.size() * 4);
  std::memcpy(post, q.data.data(), q.data.size() * 4);
  return 0;
}

int run_mha(int batch, int seq, int d, int heads, int kv_heads, int head_dim, int msl, int dtype, const float* Q,
            const float* K, const float* V, const float* O, const float* x, float* pre, float* post, char* msg) {
  welvet::mha::Config cfg = welvet::mha::decoder_causal(d, heads, kv_heads);
  cfg.head_dim = head_dim;
  cfg.max_seq_len = msl;
  welvet::mha::Layer L;
  Status st = welvet::mha::new_configured(cfg, static_cast<welvet::DType>(dtype), Q, K, V, O, &L);
  if (!st) return fail(st, msg);
  TensorF32 p, q;
  st = kMhaForward(L, tensor({batch, seq, d}, x, static_cast<size_t>(batch) * seq * d), &p, &q);
  if (!st) return fail(st, msg);
  std::memcpy(pre, p.data.data(), p.data.size() * 4);
  std::memcpy(post, q.data.data(), q.data.size() * 4);
  return 0;
}

} // extern "C"
