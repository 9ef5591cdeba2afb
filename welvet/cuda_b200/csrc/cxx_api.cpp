// cxx_api.cpp -- the reference's C++ layer API (include/welvet/{dense,swiglu,mha}.hpp) over this
// library's sessions and cells, so that code written against dense::forward_f32,
// swiglu::forward and mha::forward (the entry points the reference's other layer kinds call,
// src/layers/*) links against libwelvet_b200 unchanged.
//
// Reference behaviour kept: argument and shape checks with the reference's messages
// (src/layers/dense/dense.cpp:58-86, src/layers/swiglu/swiglu.cpp:18-136,
// src/layers/mha/mha.cpp:18-183), the lazy (re)mount on first use / invalidate_gpu() / batch
// change, host tensors in and out, synchronous calls. What differs by design: the device state
// holds packed codes instead of an fp64 mirror, and SwiGLU / MHA run the library's fused cells
// (one Gate/Up kernel with the product in its epilogue; projections on the tensor-core paths)
// instead of chaining host round trips through dense::forward_f32.
#include "../../../include/welvet/dense.hpp"
#include "../../../include/welvet/mha.hpp"
#include "../../../include/welvet/swiglu.hpp"

#include "backward.hpp"
#include "cells.hpp"
#include "codec.hpp"
#include "dense.hpp"

#include <cmath>
#include <cstring>
#include <string>
#include <vector>

namespace {

welvet::Status from_wb(const wb::Status& s) {
  return welvet::Status::Err(static_cast<welvet::StatusCode>(static_cast<int>(s.code)), s.message);
}

welvet::Status invalid(const char* m) { return welvet::Status::Err(welvet::StatusCode::InvalidArgument, m); }

// Fused cells held in a layer's device state, with their own stream and device work buffers.
struct SwigluHolder {
  wb::SwigluCell cell;
  cudaStream_t stream = nullptr;
  float *x = nullptr, *h = nullptr, *y = nullptr;
  int rows = 0;
  ~SwigluHolder() {
    cudaSetDevice(cell.device);
    if (stream) cudaStreamSynchronize(stream);
    for (float* p : {x, h, y})
      if (p) cudaFree(p);
    if (stream) cudaStreamDestroy(stream);
  }
};

struct MhaHolder {
  wb::MhaCell cell;
  cudaStream_t stream = nullptr;
  float *x = nullptr, *attn = nullptr, *y = nullptr;
  int rows = 0;
  ~MhaHolder() {
    cudaSetDevice(cell.device);
    if (stream) cudaStreamSynchronize(stream);
    for (float* p : {x, attn, y})
      if (p) cudaFree(p);
    if (stream) cudaStreamDestroy(stream);
  }
};

void drop_session(welvet::cuda::ResidentDense& r) {
  delete static_cast<wb::DenseSession*>(r.session);
  r.session = nullptr;
}

void drop_cell(welvet::cuda::ResidentDense& r) {
  if (r.cell_kind == 1) delete static_cast<SwigluHolder*>(r.cell);
  if (r.cell_kind == 2) delete static_cast<MhaHolder*>(r.cell);
  r.cell = nullptr;
  r.cell_kind = 0;
}

// A store as a cell mount reads it: its native bytes (Float32: the float payload) and scale.
wb::WeightSrc source(const welvet::WeightStore& s) {
  wb::WeightSrc w;
  if (s.dtype == welvet::DType::Float32) {
    w.native = reinterpret_cast<const uint8_t*>(s.f32.data());
    w.native_len = s.f32.size() * sizeof(float);
  } else {
    w.native = s.native.data();
    w.native_len = s.native.size();
  }
  w.scale = s.scale;
  return w;
}

// Device buffers released on every exit path.
struct DevBufs {
  std::vector<void*> p;
  ~DevBufs() {
    for (void* q : p)
      if (q) cudaFree(q);
  }
  template <typename T>
  wb::Status get(T** out, size_t n) {
    void* q = nullptr;
    WB_CUDA(cudaMalloc(&q, n > 0 ? n * sizeof(T) : 16));
    p.push_back(q);
    *out = static_cast<T*>(q);
    return wb::Status::Ok();
  }
};

// A store's payload as the GPU codec reads it (Float32: the float master).
const void* payload_of(const welvet::WeightStore& s, size_t* bytes) {
  if (s.dtype == welvet::DType::Float32) {
    *bytes = s.f32.size() * sizeof(float);
    return s.f32.data();
  }
  *bytes = s.native.size();
  return s.native.data();
}

// Checks the store's payload covers rows * cols elements (the reference's "short" errors).
welvet::Status payload_ok(const welvet::WeightStore& s) {
  const int64_t n = static_cast<int64_t>(s.rows) * s.cols;
  if (s.dtype == welvet::DType::Float32)
    return static_cast<int64_t>(s.f32.size()) < n ? invalid("f32 short") : welvet::Status::Ok();
  if (!wb::dtype_on_path(static_cast<int32_t>(s.dtype)))
    return welvet::Status::Err(welvet::StatusCode::Unsupported,
                               std::string("weights: dtype ") + std::string(welvet::dtype_name(s.dtype)) +
                                   " is not served on the GPU by this library");
  if (static_cast<int64_t>(s.native.size()) < wb::native_bytes(static_cast<wb::DType>(s.dtype), n))
    return invalid("weights: native payload short");
  return welvet::Status::Ok();
}

// Resamples gy to `need` values by bucket means (the reference's remap for gradient lengths
// that differ from batch * out, src/layers/dense/dense.cpp:122-139).
void remap_len(const std::vector<float>& src, int need, std::vector<float>* out) {
  out->assign(static_cast<size_t>(need > 0 ? need : 0), 0.0f);
  const int sn = static_cast<int>(src.size());
  if (sn <= 0 || need <= 0) return;
  if (sn == need) {
    *out = src;
    return;
  }
  for (int i = 0; i < need; ++i) {
    const int lo = static_cast<int>(static_cast<int64_t>(i) * sn / need);
    int hi = static_cast<int>(static_cast<int64_t>(i + 1) * sn / need);
    hi = hi <= lo ? lo + 1 : (hi > sn ? sn : hi);
    double acc = 0.0;
    for (int j = lo; j < hi; ++j) acc += static_cast<double>(src[static_cast<size_t>(j)]);
    (*out)[static_cast<size_t>(i)] = static_cast<float>(acc / static_cast<double>(hi - lo));
  }
}

// One backward on the layer's mounted session: host gy / x / pre in, gx and / or dW out.
welvet::Status run_backward(const welvet::dense::Layer& layer, int batch, const float* gy, const float* x,
                            const float* pre, bool linear, float* gx_host, float* dw_host) {
  if (!layer.gpu_valid || layer.gpu_batch != batch || !layer.gpu.session) {
    if (auto st = welvet::dense::sync_gpu_from_weights(layer, batch); !st) return st;
  }
  auto* s = static_cast<wb::DenseSession*>(layer.gpu.session);
  wb::Status st = wb::cuda_status(cudaSetDevice(s->device), "cudaSetDevice");
  const size_t nx = static_cast<size_t>(batch) * layer.input_height;
  const size_t ny = static_cast<size_t>(batch) * layer.output_height;
  const size_t nw = static_cast<size_t>(layer.output_height) * layer.input_height;
  DevBufs b;
  float *gyd = nullptr, *xd = nullptr, *pred = nullptr, *dpre = nullptr, *gxd = nullptr, *dwd = nullptr;
  if (st.ok()) st = b.get(&gyd, ny);
  if (st.ok()) st = b.get(&xd, nx);
  if (st.ok()) st = b.get(&pred, ny);
  if (st.ok()) st = b.get(&dpre, ny);
  if (st.ok()) st = b.get(&gxd, nx);
  if (st.ok()) st = b.get(&dwd, nw);
  if (st.ok()) st = wb::cuda_status(cudaMemcpyAsync(gyd, gy, ny * 4, cudaMemcpyHostToDevice, s->stream), "H2D");
  if (st.ok()) st = wb::cuda_status(cudaMemcpyAsync(xd, x, nx * 4, cudaMemcpyHostToDevice, s->stream), "H2D");
  if (st.ok()) st = wb::cuda_status(cudaMemcpyAsync(pred, pre, ny * 4, cudaMemcpyHostToDevice, s->stream), "H2D");
  if (st.ok()) st = wb::dense_backward_device(s->dev, batch, gyd, xd, pred, linear, dpre, gxd, dwd, s->stream);
  if (st.ok() && gx_host)
    st = wb::cuda_status(cudaMemcpyAsync(gx_host, gxd, nx * 4, cudaMemcpyDeviceToHost, s->stream), "D2H");
  if (st.ok() && dw_host)
    st = wb::cuda_status(cudaMemcpyAsync(dw_host, dwd, nw * 4, cudaMemcpyDeviceToHost, s->stream), "D2H");
  const wb::Status sync = wb::cuda_status(cudaStreamSynchronize(s->stream), "backward sync");
  if (st.ok()) st = sync;
  return st.ok() ? welvet::Status::Ok() : from_wb(st);
}

wb::Status grow(float** p, size_t n) {
  if (*p) cudaFree(*p);
  *p = nullptr;
  return wb::cuda_status(cudaMalloc(p, n * sizeof(float)), "cudaMalloc");
}

} // namespace

namespace welvet {

TensorF32 TensorF32::zeros(int64_t a, int64_t b) {
  TensorF32 t;
  t.shape = {a, b};
  t.data.assign(static_cast<std::size_t>(a * b), 0.0f);
  return t;
}

std::string_view dtype_name(DType dt) {
  static const char* const names[kNumDTypes] = {
      "float64", "float32", "float16", "bfloat16", "fp8e4m3", "fp8e5m2", "int64", "int32", "int16",
      "int8", "uint64", "uint32", "uint16", "uint8", "int4", "uint4", "fp4", "int2", "uint2", "ternary",
      "binary", "int", "uint", "uintptr", "complex64", "complex128", "nf4", "fp6", "int6", "uint6",
      "int5", "uint5", "int3", "uint3"};
  const int id = static_cast<int>(dt);
  return id >= 0 && id < kNumDTypes ? names[id] : "unknown";
}

bool dtype_implemented_forward(DType dt) { return wb::dtype_on_path(static_cast<int32_t>(dt)); }

// src/weights/store.cpp:7-22: zeros when no values are given; the FormatNone encode runs on the GPU.
Status WeightStore::make(int rows, int cols, DType dt, const float* init_or_null, WeightStore* out) {
  if (!out || rows <= 0 || cols <= 0) return Status::Err(StatusCode::InvalidArgument, "weights: bad shape");
  if (!wb::dtype_on_path(static_cast<int32_t>(dt)))
    return Status::Err(StatusCode::Unsupported, std::string("weights: dtype ") + std::string(dtype_name(dt)) +
                                                    " is not served on the GPU by this library");
  out->rows = rows;
  out->cols = cols;
  out->bias.clear();
  out->dtype = dt;
  out->format = QuantFormat::None;
  const int64_t n = static_cast<int64_t>(rows) * cols;
  std::vector<float> scratch(static_cast<size_t>(n), 0.0f);
  if (init_or_null) std::memcpy(scratch.data(), init_or_null, scratch.size() * sizeof(float));
  if (dt == DType::Float32) {
    out->native.clear();
    out->f32 = std::move(scratch);
    out->scale = 1.0f;
    return Status::Ok();
  }
  int device = 0;
  if (auto s = wb::library_device(&device); !s.ok()) return from_wb(s);
  if (cudaSetDevice(device) != cudaSuccess) return Status::Err(StatusCode::Internal, "cudaSetDevice");
  const int64_t nb = wb::native_bytes(static_cast<wb::DType>(dt), n);
  float* w = nullptr;
  uint8_t* nat = nullptr;
  float* small = nullptr;
  wb::Status st = wb::cuda_status(cudaMalloc(&w, static_cast<size_t>(n) * 4), "cudaMalloc");
  if (st.ok()) st = wb::cuda_status(cudaMalloc(&nat, static_cast<size_t>(nb)), "cudaMalloc");
  if (st.ok()) st = wb::cuda_status(cudaMalloc(&small, 16), "cudaMalloc");
  if (st.ok())
    st = wb::cuda_status(cudaMemcpy(w, scratch.data(), static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice), "H2D");
  if (st.ok())
    st = wb::encode_native(static_cast<wb::DType>(dt), w, n, nat, small,
                           reinterpret_cast<unsigned int*>(small + 2), nullptr);
  float scale = 1.0f;
  if (st.ok()) {
    out->f32.clear();
    out->native.resize(static_cast<size_t>(nb));
    st = wb::cuda_status(cudaMemcpy(out->native.data(), nat, static_cast<size_t>(nb), cudaMemcpyDeviceToHost), "D2H");
  }
  if (st.ok()) st = wb::cuda_status(cudaMemcpy(&scale, small, sizeof(float), cudaMemcpyDeviceToHost), "D2H");
  for (void* p : {static_cast<void*>(w), static_cast<void*>(nat), static_cast<void*>(small)})
    if (p) cudaFree(p);
  if (!st.ok()) return from_wb(st);
  out->scale = scale;
  return Status::Ok();
}

// src/weights/store.cpp:42-70: decoded values (weight_at per element), on the GPU.
Status WeightStore::export_f32(float* dst) const {
  if (!dst) return invalid("weights: nil dst");
  if (format != QuantFormat::None) return Status::Err(StatusCode::Gap, "gap? export_f32 packed formats");
  if (auto st = payload_ok(*this); !st) return st;
  const int64_t n = static_cast<int64_t>(rows) * cols;
  if (n <= 0) return Status::Ok();
  if (dtype == DType::Float32) {
    std::memcpy(dst, f32.data(), static_cast<size_t>(n) * sizeof(float));
    return Status::Ok();
  }
  int device = 0;
  if (auto s = wb::library_device(&device); !s.ok()) return from_wb(s);
  wb::Status st = wb::cuda_status(cudaSetDevice(device), "cudaSetDevice");
  DevBufs b;
  uint8_t* nat = nullptr;
  float* out = nullptr;
  const size_t nb = native.size();
  if (st.ok()) st = b.get(&nat, nb);
  if (st.ok()) st = b.get(&out, static_cast<size_t>(n));
  if (st.ok()) st = wb::cuda_status(cudaMemcpy(nat, native.data(), nb, cudaMemcpyHostToDevice), "H2D");
  if (st.ok()) st = wb::decode_ref(static_cast<wb::DType>(dtype), nat, n, scale, out, nullptr);
  if (st.ok())
    st = wb::cuda_status(cudaMemcpy(dst, out, static_cast<size_t>(n) * sizeof(float), cudaMemcpyDeviceToHost), "D2H");
  return st.ok() ? Status::Ok() : from_wb(st);
}

// src/weights/native_codec.cpp:1080-1133: per element decode, float(double(v) - lr * dW),
// re-encode; Float32 masters take w -= float(lr * dW). One GPU pass over the payload.
Status WeightStore::apply_sgd(const double* dW, double lr) {
  if (!dW) return invalid("weights: ApplySGD nil dW");
  if (format != QuantFormat::None) return Status::Err(StatusCode::Gap, "gap? weights.ApplySGD packed quant formats");
  if (auto st = payload_ok(*this); !st) return st;
  const int64_t n = static_cast<int64_t>(rows) * cols;
  if (n <= 0) return Status::Ok();
  int device = 0;
  if (auto s = wb::library_device(&device); !s.ok()) return from_wb(s);
  wb::Status st = wb::cuda_status(cudaSetDevice(device), "cudaSetDevice");
  size_t bytes = 0;
  const void* host = payload_of(*this, &bytes);
  DevBufs b;
  uint8_t* pay = nullptr;
  double* dwd = nullptr;
  if (st.ok()) st = b.get(&pay, bytes);
  if (st.ok()) st = b.get(&dwd, static_cast<size_t>(n));
  if (st.ok()) st = wb::cuda_status(cudaMemcpy(pay, host, bytes, cudaMemcpyHostToDevice), "H2D");
  if (st.ok())
    st = wb::cuda_status(cudaMemcpy(dwd, dW, static_cast<size_t>(n) * sizeof(double), cudaMemcpyHostToDevice), "H2D");
  if (st.ok()) st = wb::apply_sgd_native(static_cast<wb::DType>(dtype), pay, n, scale, dwd, lr, nullptr);
  void* back = dtype == DType::Float32 ? static_cast<void*>(f32.data()) : static_cast<void*>(native.data());
  if (st.ok()) st = wb::cuda_status(cudaMemcpy(back, pay, bytes, cudaMemcpyDeviceToHost), "D2H");
  return st.ok() ? Status::Ok() : from_wb(st);
}

namespace cuda {

void resident_release(ResidentDense* r) {
  if (!r) return;
  drop_session(*r);
  drop_cell(*r);
}

} // namespace cuda

namespace dense {

bool dtype_supported_cuda_forward(DType dt) { return dtype_implemented_forward(dt); }

Status new_layer(int in_h, int out_h, Activation act, DType dt, const float* init_or_null, Layer* layer) {
  if (!layer) return invalid("null Layer");
  if (in_h <= 0 || out_h <= 0) return invalid("bad dims");
  if (!dtype_supported_cuda_forward(dt))
    return Status::Err(StatusCode::Unsupported, std::string("dense CUDA unsupported dtype ") + std::string(dtype_name(dt)));
  Layer L;
  L.input_height = in_h;
  L.output_height = out_h;
  L.activation = act;
  if (auto st = WeightStore::make(out_h, in_h, dt, init_or_null, &L.weights); !st) return st;
  *layer = std::move(L);
  return Status::Ok();
}

Status sync_gpu_from_weights(const Layer& layer, int batch) {
  if (batch <= 0) return invalid("bad batch");
  drop_session(layer.gpu);
  const WeightStore& W = layer.weights;
  const wb::WeightSrc src = source(W);
  wb::DenseSession* s = nullptr;
  const double* bias = W.bias.empty() ? nullptr : W.bias.data();
  wb::Status st = wb::session_mount_native(batch, layer.input_height, layer.output_height,
                                           static_cast<int32_t>(layer.activation), static_cast<int32_t>(W.dtype),
                                           src.native, src.native_len, W.scale, bias, W.bias.size(), &s);
  if (!st.ok()) return from_wb(st);
  layer.gpu.session = s;
  layer.gpu_valid = true;
  layer.gpu_batch = batch;
  return Status::Ok();
}

Status forward_f32(const Layer& layer, const TensorF32& input, TensorF32* pre, TensorF32* post) {
  if (!pre || !post) return invalid("dense: nil out");
  if (!dtype_supported_cuda_forward(layer.weights.dtype))
    return Status::Err(StatusCode::Unsupported,
                       std::string("dense CUDA unsupported dtype ") + std::string(dtype_name(layer.weights.dtype)));
  if (input.shape.size() != 2) return invalid("dense: input shape need [batch,in]");
  const int batch = static_cast<int>(input.shape[0]);
  const int in = layer.input_height;
  const int out = layer.output_height;
  if (batch <= 0 || input.data.size() != static_cast<std::size_t>(batch) * static_cast<std::size_t>(in) ||
      static_cast<int>(input.shape[1]) != in)
    return invalid("dense: input width mismatch");
  if (layer.weights.rows != out || layer.weights.cols != in) return invalid("dense: weight shape mismatch");
  if (!layer.gpu_valid || layer.gpu_batch != batch || !layer.gpu.session) {
    if (auto st = sync_gpu_from_weights(layer, batch); !st) return st;
  }
  *pre = TensorF32::zeros(batch, out);
  *post = TensorF32::zeros(batch, out);
  return from_wb(wb::session_execute(static_cast<wb::DenseSession*>(layer.gpu.session), input.data.data(),
                                     pre->data.data(), post->data.data()));
}

// src/layers/dense/dense.cpp:88-120.
Status backward_f32(const Layer& layer, const TensorF32& grad_out, const TensorF32& input, const TensorF32& pre,
                    TensorF32* grad_in, TensorF32* grad_w) {
  if (!grad_in || !grad_w) return invalid("dense: nil grad out");
  if (input.shape.size() != 2 || grad_out.shape.size() != 2 || pre.shape.size() != 2)
    return invalid("dense: bad shapes");
  const int batch = static_cast<int>(input.shape[0]);
  const int in = layer.input_height;
  const int out = layer.output_height;
  const size_t bi = static_cast<size_t>(batch > 0 ? batch : 0) * static_cast<size_t>(in);
  const size_t bo = static_cast<size_t>(batch > 0 ? batch : 0) * static_cast<size_t>(out);
  if (batch <= 0 || input.data.size() != bi || pre.data.size() != bo || grad_out.data.size() != bo ||
      static_cast<int>(input.shape[1]) != in || static_cast<int>(grad_out.shape[0]) != batch ||
      static_cast<int>(grad_out.shape[1]) != out || static_cast<int>(pre.shape[0]) != batch ||
      static_cast<int>(pre.shape[1]) != out)
    return invalid("dense: bwd shape mismatch");
  if (layer.weights.rows != out || layer.weights.cols != in) return invalid("dense: weight shape mismatch");
  *grad_in = TensorF32::zeros(batch, in);
  *grad_w = TensorF32::zeros(out, in);
  return run_backward(layer, batch, grad_out.data.data(), input.data.data(), pre.data.data(), false,
                      grad_in->data.data(), grad_w->data.data());
}

// src/layers/dense/dense.cpp:141-166: no act', pre unused (zeros).
Status linear_grad_in(const Layer& layer, const TensorF32& gy, const TensorF32& input, TensorF32* gx) {
  if (!gx || input.shape.size() != 2 || input.data.empty() || gy.data.empty())
    return invalid("dense: LinearGradIn input");
  const int batch = static_cast<int>(input.shape[0]);
  const int in = layer.input_height;
  const int out = layer.output_height;
  if (batch <= 0 || input.data.size() != static_cast<size_t>(batch) * static_cast<size_t>(in) ||
      static_cast<int>(input.shape[1]) != in)
    return invalid("dense: LinearGradIn shape");
  std::vector<float> projected;
  remap_len(gy.data, batch * out, &projected);
  std::vector<float> pre(static_cast<size_t>(batch) * out, 0.0f);
  *gx = TensorF32::zeros(batch, in);
  return run_backward(layer, batch, projected.data(), input.data.data(), pre.data(), true, gx->data.data(), nullptr);
}

// src/layers/dense/dense.cpp:168-190: the full backward with a resampled gy; only dW is kept.
Status grad_w_only(const Layer& layer, const TensorF32& gy, const TensorF32& input, const TensorF32& pre,
                   TensorF32* dw) {
  if (!dw || input.shape.size() != 2 || gy.data.empty()) return invalid("dense: GradWOnly input");
  const int batch = static_cast<int>(input.shape[0]);
  const int in = layer.input_height;
  const int out = layer.output_height;
  if (batch <= 0 || input.data.size() != static_cast<size_t>(batch) * static_cast<size_t>(in))
    return invalid("dense: GradWOnly shape");
  TensorF32 projected;
  projected.shape = {batch, out};
  remap_len(gy.data, batch * out, &projected.data);
  TensorF32 use_pre = pre;
  if (use_pre.data.size() < static_cast<size_t>(batch) * static_cast<size_t>(out) || use_pre.shape.size() != 2)
    use_pre = TensorF32::zeros(batch, out);
  TensorF32 gx;
  return backward_f32(layer, projected, input, use_pre, &gx, dw);
}

// src/layers/dense/dense.cpp:192-209.
Status apply_grad_sgd(Layer* layer, const TensorF32& dW, double lr) {
  if (!layer) return invalid("dense: nil SGD layer");
  const int64_t n = static_cast<int64_t>(layer->weights.rows) * layer->weights.cols;
  if (static_cast<int64_t>(dW.data.size()) < n) return invalid("dense: dW short");
  std::vector<double> buf(dW.data.begin(), dW.data.begin() + n);
  if (auto st = layer->weights.apply_sgd(buf.data(), lr); !st) return st;
  layer->invalidate_gpu();
  return Status::Ok();
}

} // namespace dense

namespace swiglu {

Status validate(const Config& cfg) {
  if (cfg.input_dim <= 0 || cfg.intermediate_dim <= 0)
    return invalid("swiglu: need InputDim>0 and IntermediateDim>0");
  return Status::Ok();
}

Config default_ffn(int d_model) {
  int inter = (d_model * 8) / 3;
  inter = (inter + 7) / 8 * 8;
  if (inter < d_model) inter = d_model * 2;
  return Config{d_model, inter};
}

Status new_configured(const Config& cfg, DType dt, const float* gate_init, const float* up_init,
                      const float* down_init, Layer* out) {
  if (!out) return invalid("swiglu: nil out");
  if (auto st = validate(cfg); !st) return st;
  const int in = cfg.input_dim, inter = cfg.intermediate_dim;
  Layer layer;
  layer.cfg = cfg;
  if (auto st = dense::new_layer(in, inter, Activation::Linear, dt, gate_init, &layer.Gate); !st)
    return Status::Err(st.code, std::string("swiglu Gate: ") + st.message);
  if (auto st = dense::new_layer(in, inter, Activation::Linear, dt, up_init, &layer.Up); !st)
    return Status::Err(st.code, std::string("swiglu Up: ") + st.message);
  if (auto st = dense::new_layer(inter, in, Activation::Linear, dt, down_init, &layer.Down); !st)
    return Status::Err(st.code, std::string("swiglu Down: ") + st.message);
  *out = std::move(layer);
  return Status::Ok();
}

Status forward(Layer& layer, const TensorF32& input, TensorF32* pre, TensorF32* post) {
  if (!pre || !post) return invalid("swiglu: nil pre/post");
  if (auto st = validate(layer.cfg); !st) return st;
  // layout (src/layers/swiglu/swiglu.cpp:18-45)
  if (input.data.empty()) return invalid("swiglu: empty input");
  const int in = layer.cfg.input_dim, inter = layer.cfg.intermediate_dim;
  int batch = 1, seq = 1;
  if (input.shape.size() == 2) {
    batch = static_cast<int>(input.shape[0]);
    if (static_cast<int>(input.shape[1]) != in) return invalid("swiglu: width != InputDim");
  } else if (input.shape.size() == 3) {
    batch = static_cast<int>(input.shape[0]);
    seq = static_cast<int>(input.shape[1]);
    if (static_cast<int>(input.shape[2]) != in) return invalid("swiglu: last dim != InputDim");
  } else {
    return invalid("swiglu: need [batch,in] or [batch,seq,in]");
  }
  if (batch <= 0 || seq <= 0) return invalid("swiglu: bad batch/seq");
  const int bs = batch * seq;
  if (static_cast<int>(input.data.size()) < bs * in) return invalid("swiglu: short data");
  dense::Layer* parts[3] = {&layer.Gate, &layer.Up, &layer.Down};
  const DType dt = layer.Gate.weights.dtype;
  for (dense::Layer* p : parts) {
    if (p->weights.dtype != dt) return Status::Err(StatusCode::Unsupported, "swiglu: Gate, Up and Down differ in dtype");
    if (!dense::dtype_supported_cuda_forward(p->weights.dtype))
      return Status::Err(StatusCode::Unsupported, std::string("dense CUDA unsupported dtype ") +
                                                      std::string(dtype_name(p->weights.dtype)));
  }
  if (layer.Gate.weights.rows != inter || layer.Gate.weights.cols != in || layer.Up.weights.rows != inter ||
      layer.Up.weights.cols != in || layer.Down.weights.rows != in || layer.Down.weights.cols != inter)
    return invalid("swiglu: weight shape mismatch");
  cuda::ResidentDense& r = layer.Gate.gpu;
  bool valid = r.cell_kind == 1 && r.cell;
  for (dense::Layer* p : parts) valid = valid && p->gpu_valid;
  if (!valid) {
    drop_cell(r);
    auto* h = new SwigluHolder();
    int device = 0;
    wb::Status st = wb::library_device(&device);
    if (st.ok()) st = wb::cuda_status(cudaSetDevice(device), "cudaSetDevice");
    if (st.ok()) st = wb::cuda_status(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking), "stream");
    const wb::WeightSrc w[3] = {source(layer.Gate.weights), source(layer.Up.weights), source(layer.Down.weights)};
    if (st.ok()) st = wb::swiglu_mount_src(device, in, inter, static_cast<wb::DType>(dt), w, &h->cell, h->stream);
    if (!st.ok()) {
      delete h;
      return from_wb(st);
    }
    r.cell = h;
    r.cell_kind = 1;
    for (dense::Layer* p : parts) {  // a later dense forward of one of them remounts its own session
      drop_session(p->gpu);
      p->gpu_valid = true;
      p->gpu_batch = -1;
    }
  }
  auto* h = static_cast<SwigluHolder*>(r.cell);
  if (cudaSetDevice(h->cell.device) != cudaSuccess) return Status::Err(StatusCode::Internal, "cudaSetDevice");
  if (h->rows < bs) {
    wb::Status st = grow(&h->x, static_cast<size_t>(bs) * in);
    if (st.ok()) st = grow(&h->h, static_cast<size_t>(bs) * inter);
    if (st.ok()) st = grow(&h->y, static_cast<size_t>(bs) * in);
    if (!st.ok()) return from_wb(st);
    h->rows = bs;
  }
  pre->shape = seq == 1 ? std::vector<int64_t>{batch, inter} : std::vector<int64_t>{batch, seq, inter};
  post->shape = seq == 1 ? std::vector<int64_t>{batch, in} : std::vector<int64_t>{batch, seq, in};
  pre->data.assign(static_cast<size_t>(bs) * inter, 0.0f);
  post->data.assign(static_cast<size_t>(bs) * in, 0.0f);
  wb::Status st = wb::cuda_status(cudaMemcpyAsync(h->x, input.data.data(), static_cast<size_t>(bs) * in * 4,
                                                  cudaMemcpyHostToDevice, h->stream), "H2D x");
  if (st.ok()) st = wb::swiglu_forward_device(&h->cell, bs, h->x, h->h, h->y, h->stream, false);
  if (st.ok())
    st = wb::cuda_status(cudaMemcpyAsync(pre->data.data(), h->h, static_cast<size_t>(bs) * inter * 4,
                                         cudaMemcpyDeviceToHost, h->stream), "D2H h");
  if (st.ok())
    st = wb::cuda_status(cudaMemcpyAsync(post->data.data(), h->y, static_cast<size_t>(bs) * in * 4,
                                         cudaMemcpyDeviceToHost, h->stream), "D2H y");
  if (st.ok()) st = wb::cuda_status(cudaStreamSynchronize(h->stream), "swiglu sync");
  for (wb::DenseIO* io : {&h->cell.io_gate, &h->cell.io_up, &h->cell.io_down})
    if (st.ok()) st = wb::check_pipeline_error(*io, h->stream);
  return from_wb(st);
}

} // namespace swiglu

namespace mha {

double Config::scale() const {
  if (scale_override > 0) return scale_override;
  return 1.0 / std::sqrt(static_cast<double>(head_dim));
}

// src/layers/mha/mha.cpp:57-85
Status validate(Config* cfg) {
  if (!cfg) return invalid("mha: nil config");
  if (cfg->d_model <= 0 || cfg->num_heads <= 0) return invalid("mha: need DModel>0 and NumHeads>0");
  if (cfg->head_dim <= 0) {
    if (cfg->d_model % cfg->num_heads != 0) return invalid("mha: HeadDim unset and DModel%NumHeads!=0");
    cfg->head_dim = cfg->d_model / cfg->num_heads;
  }
  if (cfg->num_kv_heads <= 0) cfg->num_kv_heads = cfg->num_heads;
  if (cfg->num_heads % cfg->num_kv_heads != 0) return invalid("mha: NumHeads not divisible by NumKVHeads");
  if (cfg->max_seq_len <= 0) cfg->max_seq_len = 512;
  if (cfg->mask == MaskKind::Unspecified) {
    cfg->mask = MaskKind::Causal;
    cfg->causal = true;
  }
  if (cfg->mask == MaskKind::Causal) cfg->causal = true;
  if (cfg->rope_theta <= 0) cfg->rope_theta = 10000;
  if (cfg->softmax != SoftmaxKind::Standard && cfg->softmax != SoftmaxKind::Sigmoid)
    return invalid("mha: unknown Softmax");
  return Status::Ok();
}

Config decoder_causal(int d_model, int num_heads, int num_kv_heads) {
  Config c;
  c.d_model = d_model;
  c.num_heads = num_heads;
  c.num_kv_heads = num_kv_heads;
  c.mask = MaskKind::Causal;
  c.pos = PosKind::RoPE;
  c.mode = AttnMode::Self;
  c.causal = true;
  return c;
}

Status new_configured(const Config& cfg_in, DType dt, const float* q_init, const float* k_init,
                      const float* v_init, const float* o_init, Layer* out) {
  if (!out) return invalid("mha: nil out");
  Config cfg = cfg_in;
  if (auto st = validate(&cfg); !st) return st;
  const int d = cfg.d_model, q_dim = cfg.q_dim(), kv_dim = cfg.kv_dim();
  Layer layer;
  layer.cfg = cfg;
  if (auto st = dense::new_layer(d, q_dim, Activation::Linear, dt, q_init, &layer.Q); !st)
    return Status::Err(st.code, std::string("mha Q: ") + st.message);
  if (auto st = dense::new_layer(d, kv_dim, Activation::Linear, dt, k_init, &layer.K); !st)
    return Status::Err(st.code, std::string("mha K: ") + st.message);
  if (auto st = dense::new_layer(d, kv_dim, Activation::Linear, dt, v_init, &layer.V); !st)
    return Status::Err(st.code, std::string("mha V: ") + st.message);
  if (auto st = dense::new_layer(q_dim, d, Activation::Linear, dt, o_init, &layer.O); !st)
    return Status::Err(st.code, std::string("mha O: ") + st.message);
  *out = std::move(layer);
  return Status::Ok();
}

Status forward(Layer& layer, const TensorF32& input, TensorF32* pre, TensorF32* post) {
  if (!pre || !post) return invalid("mha: nil pre/post");
  Config cfg = layer.cfg;
  if (auto st = validate(&cfg); !st) return st;
  if (cfg.mode != AttnMode::Self) return Status::Gap("mha forward: ModeCross not in baseline");
  // layout (src/layers/mha/mha.cpp:18-46)
  if (input.data.empty()) return invalid("mha: empty input");
  const int d = cfg.d_model;
  int batch = 1, seq = 0;
  if (input.shape.size() == 3) {
    batch = static_cast<int>(input.shape[0]);
    seq = static_cast<int>(input.shape[1]);
    if (static_cast<int>(input.shape[2]) != d) return invalid("mha: last dim != d_model");
  } else if (input.shape.size() == 2) {
    if (static_cast<int>(input.shape[1]) != d) return invalid("mha: width != d_model");
    seq = static_cast<int>(input.shape[0]);
  } else {
    return invalid("mha: need [batch,seq,d] or [seq,d]");
  }
  if (batch <= 0 || seq <= 0) return invalid("mha: bad batch/seq");
  const int bs = batch * seq;
  if (static_cast<int>(input.data.size()) < bs * d) return invalid("mha: short data");
  if (seq > cfg.max_seq_len) return invalid("mha: seq > MaxSeqLen");
  dense::Layer* parts[4] = {&layer.Q, &layer.K, &layer.V, &layer.O};
  const DType dt = layer.Q.weights.dtype;
  for (dense::Layer* p : parts) {
    if (p->weights.dtype != dt) return Status::Err(StatusCode::Unsupported, "mha: Q, K, V and O differ in dtype");
    if (!dense::dtype_supported_cuda_forward(p->weights.dtype))
      return Status::Err(StatusCode::Unsupported, std::string("dense CUDA unsupported dtype ") +
                                                      std::string(dtype_name(p->weights.dtype)));
  }
  const int qd = cfg.q_dim(), kvd = cfg.kv_dim();
  if (layer.Q.weights.rows != qd || layer.Q.weights.cols != d || layer.K.weights.rows != kvd ||
      layer.K.weights.cols != d || layer.V.weights.rows != kvd || layer.V.weights.cols != d ||
      layer.O.weights.rows != d || layer.O.weights.cols != qd)
    return invalid("mha: weight shape mismatch");
  cuda::ResidentDense& r = layer.Q.gpu;
  bool valid = r.cell_kind == 2 && r.cell;
  for (dense::Layer* p : parts) valid = valid && p->gpu_valid;
  if (valid) {  // the cell was mounted for this configuration
    const wb::MhaConfig& g = static_cast<MhaHolder*>(r.cell)->cell.cfg;
    valid = g.mask == static_cast<int>(cfg.mask) && g.pos == static_cast<int>(cfg.pos) &&
            g.softmax == static_cast<int>(cfg.softmax) && g.max_seq_len == cfg.max_seq_len &&
            g.window == cfg.window && g.prefix_len == cfg.prefix_len &&
            g.window_causal == static_cast<int>(cfg.window_causal || cfg.causal) &&
            g.rope_theta == cfg.rope_theta && g.scale_override == cfg.scale_override;
  }
  if (!valid) {
    drop_cell(r);
    auto* h = new MhaHolder();
    wb::MhaConfig mc;
    mc.d_model = d;
    mc.num_heads = cfg.num_heads;
    mc.num_kv_heads = cfg.num_kv_heads;
    mc.head_dim = cfg.head_dim;
    mc.max_seq_len = cfg.max_seq_len;
    mc.mask = static_cast<int>(cfg.mask);
    mc.pos = static_cast<int>(cfg.pos);
    mc.softmax = static_cast<int>(cfg.softmax);
    mc.window = cfg.window;
    mc.prefix_len = cfg.prefix_len;
    mc.window_causal = (cfg.window_causal || cfg.causal) ? 1 : 0;
    mc.rope_theta = cfg.rope_theta;
    mc.scale_override = cfg.scale_override;
    int device = 0;
    wb::Status st = wb::library_device(&device);
    if (st.ok()) st = wb::cuda_status(cudaSetDevice(device), "cudaSetDevice");
    if (st.ok()) st = wb::cuda_status(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking), "stream");
    const wb::WeightSrc w[4] = {source(layer.Q.weights), source(layer.K.weights), source(layer.V.weights),
                                source(layer.O.weights)};
    if (st.ok()) st = wb::mha_mount_src(device, mc, static_cast<wb::DType>(dt), w, &h->cell, h->stream);
    if (!st.ok()) {
      delete h;
      return from_wb(st);
    }
    r.cell = h;
    r.cell_kind = 2;
    for (dense::Layer* p : parts) {
      drop_session(p->gpu);
      p->gpu_valid = true;
      p->gpu_batch = -1;
    }
  }
  auto* h = static_cast<MhaHolder*>(r.cell);
  if (cudaSetDevice(h->cell.device) != cudaSuccess) return Status::Err(StatusCode::Internal, "cudaSetDevice");
  if (h->rows < bs) {
    wb::Status st = grow(&h->x, static_cast<size_t>(bs) * d);
    if (st.ok()) st = grow(&h->attn, static_cast<size_t>(bs) * qd);
    if (st.ok()) st = grow(&h->y, static_cast<size_t>(bs) * d);
    if (!st.ok()) return from_wb(st);
    h->rows = bs;
  }
  pre->shape = {batch, seq, qd};
  post->shape = {batch, seq, d};
  pre->data.assign(static_cast<size_t>(bs) * qd, 0.0f);
  post->data.assign(static_cast<size_t>(bs) * d, 0.0f);
  wb::Status st = wb::cuda_status(cudaMemcpyAsync(h->x, input.data.data(), static_cast<size_t>(bs) * d * 4,
                                                  cudaMemcpyHostToDevice, h->stream), "H2D x");
  if (st.ok()) st = wb::mha_forward_device(&h->cell, batch, seq, h->x, h->attn, h->y, h->stream);
  if (st.ok())
    st = wb::cuda_status(cudaMemcpyAsync(pre->data.data(), h->attn, static_cast<size_t>(bs) * qd * 4,
                                         cudaMemcpyDeviceToHost, h->stream), "D2H attn");
  if (st.ok())
    st = wb::cuda_status(cudaMemcpyAsync(post->data.data(), h->y, static_cast<size_t>(bs) * d * 4,
                                         cudaMemcpyDeviceToHost, h->stream), "D2H y");
  if (st.ok()) st = wb::cuda_status(cudaStreamSynchronize(h->stream), "mha sync");
  for (wb::DenseIO* io : {&h->cell.io_q, &h->cell.io_k, &h->cell.io_v, &h->cell.io_o})
    if (st.ok()) st = wb::check_pipeline_error(*io, h->stream);
  return from_wb(st);
}

} // namespace mha

} // namespace welvet
