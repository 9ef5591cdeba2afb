// volume_abi.cpp -- extern "C" entry points of the device-resident volume (volume.hpp).
#include "abi_handles.hpp"

#include <cstring>
#include <exception>
#include <new>
#include <string>

namespace {

welvet_status to_c(const wb::Status& st) {
  welvet_status out{};
  out.code = static_cast<int32_t>(st.code);
  std::strncpy(out.message, st.message.c_str(), sizeof(out.message) - 1);
  out.message[sizeof(out.message) - 1] = '\0';
  return out;
}

template <typename F>
welvet_status guarded(F&& f) {
  try {
    return to_c(f());
  } catch (const std::bad_alloc&) {
    return to_c(wb::Status::Internal("host allocation failed"));
  } catch (const std::exception& e) {
    return to_c(wb::Status::Internal(e.what()));
  } catch (...) {
    return to_c(wb::Status::Internal("unknown exception"));
  }
}

wb::Status coord(welvet_b200_volume* h, int32_t z, int32_t y, int32_t x, int32_t l, int* idx) {
  if (!h || !h->v) return wb::Status::Invalid("volume: nil handle");
  *idx = wb::volume_index(*h->v, z, y, x, l);
  if (*idx < 0) {
    return wb::Status::Invalid("architecture: bad coord z=" + std::to_string(z) + " y=" + std::to_string(y) +
                               " x=" + std::to_string(x) + " l=" + std::to_string(l));
  }
  return wb::Status::Ok();
}

wb::Status dtype_ok(int32_t dtype) {
  if (!wb::dtype_on_path(dtype))
    return wb::Status::Unsupported("volume cell CUDA (b200) unsupported dtype id " + std::to_string(dtype));
  return wb::Status::Ok();
}

} // namespace

extern "C" {

welvet_status welvet_b200_volume_create(int32_t depth, int32_t rows, int32_t cols, int32_t layers_per_cell,
                                        welvet_b200_volume** out) {
  return guarded([&] {
    if (!out) return wb::Status::Invalid("volume: nil out");
    wb::Volume* v = nullptr;
    WB_TRY(wb::volume_create(depth, rows, cols, layers_per_cell, &v));
    *out = new welvet_b200_volume{v};
    return wb::Status::Ok();
  });
}

welvet_status welvet_b200_volume_bind_dense(welvet_b200_volume* h, int32_t z, int32_t y, int32_t x, int32_t l,
                                            int32_t in, int32_t out, int32_t act, int32_t dtype, const float* W,
                                            const double* bias, size_t bias_len, int32_t weights_on_device) {
  return guarded([&] {
    int idx = 0;
    WB_TRY(coord(h, z, y, x, l, &idx));
    WB_TRY(dtype_ok(dtype));
    if (!W) return wb::Status::Invalid("dense: nil weights");
    return wb::volume_bind_dense(h->v, idx, in, out, act, static_cast<wb::DType>(dtype), W, weights_on_device != 0,
                                 bias, bias_len);
  });
}

welvet_status welvet_b200_volume_bind_dense_native(welvet_b200_volume* h, int32_t z, int32_t y, int32_t x,
                                                   int32_t l, int32_t in, int32_t out, int32_t act, int32_t dtype,
                                                   const uint8_t* native, size_t native_len, float scale,
                                                   const double* bias, size_t bias_len) {
  return guarded([&] {
    int idx = 0;
    WB_TRY(coord(h, z, y, x, l, &idx));
    WB_TRY(dtype_ok(dtype));
    return wb::volume_bind_dense_native(h->v, idx, in, out, act, static_cast<wb::DType>(dtype), native, native_len,
                                        scale, bias, bias_len);
  });
}

welvet_status welvet_b200_volume_bind_swiglu(welvet_b200_volume* h, int32_t z, int32_t y, int32_t x, int32_t l,
                                             int32_t input_dim, int32_t intermediate_dim, int32_t dtype,
                                             const float* Gate, const float* Up, const float* Down,
                                             int32_t weights_on_device) {
  return guarded([&] {
    int idx = 0;
    WB_TRY(coord(h, z, y, x, l, &idx));
    WB_TRY(dtype_ok(dtype));
    if (!Gate || !Up || !Down) return wb::Status::Invalid("swiglu: invalid argument");
    return wb::volume_bind_swiglu(h->v, idx, input_dim, intermediate_dim, static_cast<wb::DType>(dtype), Gate, Up,
                                  Down, weights_on_device != 0);
  });
}

welvet_status welvet_b200_volume_bind_mha(welvet_b200_volume* h, int32_t z, int32_t y, int32_t x, int32_t l,
                                          int32_t d_model, int32_t num_heads, int32_t num_kv_heads,
                                          int32_t head_dim, int32_t max_seq_len, int32_t mask, int32_t pos,
                                          int32_t seq, int32_t dtype, const float* Q, const float* K, const float* V,
                                          const float* O, int32_t weights_on_device) {
  return guarded([&] {
    int idx = 0;
    WB_TRY(coord(h, z, y, x, l, &idx));
    WB_TRY(dtype_ok(dtype));
    if (!Q || !K || !V || !O) return wb::Status::Invalid("mha: invalid argument");
    wb::MhaConfig cfg;
    cfg.d_model = d_model;
    cfg.num_heads = num_heads;
    cfg.num_kv_heads = num_kv_heads;
    cfg.head_dim = head_dim;
    cfg.max_seq_len = max_seq_len;
    cfg.mask = mask;
    cfg.pos = pos;
    return wb::volume_bind_mha(h->v, idx, cfg, seq, static_cast<wb::DType>(dtype), Q, K, V, O, weights_on_device != 0);
  });
}

welvet_status welvet_b200_volume_bind_rmsnorm(welvet_b200_volume* h, int32_t z, int32_t y, int32_t x, int32_t l,
                                              int32_t dim, double eps, int32_t dtype, const float* gamma) {
  return guarded([&] {
    int idx = 0;
    WB_TRY(coord(h, z, y, x, l, &idx));
    WB_TRY(dtype_ok(dtype));
    return wb::volume_bind_rmsnorm(h->v, idx, dim, eps, static_cast<wb::DType>(dtype), gamma);
  });
}

welvet_status welvet_b200_volume_set_remote_link(welvet_b200_volume* h, int32_t z, int32_t y, int32_t x, int32_t l,
                                                 int32_t tz, int32_t ty, int32_t tx, int32_t tl) {
  return guarded([&] {
    int idx = 0;
    WB_TRY(coord(h, z, y, x, l, &idx));
    const int t = wb::volume_index(*h->v, tz, ty, tx, tl);
    return wb::volume_set_remote_link(h->v, idx, t);
  });
}

welvet_status welvet_b200_volume_set_disabled(welvet_b200_volume* h, int32_t z, int32_t y, int32_t x, int32_t l,
                                              int32_t disabled) {
  return guarded([&] {
    int idx = 0;
    WB_TRY(coord(h, z, y, x, l, &idx));
    return wb::volume_set_disabled(h->v, idx, disabled != 0);
  });
}

int32_t welvet_b200_volume_hops(welvet_b200_volume* h) {
  return (h && h->v) ? wb::volume_hops(*h->v) : 0;
}

welvet_status welvet_b200_volume_forward_device(welvet_b200_volume* h, int32_t rows, const float* x_dev,
                                                int32_t in_width, int32_t hop_begin, int32_t hop_end, float* out_dev,
                                                int32_t* out_width, void* stream) {
  return guarded([&] {
    if (!h || !h->v) return wb::Status::Invalid("volume: nil handle");
    int ow = 0;
    WB_TRY(wb::volume_forward_device(h->v, rows, x_dev, in_width, hop_begin, hop_end, out_dev, &ow,
                                     static_cast<cudaStream_t>(stream)));
    if (out_width) *out_width = ow;
    return wb::Status::Ok();
  });
}

welvet_status welvet_b200_volume_forward_f32(welvet_b200_volume* h, int32_t rows, const float* x_host, int32_t in_width,
                                             float* out_host, size_t out_cap, int32_t* out_width) {
  return guarded([&] {
    if (!h || !h->v || !x_host || !out_host || rows <= 0 || in_width <= 0)
      return wb::Status::Invalid("runtime.forward: invalid argument");
    wb::Volume* v = h->v;
    WB_CUDA(cudaSetDevice(v->device));
    struct Buf {
      void* p = nullptr;
      ~Buf() { if (p) cudaFree(p); }
    } xb, ob;
    const size_t xbytes = static_cast<size_t>(rows) * in_width * 4;
    WB_CUDA(cudaMalloc(&xb.p, xbytes));
    WB_CUDA(cudaMemcpyAsync(xb.p, x_host, xbytes, cudaMemcpyHostToDevice, v->stream));
    int ow = 0;
    WB_TRY(wb::volume_forward_device(v, rows, static_cast<float*>(xb.p), in_width, 0, -1, nullptr, &ow, v->stream));
    if (static_cast<size_t>(ow) * static_cast<size_t>(rows) > out_cap)
      return wb::Status::Invalid("runtime.forward: output buffer too small");
    // the last executed cell's post is the output (src/runtime/forward.cpp:153)
    int last = -1;
    for (int i = wb::volume_hops(*v) - 1; i >= 0 && last < 0; --i)
      if (!v->cells[static_cast<size_t>(i)].disabled && v->cells[static_cast<size_t>(i)].op != wb::OpKind::None) last = i;
    WB_CUDA(cudaMemcpyAsync(out_host, v->cells[static_cast<size_t>(last)].post, static_cast<size_t>(rows) * ow * 4,
                            cudaMemcpyDeviceToHost, v->stream));
    WB_CUDA(cudaStreamSynchronize(v->stream));
    for (auto& c : v->cells) WB_TRY(wb::check_pipeline_error(c.io, v->stream));
    if (out_width) *out_width = ow;
    return wb::Status::Ok();
  });
}

welvet_status welvet_b200_volume_cell_outputs(welvet_b200_volume* h, int32_t z, int32_t y, int32_t x, int32_t l,
                                              const float** pre, int32_t* pre_width, const float** post,
                                              int32_t* post_width) {
  return guarded([&] {
    int idx = 0;
    WB_TRY(coord(h, z, y, x, l, &idx));
    int pw = 0, ow = 0;
    WB_TRY(wb::volume_cell_outputs(h->v, idx, pre, &pw, post, &ow));
    if (pre_width) *pre_width = pw;
    if (post_width) *post_width = ow;
    return wb::Status::Ok();
  });
}

void welvet_b200_volume_release(welvet_b200_volume* h) {
  if (!h) return;
  delete h->v;
  delete h;
}

} // extern "C"
