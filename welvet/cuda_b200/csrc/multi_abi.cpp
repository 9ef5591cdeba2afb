// multi_abi.cpp -- extern "C" entry points of the multi-GPU runtime (comm.hpp, sharded.hpp).
// No counterpart in the reference, which runs on device 0 only (src/cuda/device.cpp:40-61).
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

} // namespace

extern "C" {

welvet_status welvet_b200_comm_unique_id(uint8_t* id128) {
  return guarded([&] { return wb::comm_unique_id(id128); });
}

welvet_status welvet_b200_comm_create(const uint8_t* id128, int32_t nranks, int32_t rank, int32_t device,
                                      welvet_b200_comm** out) {
  return guarded([&] {
    if (!out) return wb::Status::Invalid("null communicator out");
    *out = nullptr;
    wb::Comm* c = nullptr;
    WB_TRY(wb::comm_create(id128, nranks, rank, device, &c));
    *out = new welvet_b200_comm{c};
    return wb::Status::Ok();
  });
}

void welvet_b200_comm_release(welvet_b200_comm* c) {
  if (!c) return;
  delete c->c;
  delete c;
}

welvet_status welvet_b200_shard_rows(int32_t rows, int32_t nranks, int32_t rank, int32_t* begin, int32_t* end) {
  return guarded([&] {
    if (!begin || !end) return wb::Status::Invalid("null shard range out");
    if (rows <= 0 || nranks <= 0 || rank < 0 || rank >= nranks) return wb::Status::Invalid("shard_rows: bad arguments");
    int b = 0, e = 0;
    wb::shard_rows(rows, nranks, rank, &b, &e);
    *begin = b;
    *end = e;
    return wb::Status::Ok();
  });
}

welvet_status welvet_b200_stage_plan(int32_t cells, int32_t layers_per_cell, int32_t nranks, int32_t rank,
                                     int32_t* hop_begin, int32_t* hop_end) {
  return guarded([&] {
    if (!hop_begin || !hop_end) return wb::Status::Invalid("null stage range out");
    if (cells <= 0 || layers_per_cell <= 0 || nranks <= 0 || rank < 0 || rank >= nranks)
      return wb::Status::Invalid("stage_plan: bad arguments");
    int b = 0, e = 0;
    wb::stage_plan(cells, layers_per_cell, nranks, rank, &b, &e);
    *hop_begin = b;
    *hop_end = e;
    return wb::Status::Ok();
  });
}

welvet_status welvet_b200_sharded_dense_mount(welvet_b200_comm* comm, int32_t batch, int32_t in, int32_t out,
                                              int32_t act, int32_t dtype, const float* W_rows,
                                              int32_t weights_on_device, const double* bias, size_t bias_len,
                                              int32_t mode, welvet_b200_sharded_dense** s_out) {
  return guarded([&] {
    if (!comm || !comm->c || !s_out) return wb::Status::Invalid("null sharded mount args");
    *s_out = nullptr;
    wb::ShardedDense* s = nullptr;
    WB_TRY(wb::sharded_mount(comm->c, batch, in, out, act, static_cast<wb::DType>(dtype), W_rows,
                             weights_on_device != 0, bias, bias_len, static_cast<wb::GatherMode>(mode), &s));
    *s_out = new welvet_b200_sharded_dense{s};
    return wb::Status::Ok();
  });
}

welvet_status welvet_b200_sharded_dense_execute_device(welvet_b200_sharded_dense* s, const float* x_dev,
                                                       void* stream, const float** post_dev,
                                                       const float** pre_dev) {
  return guarded([&] {
    if (!s || !s->s) return wb::Status::Invalid("null sharded session");
    return wb::sharded_execute_device(s->s, x_dev, static_cast<cudaStream_t>(stream), post_dev, pre_dev);
  });
}

welvet_status welvet_b200_sharded_dense_execute(welvet_b200_sharded_dense* s, const float* x, float* pre,
                                                float* post) {
  return guarded([&] {
    if (!s || !s->s) return wb::Status::Invalid("null sharded session");
    return wb::sharded_execute(s->s, x, pre, post);
  });
}

welvet_status welvet_b200_sharded_dense_check_error(welvet_b200_sharded_dense* s, void* stream) {
  return guarded([&] {
    if (!s || !s->s) return wb::Status::Invalid("null sharded session");
    return wb::sharded_check_error(s->s, static_cast<cudaStream_t>(stream));
  });
}

welvet_status welvet_b200_sharded_dense_rows(welvet_b200_sharded_dense* s, int32_t* row_begin, int32_t* row_end) {
  return guarded([&] {
    if (!s || !s->s || !row_begin || !row_end) return wb::Status::Invalid("null sharded rows args");
    *row_begin = s->s->row_begin;
    *row_end = s->s->row_end;
    return wb::Status::Ok();
  });
}

void welvet_b200_sharded_dense_release(welvet_b200_sharded_dense* s) {
  if (!s) return;
  delete s->s;
  delete s;
}

welvet_status welvet_b200_volume_pipeline_forward_device(welvet_b200_volume* v, welvet_b200_comm* comm,
                                                         int32_t hop_begin, int32_t hop_end, int32_t rows,
                                                         const float* x_dev, int32_t stage_in_width,
                                                         int32_t micro, float* out_dev, int32_t out_width,
                                                         void* stream) {
  return guarded([&] {
    if (!v || !v->v || !comm || !comm->c) return wb::Status::Invalid("null pipeline args");
    return wb::volume_pipeline_forward(v->v, comm->c, hop_begin, hop_end, rows, x_dev, stage_in_width, micro,
                                       out_dev, out_width, static_cast<cudaStream_t>(stream));
  });
}

int32_t welvet_b200_nccl_available(void) { return wb::nccl_available() ? 1 : 0; }

} // extern "C"
