// train.cpp -- the reference's Dense training leaf (welvet_dense_normalbp_f32,
// src/interop/c_abi.cpp:119-184) on the GPU: mount, forward, MSE from a target or the given
// output gradient, backward, optional SGD on the packed store, export of the updated weights.
// Every step runs on the device; the host only moves the caller's buffers.
#include "train.hpp"

#include "backward.hpp"
#include "codec.hpp"

#include <string>
#include <vector>

namespace wb {

namespace {

struct Scratch {  // device buffers freed on every exit path
  std::vector<void*> p;
  ~Scratch() {
    for (void* q : p)
      if (q) cudaFree(q);
  }
  template <typename T>
  Status get(T** out, size_t n) {
    void* q = nullptr;
    WB_CUDA(cudaMalloc(&q, n * sizeof(T) > 0 ? n * sizeof(T) : 16));
    p.push_back(q);
    *out = static_cast<T*>(q);
    return Status::Ok();
  }
};

} // namespace

Status dense_normalbp(int batch, int in, int out, int act, int32_t dtype, const float* W_init, const double* bias,
                      size_t bias_len, const float* x, const float* grad_or_target, bool use_target, double lr,
                      float* pre, float* post, float* dX, float* dW, float* W_after, double* loss) {
  if (batch <= 0 || in <= 0 || out <= 0 || !W_init || !x || !grad_or_target || !pre || !post || !dX || !dW ||
      !W_after || !loss)
    return Status::Invalid("invalid argument");
  if (dtype < 0 || dtype >= 34) return Status::Invalid("bad dtype " + std::to_string(dtype));
  if (!dtype_on_path(dtype))
    return Status::Unsupported(std::string("dense CUDA (b200) unsupported dtype id ") + std::to_string(dtype));
  if (!activation_valid(act)) return Status::Invalid("bad activation");
  int device = 0;
  WB_TRY(library_device(&device));
  WB_CUDA(cudaSetDevice(device));
  cudaStream_t st = nullptr;
  WB_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  } guard{st};

  const DType dt = static_cast<DType>(dtype);
  WeightStore store;
  DeviceDense dev;
  WB_TRY(mount_dense(device, out, in, dt, act, W_init, false, bias, bias_len, &store, &dev, st, batch));
  DenseIO io;
  struct IoGuard {
    DenseIO& io;
    ~IoGuard() { io.release(); }
  } ioguard{io};
  WB_TRY(alloc_io(dev, batch, &io, st));

  const size_t nx = static_cast<size_t>(batch) * in, ny = static_cast<size_t>(batch) * out;
  const size_t nw = static_cast<size_t>(out) * in;
  Scratch s;
  float *xd = nullptr, *pred = nullptr, *postd = nullptr, *gyd = nullptr, *tgt = nullptr, *dpre = nullptr,
        *gxd = nullptr, *dwd = nullptr, *wout = nullptr;
  double* lossd = nullptr;
  WB_TRY(s.get(&xd, nx));
  WB_TRY(s.get(&pred, ny));
  WB_TRY(s.get(&postd, ny));
  WB_TRY(s.get(&gyd, ny));
  WB_TRY(s.get(&tgt, ny));
  WB_TRY(s.get(&dpre, ny));
  WB_TRY(s.get(&gxd, nx));
  WB_TRY(s.get(&dwd, nw));
  WB_TRY(s.get(&wout, nw));
  WB_TRY(s.get(&lossd, 1));
  WB_CUDA(cudaMemcpyAsync(xd, x, nx * 4, cudaMemcpyHostToDevice, st));
  WB_TRY(forward_device(dev, batch, xd, in, pred, postd, &io, st, false));
  WB_TRY(check_pipeline_error(io, st));
  *loss = 0.0;
  if (use_target) {
    WB_CUDA(cudaMemcpyAsync(tgt, grad_or_target, ny * 4, cudaMemcpyHostToDevice, st));
    WB_TRY(mse_device(postd, tgt, static_cast<int64_t>(ny), gyd, lossd, st));
  } else {
    WB_CUDA(cudaMemcpyAsync(gyd, grad_or_target, ny * 4, cudaMemcpyHostToDevice, st));
  }
  WB_TRY(dense_backward_device(dev, batch, gyd, xd, pred, false, dpre, gxd, dwd, st));
  // The store's payload on the device: updated by the SGD when lr != 0, then exported with the
  // reference's decode (weight_at).
  const bool f32 = dt == DType::Float32;
  const size_t pb = f32 ? nw * 4 : store.native.size();
  uint8_t* payload = nullptr;
  WB_TRY(s.get(&payload, pb));
  WB_CUDA(cudaMemcpyAsync(payload, f32 ? static_cast<const void*>(store.f32.data()) : store.native.data(), pb,
                          cudaMemcpyHostToDevice, st));
  if (lr != 0.0) WB_TRY(apply_sgd_native(dt, payload, static_cast<int64_t>(nw), store.scale, dwd, lr, st));
  WB_TRY(decode_ref(dt, payload, static_cast<int64_t>(nw), store.scale, wout, st));
  WB_CUDA(cudaMemcpyAsync(pre, pred, ny * 4, cudaMemcpyDeviceToHost, st));
  WB_CUDA(cudaMemcpyAsync(post, postd, ny * 4, cudaMemcpyDeviceToHost, st));
  WB_CUDA(cudaMemcpyAsync(dX, gxd, nx * 4, cudaMemcpyDeviceToHost, st));
  WB_CUDA(cudaMemcpyAsync(dW, dwd, nw * 4, cudaMemcpyDeviceToHost, st));
  WB_CUDA(cudaMemcpyAsync(W_after, wout, nw * 4, cudaMemcpyDeviceToHost, st));
  if (use_target) WB_CUDA(cudaMemcpyAsync(loss, lossd, sizeof(double), cudaMemcpyDeviceToHost, st));
  WB_CUDA(cudaStreamSynchronize(st));
  return Status::Ok();
}

} // namespace wb
