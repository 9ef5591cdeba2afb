// dense.cpp -- Dense layer mount / execute over the packed device mirror.
//
// Mount follows the reference's resident session (src/layers/dense/session.cpp:34-69):
// float32 W -> FormatNone store (WeightStore::make, src/weights/store.cpp:7-22) -> device.
// Here the encode runs as GPU kernels (bit-exact with the host codec) and the native bytes
// are copied back so the host store stays authoritative, as in the reference. Execute keeps
// resident_execute's contract (src/cuda/kernels.cu:873-915): host x in, host pre/post out,
// synchronous; plus an asynchronous device-pointer variant.
#include "dense.hpp"

#include "cell_kernels.hpp"
#include "codec.hpp"
#include "gemm_tc.hpp"
#include "gemv.hpp"
#include "gemv_tc.hpp"

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <sstream>
#include <vector>

namespace wb {

namespace {

template <typename T>
void free_dev(T*& p) {
  if (p) cudaFree(p);
  p = nullptr;
}

struct DevBuf {  // scoped temporary device allocation
  void* p = nullptr;
  ~DevBuf() { if (p) cudaFree(p); }
};

} // namespace

DeviceDense& DeviceDense::operator=(DeviceDense&& o) noexcept {
  if (this == &o) return *this;
  release();
  device = o.device; dtype = o.dtype; rows = o.rows; cols = o.cols;
  row_stride = o.row_stride; x_stride = o.x_stride; W = o.W; Wt = o.Wt; Wg = o.Wg; scale = o.scale;
  bias = o.bias; bias_len = o.bias_len; act = o.act; exact = o.exact;
  o.W = nullptr; o.Wt = nullptr; o.Wg = nullptr; o.bias = nullptr;
  return *this;
}

void DeviceDense::release() {
  if (W || Wt || Wg || bias) {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    free_dev(W);
    free_dev(Wt);
    free_dev(Wg);
    free_dev(bias);
    cudaSetDevice(cur);
  }
}

void DenseIO::release() {
  free_dev(x);
  free_dev(pre);
  free_dev(post);
  free_dev(scratch);
  free_dev(err);
  free_dev(prep);
  scratch_bytes = 0;
  batch = 0;
}

bool use_gemv_tc(const DeviceDense& d, int batch) {
  const char* env = std::getenv("WELVET_B200_GEMV");
  if (env && std::strcmp(env, "simt") == 0) return false;
  if (batch > 8) {
    // 9..16 tokens run the tcgen05 GEMM: measured faster on B200 than the register-path GEMV,
    // whose mma.sync work grows with the token count (14336 x 4096 E4M3, 16 tokens: GEMM
    // 46 us, GEMV 144 us). WELVET_B200_GEMV16=1 selects the GEMV where it fits.
    const char* b = std::getenv("WELVET_B200_BATCHED");
    if (b && (std::strcmp(b, "tc") == 0)) return false;
    const char* g16 = std::getenv("WELVET_B200_GEMV16");
    if (!(g16 && g16[0] == '1')) return false;
  }
  return batch >= 1 && batch <= kGemvMaxBatch && !d.exact && d.Wt != nullptr &&
         gemv_tc_fits(d.dtype, d.rows, d.cols, batch);
}

// f16 planes that carry x on the batched tensor-core path. Default 2 (22 bits of x, as the
// tensor GEMV): the measured error against the fp64 oracle is the same as with 3 (fp32 tensor
// accumulation dominates it), and fp32-valued activations cost two MMA columns per token
// instead of three.
int xsplit_policy() {
  const char* env = std::getenv("WELVET_B200_XSPLIT");
  if (env && env[0] >= '1' && env[0] <= '3') return env[0] - '0';
  return 2;
}

bool use_tensor_path(const DeviceDense& d, int batch) {
  const char* env = std::getenv("WELVET_B200_BATCHED");
  if (env && std::strcmp(env, "gemv") == 0) return false;
  if (env && std::strcmp(env, "tc") == 0) return !d.exact && gemm_supported(d.dtype) && d.Wg != nullptr;
  return batch > 8 && !use_gemv_tc(d, batch) && !d.exact && gemm_supported(d.dtype) && d.Wg != nullptr;
}

bool exact_policy(int rows, int cols) {
  const char* env = std::getenv("WELVET_B200_EXACT");
  if (env && env[0] == '1') return true;
  if (env && env[0] == '0') return false;
  return static_cast<int64_t>(rows) * cols <= (static_cast<int64_t>(1) << 20);
}

int64_t mirror_row_stride(DType dt, int cols) { return round_up(row_bytes(dt, cols), 16); }

int64_t activation_stride(DType dt, int cols) {
  return mirror_row_stride(dt, cols) / 16 * elems_per_16B(dt);
}

static Status check_dims(int rows, int cols, int32_t dtype) {
  if (rows <= 0 || cols <= 0) return Status::Invalid("dense: bad dims");
  if (!dtype_on_path(dtype))
    return Status::Unsupported(std::string("dense CUDA (b200) unsupported dtype id ") + std::to_string(dtype));
  if (static_cast<int64_t>(rows) * cols > (static_cast<int64_t>(1) << 31) - 1)
    return Status::Invalid("dense: rows*cols exceeds the reference's int element count");
  return Status::Ok();
}

static Status finish_mirror(int device, int rows, int cols, DType dt, int act, const uint8_t* native_dev,
                            float scale, const double* bias, size_t bias_len, WeightStore* store,
                            DeviceDense* dev, cudaStream_t st, int batch_hint) {
  DeviceDense d;
  d.device = device;
  d.dtype = dt;
  d.rows = rows;
  d.cols = cols;
  d.row_stride = mirror_row_stride(dt, cols);
  d.x_stride = activation_stride(dt, cols);
  d.scale = scale;
  d.act = act;
  d.exact = exact_policy(rows, cols);
  WB_CUDA(cudaMalloc(&d.W, static_cast<size_t>(d.row_stride) * rows));
  WB_TRY(build_mirror(dt, native_dev, rows, cols, d.row_stride, d.W, st));
  if (gemv_tc_supported(dt) && !d.exact && (batch_hint <= 0 || batch_hint <= kGemvMaxBatch)) {
    WB_CUDA(cudaMalloc(&d.Wt, static_cast<size_t>(tiled_geom(dt, rows, cols).bytes())));
    WB_TRY(build_tiled_mirror(dt, native_dev, rows, cols, d.Wt, st));
  }
  if (gemm_supported(dt) && !d.exact && (batch_hint <= 0 || batch_hint > 4)) {
    WB_CUDA(cudaMalloc(&d.Wg, gemm_mirror_bytes(dt, rows, cols)));
    WB_TRY(build_gemm_mirror(dt, d.W, rows, d.row_stride, cols, d.Wg, st));
  }
  store->bias.clear();
  if (bias && bias_len > 0) {
    store->bias.assign(bias, bias + bias_len);
    d.bias_len = static_cast<int>(bias_len);
    WB_CUDA(cudaMalloc(&d.bias, bias_len * sizeof(double)));
    WB_CUDA(cudaMemcpyAsync(d.bias, bias, bias_len * sizeof(double), cudaMemcpyHostToDevice, st));
  }
  WB_CUDA(cudaStreamSynchronize(st));
  *dev = std::move(d);
  return Status::Ok();
}

Status mount_dense(int device, int rows, int cols, DType dt, int act, const float* W, bool w_is_device,
                   const double* bias, size_t bias_len, WeightStore* store, DeviceDense* dev,
                   cudaStream_t st, int batch_hint) {
  WB_TRY(check_dims(rows, cols, static_cast<int32_t>(dt)));
  if (!W) return Status::Invalid("null mount args");
  WB_CUDA(cudaSetDevice(device));
  const int64_t n = static_cast<int64_t>(rows) * cols;
  DevBuf wtmp, ntmp, small;
  const float* wdev = W;
  if (!w_is_device) {
    WB_CUDA(cudaMalloc(&wtmp.p, static_cast<size_t>(n) * 4));
    WB_CUDA(cudaMemcpyAsync(wtmp.p, W, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, st));
    wdev = static_cast<const float*>(wtmp.p);
  }
  const int64_t nb = native_bytes(dt, n);
  WB_CUDA(cudaMalloc(&ntmp.p, static_cast<size_t>(nb)));
  WB_CUDA(cudaMalloc(&small.p, 16));
  float* scale_dev = static_cast<float*>(small.p);
  unsigned int* absmax = reinterpret_cast<unsigned int*>(static_cast<char*>(small.p) + 8);
  uint8_t* native_dev = static_cast<uint8_t*>(ntmp.p);
  WB_TRY(encode_native(dt, wdev, n, native_dev, scale_dev, absmax, st));

  store->dtype = dt;
  store->format = 0;
  store->rows = rows;
  store->cols = cols;
  float scale = 1.0f;
  if (dt == DType::Float32) {
    store->native.clear();
    store->f32.resize(static_cast<size_t>(n));
    WB_CUDA(cudaMemcpyAsync(store->f32.data(), wdev, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, st));
  } else {
    store->f32.clear();
    store->native.resize(static_cast<size_t>(nb));
    WB_CUDA(cudaMemcpyAsync(store->native.data(), native_dev, static_cast<size_t>(nb), cudaMemcpyDeviceToHost, st));
    WB_CUDA(cudaMemcpyAsync(&scale, scale_dev, sizeof(float), cudaMemcpyDeviceToHost, st));
  }
  WB_CUDA(cudaStreamSynchronize(st));
  store->scale = scale;
  return finish_mirror(device, rows, cols, dt, act, native_dev, scale, bias, bias_len, store, dev, st, batch_hint);
}

Status mount_dense_native(int device, int rows, int cols, DType dt, int act, const uint8_t* native,
                          size_t native_len, float scale, const double* bias, size_t bias_len,
                          WeightStore* store, DeviceDense* dev, cudaStream_t st, int batch_hint) {
  WB_TRY(check_dims(rows, cols, static_cast<int32_t>(dt)));
  if (!native) return Status::Invalid("null native bytes");
  const int64_t n = static_cast<int64_t>(rows) * cols;
  const int64_t nb = native_bytes(dt, n);
  if (static_cast<int64_t>(native_len) < nb) return Status::Invalid(std::string(dtype_name(static_cast<int32_t>(dt))) + " short");
  WB_CUDA(cudaSetDevice(device));
  DevBuf ntmp;
  WB_CUDA(cudaMalloc(&ntmp.p, static_cast<size_t>(nb)));
  WB_CUDA(cudaMemcpyAsync(ntmp.p, native, static_cast<size_t>(nb), cudaMemcpyHostToDevice, st));
  store->dtype = dt;
  store->format = 0;
  store->rows = rows;
  store->cols = cols;
  store->scale = dt == DType::Float32 ? 1.0f : scale;
  if (dt == DType::Float32) {
    store->native.clear();
    store->f32.assign(reinterpret_cast<const float*>(native), reinterpret_cast<const float*>(native) + n);
  } else {
    store->f32.clear();
    store->native.assign(native, native + nb);
  }
  // weight_at treats a zero scale as 1 (src/weights/native_codec.cpp:514-515).
  const float eff = (store->scale == 0.0f) ? 1.0f : store->scale;
  return finish_mirror(device, rows, cols, dt, act, static_cast<const uint8_t*>(ntmp.p), eff, bias,
                       bias_len, store, dev, st, batch_hint);
}

Status alloc_io(const DeviceDense& d, int batch, DenseIO* io, cudaStream_t st) {
  io->release();
  io->batch = batch;
  const size_t xb = static_cast<size_t>(batch) * static_cast<size_t>(d.x_stride) * 4;
  const size_t yb = static_cast<size_t>(batch) * static_cast<size_t>(d.rows) * 4;
  WB_CUDA(cudaMalloc(&io->x, xb));
  WB_CUDA(cudaMemsetAsync(io->x, 0, xb, st));
  WB_CUDA(cudaMalloc(&io->pre, yb));
  WB_CUDA(cudaMalloc(&io->post, yb));
  WB_CUDA(cudaMalloc(&io->err, sizeof(int)));
  WB_CUDA(cudaMemsetAsync(io->err, 0, sizeof(int), st));
  if (use_tensor_path(d, batch)) {
    io->scratch_bytes = gemm_scratch_bytes(batch, d.cols, d.rows, xsplit_policy(), true, io->max_tb);
    WB_CUDA(cudaMalloc(&io->scratch, io->scratch_bytes));
  }
  if (use_gemv_tc(d, batch)) {
    if (const size_t pb = gemv_prep_bytes(d.dtype, d.rows, d.cols, batch)) WB_CUDA(cudaMalloc(&io->prep, pb));
  }
  return Status::Ok();
}

Status forward_device(const DeviceDense& d, int batch, const float* x, int64_t x_ld, float* pre,
                      float* post, DenseIO* io, cudaStream_t st, bool pdl, int64_t ld_out,
                      const PeerOut* peers, const SplitNorm* norm) {
  if (batch <= 0 || !x || !pre || !post) return Status::Invalid("null execute args");
  if (ld_out <= 0) ld_out = d.rows;
  if (ld_out < d.rows) return Status::Invalid("dense: output pitch below the layer's rows");
  const bool gemm = use_tensor_path(d, batch) && io && io->scratch;
  if (norm && norm->gamma) {
    if (!norm->pre || !norm->post) return Status::Invalid("rmsnorm: null outputs");
    if (!gemm) {  // the norm as its own kernel, then the layer on its post
      if (x_ld != d.cols) return Status::Invalid("rmsnorm: input rows must be dense");
      WB_TRY(launch_rmsnorm(x, norm->gamma, norm->pre, norm->post, batch, d.cols, norm->eps, st));
      x = norm->post;
      pdl = false;
    }
  }
  const PeerOut no_peers{};
  const PeerOut& pe = peers ? *peers : no_peers;
  const float* xs = x;  // the tensor-core paths read x in any layout
  int64_t xst = x_ld;
  const bool pdl_in = pdl;
  if (gemm) {
    GemmArgs g;
    g.dtype = d.dtype;
    g.W = d.W;
    g.Wg = d.Wg;
    g.row_stride = d.row_stride;
    g.rows = d.rows;
    g.cols = d.cols;
    g.scale = d.scale;
    g.x = xs;
    g.x_ld = xst;
    g.M = batch;
    g.pre = pre;
    g.post = post;
    g.ld_out = ld_out;
    g.peers = pe;
    g.bias = d.bias;
    g.bias_len = d.bias_len;
    g.act = d.act;
    g.xsplit = xsplit_policy();
    g.max_tb = io->max_tb;
    g.scratch = io->scratch;
    g.scratch_bytes = io->scratch_bytes;
    g.err = io->err;
    g.pdl = pdl_in;
    if (norm) g.norm = *norm;
    return launch_gemm_tc(g, st);
  }
  if (use_gemv_tc(d, batch) && io && io->prep && gemv_prefers_prepared(d.dtype, d.rows, d.cols, batch)) {
    // a layer that fills the GPU by itself: x prepared once, longer K ranges per CTA
    GemvGroupLayer L;
    L.Wt = d.Wt;
    L.x = x;
    L.pre = pre;
    L.post = post;
    L.bias = d.bias;
    L.bias_len = d.bias_len;
    L.act = d.act;
    L.scale = d.scale;
    L.prep = io->prep;
    return launch_gemv_tc_group(d.dtype, d.rows, d.cols, batch, x_ld, ld_out, &L, 1, st, pdl_in, &pe);
  }
  if (use_gemv_tc(d, batch)) {
    GemvTcArgs g;
    g.dtype = d.dtype;
    g.Wt = d.Wt;
    g.rows = d.rows;
    g.cols = d.cols;
    g.scale = d.scale;
    g.x = x;  // any layout: the kernel reads x with bounds checks, no staging needed
    g.x_ld = x_ld;
    g.batch = batch;
    g.pre = pre;
    g.post = post;
    g.ld_out = ld_out;
    g.peers = pe;
    g.bias = d.bias;
    g.bias_len = d.bias_len;
    g.act = d.act;
    g.prep = io ? io->prep : nullptr;
    return launch_gemv_tc(g, st, pdl_in);
  }
  // The SIMT GEMV reads x in 16-byte vectors over the padded row: stage unpadded inputs (the
  // session's own staging rows keep zero pads).
  const bool own = io && x == io->x && x_ld == d.x_stride && io->batch >= batch;
  const bool direct = own || (d.cols == d.x_stride && x_ld == d.cols && (reinterpret_cast<uintptr_t>(x) & 15) == 0);
  if (!direct) {
    if (!io || !io->x || io->batch < batch) return Status::Internal("dense: no staging buffer for this batch");
    WB_CUDA(cudaMemcpy2DAsync(io->x, static_cast<size_t>(d.x_stride) * 4, x, static_cast<size_t>(x_ld) * 4,
                              static_cast<size_t>(d.cols) * 4, static_cast<size_t>(batch),
                              cudaMemcpyDeviceToDevice, st));
    xs = io->x;
    xst = d.x_stride;
    pdl = false;
  }
  GemvArgs a;
  a.dtype = d.dtype;
  a.W = d.W;
  a.row_stride = d.row_stride;
  a.rows = d.rows;
  a.cols = d.cols;
  a.scale = d.scale;
  a.x = xs;
  a.x_stride = xst;
  a.batch = batch;
  a.pre = pre;
  a.post = post;
  a.ld_out = ld_out;
  a.peers = pe;
  a.bias = d.bias;
  a.bias_len = d.bias_len;
  a.act = d.act;
  a.exact = d.exact;
  return launch_gemv(a, st, pdl);
}

DenseSession::~DenseSession() {
  cudaSetDevice(device);
  if (stream) cudaStreamSynchronize(stream);
  if (graph) cudaGraphExecDestroy(graph);
  for (auto& g : caller_graphs) cudaGraphExecDestroy(g.exec);
  for (void* p : {static_cast<void*>(x_pin), static_cast<void*>(pre_pin), static_cast<void*>(post_pin),
                  static_cast<void*>(err_pin)})
    if (p) cudaFreeHost(p);
  io.release();
  dev.release();
  if (stream) cudaStreamDestroy(stream);
}

Status library_device(int* device) {
  static std::once_flag once;
  static int dev = 0;
  static Status st;
  std::call_once(once, [] {
    int count = 0;
    st = cuda_status(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (!st.ok()) return;
    if (count <= 0) {
      st = Status::Unsupported("no CUDA device available");
      return;
    }
    const char* env = std::getenv("WELVET_B200_DEVICE");
    if (env && *env) {
      dev = std::atoi(env);
    } else {
      st = cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
    }
    if (st.ok() && (dev < 0 || dev >= count)) st = Status::Invalid("WELVET_B200_DEVICE out of range");
  });
  *device = dev;
  return st;
}

std::string runtime_identity() {
  int d = 0;
  if (!library_device(&d).ok()) return "cuda:unavailable";
  cudaDeviceProp p{};
  if (cudaGetDeviceProperties(&p, d) != cudaSuccess) return "cuda:unavailable";
  std::ostringstream os;
  os << "cuda:" << p.name << ":idx=" << d << ":sm=" << p.major << "." << p.minor << ":mem=" << p.totalGlobalMem;
  return os.str();
}

static Status new_session(int32_t batch, DenseSession** out) {
  if (!out) return Status::Invalid("null mount args");
  if (batch <= 0) return Status::Invalid("bad dims");
  auto* s = new DenseSession();
  Status st = library_device(&s->device);
  if (st.ok()) st = cuda_status(cudaSetDevice(s->device), "cudaSetDevice");
  if (st.ok()) st = cuda_status(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "stream");
  if (!st.ok()) {
    delete s;
    return st;
  }
  s->batch = batch;
  *out = s;
  return Status::Ok();
}

Status session_mount(int32_t batch, int32_t in, int32_t out, int32_t act, int32_t dtype, const float* W,
                     bool w_is_device, const double* bias, size_t bias_len, DenseSession** out_sess) {
  if (!out_sess || !W) return Status::Invalid("null mount args");
  WB_TRY(check_dims(out, in, dtype));
  DenseSession* s = nullptr;
  WB_TRY(new_session(batch, &s));
  Status st = mount_dense(s->device, out, in, static_cast<DType>(dtype), act, W, w_is_device, bias, bias_len,
                          &s->store, &s->dev, s->stream, batch);
  if (st.ok()) st = alloc_io(s->dev, batch, &s->io, s->stream);
  if (st.ok()) st = cuda_status(cudaStreamSynchronize(s->stream), "mount sync");
  if (!st.ok()) {
    delete s;
    return st;
  }
  *out_sess = s;
  return Status::Ok();
}

Status session_mount_native(int32_t batch, int32_t in, int32_t out, int32_t act, int32_t dtype,
                            const uint8_t* native, size_t native_len, float scale, const double* bias,
                            size_t bias_len, DenseSession** out_sess) {
  if (!out_sess || !native) return Status::Invalid("null mount args");
  WB_TRY(check_dims(out, in, dtype));
  DenseSession* s = nullptr;
  WB_TRY(new_session(batch, &s));
  Status st = mount_dense_native(s->device, out, in, static_cast<DType>(dtype), act, native, native_len, scale,
                                 bias, bias_len, &s->store, &s->dev, s->stream, batch);
  if (st.ok()) st = alloc_io(s->dev, batch, &s->io, s->stream);
  if (st.ok()) st = cuda_status(cudaStreamSynchronize(s->stream), "mount sync");
  if (!st.ok()) {
    delete s;
    return st;
  }
  *out_sess = s;
  return Status::Ok();
}

namespace {
// The device side of a host-buffer forward over device-accessible host memory (mapped pinned
// buffers), moving no data with copy-engine transfers: a staging kernel reads x over the bus
// with all its loads in flight at once into the session's padded x (a GEMV, launched as its
// programmatic dependent, streams its weights meanwhile); the epilogues store pre / post
// straight into host memory. Only the GEMM pipeline's error word is copied back (4 bytes, to
// err_pin).
Status enqueue_mapped_execute(DenseSession* s, const float* x_dev, float* pre_dev, float* post_dev) {
  const DeviceDense& d = s->dev;
  WB_TRY(launch_stage_rows(s->io.x, d.x_stride, x_dev, d.cols, d.cols, s->batch, s->stream));
  WB_TRY(forward_device(d, s->batch, s->io.x, d.x_stride, pre_dev, post_dev, &s->io, s->stream, true));
  if (s->io.err && s->io.scratch)
    WB_CUDA(cudaMemcpyAsync(s->err_pin, s->io.err, sizeof(int), cudaMemcpyDeviceToHost, s->stream));
  return Status::Ok();
}

// Records enqueue_mapped_execute over the given device addresses as a graph.
Status record_execute_graph(DenseSession* s, const float* x_dev, float* pre_dev, float* post_dev,
                            cudaGraphExec_t* exec) {
  cudaGraph_t g = nullptr;
  WB_CUDA(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  Status st = enqueue_mapped_execute(s, x_dev, pre_dev, post_dev);
  const cudaError_t end = cudaStreamEndCapture(s->stream, &g);
  if (st.ok()) st = cuda_status(end, "end capture");
  if (st.ok()) st = cuda_status(cudaGraphInstantiate(exec, g, 0), "graph instantiate");
  if (g) cudaGraphDestroy(g);
  cudaGetLastError();  // a failed capture leaves nothing pending for the direct path
  return st;
}

// Allocates the session's mapped staging and records the graph over it.
Status build_execute_graph(DenseSession* s) {
  const DeviceDense& d = s->dev;
  const size_t xb = static_cast<size_t>(s->batch) * static_cast<size_t>(d.cols) * 4;
  const size_t yb = static_cast<size_t>(s->batch) * static_cast<size_t>(d.rows) * 4;
  WB_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&s->x_pin), xb, cudaHostAllocMapped));
  WB_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&s->pre_pin), yb, cudaHostAllocMapped));
  WB_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&s->post_pin), yb, cudaHostAllocMapped));
  WB_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&s->err_pin), sizeof(int), cudaHostAllocMapped));
  *s->err_pin = 0;
  float *x_dev = nullptr, *pre_dev = nullptr, *post_dev = nullptr;
  WB_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&x_dev), s->x_pin, 0));
  WB_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&pre_dev), s->pre_pin, 0));
  WB_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&post_dev), s->post_pin, 0));
  return record_execute_graph(s, x_dev, pre_dev, post_dev, &s->graph);
}

// The graph over pinned caller buffers at these device addresses: a kept one, or a new
// recording that replaces the least recently used. nullptr when recording fails.
cudaGraphExec_t caller_graph(DenseSession* s, const float* x_dev, float* pre_dev, float* post_dev) {
  auto& gs = s->caller_graphs;
  const uint64_t now = static_cast<uint64_t>(s->calls);
  for (auto& g : gs)
    if (g.x == x_dev && g.pre == pre_dev && g.post == post_dev) {
      g.used = now;
      return g.exec;
    }
  cudaGraphExec_t exec = nullptr;
  if (!record_execute_graph(s, x_dev, pre_dev, post_dev, &exec).ok()) return nullptr;
  DenseSession::ExecGraph e;
  e.x = x_dev;
  e.pre = pre_dev;
  e.post = post_dev;
  e.exec = exec;
  e.used = now;
  if (static_cast<int>(gs.size()) < DenseSession::kMaxExecGraphs) {
    gs.push_back(e);
  } else {
    size_t lru = 0;
    for (size_t i = 1; i < gs.size(); ++i)
      if (gs[i].used < gs[lru].used) lru = i;
    cudaGraphExecDestroy(gs[lru].exec);
    gs[lru] = e;
  }
  return exec;
}

// The address under which the current device reads host buffer p, when p lies in pinned host
// memory mapped into the device's address space (cudaHostAlloc / cudaHostRegister); nullptr
// for pageable memory.
void* mapped_address(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

Status finish_mapped_execute(DenseSession* s) {
  WB_CUDA(cudaStreamSynchronize(s->stream));
  if (*s->err_pin == 0) return Status::Ok();
  const int e = *s->err_pin;
  *s->err_pin = 0;
  WB_CUDA(cudaMemsetAsync(s->io.err, 0, sizeof(int), s->stream));
  WB_CUDA(cudaStreamSynchronize(s->stream));
  return Status::Internal("tensor-core pipeline wait timed out (stage code " + std::to_string(e) + ")");
}
} // namespace

// WELVET_B200_EXEC_GRAPH=0 keeps the host-buffer execute on the direct path.
static bool exec_graph_policy() {
  const char* env = std::getenv("WELVET_B200_EXEC_GRAPH");
  return !(env && env[0] == '0');
}

Status session_execute(DenseSession* s, const float* x, float* pre, float* post) {
  if (!s || !x || !pre || !post) return Status::Invalid("null execute args");
  WB_CUDA(cudaSetDevice(s->device));
  const DeviceDense& d = s->dev;
  if (s->graph_state == 0 && s->calls >= 1)
    s->graph_state = exec_graph_policy() && build_execute_graph(s).ok() ? 1 : -1;
  ++s->calls;
  if (s->graph_state == 1) {
    // Pinned caller buffers are read and written where they lie; others go through the
    // session's mapped staging and its recorded graph.
    auto* xd = static_cast<const float*>(mapped_address(x));
    auto* pd = static_cast<float*>(mapped_address(pre));
    auto* qd = static_cast<float*>(mapped_address(post));
    if (xd && pd && qd) {
      if (cudaGraphExec_t exec = caller_graph(s, xd, pd, qd)) {
        WB_CUDA(cudaGraphLaunch(exec, s->stream));
        return finish_mapped_execute(s);
      }
    }
    const size_t xb = static_cast<size_t>(s->batch) * static_cast<size_t>(d.cols) * 4;
    const size_t yb = static_cast<size_t>(s->batch) * static_cast<size_t>(d.rows) * 4;
    std::memcpy(s->x_pin, x, xb);
    WB_CUDA(cudaGraphLaunch(s->graph, s->stream));
    WB_TRY(finish_mapped_execute(s));
    std::memcpy(pre, s->pre_pin, yb);
    std::memcpy(post, s->post_pin, yb);
    return Status::Ok();
  }
  WB_CUDA(cudaMemcpy2DAsync(s->io.x, static_cast<size_t>(d.x_stride) * 4, x, static_cast<size_t>(d.cols) * 4,
                            static_cast<size_t>(d.cols) * 4, static_cast<size_t>(s->batch),
                            cudaMemcpyHostToDevice, s->stream));
  WB_TRY(forward_device(d, s->batch, s->io.x, d.x_stride, s->io.pre, s->io.post, &s->io, s->stream, false));
  const size_t yb = static_cast<size_t>(s->batch) * static_cast<size_t>(d.rows) * 4;
  WB_CUDA(cudaMemcpyAsync(pre, s->io.pre, yb, cudaMemcpyDeviceToHost, s->stream));
  WB_CUDA(cudaMemcpyAsync(post, s->io.post, yb, cudaMemcpyDeviceToHost, s->stream));
  WB_CUDA(cudaStreamSynchronize(s->stream));
  return check_pipeline_error(s->io, s->stream);
}

Status check_pipeline_error(DenseIO& io, cudaStream_t st) {
  if (!io.err || !io.scratch) return Status::Ok();
  int e = 0;
  WB_CUDA(cudaMemcpyAsync(&e, io.err, sizeof(int), cudaMemcpyDeviceToHost, st));
  WB_CUDA(cudaStreamSynchronize(st));
  if (e == 0) return Status::Ok();
  WB_CUDA(cudaMemsetAsync(io.err, 0, sizeof(int), st));
  return Status::Internal("tensor-core pipeline wait timed out (stage code " + std::to_string(e) + ")");
}

// The batched tensor-core forward with its scratch in the library's static device array
// (gemm_tc.hpp: launch_gemm_tc_static) instead of the session's: makes no allocation.
Status session_execute_device_noalloc(DenseSession* s, const float* x, float* pre, float* post, cudaStream_t st) {
  if (!s || !x || !pre || !post) return Status::Invalid("null execute args");
  const DeviceDense& d = s->dev;
  if (!use_tensor_path(d, s->batch))
    return Status::Unsupported("allocation-free forward serves the batched tensor-core path only "
                               "(FP8/FP4/Int8 sessions with batch > 8 outside exact mode)");
  WB_CUDA(cudaSetDevice(s->device));
  GemmArgs g;
  g.dtype = d.dtype;
  g.W = d.W;
  g.Wg = d.Wg;
  g.row_stride = d.row_stride;
  g.rows = d.rows;
  g.cols = d.cols;
  g.scale = d.scale;
  g.x = x;
  g.x_ld = d.cols;
  g.M = s->batch;
  g.pre = pre;
  g.post = post;
  g.ld_out = d.rows;
  g.bias = d.bias;
  g.bias_len = d.bias_len;
  g.act = d.act;
  g.xsplit = xsplit_policy();
  g.err = s->io.err;
  return launch_gemm_tc_static(g, st);
}

Status session_execute_group(DenseSession* const* s, int n, const float* const* x, float* const* pre,
                             float* const* post, cudaStream_t st) {
  if (n < 0 || (n > 0 && (!s || !x || !pre || !post))) return Status::Invalid("null group execute args");
  if (n == 0) return Status::Ok();
  for (int i = 0; i < n; ++i)
    if (!s[i] || !x[i] || !pre[i] || !post[i]) return Status::Invalid("null group execute args");
  WB_CUDA(cudaSetDevice(s[0]->device));
  const DeviceDense& d0 = s[0]->dev;
  bool grouped = s[0]->batch <= 4 && use_gemv_tc(d0, s[0]->batch);
  for (int i = 1; i < n && grouped; ++i) {
    const DeviceDense& d = s[i]->dev;
    grouped = s[i]->device == s[0]->device && s[i]->batch == s[0]->batch && d.dtype == d0.dtype &&
              d.rows == d0.rows && d.cols == d0.cols && use_gemv_tc(d, s[i]->batch);
  }
  if (!grouped) {
    for (int i = 0; i < n; ++i) WB_TRY(session_execute_device(s[i], x[i], pre[i], post[i], st));
    return Status::Ok();
  }
  std::vector<GemvGroupLayer> layers(static_cast<size_t>(n));
  for (int i = 0; i < n; ++i) {
    const DeviceDense& d = s[i]->dev;
    GemvGroupLayer& L = layers[static_cast<size_t>(i)];
    L.Wt = d.Wt;
    L.x = x[i];
    L.pre = pre[i];
    L.post = post[i];
    L.bias = d.bias;
    L.bias_len = d.bias_len;
    L.act = d.act;
    L.scale = d.scale;
    L.prep = s[i]->io.prep;  // one session's layer at a time: its scratch is free
  }
  return launch_gemv_tc_group(d0.dtype, d0.rows, d0.cols, s[0]->batch, d0.cols, d0.rows, layers.data(), n, st,
                              true);
}

Status session_execute_device(DenseSession* s, const float* x, float* pre, float* post, cudaStream_t st) {
  if (!s || !x || !pre || !post) return Status::Invalid("null execute args");
  WB_CUDA(cudaSetDevice(s->device));
  return forward_device(s->dev, s->batch, x, s->dev.cols, pre, post, &s->io, st, true);
}

} // namespace wb
