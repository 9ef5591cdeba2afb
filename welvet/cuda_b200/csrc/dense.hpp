// dense.hpp -- Dense layer: host WeightStore, device mirror, resident session.
//
// Reference interfaces mirrored (same field meaning and error behaviour):
//   WeightStore          include/welvet/weights.hpp:18-26
//   dense::Layer         include/welvet/dense.hpp:13-51  (lazy device mirror, invalidation)
//   dense::Session       src/layers/dense/session.cpp:10-18, :34-82
//   cuda::ResidentDense  include/welvet/cuda/matvec.hpp:14-25
// What differs by design: the device mirror holds the packed codes (row-padded, canonical)
// instead of a host-decoded fp64 matrix, codecs run on the GPU, and every call works on the
// session's own stream instead of the default stream.
#pragma once

#include "common.hpp"
#include "gemv_tc.hpp"

#include <vector>

namespace wb {

// Authoritative host store, field for field the reference's FormatNone WeightStore.
struct WeightStore {
  DType dtype = DType::Float32;
  int32_t format = 0;            // QuantFormat::None
  int rows = 0;                  // out
  int cols = 0;                  // in
  std::vector<float> f32;        // Float32 payload
  std::vector<uint8_t> native;   // FP8 / FP4 / Int8 payload, reference layout
  float scale = 1.0f;
  std::vector<double> bias;
};

// Device-resident mirror of one Dense layer's weights.
struct DeviceDense {
  int device = 0;
  DType dtype = DType::Float32;
  int rows = 0, cols = 0;
  int64_t row_stride = 0;   // bytes per padded mirror row (multiple of 16)
  int64_t x_stride = 0;     // floats per padded activation row this layer consumes
  uint8_t* W = nullptr;     // mirror [rows][row_stride]
  uint8_t* Wt = nullptr;    // fragment-tiled mirror for the small-batch tensor GEMV (gemv_tc.hpp)
  uint8_t* Wg = nullptr;    // 128-row tiled mirror for the batched tcgen05 GEMM (gemm_tc.hpp)
  float scale = 1.0f;
  double* bias = nullptr;   // [bias_len]
  int bias_len = 0;
  int act = -1;
  bool exact = false;       // fp64-accumulating GEMV (see exact_policy)

  DeviceDense() = default;
  DeviceDense(const DeviceDense&) = delete;
  DeviceDense& operator=(const DeviceDense&) = delete;
  DeviceDense(DeviceDense&& o) noexcept { *this = std::move(o); }
  DeviceDense& operator=(DeviceDense&& o) noexcept;
  ~DeviceDense() { release(); }
  void release();
};

// Whether a layer of rows x cols weights runs the fp64-accumulating GEMV: forced by
// WELVET_B200_EXACT=1 / =0, otherwise for layers of at most 2^20 weights (latency-bound
// sizes where fp64 costs nothing). Read at mount.
bool exact_policy(int rows, int cols);

// Padded geometry of a layer's mirror rows and of the activations it reads.
int64_t mirror_row_stride(DType dt, int cols);
int64_t activation_stride(DType dt, int cols);

// Quantize host float32 weights W[rows*cols] on the GPU into `store` (reference bytes and
// scale, copied back to the host) and build the device mirror. `w_is_device` selects whether
// W is a device pointer (no H2D copy of the float32 matrix).
// `batch_hint` > 0: the only batch size the mirror will serve (a session's), so that only the
// mirrors that batch reads are built (the fragment-tiled one up to kGemvMaxBatch tokens, the
// GEMM one above 4); 0 builds every mirror.
Status mount_dense(int device, int rows, int cols, DType dt, int act, const float* W, bool w_is_device,
                   const double* bias, size_t bias_len, WeightStore* store, DeviceDense* dev,
                   cudaStream_t st, int batch_hint = 0);

// Mirror from reference-layout native bytes (+ scale), as a stored model is re-mounted
// (src/interop/model_session.cpp:135-153 reads native bytes and scale back into a store).
Status mount_dense_native(int device, int rows, int cols, DType dt, int act, const uint8_t* native,
                          size_t native_len, float scale, const double* bias, size_t bias_len,
                          WeightStore* store, DeviceDense* dev, cudaStream_t st, int batch_hint = 0);

// Device buffers for one batch size: padded x, pre, post, and the tensor-core path's scratch.
struct DenseIO {
  int batch = 0;
  float* x = nullptr;     // [batch][x_stride], padding zero
  float* pre = nullptr;   // [batch][rows]
  float* post = nullptr;  // [batch][rows]
  void* scratch = nullptr;  // gemm_scratch_bytes(batch, cols, rows, xsplit)
  size_t scratch_bytes = 0;
  int* err = nullptr;     // device error word of the tensor-core path
  void* prep = nullptr;   // gemv_group_prep_bytes: x prepared once per grouped launch (batch <= 4)
  // Tokens per GEMM token block at most (0: the plan's own), set before alloc_io by a caller
  // whose activations are fp32 results (two x planes): blocks of 128 make one pass each, so
  // more tiles fill the GPU without split-K.
  int max_tb = 0;
  void release();
};

// Batched path selection: batches above 8 tokens run the tcgen05 GEMM (FP8/FP4/Int8 layers
// that are not in exact mode) unless WELVET_B200_GEMV16=1 puts 9..16 on the tensor GEMV;
// WELVET_B200_BATCHED=gemv keeps every batch on the GEMV, =tc every batch on the GEMM.
bool use_tensor_path(const DeviceDense& d, int batch);
// Batches of 1..8 on quantized, non-exact layers run the tensor-core GEMV (gemv_tc.hpp); 9..16
// with WELVET_B200_GEMV16=1 where it fits (else the GEMM); WELVET_B200_GEMV=simt keeps them on
// the SIMT GEMV.
bool use_gemv_tc(const DeviceDense& d, int batch);
// Number of f16 planes x is split into on the tensor path (WELVET_B200_XSPLIT, default 3).
int xsplit_policy();

Status alloc_io(const DeviceDense& d, int batch, DenseIO* io, cudaStream_t st);
// Synchronizes `st` and reports (then clears) a timed-out tensor-core pipeline wait.
Status check_pipeline_error(DenseIO& io, cudaStream_t st);

// y = Dense(x) on the device: x [batch][x_ld] (any alignment; staged into io.x when it is
// not already padded), outputs [batch][rows] into pre/post (device pointers).
// `ld_out` (0: rows) is the row pitch of pre/post; `peers` (may be nullptr) lists further
// destinations of post with the same layout (column-sharded layers, sharded.hpp).
// `norm` (may be nullptr) puts an RMSNorm layer of width cols in front: x is the norm's input
// ([batch][x_ld]), the norm's pre / post ([batch][cols]) are written, and the layer reads
// post. On the tensor-core GEMM the norm is the launch's prologue; elsewhere it runs first as
// its own kernel, with the same bits.
Status forward_device(const DeviceDense& d, int batch, const float* x, int64_t x_ld, float* pre,
                      float* post, DenseIO* io, cudaStream_t st, bool pdl, int64_t ld_out = 0,
                      const PeerOut* peers = nullptr, const SplitNorm* norm = nullptr);

struct DenseSession {
  int device = 0;
  int batch = 0;
  cudaStream_t stream = nullptr;
  WeightStore store;
  DeviceDense dev;
  DenseIO io;
  // Host-buffer execute (session_execute): after a first direct call, the device side of a
  // call is a CUDA graph replayed per call, recorded over device-accessible host memory: the
  // caller's own buffers when they are pinned (one graph per buffer triple, the most recent
  // kMaxExecGraphs kept), else the session's mapped staging, to and from which the caller's
  // buffers are copied on the host. `graph_state` 0: not built yet, 1: built, -1: capture
  // failed (the direct path is used).
  struct ExecGraph {
    const void *x = nullptr, *pre = nullptr, *post = nullptr;  // device addresses recorded
    cudaGraphExec_t exec = nullptr;
    uint64_t used = 0;
  };
  static constexpr int kMaxExecGraphs = 4;
  int calls = 0;
  int graph_state = 0;
  cudaGraphExec_t graph = nullptr;      // over the staging buffers
  std::vector<ExecGraph> caller_graphs;  // over pinned caller buffers
  float* x_pin = nullptr;
  float* pre_pin = nullptr;
  float* post_pin = nullptr;
  int* err_pin = nullptr;
  ~DenseSession();
};

Status session_mount(int32_t batch, int32_t in, int32_t out, int32_t act, int32_t dtype,
                     const float* W, bool w_is_device, const double* bias, size_t bias_len,
                     DenseSession** out_sess);
Status session_mount_native(int32_t batch, int32_t in, int32_t out, int32_t act, int32_t dtype,
                            const uint8_t* native, size_t native_len, float scale,
                            const double* bias, size_t bias_len, DenseSession** out_sess);
// Host buffers in and out, synchronous (the reference's resident_execute contract).
Status session_execute(DenseSession* s, const float* x, float* pre, float* post);
// Device buffers on a caller stream (0 = the legacy default stream), asynchronous.
Status session_execute_device(DenseSession* s, const float* x, float* pre, float* post,
                              cudaStream_t st);

// n independent forwards on one stream: sessions that share dtype, shape and batch and run
// the small-batch tensor GEMV go out together in grouped launches (up to 32 layers each);
// any others run one by one. x[i], pre[i], post[i] are device pointers of session i.
Status session_execute_group(DenseSession* const* s, int n, const float* const* x, float* const* pre,
                             float* const* post, cudaStream_t st);

// Same forward for batched sessions (> 8 tokens on the tcgen05 path), with the GEMM's scratch
// in the library's fixed static device array: no allocation of any kind.
Status session_execute_device_noalloc(DenseSession* s, const float* x, float* pre, float* post,
                                      cudaStream_t st);

// Library device selection: the device current on the first call of the process (0 unless
// the host application selected another), unless WELVET_B200_DEVICE is set.
Status library_device(int* device);
std::string runtime_identity();

} // namespace wb
