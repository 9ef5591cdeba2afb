// volume.hpp -- device-resident volume (Grid) forward.
//
// Reference interfaces mirrored:
//   architecture::Grid / Cell / new_grid / index / hop_order / set_remote_link / bind_*
//                                             include/welvet/architecture.hpp:34-141,
//                                             src/architecture/grid.cpp:31-117
//   runtime::forward::volume_dense / cell     src/runtime/forward.cpp:45-156
// Differences by design: activations stay on the device from hop to hop (the reference
// round-trips every hop through host TensorF32), and a forward can run a contiguous range
// of the hop order so that consecutive ranges can live on different GPUs.
#pragma once

#include "cells.hpp"
#include "dense.hpp"

#include <memory>
#include <vector>

namespace wb {

// OpKind values of the reference (include/welvet/architecture.hpp:41-65) served here.
enum class OpKind : int32_t { None = 0, Dense = 1, RMSNorm = 2, SwiGLU = 4, MHA = 7 };

struct VolumeCell {
  OpKind op = OpKind::None;
  bool disabled = false;
  bool remote = false;
  int target = -1;          // flat index of the remote-link target
  int in_width = 0, out_width = 0, pre_width = 0;
  // ops
  std::unique_ptr<WeightStore> store;
  std::unique_ptr<DeviceDense> dense;
  std::unique_ptr<SwigluCell> swiglu;
  std::unique_ptr<MhaCell> mha;
  int mha_seq = 1;          // tokens per sequence for MHA cells (rows = batch * seq)
  double* gamma64 = nullptr;  // RMSNorm
  double eps = 1e-6;
  // per-forward device buffers
  DenseIO io;
  float* pre = nullptr;
  float* post = nullptr;
  int rows = 0;             // rows the buffers are sized for
  uint64_t epoch = 0;       // forward in which pre/post were last written (0: never)
  int epoch_rows = 0;       // rows of that forward
  ~VolumeCell();
};

struct Volume {
  int device = 0;
  int depth = 1, rows = 1, cols = 1, lpc = 1;
  std::vector<VolumeCell> cells;  // flat index ((z*rows + y)*cols + x)*lpc + l
  cudaStream_t stream = nullptr;
  uint64_t epoch = 0;             // current forward; a forward starting at hop 0 opens a new one
  ~Volume();
};

Status volume_create(int depth, int rows, int cols, int lpc, Volume** out);
int volume_index(const Volume& v, int z, int y, int x, int l);  // -1 when out of range
// Hop order is the flat index order (z, y, x, l nested), src/architecture/grid.cpp:82-95.
int volume_hops(const Volume& v);

Status volume_bind_dense(Volume* v, int idx, int in, int out, int act, DType dt, const float* W, bool w_dev,
                         const double* bias, size_t bias_len);
Status volume_bind_dense_native(Volume* v, int idx, int in, int out, int act, DType dt, const uint8_t* native,
                                size_t native_len, float scale, const double* bias, size_t bias_len);
Status volume_bind_swiglu(Volume* v, int idx, int in, int inter, DType dt, const float* G, const float* U,
                          const float* D, bool w_dev);
Status volume_bind_mha(Volume* v, int idx, const MhaConfig& cfg, int seq, DType dt, const float* Q, const float* K,
                       const float* V, const float* O, bool w_dev);
Status volume_bind_rmsnorm(Volume* v, int idx, int dim, double eps, DType dt, const float* gamma);
// The same cells from weight sources (float32 values or a stored model's native bytes).
Status volume_bind_swiglu_src(Volume* v, int idx, int in, int inter, DType dt, const WeightSrc (&w)[3]);
Status volume_bind_mha_src(Volume* v, int idx, const MhaConfig& cfg, int seq, DType dt, const WeightSrc (&w)[4]);
Status volume_bind_rmsnorm_src(Volume* v, int idx, int dim, double eps, DType dt, const WeightSrc& gamma);
// Tokens per sequence of an MHA cell (rows = batch * seq), as the input shape of a forward sets it.
Status volume_set_mha_seq(Volume* v, int idx, int seq);
Status volume_set_remote_link(Volume* v, int idx, int target);
Status volume_set_disabled(Volume* v, int idx, bool disabled);

// Runs hops [hop_begin, hop_end) on `rows` input rows x (device, [rows][in_width]) and copies
// the last executed cell's post to `out` ([rows][out_width], may be nullptr). `out_width`
// receives that width. As in the reference, a remote link reads the post its target recorded
// earlier in the same forward: a range starting at hop 0 opens a forward, a range starting
// later continues the current one (consecutive ranges of one pipelined forward), and a
// target not executed in it -- later in hop order, disabled, or run on other rows -- is an
// error.
Status volume_forward_device(Volume* v, int rows, const float* x, int in_width, int hop_begin, int hop_end,
                             float* out, int* out_width, cudaStream_t st);

// The same over an explicit forward: `open` starts a new one (remote-link targets must then be
// executed within this call); *last_post (may be nullptr) receives the device address of the
// last executed cell's post, valid until that cell runs again.
Status volume_forward_range(Volume* v, int rows, const float* x, int in_width, int hop_begin, int hop_end,
                            float* out, int* out_width, cudaStream_t st, bool open, const float** last_post);

// Device pointers of a cell's last pre / post ([rows][width]) for step records.
Status volume_cell_outputs(Volume* v, int idx, const float** pre, int* pre_width, const float** post,
                           int* post_width);

} // namespace wb
