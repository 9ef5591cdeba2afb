// volume.cpp -- device-resident volume forward (src/runtime/forward.cpp:98-156 semantics).
//
// For every coordinate in hop order: disabled cells are skipped; a cell with a remote link
// reads the recorded post of its target instead of the running activation; otherwise it
// reads the previous executed cell's post; its post becomes the running activation. An
// empty grid or an unbound enabled cell is an error, as in the reference.
#include "volume.hpp"

#include "cell_kernels.hpp"

#include <cstdlib>
#include <string>

namespace wb {

namespace {
template <typename T>
void free_dev(T*& p) {
  if (p) cudaFree(p);
  p = nullptr;
}

std::string coord_str(const Volume& v, int idx) {
  int l = idx % v.lpc, r = idx / v.lpc;
  int x = r % v.cols;
  r /= v.cols;
  int y = r % v.rows, z = r / v.rows;
  return "z=" + std::to_string(z) + " y=" + std::to_string(y) + " x=" + std::to_string(x) + " l=" + std::to_string(l);
}

Status reserve_cell(VolumeCell& c, int rows, cudaStream_t st) {
  if (c.rows >= rows) return Status::Ok();
  free_dev(c.pre);
  free_dev(c.post);
  c.io.release();
  c.rows = 0;
  WB_CUDA(cudaMalloc(&c.pre, static_cast<size_t>(rows) * c.pre_width * 4));
  WB_CUDA(cudaMalloc(&c.post, static_cast<size_t>(rows) * c.out_width * 4));
  if (c.op == OpKind::Dense) WB_TRY(alloc_io(*c.dense, rows, &c.io, st));
  c.rows = rows;
  return Status::Ok();
}
} // namespace

VolumeCell::~VolumeCell() {
  free_dev(pre);
  free_dev(post);
  free_dev(gamma64);
  io.release();
}

Volume::~Volume() {
  cudaSetDevice(device);
  if (stream) cudaStreamSynchronize(stream);
  cells.clear();
  if (stream) cudaStreamDestroy(stream);
}

Status volume_create(int depth, int rows, int cols, int lpc, Volume** out) {
  if (!out) return Status::Invalid("volume: nil out");
  // src/architecture/grid.cpp:31-36: non-positive dims become 1
  auto* v = new Volume();
  v->depth = depth < 1 ? 1 : depth;
  v->rows = rows < 1 ? 1 : rows;
  v->cols = cols < 1 ? 1 : cols;
  v->lpc = lpc < 1 ? 1 : lpc;
  Status st = library_device(&v->device);
  if (st.ok()) st = cuda_status(cudaSetDevice(v->device), "cudaSetDevice");
  if (st.ok()) st = cuda_status(cudaStreamCreateWithFlags(&v->stream, cudaStreamNonBlocking), "stream");
  if (!st.ok()) {
    delete v;
    return st;
  }
  v->cells = std::vector<VolumeCell>(static_cast<size_t>(v->depth) * v->rows * v->cols * v->lpc);
  *out = v;
  return Status::Ok();
}

int volume_index(const Volume& v, int z, int y, int x, int l) {
  if (z < 0 || z >= v.depth || y < 0 || y >= v.rows || x < 0 || x >= v.cols || l < 0 || l >= v.lpc) return -1;
  return ((z * v.rows + y) * v.cols + x) * v.lpc + l;
}

int volume_hops(const Volume& v) { return static_cast<int>(v.cells.size()); }

static Status check_idx(Volume* v, int idx) {
  if (!v || idx < 0 || idx >= volume_hops(*v)) return Status::Invalid("architecture: bad bind coord");
  return Status::Ok();
}

static void reset_cell(VolumeCell& c) {
  const bool remote = c.remote;
  const int target = c.target;
  const bool disabled = c.disabled;
  c.~VolumeCell();
  new (&c) VolumeCell();
  c.remote = remote;
  c.target = target;
  c.disabled = disabled;
}

Status volume_bind_dense(Volume* v, int idx, int in, int out, int act, DType dt, const float* W, bool w_dev,
                         const double* bias, size_t bias_len) {
  WB_TRY(check_idx(v, idx));
  VolumeCell& c = v->cells[static_cast<size_t>(idx)];
  reset_cell(c);
  c.store = std::make_unique<WeightStore>();
  c.dense = std::make_unique<DeviceDense>();
  WB_TRY(mount_dense(v->device, out, in, dt, act, W, w_dev, bias, bias_len, c.store.get(), c.dense.get(), v->stream));
  c.op = OpKind::Dense;
  c.in_width = in;
  c.out_width = out;
  c.pre_width = out;
  return Status::Ok();
}

Status volume_bind_dense_native(Volume* v, int idx, int in, int out, int act, DType dt, const uint8_t* native,
                                size_t native_len, float scale, const double* bias, size_t bias_len) {
  WB_TRY(check_idx(v, idx));
  VolumeCell& c = v->cells[static_cast<size_t>(idx)];
  reset_cell(c);
  c.store = std::make_unique<WeightStore>();
  c.dense = std::make_unique<DeviceDense>();
  WB_TRY(mount_dense_native(v->device, out, in, dt, act, native, native_len, scale, bias, bias_len, c.store.get(),
                            c.dense.get(), v->stream));
  c.op = OpKind::Dense;
  c.in_width = in;
  c.out_width = out;
  c.pre_width = out;
  return Status::Ok();
}

Status volume_bind_swiglu(Volume* v, int idx, int in, int inter, DType dt, const float* G, const float* U,
                          const float* D, bool w_dev) {
  WeightSrc w[3];
  const float* m[3] = {G, U, D};
  for (int i = 0; i < 3; ++i) {
    w[i].f32 = m[i];
    w[i].f32_on_device = w_dev;
  }
  return volume_bind_swiglu_src(v, idx, in, inter, dt, w);
}

Status volume_bind_swiglu_src(Volume* v, int idx, int in, int inter, DType dt, const WeightSrc (&w)[3]) {
  WB_TRY(check_idx(v, idx));
  VolumeCell& c = v->cells[static_cast<size_t>(idx)];
  reset_cell(c);
  c.swiglu = std::make_unique<SwigluCell>();
  WB_TRY(swiglu_mount_src(v->device, in, inter, dt, w, c.swiglu.get(), v->stream));
  c.op = OpKind::SwiGLU;
  c.in_width = in;
  c.out_width = in;
  c.pre_width = inter;
  return Status::Ok();
}

Status volume_bind_mha(Volume* v, int idx, const MhaConfig& cfg, int seq, DType dt, const float* Q, const float* K,
                       const float* V, const float* O, bool w_dev) {
  WeightSrc w[4];
  const float* m[4] = {Q, K, V, O};
  for (int i = 0; i < 4; ++i) {
    w[i].f32 = m[i];
    w[i].f32_on_device = w_dev;
  }
  return volume_bind_mha_src(v, idx, cfg, seq, dt, w);
}

Status volume_bind_mha_src(Volume* v, int idx, const MhaConfig& cfg, int seq, DType dt, const WeightSrc (&w)[4]) {
  WB_TRY(check_idx(v, idx));
  if (seq <= 0) return Status::Invalid("mha: bad seq");
  VolumeCell& c = v->cells[static_cast<size_t>(idx)];
  reset_cell(c);
  c.mha = std::make_unique<MhaCell>();
  WB_TRY(mha_mount_src(v->device, cfg, dt, w, c.mha.get(), v->stream));
  c.op = OpKind::MHA;
  c.mha_seq = seq;
  c.in_width = c.mha->cfg.d_model;
  c.out_width = c.mha->cfg.d_model;
  c.pre_width = c.mha->cfg.num_heads * c.mha->cfg.head_dim;
  return Status::Ok();
}

Status volume_set_mha_seq(Volume* v, int idx, int seq) {
  WB_TRY(check_idx(v, idx));
  VolumeCell& c = v->cells[static_cast<size_t>(idx)];
  if (c.op != OpKind::MHA || seq <= 0) return Status::Invalid("mha: bad seq");
  c.mha_seq = seq;
  return Status::Ok();
}

Status volume_bind_rmsnorm(Volume* v, int idx, int dim, double eps, DType dt, const float* gamma) {
  if (dim <= 0 || !gamma) return Status::Invalid("rmsnorm: invalid argument");
  WeightSrc w;
  w.f32 = gamma;
  return volume_bind_rmsnorm_src(v, idx, dim, eps, dt, w);
}

Status volume_bind_rmsnorm_src(Volume* v, int idx, int dim, double eps, DType dt, const WeightSrc& gamma) {
  WB_TRY(check_idx(v, idx));
  if (dim <= 0) return Status::Invalid("rmsnorm: invalid argument");
  VolumeCell& c = v->cells[static_cast<size_t>(idx)];
  reset_cell(c);
  WB_TRY(rmsnorm_gamma_src(v->device, dim, dt, gamma, &c.gamma64, v->stream));
  c.op = OpKind::RMSNorm;
  c.eps = eps <= 0.0 ? 1e-6 : eps;
  c.in_width = c.out_width = c.pre_width = dim;
  return Status::Ok();
}

Status volume_set_remote_link(Volume* v, int idx, int target) {
  if (!v || idx < 0 || idx >= volume_hops(*v)) return Status::Invalid("architecture: bad source coord");
  if (target < 0 || target >= volume_hops(*v)) return Status::Invalid("architecture: bad target coord");
  VolumeCell& c = v->cells[static_cast<size_t>(idx)];
  c.remote = true;
  c.target = target;
  return Status::Ok();
}

Status volume_set_disabled(Volume* v, int idx, bool disabled) {
  WB_TRY(check_idx(v, idx));
  v->cells[static_cast<size_t>(idx)].disabled = disabled;
  return Status::Ok();
}

Status volume_forward_device(Volume* v, int rows, const float* x, int in_width, int hop_begin, int hop_end,
                             float* out, int* out_width, cudaStream_t st) {
  if (!v) return Status::Invalid("runtime.forward: nil volume");
  return volume_forward_range(v, rows, x, in_width, hop_begin, hop_end, out, out_width, st,
                              hop_begin <= 0 || v->epoch == 0, nullptr);
}

// Whether the RMSNorm cell at hop h runs inside the next enabled hop: that hop reads the norm's
// output as its own input (not a remote link) and is a Dense, SwiGLU or MHA cell of the same
// width, within this range. WELVET_B200_NORM_PROLOGUE=0 keeps the norm a kernel of its own.
static bool norm_prologue_wanted(const Volume& v, int h, int hop_end, int rows, int width) {
  const char* env = std::getenv("WELVET_B200_NORM_PROLOGUE");
  if (env && env[0] == '0') return false;
  for (int n = h + 1; n < hop_end; ++n) {
    const VolumeCell& c = v.cells[static_cast<size_t>(n)];
    if (c.disabled) continue;
    if (c.remote || c.in_width != width) return false;
    if (c.op == OpKind::MHA) return c.mha_seq > 0 && rows % c.mha_seq == 0;
    return c.op == OpKind::Dense || c.op == OpKind::SwiGLU;
  }
  return false;
}

Status volume_forward_range(Volume* v, int rows, const float* x, int in_width, int hop_begin, int hop_end,
                            float* out, int* out_width, cudaStream_t st, bool open, const float** last_post) {
  if (!v) return Status::Invalid("runtime.forward: nil volume");
  if (rows <= 0 || !x || in_width <= 0) return Status::Invalid("runtime.forward: empty input");
  const int hops = volume_hops(*v);
  if (hop_begin < 0) hop_begin = 0;
  if (hop_end > hops || hop_end < 0) hop_end = hops;
  WB_CUDA(cudaSetDevice(v->device));
  if (open) ++v->epoch;
  const float* cur = x;
  int cur_w = in_width;
  int last = -1;
  // An RMSNorm cell whose post feeds the next enabled cell's projections directly is run by
  // that cell (the projection GEMM's prologue): `norm` holds it and norm_in its input.
  SplitNorm norm;
  const float* norm_in = nullptr;
  for (int h = hop_begin; h < hop_end; ++h) {
    VolumeCell& c = v->cells[static_cast<size_t>(h)];
    if (c.disabled) continue;
    if (c.op == OpKind::None) return Status::Invalid("runtime.forward: no op at " + coord_str(*v, h));
    const float* in = cur;
    int in_w = cur_w;
    const SplitNorm* pn = nullptr;
    if (norm.gamma && !c.remote) {
      pn = &norm;
      in = norm_in;
    }
    if (c.remote) {
      const VolumeCell& t = v->cells[static_cast<size_t>(c.target)];
      if (t.epoch != v->epoch || t.epoch_rows != rows)
        return Status::Invalid("runtime.forward: remote hop has no recorded activation -> " + coord_str(*v, c.target));
      in = t.post;
      in_w = t.out_width;
    }
    if (in_w != c.in_width)  // dense: src/layers/dense/dense.cpp:70-73
      return Status::Invalid(std::string(c.op == OpKind::Dense ? "dense" : "cell") + ": input width mismatch (" +
                             std::to_string(in_w) + " != " + std::to_string(c.in_width) + ") at " +
                             coord_str(*v, h));
    WB_TRY(reserve_cell(c, rows, st));
    switch (c.op) {
    case OpKind::Dense:
      WB_TRY(forward_device(*c.dense, rows, in, in_w, c.pre, c.post, &c.io, st, true, 0, nullptr, pn));
      break;
    case OpKind::SwiGLU:
      WB_TRY(swiglu_forward_device(c.swiglu.get(), rows, in, c.pre, c.post, st, true, pn));
      break;
    case OpKind::MHA:
      if (rows % c.mha_seq != 0) return Status::Invalid("mha: rows not a multiple of seq at " + coord_str(*v, h));
      WB_TRY(mha_forward_device(c.mha.get(), rows / c.mha_seq, c.mha_seq, in, c.pre, c.post, st, pn));
      break;
    case OpKind::RMSNorm:
      if (norm_prologue_wanted(*v, h, hop_end, rows, c.out_width)) {
        norm.gamma = c.gamma64;
        norm.eps = c.eps;
        norm.pre = c.pre;
        norm.post = c.post;
        norm_in = in;
      } else {
        WB_TRY(launch_rmsnorm(in, c.gamma64, c.pre, c.post, rows, c.in_width, c.eps, st));
      }
      break;
    default:
      return Status::Err(StatusCode::Gap, "gap? runtime.forward: unsupported cell Op");
    }
    if (pn) norm = SplitNorm{};
    c.epoch = v->epoch;
    c.epoch_rows = rows;
    cur = c.post;
    cur_w = c.out_width;
    last = h;
  }
  if (last < 0) return Status::Invalid("runtime.forward: grid has no enabled cells with ops");
  if (out_width) *out_width = cur_w;
  if (last_post) *last_post = cur;
  if (out) {
    WB_CUDA(cudaMemcpyAsync(out, cur, static_cast<size_t>(rows) * cur_w * 4, cudaMemcpyDeviceToDevice, st));
  }
  return Status::Ok();
}

Status volume_cell_outputs(Volume* v, int idx, const float** pre, int* pre_width, const float** post,
                           int* post_width) {
  WB_TRY(check_idx(v, idx));
  const VolumeCell& c = v->cells[static_cast<size_t>(idx)];
  if (pre) *pre = c.pre;
  if (pre_width) *pre_width = c.pre_width;
  if (post) *post = c.post;
  if (post_width) *post_width = c.out_width;
  return Status::Ok();
}

} // namespace wb
