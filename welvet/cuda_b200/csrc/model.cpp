// model.cpp -- persistent model sessions over a stored model descriptor (WMN1).
//
// The descriptor is read in the order of the reference's welvet_model_mount
// (src/interop/model_session.cpp:317-396): magic, root, child count, grid dims, the children
// (include/welvet/interop/child_wire.hpp:21-192), the root's training controls and each
// child's control tree (model_wire.hpp:195-263; read and checked, not used by a forward), the
// store section (model_session.cpp:135-153: each store's dtype, shape, scale, float32 values,
// native bytes and bias, in the order cam_sync.cpp:8-40 collects them), then, for a Grid root,
// each cell's enabled flag and remote link. The layers are mounted from the stores -- the
// stored native bytes, not a re-encoding of the children's float32 initial weights -- into a
// volume whose hop order is the child order.
#include "model.hpp"

#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>

namespace wb {

namespace {

struct GapError : std::runtime_error {
  explicit GapError(const std::string& m) : std::runtime_error(m) {}
};
struct StatusError : std::runtime_error {
  Status st;
  explicit StatusError(Status s) : std::runtime_error(s.message), st(std::move(s)) {}
};

void require(bool ok, const char* why) {
  if (!ok) throw std::invalid_argument(why);
}

void good(Status s) {
  if (!s.ok()) throw StatusError(std::move(s));
}

// Bounds-checked little-endian reader of the descriptor (model_session.cpp:3-36).
struct Reader {
  const uint8_t* p;
  size_t left;
  template <class T>
  T one() {
    T v{};
    if (left < sizeof(T)) throw std::invalid_argument("truncated descriptor");
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    left -= sizeof(T);
    return v;
  }
  // n elements of T, skipped (their bytes are bounds-checked)
  template <class T>
  void skip(int64_t n) {
    if (n < 0 || static_cast<uint64_t>(n) > left / sizeof(T)) throw std::invalid_argument("short model payload");
    p += static_cast<size_t>(n) * sizeof(T);
    left -= static_cast<size_t>(n) * sizeof(T);
  }
  template <class T>
  std::vector<T> vec() {
    const int32_t n = one<int32_t>();
    if (n < 0 || static_cast<size_t>(n) > left / sizeof(T)) throw std::invalid_argument("invalid vector length");
    std::vector<T> v(static_cast<size_t>(n));
    if (n) std::memcpy(v.data(), p, static_cast<size_t>(n) * sizeof(T));
    p += static_cast<size_t>(n) * sizeof(T);
    left -= static_cast<size_t>(n) * sizeof(T);
    return v;
  }
  void end() const {
    if (left) throw std::invalid_argument("trailing descriptor bytes");
  }
};

// child_wire.hpp:15-20: a payload count is positive (or zero where allowed), at most 2^26,
// and within the bytes left.
int64_t checked_count(const Reader& r, int64_t n, bool empty = false) {
  if (n < 0 || (!empty && n == 0) || n > (int64_t(1) << 26) || static_cast<uint64_t>(n) > r.left / 4)
    throw std::invalid_argument("invalid model payload size");
  return n;
}

// stack::Kind values (include/welvet/stack.hpp:50-58) of the children served here.
enum : int32_t { kNone = 0, kDense = 1, kRMSNorm = 2, kSwiGLU = 4, kMHA = 7 };

struct Child {
  int kind = kNone;
  int in = 0, out = 0, act = -1, dtype = 1;  // Dense (dtype for every kind)
  int dim = 0;                               // RMSNorm
  double eps = 0.0;
  int inter = 0;                             // SwiGLU (in, inter)
  MhaConfig mha;                             // MHA
  int seq = 0;
  std::vector<std::pair<int, int>> stores;   // (rows, cols) of its stores, collect_stores order
};

Child read_child(Reader& r) {
  Child c;
  c.kind = r.one<int32_t>();
  switch (c.kind) {
  case kNone:
    return c;
  case kDense: {  // child_wire.hpp:29-55
    c.in = r.one<int32_t>();
    c.out = r.one<int32_t>();
    c.act = r.one<int32_t>();
    c.dtype = r.one<int32_t>();
    require(c.in > 0 && c.out > 0, "invalid model child");
    r.skip<float>(checked_count(r, int64_t(c.out) * c.in));
    const uint32_t bias_len = r.one<uint32_t>();
    r.skip<double>(checked_count(r, bias_len, true));
    c.stores = {{c.out, c.in}};
    return c;
  }
  case kRMSNorm: {  // child_wire.hpp:56-73
    c.dim = r.one<int32_t>();
    c.dtype = r.one<int32_t>();
    c.eps = r.one<double>();
    r.skip<float>(checked_count(r, c.dim));
    c.stores = {{1, c.dim}};
    return c;
  }
  case kSwiGLU: {  // child_wire.hpp:94-114
    c.in = r.one<int32_t>();
    c.inter = r.one<int32_t>();
    c.dtype = r.one<int32_t>();
    require(c.in > 0 && c.inter > 0, "invalid model child");
    r.skip<float>(checked_count(r, 3 * int64_t(c.inter) * c.in));
    c.stores = {{c.inter, c.in}, {c.inter, c.in}, {c.in, c.inter}};
    return c;
  }
  case kMHA: {  // child_wire.hpp:153-192
    const int32_t seq = r.one<int32_t>(), d_model = r.one<int32_t>(), num_heads = r.one<int32_t>();
    const int32_t num_kv = r.one<int32_t>(), head_dim = r.one<int32_t>(), msl = r.one<int32_t>();
    const int32_t mask = r.one<int32_t>(), pos = r.one<int32_t>();
    c.dtype = r.one<int32_t>();
    require(num_heads > 0 && d_model > 0 && num_kv >= 0 && head_dim >= 0, "invalid model child");
    const int hd = head_dim > 0 ? head_dim : d_model / num_heads;
    const int kv_heads = num_kv > 0 ? num_kv : num_heads;
    const int64_t q_dim = int64_t(num_heads) * hd, kv_dim = int64_t(kv_heads) * hd;
    r.skip<float>(checked_count(r, q_dim * d_model));
    r.skip<float>(checked_count(r, kv_dim * d_model));
    r.skip<float>(checked_count(r, kv_dim * d_model));
    r.skip<float>(checked_count(r, d_model * q_dim));
    // mha::decoder_causal (src/layers/mha/mha.cpp:83-93) with the descriptor's overrides
    c.mha.d_model = d_model;
    c.mha.num_heads = num_heads;
    c.mha.num_kv_heads = kv_heads;
    c.mha.head_dim = head_dim;
    c.mha.max_seq_len = msl > 0 ? msl : seq;
    c.mha.mask = mask;
    c.mha.pos = pos;
    c.seq = seq;
    c.stores = {{static_cast<int>(q_dim), d_model},
                {static_cast<int>(kv_dim), d_model},
                {static_cast<int>(kv_dim), d_model},
                {d_model, static_cast<int>(q_dim)}};
    return c;
  }
  default:
    throw GapError("model child kind " + std::to_string(c.kind) +
                   " (served: Dense, RMSNorm, SwiGLU, MHA)");
  }
}

// model_wire.hpp:195-253: training modes, branch rates, coefficients and an optional sync
// configuration -- scheduling state of the reference's trainers, checked and skipped.
void skip_controls(Reader& r) {
  int32_t n = r.one<int32_t>();
  require(n >= 0 && n <= 4096, "invalid root controls");
  for (int i = 0; i < n; ++i) {
    const int32_t m = r.one<int32_t>();
    require(m >= 0 && m <= 33, "invalid root controls");
  }
  n = r.one<int32_t>();
  require(n >= 0 && n <= 4096, "invalid root controls");
  r.skip<double>(n);
  r.skip<double>(3);  // shadow_coef, surprise_thresh, last_loss
  if (!r.one<int32_t>()) return;
  r.one<int32_t>();   // enabled
  r.one<double>();    // alpha
  const int32_t when = r.one<int32_t>();
  require(when >= 0 && when <= 3, "invalid root controls");
  n = r.one<int32_t>();
  require(n >= 0 && n <= 4096, "invalid root controls");
  r.skip<double>(n);  // branch_alpha
  n = r.one<int32_t>();
  require(n >= 0 && n <= 4096, "invalid root controls");
  for (int g = 0; g < n; ++g) {
    const int32_t count = r.one<int32_t>();
    require(count >= 0 && count <= 4096, "invalid root controls");
    r.skip<int32_t>(count);
  }
  n = r.one<int32_t>();
  require(n >= 0 && n <= 4096, "invalid root controls");
  r.skip<int32_t>(int64_t(n) * 6);  // cross pairs: two (stack_idx, branch, store) endpoints
}

struct Store {
  DType dtype = DType::Float32;
  float scale = 1.0f;
  std::vector<float> f32;
  std::vector<uint8_t> native;
  std::vector<double> bias;
  WeightSrc src() const {
    WeightSrc w;
    if (dtype == DType::Float32) {
      w.f32 = f32.data();
    } else {
      w.native = native.data();
      w.native_len = native.size();
      w.scale = scale;
    }
    return w;
  }
};

bool served_dtype(int dt) { return dt == 1 || dt == 4 || dt == 5 || dt == 9 || dt == 16; }

// read_store (model_session.cpp:135-153): metadata must match the layer's store shape, and
// the payload lengths those of a fresh store of that dtype (float32 values for Float32,
// native bytes otherwise).
Store read_store(Reader& r, int rows, int cols) {
  Store s;
  const int32_t dt = r.one<int32_t>(), sr = r.one<int32_t>(), sc = r.one<int32_t>();
  s.scale = r.one<float>();
  require(dt >= 0 && dt <= 33 && sr == rows && sc == cols && std::isfinite(s.scale),
          "native store metadata mismatch");
  s.f32 = r.vec<float>();
  s.native = r.vec<uint8_t>();
  s.bias = r.vec<double>();
  if (!served_dtype(dt))
    throw StatusError(Status::Unsupported("model store dtype " + std::to_string(dt) +
                                          " (served: Float32, FP8 E4M3/E5M2, Int8, FP4)"));
  s.dtype = static_cast<DType>(dt);
  const int64_t n = int64_t(rows) * cols;
  const int64_t nat = dt == 1 ? 0 : (dt == 16 ? (n + 1) / 2 : n);
  require(static_cast<int64_t>(s.f32.size()) == (dt == 1 ? n : 0) && static_cast<int64_t>(s.native.size()) == nat,
          "native store payload length mismatch");
  return s;
}

DType common_dtype(const std::vector<Store>& st, size_t first, size_t n, const char* what) {
  for (size_t i = first + 1; i < first + n; ++i)
    if (st[i].dtype != st[first].dtype)
      throw GapError(std::string(what) + " with stores of different dtypes");
  return st[first].dtype;
}

Status mount_impl(const uint8_t* desc, size_t size, ModelSession* s) {
  require(desc && size >= 28 && size <= (size_t(1) << 28), "invalid mount arguments");
  Reader r{desc, size};
  require(r.one<uint32_t>() == 0x314e4d57u, "unsupported model descriptor version");
  s->root = r.one<int32_t>();
  const int count = r.one<int32_t>();
  require(s->root >= 0 && s->root <= 2 && count > 0 && count <= 4096, "invalid model root/count");
  int dims[4];
  for (int& d : dims) d = r.one<int32_t>();
  if (s->root == 1) throw GapError("Parallel model root");
  std::vector<Child> ch;
  ch.reserve(static_cast<size_t>(count));
  for (int i = 0; i < count; ++i) ch.push_back(read_child(r));
  skip_controls(r);                            // root controls
  for (int i = 0; i < count; ++i) skip_controls(r);  // each child's tree (no nested children here)
  size_t nstores = 0;
  for (const Child& c : ch) nstores += c.stores.size();
  require(r.one<int32_t>() == static_cast<int32_t>(nstores), "store count mismatch");
  std::vector<Store> st;
  st.reserve(nstores);
  for (const Child& c : ch)
    for (const auto& rc : c.stores) st.push_back(read_store(r, rc.first, rc.second));

  struct CellLink {
    bool enabled = true, remote = false;
    int tz = 0, ty = 0, tx = 0, tl = 0;
  };
  std::vector<CellLink> links(static_cast<size_t>(count));
  if (s->root == 2) {
    int64_t n = 1;
    for (int d : dims) {
      require(d > 0 && d <= 4096 && n <= 4096 / d, "invalid grid dimensions");
      n *= d;
    }
    require(n == count, "grid cell count mismatch");
    for (int i = 0; i < count; ++i) {
      CellLink& l = links[static_cast<size_t>(i)];
      l.enabled = r.one<int32_t>() != 0;
      require(!l.enabled || ch[static_cast<size_t>(i)].kind != kNone, "enabled grid cell has no operation");
      l.remote = r.one<int32_t>() != 0;
      l.tz = r.one<int32_t>();
      l.ty = r.one<int32_t>();
      l.tx = r.one<int32_t>();
      l.tl = r.one<int32_t>();
    }
  }
  r.end();

  // a Stack runs its children in order: a volume of one cell with `count` layers
  if (s->root == 0) dims[0] = dims[1] = dims[2] = 1, dims[3] = count;
  good(volume_create(dims[0], dims[1], dims[2], dims[3], &s->vol));
  Volume* v = s->vol;
  size_t si = 0;
  for (int i = 0; i < count; ++i) {
    const Child& c = ch[static_cast<size_t>(i)];
    const CellLink& l = links[static_cast<size_t>(i)];
    switch (c.kind) {
    case kNone:
      break;
    case kDense: {
      const Store& w = st[si];
      if (w.dtype == DType::Float32)
        good(volume_bind_dense(v, i, c.in, c.out, c.act, w.dtype, w.f32.data(), false,
                               w.bias.empty() ? nullptr : w.bias.data(), w.bias.size()));
      else
        good(volume_bind_dense_native(v, i, c.in, c.out, c.act, w.dtype, w.native.data(), w.native.size(), w.scale,
                                      w.bias.empty() ? nullptr : w.bias.data(), w.bias.size()));
      if (l.enabled) s->dense = true;
      break;
    }
    case kRMSNorm:
      good(volume_bind_rmsnorm_src(v, i, c.dim, c.eps, st[si].dtype, st[si].src()));
      break;
    case kSwiGLU: {
      const DType dt = common_dtype(st, si, 3, "SwiGLU");
      const WeightSrc w[3] = {st[si].src(), st[si + 1].src(), st[si + 2].src()};
      good(volume_bind_swiglu_src(v, i, c.in, c.inter, dt, w));
      break;
    }
    case kMHA: {
      const DType dt = common_dtype(st, si, 4, "MHA");
      const WeightSrc w[4] = {st[si].src(), st[si + 1].src(), st[si + 2].src(), st[si + 3].src()};
      good(volume_bind_mha_src(v, i, c.mha, c.seq > 0 ? c.seq : 1, dt, w));
      s->mha.push_back(i);
      break;
    }
    default:
      break;
    }
    si += c.stores.size();
    const VolumeCell& cell = v->cells[static_cast<size_t>(i)];
    if (cell.out_width > s->max_width) s->max_width = cell.out_width;
    if (c.kind == kNone || !l.enabled) good(volume_set_disabled(v, i, true));
    if (l.remote) {
      const int t = volume_index(*v, l.tz, l.ty, l.tx, l.tl);
      require(t >= 0, "invalid remote link");
      good(volume_set_remote_link(v, i, t));
    }
  }
  return Status::Ok();
}

template <class F>
Status guarded(F fn) {
  try {
    return fn();
  } catch (const GapError& e) {
    return Status::Err(StatusCode::Gap, std::string("gap? ") + e.what());
  } catch (const StatusError& e) {
    return e.st;
  } catch (const std::invalid_argument& e) {
    return Status::Invalid(e.what());
  } catch (const std::exception& e) {
    return Status::Internal(e.what());
  }
}

} // namespace

ModelSession::~ModelSession() {
  if (vol) {
    cudaSetDevice(vol->device);
    if (x_dev) cudaFree(x_dev);
    if (y_dev) cudaFree(y_dev);
  }
  delete vol;
}

Status model_mount(const uint8_t* desc, size_t size, ModelSession** out) {
  if (out) *out = nullptr;
  if (!out) return Status::Invalid("invalid mount arguments");
  auto* s = new ModelSession();
  const Status st = guarded([&] { return mount_impl(desc, size, s); });
  if (!st.ok()) {
    delete s;
    return st;
  }
  *out = s;
  return Status::Ok();
}

Status model_forward(ModelSession* s, const uint8_t* input, size_t size, std::vector<uint8_t>* out) {
  if (!s || !input || !out) return Status::Invalid("invalid forward arguments");
  std::lock_guard<std::mutex> lock(s->mu);
  return guarded([&]() -> Status {
    // tensor (model_session.cpp:101-116)
    Reader r{input, size};
    const int32_t rank = r.one<int32_t>();
    require(rank > 0 && rank <= 5, "tensor rank must be 1..5");
    std::vector<int32_t> dims(static_cast<size_t>(rank));
    int64_t n = 1;
    for (auto& d : dims) {
      d = r.one<int32_t>();
      require(d > 0 && n <= (int64_t(1) << 26) / d, "invalid tensor shape");
      n *= d;
    }
    require(static_cast<uint64_t>(n) <= r.left / 4, "short tensor data");
    const float* x = reinterpret_cast<const float*>(r.p);
    r.skip<float>(n);
    r.end();
    // the layers' shape rules: Dense takes [batch, in]; RMSNorm, SwiGLU and MHA [batch, in] or
    // [batch, seq, in] ([seq, d] is one sequence for MHA); every layer keeps the leading dims
    if (s->dense && rank != 2) return Status::Invalid("dense: input shape need [batch,in]");
    require(rank == 2 || rank == 3, "model input must be [batch, in] or [batch, seq, in]");
    const int width = dims.back();
    const int rows = static_cast<int>(n / width);
    const int seq = rank == 3 ? dims[1] : rows;
    for (int idx : s->mha) WB_TRY(volume_set_mha_seq(s->vol, idx, seq));
    Volume* v = s->vol;
    WB_CUDA(cudaSetDevice(v->device));
    const size_t xn = static_cast<size_t>(n), yn = static_cast<size_t>(rows) * static_cast<size_t>(s->max_width);
    if (s->x_cap < xn) {
      if (s->x_dev) cudaFree(s->x_dev);
      s->x_dev = nullptr;
      s->x_cap = 0;
      WB_CUDA(cudaMalloc(&s->x_dev, xn * 4));
      s->x_cap = xn;
    }
    if (s->y_cap < yn) {
      if (s->y_dev) cudaFree(s->y_dev);
      s->y_dev = nullptr;
      s->y_cap = 0;
      WB_CUDA(cudaMalloc(&s->y_dev, yn * 4));
      s->y_cap = yn;
    }
    WB_CUDA(cudaMemcpyAsync(s->x_dev, x, xn * 4, cudaMemcpyHostToDevice, v->stream));
    int ow = 0;
    WB_TRY(volume_forward_device(v, rows, s->x_dev, width, 0, -1, s->y_dev, &ow, v->stream));
    const size_t on = static_cast<size_t>(rows) * static_cast<size_t>(ow);
    // output tensor: the input's leading dims and the last cell's width (tensor_out,
    // model_session.cpp:117-122)
    out->assign(4 * (1 + dims.size()) + on * 4, 0);
    uint8_t* o = out->data();
    std::memcpy(o, &rank, 4);
    for (size_t i = 0; i + 1 < dims.size(); ++i) std::memcpy(o + 4 * (1 + i), &dims[i], 4);
    std::memcpy(o + 4 * dims.size(), &ow, 4);
    WB_CUDA(cudaMemcpyAsync(o + 4 * (1 + dims.size()), s->y_dev, on * 4, cudaMemcpyDeviceToHost, v->stream));
    WB_CUDA(cudaStreamSynchronize(v->stream));
    return Status::Ok();
  });
}

} // namespace wb
