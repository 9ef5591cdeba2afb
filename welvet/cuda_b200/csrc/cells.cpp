// cells.cpp -- SwiGLU / MHA / RMSNorm cells over the packed Dense mirror.
//
// SwiGLU (src/layers/swiglu/swiglu.cpp:87-136): the reference runs Gate and Up as two Dense
// forwards, copies both back to the host, launches the SiLU product with a per-call
// allocation and runs Down. Here Gate and Up stream in one fused GEMV whose epilogue writes
// h directly (padded for Down), and Down reads h on the device.
// MHA (src/layers/mha/mha.cpp:123-183): Q/K/V Dense, attention core, O Dense -- all on the
// device with no host round trip.
#include "cells.hpp"

#include "codec.hpp"
#include "gemm_tc.hpp"
#include "gemv.hpp"
#include "gemv_tc.hpp"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace wb {

namespace {
template <typename T>
void free_dev(T*& p) {
  if (p) cudaFree(p);
  p = nullptr;
}
} // namespace

SwigluCell::~SwigluCell() {
  release_work();
  cudaSetDevice(device);
  free_dev(Wg_pair);
}

void SwigluCell::release_work() {
  cudaSetDevice(device);
  free_dev(x_pad);
  free_dev(h_pad);
  free_dev(g_buf);
  free_dev(u_buf);
  free_dev(pair_scratch);
  pair_scratch_bytes = 0;
  io_gate.release();
  io_up.release();
  io_down.release();
  bs = 0;
}

Status mount_dense_src(int device, int rows, int cols, DType dt, int act, const WeightSrc& w,
                       const double* bias, size_t bias_len, WeightStore* store, DeviceDense* dev,
                       cudaStream_t st) {
  if (w.native)
    return mount_dense_native(device, rows, cols, dt, act, w.native, w.native_len, w.scale, bias, bias_len, store,
                              dev, st);
  return mount_dense(device, rows, cols, dt, act, w.f32, w.f32_on_device, bias, bias_len, store, dev, st);
}

static WeightSrc f32_src(const float* W, bool on_device) {
  WeightSrc s;
  s.f32 = W;
  s.f32_on_device = on_device;
  return s;
}

Status swiglu_mount(int device, int in, int inter, DType dt, const float* G, const float* U, const float* D,
                    bool w_is_device, SwigluCell* c, cudaStream_t st) {
  const WeightSrc w[3] = {f32_src(G, w_is_device), f32_src(U, w_is_device), f32_src(D, w_is_device)};
  return swiglu_mount_src(device, in, inter, dt, w, c, st);
}

Status swiglu_mount_src(int device, int in, int inter, DType dt, const WeightSrc (&w)[3], SwigluCell* c,
                        cudaStream_t st) {
  if (in <= 0 || inter <= 0) return Status::Invalid("swiglu: need InputDim>0 and IntermediateDim>0");
  c->device = device;
  c->in = in;
  c->inter = inter;
  Status s = mount_dense_src(device, inter, in, dt, -1, w[0], nullptr, 0, &c->sg, &c->gate, st);
  if (!s.ok()) return Status::Err(s.code, "swiglu Gate: " + s.message);
  s = mount_dense_src(device, inter, in, dt, -1, w[1], nullptr, 0, &c->su, &c->up, st);
  if (!s.ok()) return Status::Err(s.code, "swiglu Up: " + s.message);
  s = mount_dense_src(device, in, inter, dt, -1, w[2], nullptr, 0, &c->sd, &c->down, st);
  if (!s.ok()) return Status::Err(s.code, "swiglu Down: " + s.message);
  if (c->gate.Wg && c->up.Wg && c->gate.row_stride == c->up.row_stride) {
    // Gate and Up run batched as one pair GEMM; their own GEMM mirrors are then unused
    WB_CUDA(cudaMalloc(&c->Wg_pair, gemm_mirror_bytes(dt, 2 * inter, in)));
    WB_TRY(build_gemm_pair_mirror(dt, c->gate.W, c->up.W, inter, c->gate.row_stride, in, c->Wg_pair, st));
    WB_CUDA(cudaStreamSynchronize(st));
    free_dev(c->gate.Wg);
    free_dev(c->up.Wg);
  }
  return Status::Ok();
}

// SwiGLU's own batch split: the fused Gate/Up tensor GEMV takes 1..4 rows; the Gate/Up pair GEMM
// (tcgen05) every larger batch of quantized, non-exact layers. WELVET_B200_GEMV16=1 runs 5..16
// rows as two tensor GEMVs (Gate, Up) and the reference's product instead (measured slower on
// B200: 16 rows of the 4096 / 14336 E4M3 cell take 370 us against 130 us on the pair GEMM).
// 1..4 rows on the tensor GEMV: Gate and Up as one grouped launch of two layers (x prepared
// once per layer, 4 CTAs per SM) followed by the product kernel, or, with
// WELVET_B200_SWIGLU_GEMV=dual, the fused Gate/Up form (one kernel streams both weight sets at
// 2 CTAs per SM and its epilogue writes h). Measured on the 4096 / 14336 E4M3 cell at 1 row:
// grouped 52.2 us, fused 60.3 us.
static bool swiglu_group_mode() {
  const char* e = std::getenv("WELVET_B200_SWIGLU_GEMV");
  return !(e && std::strcmp(e, "dual") == 0);
}
static bool swiglu_small_gemv(const SwigluCell* c, int bs) {
  return bs <= 4 && use_gemv_tc(c->gate, bs) && c->up.Wt;
}
static bool swiglu_group_gemv(const SwigluCell* c, int bs) {
  return swiglu_small_gemv(c, bs) && swiglu_group_mode() && use_gemv_tc(c->up, bs);
}
static bool swiglu_split_gemv(const SwigluCell* c, int bs) {
  if (std::getenv("WELVET_B200_BATCHED") != nullptr) return false;
  const char* g16 = std::getenv("WELVET_B200_GEMV16");
  if (!(g16 && g16[0] == '1')) return false;
  return bs > 4 && bs <= kGemvMaxBatch && use_gemv_tc(c->gate, bs) && use_gemv_tc(c->up, bs);
}
static bool swiglu_batched(const SwigluCell* c, int bs) {
  if (std::getenv("WELVET_B200_BATCHED") != nullptr) return use_tensor_path(c->gate, bs);
  return bs > 4 && !swiglu_split_gemv(c, bs) && !c->gate.exact && gemm_supported(c->gate.dtype);
}

Status swiglu_reserve(SwigluCell* c, int bs, cudaStream_t st) {
  if (c->bs >= bs) return Status::Ok();
  c->release_work();
  WB_CUDA(cudaSetDevice(c->device));
  const size_t xb = static_cast<size_t>(bs) * c->gate.x_stride * 4;
  const size_t hb = static_cast<size_t>(bs) * c->down.x_stride * 4;
  WB_CUDA(cudaMalloc(&c->x_pad, xb));
  WB_CUDA(cudaMemsetAsync(c->x_pad, 0, xb, st));
  WB_CUDA(cudaMalloc(&c->h_pad, hb));
  WB_CUDA(cudaMemsetAsync(c->h_pad, 0, hb, st));
  if (swiglu_split_gemv(c, bs) || swiglu_group_gemv(c, bs)) {
    WB_CUDA(cudaMalloc(&c->g_buf, static_cast<size_t>(bs) * c->inter * 4));
    WB_CUDA(cudaMalloc(&c->u_buf, static_cast<size_t>(bs) * c->inter * 4));
    WB_TRY(alloc_io(c->gate, bs, &c->io_gate, st));  // prepared-fragment scratch of each GEMV
    WB_TRY(alloc_io(c->up, bs, &c->io_up, st));
  } else if (swiglu_batched(c, bs)) {
    WB_TRY(alloc_io(c->gate, bs, &c->io_gate, st));  // error word (and the unfused path's scratch)
    if (c->Wg_pair && gemm_uses_tmem()) {
      c->pair_scratch_bytes = gemm_scratch_bytes(bs, c->in, 2 * c->inter, xsplit_policy());
      WB_CUDA(cudaMalloc(&c->pair_scratch, c->pair_scratch_bytes));
    } else {
      WB_CUDA(cudaMalloc(&c->g_buf, static_cast<size_t>(bs) * c->inter * 4));
      WB_CUDA(cudaMalloc(&c->u_buf, static_cast<size_t>(bs) * c->inter * 4));
      WB_TRY(alloc_io(c->up, bs, &c->io_up, st));
    }
  }
  c->io_down.max_tb = xsplit_policy() >= 2 ? 128 : 0;  // h: fp32 products, two x planes
  WB_TRY(alloc_io(c->down, bs, &c->io_down, st));
  c->bs = bs;
  return Status::Ok();
}

// x [bs][in] -> h [bs][inter] (= SiLU(Gate x) * (Up x), the reference's pre) -> y = Down h.
Status swiglu_forward_device(SwigluCell* c, int bs, const float* x, float* h, float* y, cudaStream_t st,
                             bool pdl, const SplitNorm* norm) {
  WB_TRY(swiglu_reserve(c, bs, st));
  const float* hsrc = nullptr;  // h as Down's input
  int64_t h_ld = 0;
  const bool group = swiglu_group_gemv(c, bs) && c->g_buf && c->io_gate.prep && c->io_up.prep;
  const bool pair = !group && !swiglu_small_gemv(c, bs) && swiglu_batched(c, bs) && c->pair_scratch;
  if (norm && norm->gamma && !pair) {
    // an RMSNorm in front, as its own kernel (the pair GEMM takes it as its prologue)
    if (!norm->pre || !norm->post) return Status::Invalid("rmsnorm: null outputs");
    WB_TRY(launch_rmsnorm(x, norm->gamma, norm->pre, norm->post, bs, c->in, norm->eps, st));
    x = norm->post;
  }
  if (group) {
    // 1..4 rows, grouped: Gate and Up in one launch of two layers, then the reference's
    // SiLU product into h
    GemvGroupLayer L[2];
    const DeviceDense* d[2] = {&c->gate, &c->up};
    float* out[2] = {c->g_buf, c->u_buf};
    DenseIO* io[2] = {&c->io_gate, &c->io_up};
    for (int i = 0; i < 2; ++i) {
      L[i].Wt = d[i]->Wt;
      L[i].x = x;
      L[i].pre = out[i];
      L[i].post = out[i];
      L[i].bias = d[i]->bias;
      L[i].bias_len = d[i]->bias_len;
      L[i].act = d[i]->act;
      L[i].scale = d[i]->scale;
      L[i].prep = io[i]->prep;
    }
    WB_TRY(launch_gemv_tc_group(c->gate.dtype, c->inter, c->in, bs, c->in, c->inter, L, 2, st, pdl, nullptr));
    float* hout = h ? h : c->h_pad;
    const int64_t ld = h ? c->inter : c->down.x_stride;
    if (ld == c->inter) {
      WB_TRY(launch_swiglu_product(c->g_buf, c->u_buf, hout, static_cast<int64_t>(bs) * c->inter, st));
    } else {
      WB_TRY(launch_swiglu_product(c->g_buf, c->u_buf, c->g_buf, static_cast<int64_t>(bs) * c->inter, st));
      WB_CUDA(cudaMemcpy2DAsync(hout, static_cast<size_t>(ld) * 4, c->g_buf, static_cast<size_t>(c->inter) * 4,
                                static_cast<size_t>(c->inter) * 4, static_cast<size_t>(bs),
                                cudaMemcpyDeviceToDevice, st));
    }
    hsrc = hout;
    h_ld = ld;
  } else if (swiglu_small_gemv(c, bs)) {
    // 1..4 rows: Gate and Up stream together through the tensor-core GEMV, whose epilogue
    // writes h directly.
    GemvTcArgs a;
    a.dtype = c->gate.dtype;
    a.Wt = c->gate.Wt;
    a.Wt2 = c->up.Wt;
    a.rows = c->inter;
    a.cols = c->in;
    a.scale = c->gate.scale;
    a.scale2 = c->up.scale;
    a.x = x;
    a.x_ld = c->in;
    a.batch = bs;
    a.pre = h ? h : c->h_pad;
    a.post = nullptr;
    a.ld_out = h ? c->inter : c->down.x_stride;
    WB_TRY(launch_gemv_tc(a, st, pdl));
    hsrc = a.pre;
    h_ld = a.ld_out;
  } else if (pair) {
    // batched: Gate and Up as one pair GEMM (2 x inter interleaved rows) whose epilogue
    // writes h = SiLU(gate)·up directly
    float* hout = h ? h : c->h_pad;
    const int64_t ld = h ? c->inter : c->down.x_stride;
    GemmArgs g;
    g.dtype = c->gate.dtype;
    g.Wg = c->Wg_pair;
    g.row_stride = c->gate.row_stride;
    g.rows = 2 * c->inter;
    g.cols = c->in;
    g.scale = c->gate.scale;
    g.scale2 = c->up.scale;
    g.x = x;
    g.x_ld = c->in;
    g.M = bs;
    g.pair = true;
    g.h = hout;
    g.ld_h = ld;
    g.xsplit = xsplit_policy();
    g.scratch = c->pair_scratch;
    g.scratch_bytes = c->pair_scratch_bytes;
    g.err = c->io_gate.err;
    if (norm) g.norm = *norm;
    WB_TRY(launch_gemm_tc(g, st));
    hsrc = hout;
    h_ld = ld;
  } else if ((swiglu_split_gemv(c, bs) || swiglu_batched(c, bs)) && c->g_buf) {
    // 5..16 rows: Gate and Up on the tensor GEMV; batched (unfused): on the tcgen05 GEMM; then
    // the reference's SiLU product.
    WB_TRY(forward_device(c->gate, bs, x, c->in, c->g_buf, c->g_buf, &c->io_gate, st, false));
    WB_TRY(forward_device(c->up, bs, x, c->in, c->u_buf, c->u_buf, &c->io_up, st, false));
    float* hout = h ? h : c->h_pad;
    const int64_t ld = h ? c->inter : c->down.x_stride;
    if (ld == c->inter) {
      WB_TRY(launch_swiglu_product(c->g_buf, c->u_buf, hout, static_cast<int64_t>(bs) * c->inter, st));
    } else {
      WB_TRY(launch_swiglu_product(c->g_buf, c->u_buf, c->g_buf, static_cast<int64_t>(bs) * c->inter, st));
      WB_CUDA(cudaMemcpy2DAsync(hout, static_cast<size_t>(ld) * 4, c->g_buf, static_cast<size_t>(c->inter) * 4,
                                static_cast<size_t>(c->inter) * 4, static_cast<size_t>(bs),
                                cudaMemcpyDeviceToDevice, st));
    }
    hsrc = hout;
    h_ld = ld;
  } else {
    // exact / Float32 layers: SIMT GEMV over x padded to the mirror's row length
    const float* xs = x;
    int64_t xst = c->in;
    if (!(c->gate.x_stride == c->in && (reinterpret_cast<uintptr_t>(x) & 15) == 0)) {
      WB_CUDA(cudaMemcpy2DAsync(c->x_pad, static_cast<size_t>(c->gate.x_stride) * 4, x,
                                static_cast<size_t>(c->in) * 4, static_cast<size_t>(c->in) * 4,
                                static_cast<size_t>(bs), cudaMemcpyDeviceToDevice, st));
      xs = c->x_pad;
      xst = c->gate.x_stride;
      pdl = false;
    }
    GemvArgs a;
    a.dtype = c->gate.dtype;
    a.W = c->gate.W;
    a.W2 = c->up.W;
    a.row_stride = c->gate.row_stride;
    a.rows = c->inter;
    a.cols = c->in;
    a.scale = c->gate.scale;
    a.scale2 = c->up.scale;
    a.x = xs;
    a.x_stride = xst;
    a.batch = bs;
    a.pre = c->h_pad;
    a.post = nullptr;
    a.ld_out = c->down.x_stride;
    a.exact = c->gate.exact && c->up.exact;
    WB_TRY(launch_gemv(a, st, pdl));
    if (h) {
      WB_CUDA(cudaMemcpy2DAsync(h, static_cast<size_t>(c->inter) * 4, c->h_pad,
                                static_cast<size_t>(c->down.x_stride) * 4, static_cast<size_t>(c->inter) * 4,
                                static_cast<size_t>(bs), cudaMemcpyDeviceToDevice, st));
    }
    hsrc = c->h_pad;
    h_ld = c->down.x_stride;
  }
  // Down: Linear, no bias, so pre == post (written by the same thread).
  return forward_device(c->down, bs, hsrc, h_ld, y, y, &c->io_down, st, true);
}

Status mha_validate(MhaConfig* cfg) {
  if (cfg->d_model <= 0 || cfg->num_heads <= 0) return Status::Invalid("mha: need DModel>0 and NumHeads>0");
  if (cfg->head_dim <= 0) {
    if (cfg->d_model % cfg->num_heads != 0) return Status::Invalid("mha: HeadDim unset and DModel%NumHeads!=0");
    cfg->head_dim = cfg->d_model / cfg->num_heads;
  }
  if (cfg->num_kv_heads <= 0) cfg->num_kv_heads = cfg->num_heads;
  if (cfg->num_heads % cfg->num_kv_heads != 0) return Status::Invalid("mha: NumHeads not divisible by NumKVHeads");
  if (cfg->max_seq_len <= 0) cfg->max_seq_len = 512;
  if (cfg->mask == 0) cfg->mask = 1;
  if (cfg->rope_theta <= 0) cfg->rope_theta = 10000;
  if (cfg->softmax != 0 && cfg->softmax != 1) return Status::Invalid("mha: unknown Softmax");
  return Status::Ok();
}

void MhaCell::release_work() {
  cudaSetDevice(device);
  free_dev(x_pad); free_dev(qb); free_dev(kb); free_dev(vb); free_dev(attn); free_dev(attn_pad);
  free_dev(Qr); free_dev(Kr); free_dev(Vd);
  io_q.release(); io_k.release(); io_v.release(); io_o.release();
  bs = 0;
}

Status mha_mount(int device, const MhaConfig& cfg_in, DType dt, const float* Q, const float* K, const float* V,
                 const float* O, bool w_is_device, MhaCell* c, cudaStream_t st) {
  const WeightSrc w[4] = {f32_src(Q, w_is_device), f32_src(K, w_is_device), f32_src(V, w_is_device),
                          f32_src(O, w_is_device)};
  return mha_mount_src(device, cfg_in, dt, w, c, st);
}

Status mha_mount_src(int device, const MhaConfig& cfg_in, DType dt, const WeightSrc (&w)[4], MhaCell* c,
                     cudaStream_t st) {
  MhaConfig cfg = cfg_in;
  WB_TRY(mha_validate(&cfg));
  c->device = device;
  c->cfg = cfg;
  const int d = cfg.d_model, qd = cfg.num_heads * cfg.head_dim, kvd = cfg.num_kv_heads * cfg.head_dim;
  Status s = mount_dense_src(device, qd, d, dt, -1, w[0], nullptr, 0, &c->sq, &c->q, st);
  if (!s.ok()) return Status::Err(s.code, "mha Q: " + s.message);
  s = mount_dense_src(device, kvd, d, dt, -1, w[1], nullptr, 0, &c->sk, &c->k, st);
  if (!s.ok()) return Status::Err(s.code, "mha K: " + s.message);
  s = mount_dense_src(device, kvd, d, dt, -1, w[2], nullptr, 0, &c->sv, &c->v, st);
  if (!s.ok()) return Status::Err(s.code, "mha V: " + s.message);
  s = mount_dense_src(device, d, qd, dt, -1, w[3], nullptr, 0, &c->so, &c->o, st);
  if (!s.ok()) return Status::Err(s.code, "mha O: " + s.message);
  return Status::Ok();
}

Status mha_reserve(MhaCell* c, int bs, cudaStream_t st) {
  if (c->bs >= bs) return Status::Ok();
  c->release_work();
  WB_CUDA(cudaSetDevice(c->device));
  const MhaConfig& g = c->cfg;
  const size_t qd = static_cast<size_t>(g.num_heads) * g.head_dim, kvd = static_cast<size_t>(g.num_kv_heads) * g.head_dim;
  const size_t n = static_cast<size_t>(bs);
  WB_CUDA(cudaMalloc(&c->x_pad, n * c->q.x_stride * 4));
  WB_CUDA(cudaMemsetAsync(c->x_pad, 0, n * c->q.x_stride * 4, st));
  WB_CUDA(cudaMalloc(&c->qb, n * qd * 4));
  WB_CUDA(cudaMalloc(&c->kb, n * kvd * 4));
  WB_CUDA(cudaMalloc(&c->vb, n * kvd * 4));
  WB_CUDA(cudaMalloc(&c->attn, n * qd * 4));
  WB_CUDA(cudaMalloc(&c->attn_pad, n * c->o.x_stride * 4));
  WB_CUDA(cudaMemsetAsync(c->attn_pad, 0, n * c->o.x_stride * 4, st));
  WB_CUDA(cudaMalloc(&c->Qr, n * qd * 8));
  WB_CUDA(cudaMalloc(&c->Kr, n * kvd * 8));
  WB_CUDA(cudaMalloc(&c->Vd, n * kvd * 8));
  WB_TRY(alloc_io(c->q, bs, &c->io_q, st));
  WB_TRY(alloc_io(c->k, bs, &c->io_k, st));
  WB_TRY(alloc_io(c->v, bs, &c->io_v, st));
  c->io_o.max_tb = xsplit_policy() >= 2 ? 128 : 0;  // attention output: fp32, two x planes
  WB_TRY(alloc_io(c->o, bs, &c->io_o, st));
  c->bs = bs;
  return Status::Ok();
}

Status mha_forward_device(MhaCell* c, int batch, int seq, const float* x, float* attn, float* y, cudaStream_t st,
                          const SplitNorm* norm) {
  const MhaConfig& g = c->cfg;
  if (batch <= 0 || seq <= 0) return Status::Invalid("mha: bad batch/seq");
  if (seq > g.max_seq_len) return Status::Invalid("mha: seq > MaxSeqLen");
  const int bs = batch * seq;
  WB_TRY(mha_reserve(c, bs, st));
  // an RMSNorm in front runs with Q's projection (its prologue on the tensor-core GEMM); K and
  // V read the norm's post
  WB_TRY(forward_device(c->q, bs, x, g.d_model, c->qb, c->qb, &c->io_q, st, false, 0, nullptr, norm));
  const float* xn = norm && norm->gamma ? norm->post : x;
  WB_TRY(forward_device(c->k, bs, xn, g.d_model, c->kb, c->kb, &c->io_k, st, false));
  WB_TRY(forward_device(c->v, bs, xn, g.d_model, c->vb, c->vb, &c->io_v, st, false));
  AttnParams p;
  p.batch = batch; p.seq = seq; p.num_heads = g.num_heads; p.num_kv = g.num_kv_heads; p.head_dim = g.head_dim;
  p.max_seq_len = g.max_seq_len; p.mask = g.mask; p.pos_kind = g.pos; p.softmax_kind = g.softmax;
  p.window = g.window; p.prefix_len = g.prefix_len; p.window_causal = g.window_causal;
  p.rope_theta = g.rope_theta; p.scale_override = g.scale_override;
  float* attn_out = attn ? attn : c->attn;
  WB_TRY(launch_mha_attention(c->qb, c->kb, c->vb, c->Qr, c->Kr, c->Vd, attn_out, p, st));
  const int qd = g.num_heads * g.head_dim;
  return forward_device(c->o, bs, attn_out, qd, y, y, &c->io_o, st, false);
}

Status rmsnorm_gamma(int device, int dim, DType dt, const float* gamma, double** gamma64_dev, cudaStream_t st) {
  return rmsnorm_gamma_src(device, dim, dt, f32_src(gamma, false), gamma64_dev, st);
}

Status rmsnorm_gamma_src(int device, int dim, DType dt, const WeightSrc& w, double** gamma64_dev, cudaStream_t st) {
  if (dim <= 0) return Status::Invalid("rmsnorm: invalid argument");
  // decode_row_f64 of the store: weight_at -> float -> double
  std::vector<double> g(static_cast<size_t>(dim));
  if (dt == DType::Float32) {
    if (!w.f32 || w.f32_on_device) return Status::Invalid("rmsnorm: float32 gamma must be host values");
    for (int i = 0; i < dim; ++i) g[static_cast<size_t>(i)] = static_cast<double>(w.f32[static_cast<size_t>(i)]);
  } else {
    // the store's native bytes: given, or the reference codec applied to the float values
    WeightStore s;
    DeviceDense d;
    const uint8_t* native = w.native;
    size_t native_len = w.native_len;
    float scale = w.scale;
    if (!native) {
      WB_TRY(mount_dense(device, 1, dim, dt, -1, w.f32, w.f32_on_device, nullptr, 0, &s, &d, st));
      native = s.native.data();
      native_len = s.native.size();
      scale = s.scale;
    }
    float* dec = nullptr;
    uint8_t* nat = nullptr;
    WB_CUDA(cudaMalloc(&dec, static_cast<size_t>(dim) * 4));
    WB_CUDA(cudaMalloc(&nat, native_len));
    Status stt = cuda_status(cudaMemcpyAsync(nat, native, native_len, cudaMemcpyHostToDevice, st), "gamma h2d");
    if (stt.ok()) stt = decode_ref(dt, nat, dim, scale, dec, st);
    std::vector<float> f(static_cast<size_t>(dim));
    if (stt.ok()) stt = cuda_status(cudaMemcpyAsync(f.data(), dec, static_cast<size_t>(dim) * 4, cudaMemcpyDeviceToHost, st), "gamma d2h");
    if (stt.ok()) stt = cuda_status(cudaStreamSynchronize(st), "gamma sync");
    cudaFree(dec);
    cudaFree(nat);
    WB_TRY(stt);
    for (int i = 0; i < dim; ++i) g[static_cast<size_t>(i)] = static_cast<double>(f[static_cast<size_t>(i)]);
  }
  WB_CUDA(cudaMalloc(gamma64_dev, static_cast<size_t>(dim) * 8));
  WB_CUDA(cudaMemcpyAsync(*gamma64_dev, g.data(), static_cast<size_t>(dim) * 8, cudaMemcpyHostToDevice, st));
  return cuda_status(cudaStreamSynchronize(st), "gamma sync");
}

} // namespace wb
