// cell_kernels.cu -- the non-projection kernels of the RMSNorm / MHA cells (sm_100a), in
// float64 like the reference, but parallel instead of one thread per token / one thread
// for the whole attention.
//
//   rmsnorm_forward   src/cuda/kernels.cu:172-204 (norm_forward_f64 with center = 0)
//   mha rope prep     src/cuda/kernels.cu:487-505 (mha_apply_rope at the global position)
//   mha attention     src/cuda/kernels.cu:536-632 (mha_attention_forward_f64, ModeSelf)
//
// Attention semantics kept from the reference: batches run in order against one KV ring of
// max_seq_len slots; token (b, s) has global position p = b*seq + s and is written to slot
// p % msl before batch b's queries run; a query of batch b scans k_pos in [0, (b+1)*seq)
// and, for an allowed k_pos, reads slot k_pos % msl -- which then holds the latest position
// p' <= (b+1)*seq-1 with p' == k_pos (mod msl). Masks and ALiBi use k_pos; RoPE of the key
// was applied at p'. The running max starts at -1e9 as in the reference.
#include "cell_kernels.hpp"
#include "rmsnorm.cuh"

#include <cstdlib>
#include <cstring>
#include <type_traits>

namespace wb {
namespace {

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_max_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One block of kNormThreads per token, its sum of squares in rms_block_ss's order (the
// projection GEMM's prologue gives the same bits). x, pre and post are [n_tok][dim].
__global__ void __launch_bounds__(kNormThreads)
    k_rmsnorm(const float* __restrict__ x, const double* __restrict__ gamma, float* __restrict__ pre,
              float* __restrict__ post, int n_tok, int dim, double eps) {
  __shared__ double s_part[kNormThreads / 32];
  const int t = blockIdx.x;
  if (t >= n_tok) return;
  const float* xt = x + static_cast<int64_t>(t) * dim;
  float* pt = pre + static_cast<int64_t>(t) * dim;
  float* qt = post + static_cast<int64_t>(t) * dim;
  const bool vec = (reinterpret_cast<uintptr_t>(xt) & 15) == 0;
  const bool vec_out = ((reinterpret_cast<uintptr_t>(pt) | reinterpret_cast<uintptr_t>(qt)) & 15) == 0;
  auto load4 = [&](int k) -> float4 {
    if (vec && k + 3 < dim) return *reinterpret_cast<const float4*>(xt + k);
    float4 v;
    v.x = xt[k];
    v.y = k + 1 < dim ? xt[k + 1] : 0.0f;
    v.z = k + 2 < dim ? xt[k + 2] : 0.0f;
    v.w = k + 3 < dim ? xt[k + 3] : 0.0f;
    return v;
  };
  const double inv = rms_inv(rms_block_ss(load4, dim, s_part), dim, eps);
  for (int k = 4 * threadIdx.x; k < dim; k += 4 * kNormThreads)
    rms_apply4(load4(k), k, dim, inv, gamma, pt, qt, true, vec_out);
}

// Widen projections to f64 and rotate Q and K at each token's global position.
// One thread per (token, head, d < half) pair, plus plain copies for V / unrotated tails.
__global__ void k_rope_prep(const float* __restrict__ q, const float* __restrict__ k,
                            const float* __restrict__ v, double* __restrict__ Qr,
                            double* __restrict__ Kr, double* __restrict__ Vd, int bs, int num_heads,
                            int num_kv, int head_dim, int use_rope, double theta) {
  const int q_dim = num_heads * head_dim;
  const int kv_dim = num_kv * head_dim;
  const int64_t total = static_cast<int64_t>(bs) * (q_dim + 2 * kv_dim);
  const int half = head_dim / 2;
  const bool rot = use_rope && half > 0 && theta > 0.0;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int tok = static_cast<int>(t / (q_dim + 2 * kv_dim));
    int c = static_cast<int>(t - static_cast<int64_t>(tok) * (q_dim + 2 * kv_dim));
    const float* src;
    double* dst;
    bool rotate = rot;
    if (c < q_dim) {
      src = q + static_cast<int64_t>(tok) * q_dim; dst = Qr + static_cast<int64_t>(tok) * q_dim;
    } else if (c < q_dim + kv_dim) {
      c -= q_dim;
      src = k + static_cast<int64_t>(tok) * kv_dim; dst = Kr + static_cast<int64_t>(tok) * kv_dim;
    } else {
      c -= q_dim + kv_dim;
      src = v + static_cast<int64_t>(tok) * kv_dim; dst = Vd + static_cast<int64_t>(tok) * kv_dim;
      rotate = false;
    }
    const int d = c % head_dim;
    const int base = c - d;
    if (!rotate || d >= 2 * half) {
      dst[c] = static_cast<double>(src[c]);
      continue;
    }
    const int dd = d < half ? d : d - half;
    const double angle = static_cast<double>(tok) /
                         pow(theta, static_cast<double>(2 * dd) / static_cast<double>(head_dim));
    const double cs = cos(angle);
    const double sn = sin(angle);
    const double v0 = static_cast<double>(src[base + dd]);
    const double v1 = static_cast<double>(src[base + dd + half]);
    dst[c] = d < half ? v0 * cs - v1 * sn : v0 * sn + v1 * cs;
  }
}

__device__ __forceinline__ bool attn_allow(int q_pos, int k_pos, int mask, int window, int msl,
                                           int prefix_len, int window_causal) {
  if (mask == 2) return true;
  if (mask == 3) {
    const int w = window > 0 ? window : msl;
    if (window_causal) return k_pos <= q_pos && k_pos >= q_pos - w + 1;
    int d = q_pos - k_pos;
    if (d < 0) d = -d;
    return d < w;
  }
  if (mask == 4) {
    if (q_pos < prefix_len && k_pos < prefix_len) return true;
    return k_pos <= q_pos;
  }
  return k_pos <= q_pos;
}

__device__ __forceinline__ double alibi(int head, int num_heads, int q_pos, int k_pos) {
  const int n = num_heads <= 0 ? 1 : num_heads;
  const double slope = pow(2.0, -static_cast<double>(head + 1) * 8.0 / static_cast<double>(n));
  const int diff = q_pos - k_pos;
  return -slope * static_cast<double>(diff < 0 ? -diff : diff);
}

constexpr int kMaxHeadDim = 256;

// One warp per (token, head). Lanes score 32 keys at a time (one each), then the warp
// folds them into an online softmax with lanes owning head_dim/32 output dimensions.
__global__ void k_attention(const double* __restrict__ Qr, const double* __restrict__ Kr,
                            const double* __restrict__ Vd, float* __restrict__ out, int batch,
                            int seq, int num_heads, int num_kv, int head_dim, int msl, int mask,
                            int use_alibi, int use_sigmoid, int window, int prefix_len,
                            int window_causal, double scale) {
  __shared__ double qs[4][kMaxHeadDim];
  const int wib = threadIdx.x >> 5;
  const int warp = blockIdx.x * 4 + wib;
  const int lane = threadIdx.x & 31;
  const int bs = batch * seq;
  if (warp >= bs * num_heads) return;
  const int tok = warp / num_heads;
  const int h = warp - tok * num_heads;
  const int b = tok / seq;
  const int q_pos = tok;  // b*seq + s
  const int kv_len = (b + 1) * seq;
  const int q_dim = num_heads * head_dim;
  const int kv_dim = num_kv * head_dim;
  const int kvh = h / (num_heads / num_kv);
  for (int d = lane; d < head_dim; d += 32) qs[wib][d] = Qr[static_cast<int64_t>(tok) * q_dim + h * head_dim + d];
  __syncwarp();

  constexpr int kPer = kMaxHeadDim / 32;
  double acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) acc[i] = 0.0;
  double m = -1e9;  // running max (reference initial value)
  double l = 0.0;   // running sum of exp(score - m)
  int n = 0;

  for (int k0 = 0; k0 < kv_len; k0 += 32) {
    const int k_pos = k0 + lane;
    bool ok = k_pos < kv_len && attn_allow(q_pos, k_pos, mask, window, msl, prefix_len, window_causal);
    double score = 0.0;
    int p = 0;
    if (ok) {
      const int slot = k_pos % msl;
      p = slot + msl * ((kv_len - 1 - slot) / msl);  // latest position written to this slot
      const double* kr = Kr + static_cast<int64_t>(p) * kv_dim + kvh * head_dim;
      double dot = 0.0;
      for (int d = 0; d < head_dim; ++d) dot += qs[wib][d] * kr[d];
      score = dot * scale + (use_alibi ? alibi(h, num_heads, q_pos, k_pos) : 0.0);
    }
    const unsigned okmask = __ballot_sync(0xffffffffu, ok);
    if (okmask == 0) continue;
    n += __popc(okmask);
    double w;
    if (use_sigmoid) {
      w = ok ? 1.0 / (1.0 + exp(-score)) : 0.0;
    } else {
      const double cm = warp_max_d(ok ? score : -INFINITY);
      const double m_new = fmax(m, cm);
      const double corr = exp(m - m_new);
      w = ok ? exp(score - m_new) : 0.0;
      l = l * corr + warp_sum_d(w);
#pragma unroll
      for (int i = 0; i < kPer; ++i) acc[i] *= corr;
      m = m_new;
    }
    // Fold the chunk's weighted V rows: lanes own dims lane, lane+32, ...
    unsigned rem = okmask;
    while (rem) {
      const int j = __ffs(rem) - 1;
      rem &= rem - 1;
      const double wj = __shfl_sync(0xffffffffu, w, j);
      const int pj = __shfl_sync(0xffffffffu, p, j);
      const double* vr = Vd + static_cast<int64_t>(pj) * kv_dim + kvh * head_dim;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int d = lane + 32 * i;
        if (d < head_dim) acc[i] += wj * vr[d];
      }
    }
  }
  float* o = out + static_cast<int64_t>(tok) * q_dim + h * head_dim;
  const double inv = (n == 0 || use_sigmoid) ? 1.0 : 1.0 / l;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int d = lane + 32 * i;
    if (d < head_dim) o[d] = n == 0 ? 0.0f : static_cast<float>(acc[i] * inv);
  }
}

// The same attention, tiled: one CTA per (8 x QW consecutive queries of one batch, head).
// Each tile of 64 key positions k_pos has its ring rows (the latest position written to slot
// k_pos % msl, as above) gathered once into shared memory -- K transposed, V row-major -- and
// serves all the CTA's queries, instead of every (query, head) warp re-reading K and V from
// L2. Scores, online softmax (running max from -1e9, as the reference) and the weighted V sum
// stay in fp64. Warp w owns queries QW w .. QW w + QW - 1; for the scores lane l takes key
// positions l and l + 32 of the tile, for the output the head dimensions l, l + 32, l + 64,
// l + 96. QW = 8 (64 queries per CTA) makes twice the FMAs per shared-memory load of QW = 4.
constexpr int kAK = 64, kAHd = 128;
// K is stored transposed with rows of kAK + 1 doubles: the gather writes consecutive head
// dimensions of one key, which a row of exactly kAK doubles would put in one bank
constexpr int kAKs = kAK + 1;

// NW warps per CTA, QW queries per warp: 16 x 4 by default (64 queries; the FP64 pipe needs
// the warps to hide its latency), 8 x 8, 32 x 2 or 8 x 4 (32 queries) on request.
template <int QW, int NW = 8>
__host__ __device__ constexpr int attn_queries() { return NW * QW; }

template <int QW, int NW = 8>
size_t attention_tiled_smem() {
  constexpr int kAQ = attn_queries<QW, NW>();
  return sizeof(double) * (kAHd * kAQ + kAHd * kAKs + kAK * kAHd + kAK * kAQ) + sizeof(int) * kAK;
}

template <int QW, int NW = 8>
__global__ void __launch_bounds__(32 * NW, 1)
    k_attention_tiled(const double* __restrict__ Qr, const double* __restrict__ Kr, const double* __restrict__ Vd,
                      float* __restrict__ out, int batch, int seq, int num_heads, int num_kv, int head_dim, int msl,
                      int mask, int use_alibi, int use_sigmoid, int window, int prefix_len, int window_causal,
                      double scale) {
  constexpr int kAQ = attn_queries<QW, NW>();
  constexpr int kAThreads = 32 * NW;
  extern __shared__ double sm[];
  double* Qs = sm;                  // [kAHd][kAQ]: queries' rotated Q, d-major
  double* Kt = Qs + kAHd * kAQ;     // [kAHd][kAKs]: the tile's keys, d-major
  double* Vs = Kt + kAHd * kAKs;    // [kAK][kAHd]
  double* Ps = Vs + kAK * kAHd;     // [kAK][kAQ]: the tile's weights, key-major
  int* prow = reinterpret_cast<int*>(Ps + kAK * kAQ);  // [kAK] ring row of each key position (-1: none)
  const int qtiles = (seq + kAQ - 1) / kAQ;
  // blocks run longest first: later batches and later queries see more key positions, and
  // the scheduler starts blocks roughly in index order
  const int bx = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);
  const int b = bx / qtiles, s0 = (bx - b * qtiles) * kAQ;
  const int h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int nq = seq - s0 < kAQ ? seq - s0 : kAQ;
  const int tok0 = b * seq + s0;  // global position of the tile's first query
  const int kv_len = (b + 1) * seq;
  const int q_dim = num_heads * head_dim, kv_dim = num_kv * head_dim;
  const int kvh = h / (num_heads / num_kv);
  // kAQ * kAHd / kAThreads loads per thread, all in flight (the loop is unrolled)
#pragma unroll 8
  for (int i = tid; i < kAQ * kAHd; i += kAThreads) {
    const int q = i / kAHd, d = i - q * kAHd;
    Qs[d * kAQ + q] = q < nq && d < head_dim ? Qr[static_cast<int64_t>(tok0 + q) * q_dim + h * head_dim + d] : 0.0;
  }
  const int qb = QW * w;
  double m[QW], l[QW], acc[QW][4];
  int n[QW];
#pragma unroll
  for (int i = 0; i < QW; ++i) {
    m[i] = -1e9;  // the reference's initial running max
    l[i] = 0.0;
    n[i] = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
  }
  // causal: no key beyond the tile's last query position is allowed
  const int k_end = mask == 1 ? (tok0 + nq < kv_len ? tok0 + nq : kv_len) : kv_len;
  for (int k0 = 0; k0 < k_end; k0 += kAK) {
    __syncthreads();  // the previous tile's K / V / P are consumed (and Qs written, first time)
    if (tid < kAK) {
      const int kp = k0 + tid;
      const int slot = kp % msl;
      prow[tid] = kp < k_end ? slot + msl * ((kv_len - 1 - slot) / msl) : -1;
    }
    __syncthreads();
    // the tile's K and V rows: 32 loads of each per thread, 8 iterations' worth in flight
#pragma unroll 8
    for (int i = tid; i < kAK * kAHd; i += kAThreads) {
      const int j = i / kAHd, d = i - j * kAHd;
      const int p = prow[j];
      const bool ok = p >= 0 && d < head_dim;
      const int64_t off = static_cast<int64_t>(p) * kv_dim + kvh * head_dim + d;
      Kt[d * kAKs + j] = ok ? Kr[off] : 0.0;
      Vs[j * kAHd + d] = ok ? Vd[off] : 0.0;
    }
    __syncthreads();
    // scores of queries qb..qb+QW-1 against key positions k0 + lane, k0 + lane + 32
    double sc[QW][2];
#pragma unroll
    for (int i = 0; i < QW; ++i) sc[i][0] = sc[i][1] = 0.0;
    for (int d = 0; d < head_dim; ++d) {
      const double k0v = Kt[d * kAKs + lane], k1v = Kt[d * kAKs + lane + 32];
#pragma unroll
      for (int i2 = 0; i2 < QW; i2 += 2) {
        const double2 qa = *reinterpret_cast<const double2*>(Qs + d * kAQ + qb + i2);
        sc[i2][0] += qa.x * k0v; sc[i2][1] += qa.x * k1v;
        sc[i2 + 1][0] += qa.y * k0v; sc[i2 + 1][1] += qa.y * k1v;
      }
    }
#pragma unroll
    for (int i = 0; i < QW; ++i) {
      const int q_pos = tok0 + qb + i;
      const bool qv = qb + i < nq;
      bool ok[2];
      double s[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int kp = k0 + lane + 32 * j;
        ok[j] = qv && kp < k_end && attn_allow(q_pos, kp, mask, window, msl, prefix_len, window_causal);
        s[j] = ok[j] ? sc[i][j] * scale + (use_alibi ? alibi(h, num_heads, q_pos, kp) : 0.0) : 0.0;
      }
      n[i] += __popc(__ballot_sync(0xffffffffu, ok[0])) + __popc(__ballot_sync(0xffffffffu, ok[1]));
      double pw[2];
      if (use_sigmoid) {
#pragma unroll
        for (int j = 0; j < 2; ++j) pw[j] = ok[j] ? 1.0 / (1.0 + exp(-s[j])) : 0.0;
      } else {
        const double cm = warp_max_d(fmax(ok[0] ? s[0] : -INFINITY, ok[1] ? s[1] : -INFINITY));
        const double m_new = fmax(m[i], cm);
        const double corr = exp(m[i] - m_new);
#pragma unroll
        for (int j = 0; j < 2; ++j) pw[j] = ok[j] ? exp(s[j] - m_new) : 0.0;
        l[i] = l[i] * corr + warp_sum_d(pw[0] + pw[1]);
#pragma unroll
        for (int dd = 0; dd < 4; ++dd) acc[i][dd] *= corr;
        m[i] = m_new;
      }
      Ps[lane * kAQ + qb + i] = pw[0];
      Ps[(lane + 32) * kAQ + qb + i] = pw[1];
    }
    __syncwarp();  // the warp's own rows of Ps
    const int kn = k_end - k0 < kAK ? k_end - k0 : kAK;
    for (int j = 0; j < kn; ++j) {
      double v[4];
#pragma unroll
      for (int dd = 0; dd < 4; ++dd) v[dd] = Vs[j * kAHd + lane + 32 * dd];
#pragma unroll
      for (int i2 = 0; i2 < QW; i2 += 2) {
        const double2 pa = *reinterpret_cast<const double2*>(Ps + j * kAQ + qb + i2);
#pragma unroll
        for (int dd = 0; dd < 4; ++dd) {
          acc[i2][dd] += pa.x * v[dd];
          acc[i2 + 1][dd] += pa.y * v[dd];
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < QW; ++i) {
    if (qb + i >= nq) continue;
    const double inv = (n[i] == 0 || use_sigmoid) ? 1.0 : 1.0 / l[i];
    float* o = out + static_cast<int64_t>(tok0 + qb + i) * q_dim + h * head_dim;
#pragma unroll
    for (int dd = 0; dd < 4; ++dd) {
      const int d = lane + 32 * dd;
      if (d < head_dim) o[d] = n[i] == 0 ? 0.0f : static_cast<float>(acc[i][dd] * inv);
    }
  }
}

// h = float(double(float(SiLU(double(g)))) * double(up)) -- src/cuda/kernels.cu:296-305.
__global__ void k_swiglu_product(const float* __restrict__ g, const float* __restrict__ u,
                                 float* __restrict__ h, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const double x = static_cast<double>(g[i]);
    const float gf = static_cast<float>(x / (1.0 + exp(-x)));
    h[i] = static_cast<float>(static_cast<double>(gf) * static_cast<double>(u[i]));
  }
}

} // namespace

Status launch_rmsnorm(const float* x, const double* gamma, float* pre, float* post, int n_tok, int dim,
                      double eps, cudaStream_t st) {
  if (n_tok <= 0 || dim <= 0) return Status::Ok();
  if ((reinterpret_cast<uintptr_t>(gamma) & 15) != 0) return Status::Invalid("rmsnorm: gamma not 16-byte aligned");
  k_rmsnorm<<<n_tok, kNormThreads, 0, st>>>(x, gamma, pre, post, n_tok, dim, eps);
  return cuda_status(cudaGetLastError(), "rmsnorm launch");
}

Status launch_mha_attention(const float* q, const float* k, const float* v, double* Qr, double* Kr,
                            double* Vd, float* out, const AttnParams& p, cudaStream_t st) {
  if (p.head_dim > kMaxHeadDim) return Status::Unsupported("mha: head_dim > 256");
  const int bs = p.batch * p.seq;
  const int64_t total = static_cast<int64_t>(bs) * (p.num_heads + 2 * p.num_kv) * p.head_dim;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  const bool use_rope = p.pos_kind == 0 || p.pos_kind == 3;
  k_rope_prep<<<blocks, 256, 0, st>>>(q, k, v, Qr, Kr, Vd, bs, p.num_heads, p.num_kv, p.head_dim,
                                      use_rope ? 1 : 0, p.rope_theta);
  WB_CUDA(cudaGetLastError());
  double scale = p.scale_override;
  if (scale <= 0.0) scale = 1.0 / sqrt(static_cast<double>(p.head_dim));
  const bool use_alibi = p.pos_kind == 2 || p.pos_kind == 3;
  const char* env = std::getenv("WELVET_B200_ATTN");
  if (p.head_dim <= kAHd && !(env && std::strcmp(env, "warp") == 0)) {
    // 64 queries on 16 warps per CTA (4 per warp) unless WELVET_B200_ATTN=tiled8w (64 on 8
    // warps), =tiled32w (64 on 32 warps) or =tiled32 (32 queries on 8 warps). Measured on C4's
    // MHA cell: 8 warps x 4 queries 3.25 ms, 8 x 8 2.84 ms, 16 x 4 2.39 ms.
    const bool q32 = env && std::strcmp(env, "tiled32") == 0;
    const bool w8 = env && std::strcmp(env, "tiled8w") == 0;
    const bool w32 = env && std::strcmp(env, "tiled32w") == 0;
    auto launch = [&](auto qw_c, auto nw_c) -> Status {
      constexpr int QW = decltype(qw_c)::value;
      constexpr int NW = decltype(nw_c)::value;
      constexpr int kAQ = attn_queries<QW, NW>();
      const size_t smem = attention_tiled_smem<QW, NW>();
      // per device (the attribute belongs to the current device's context); a cheap host call
      WB_CUDA(cudaFuncSetAttribute(k_attention_tiled<QW, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(smem)));
      const dim3 grid(static_cast<unsigned>(p.batch * ((p.seq + kAQ - 1) / kAQ)), static_cast<unsigned>(p.num_heads));
      k_attention_tiled<QW, NW><<<grid, 32 * NW, smem, st>>>(Qr, Kr, Vd, out, p.batch, p.seq, p.num_heads, p.num_kv,
                                                             p.head_dim, p.max_seq_len, p.mask, use_alibi ? 1 : 0,
                                                             p.softmax_kind == 1 ? 1 : 0, p.window, p.prefix_len,
                                                             p.window_causal, scale);
      return cuda_status(cudaGetLastError(), "attention launch");
    };
    if (q32) return launch(std::integral_constant<int, 4>{}, std::integral_constant<int, 8>{});
    if (w8) return launch(std::integral_constant<int, 8>{}, std::integral_constant<int, 8>{});
    if (w32) return launch(std::integral_constant<int, 2>{}, std::integral_constant<int, 32>{});
    return launch(std::integral_constant<int, 4>{}, std::integral_constant<int, 16>{});
  }
  const int warps = bs * p.num_heads;
  k_attention<<<(warps + 3) / 4, 128, 0, st>>>(Qr, Kr, Vd, out, p.batch, p.seq, p.num_heads, p.num_kv,
                                              p.head_dim, p.max_seq_len, p.mask, use_alibi ? 1 : 0,
                                              p.softmax_kind == 1 ? 1 : 0, p.window, p.prefix_len,
                                              p.window_causal, scale);
  return cuda_status(cudaGetLastError(), "attention launch");
}

Status launch_swiglu_product(const float* g, const float* u, float* h, int64_t n, cudaStream_t st) {
  int blocks = static_cast<int>((n + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  k_swiglu_product<<<blocks, 256, 0, st>>>(g, u, h, n);
  return cuda_status(cudaGetLastError(), "swiglu product launch");
}

} // namespace wb
