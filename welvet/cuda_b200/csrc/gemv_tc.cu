// gemv_tc.cu -- small-batch dequant GEMV on the tensor cores' register path (sm_100a).
//
// Replaces, for 1..8 tokens, the reference's dense_matvec_f64_batch + dense_bias_act
// (src/cuda/kernels.cu:130-161) over a host-decoded fp64 W. It streams the packed codes once:
//
//  * Weights come from a fragment-tiled mirror: one 16-byte load per lane and row group
//    holds that lane's mma.m16n8k16 A fragments for 4 (FP4) or 2 (FP8/Int8) K blocks; each
//    code byte becomes one f16x2 A register through cvt.rn.f16x2.{e2m1x2,e4m3x2,e5m2x2} (Int8
//    through an exact f16 bias trick). FP8/FP4/Int8 values are exact in f16.
//  * x is split per token into two f16 planes after scaling by a power of two chosen from
//    the CTA's own K range (x * 2^e = h0 + h1, 22 significant bits); the planes sit in the
//    MMA's N columns (n = 2 * token + plane), so each thread's D fragment holds both planes of
//    one token. Up to 4 tokens fill one n8 tile; 5..8 tokens use two, and each converted A
//    fragment then feeds two MMAs. The CTA's 128 threads build these B fragments once into shared memory.
//    Products are exact, accumulation is fp32 within a chunk and fp64 across chunks, warps
//    and CTAs: |y - y_fp64| <= ~2^-22 * sum_k |W x| before the final rounding.
//  * A CTA owns 64 rows x a K range, its 4 warps a quarter each. All of a warp's weight
//    loads for its first chunk are issued before griddepcontrol.wait (programmatic dependent
//    launch: the weights do not depend on the previous kernel), so a chained layer streams
//    its weights while the previous one finishes.
//  * The K ranges of one 64-row set are the CTAs of one thread-block cluster (up to 8); their
//    fp64 partials are summed in rank order by rank 0 through distributed shared memory,
//    which then runs the epilogue (bias / activation, or the SwiGLU product, as in
//    src/cuda/kernels.cu:147-161 and :296-305). No global scratch and no atomics: the result
//    is deterministic.
#include "gemv_tc.hpp"
#include "codec.cuh"

#include <cooperative_groups.h>

#include <cstdlib>
#include <mutex>
#include <tuple>
#include <vector>

namespace wb {
namespace {

constexpr int kWarps = 4;   // warps per CTA (K slices of the CTA's K range)
constexpr int kRG = TiledGeom::kSetGroups;  // row groups of 16 rows per warp -> 64-row sets
constexpr int kRowsPerSet = kRG * 16;
constexpr int kMaxCluster = 8;

struct Plan {
  TiledGeom g;
  int64_t row_sets = 0;
  int64_t chunks = 0;       // chunks of 2 units along K
  int cpw = 1;              // chunks per warp
  int csize = 1;            // CTAs per cluster (split of K)
  int nkb_cta = 0;          // K blocks of 16 per CTA
  int64_t grid_y = 0;       // CTAs along the row sets (a CTA loops over row sets grid_y apart)
};

// grouped = false: one layer per launch, latency first -- the K range is split over up to 8
// CTAs of a cluster so that a single small layer spreads over many SMs.
// grouped = true: many layers per launch fill the GPU by themselves, so each CTA streams a
// longer K range (up to 8 chunks per warp, double-buffered) and the fixed cost of a CTA (x
// staging, fragment build, reduction, epilogue) is paid over more bytes.
// batch > 8 (one layer per launch, prepared fragments of 12 or 16 tokens): the shortest K
// range per CTA the cluster limit allows, so that the fragments fit in shared memory.
Plan make_plan(DType dt, int rows, int cols, bool grouped = false, int batch = 1, bool dual = false) {
  Plan p;
  p.g = tiled_geom(dt, rows, cols);
  p.row_sets = (p.g.row_groups + kRG - 1) / kRG;
  p.chunks = (p.g.units_k + 1) / 2;
  // At least two chunks per warp: both are loaded before griddepcontrol.wait, and a launch
  // then takes about half of the GPU's CTA slots, so the next launch can co-reside and
  // prefetch its weights.
  p.cpw = static_cast<int>((p.chunks + kWarps * kMaxCluster - 1) / (kWarps * kMaxCluster));
  if (!grouped && batch <= 8) {
    // A layer with many row sets fills the GPU by itself: give each CTA a longer K range
    // (fewer CTAs, each paying its fixed x-staging / reduction cost over more bytes) while
    // keeping at least two waves of CTAs for balance (4 CTAs per SM). The fused Gate/Up form
    // runs 2 CTAs per SM and is best at about one and a half waves (14336 x 4096 E4M3 pair,
    // 1 token: 3 waves of 4 chunks per warp 56.4 us for the SwiGLU cell, 1.5 waves of 8 chunks
    // 52.3 us, 6 waves of 2 chunks 64.6 us).
    const int64_t kMinCtas = dual ? 148 * 2 : 2 * 148 * 4;
    for (int c = 16; c > p.cpw; c >>= 1) {
      const int64_t cs = (p.chunks + kWarps * c - 1) / (kWarps * c);
      if (p.row_sets * cs >= kMinCtas) {
        p.cpw = c;
        break;
      }
    }
  }
  // Tuning override, read once per process: the prepared-fragment scratch a session
  // allocates is sized from this plan, so the plan must not change under it.
  static const int cpw_env = [] {
    const char* e = std::getenv("WELVET_B200_GEMV_CPW");
    return e ? std::atoi(e) : 0;
  }();
  if (batch <= 8 && cpw_env >= 1 && cpw_env <= 64 &&
      (p.chunks + kWarps * cpw_env - 1) / (kWarps * cpw_env) <= kMaxCluster)
    p.cpw = cpw_env;
  if (grouped) {
    // Up to 8 chunks per warp; 16 for layers of 256 row sets or more, which fill the GPU
    // with half as many CTAs of twice the K range (measured, 16384-column FP4 at 1 token:
    // 65536 rows 102.7 -> 96.1 us, 32768 rows 56.5 -> 54.2, 16384 rows 31.2 -> 30.0; at 8192
    // rows 16 was slower, 17.5 -> 27.7).
    const int64_t per_warp = (p.chunks + kWarps - 1) / kWarps;
    const int cap = p.row_sets >= 256 ? 16 : 8;
    const int longer = static_cast<int>(per_warp < cap ? per_warp : cap);
    if (longer > p.cpw) p.cpw = longer;  // never fewer chunks than the cluster limit needs
  }
  if (p.cpw < 2) p.cpw = 2;
  p.csize = static_cast<int>((p.chunks + kWarps * p.cpw - 1) / (kWarps * p.cpw));
  const int kbpu = dt == DType::FP4 ? 4 : 2;
  p.nkb_cta = kWarps * p.cpw * 2 * kbpu;
  p.grid_y = p.row_sets;
  return p;
}

struct KArgs {
  const uint8_t* Wt;
  const uint8_t* Wt2;
  int rows, cols;
  int64_t units_k;
  int64_t row_groups;
  int64_t chunks;
  int cpw, csize, nkb_cta;
  float scale, scale2;
  const float* x;
  int64_t x_ld;
  float* pre;
  float* post;
  int64_t ld_out;
  const double* bias;
  int bias_len;
  int act;
  const uint2* frags;   // prepared B fragments [csize * nkb_cta][2 kB][4] (nullptr: built per CTA)
  const float* fscale;  // prepared 2^-e per K segment and token [csize][kB]
  PeerOut peers;        // further destinations of post (column-sharded layers)
  int nb;               // tokens present (<= kB; kB rounds a batch of 9..16 up to 12 or 16)
};

__device__ __forceinline__ uint4 ld_stream(const uint8_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment of K block j (within a unit) from the lane's 16-byte share of the unit.
template <int kDt>
__device__ __forceinline__ void a_frag(const uint4& u, int j, uint32_t (&a)[4]) {
  if constexpr (kDt == 16) {
    const uint32_t w = j == 0 ? u.x : (j == 1 ? u.y : (j == 2 ? u.z : u.w));
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
        : "r"(w));
  } else {
    const uint32_t w0 = j == 0 ? u.x : u.z;
    const uint32_t w1 = j == 0 ? u.y : u.w;
    if constexpr (kDt == 4) {
      asm("{\n\t.reg .b16 l0, h0, l1, h1;\n\t"
          "mov.b32 {l0, h0}, %4;\n\t"
          "mov.b32 {l1, h1}, %5;\n\t"
          "cvt.rn.f16x2.e4m3x2 %0, l0;\n\t"
          "cvt.rn.f16x2.e4m3x2 %1, h0;\n\t"
          "cvt.rn.f16x2.e4m3x2 %2, l1;\n\t"
          "cvt.rn.f16x2.e4m3x2 %3, h1;\n\t}"
          : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
          : "r"(w0), "r"(w1));
    } else if constexpr (kDt == 5) {
      asm("{\n\t.reg .b16 l0, h0, l1, h1;\n\t"
          "mov.b32 {l0, h0}, %4;\n\t"
          "mov.b32 {l1, h1}, %5;\n\t"
          "cvt.rn.f16x2.e5m2x2 %0, l0;\n\t"
          "cvt.rn.f16x2.e5m2x2 %1, h0;\n\t"
          "cvt.rn.f16x2.e5m2x2 %2, l1;\n\t"
          "cvt.rn.f16x2.e5m2x2 %3, h1;\n\t}"
          : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
          : "r"(w0), "r"(w1));
    } else {  // Int8: f16 bits 0x6400 | (q ^ 0x80) = 1152 + q, minus 1152
      const uint32_t u0 = w0 ^ 0x80808080u, u1 = w1 ^ 0x80808080u;
      const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
      uint32_t p[4] = {__byte_perm(u0, 0x64646464u, 0x4140), __byte_perm(u0, 0x64646464u, 0x4342),
                       __byte_perm(u1, 0x64646464u, 0x4140), __byte_perm(u1, 0x64646464u, 0x4342)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __half2 h = __hsub2(*reinterpret_cast<__half2*>(&p[i]), bias);
        a[i] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
  }
}

// Two x values scaled by s, split into plane 0 (their f16 rounding) and plane 1 (the f16
// rounding of the residual).
__device__ __forceinline__ void x_planes(float v0, float v1, float s, uint32_t& p0, uint32_t& p1) {
  float a = v0 * s, b = v1 * s;
  const bool fa = isfinite(a), fb = isfinite(b);
  if (!fa) a = v0;  // Inf / NaN pass through plane 0 (w * Inf as in fp64)
  if (!fb) b = v1;
  __half2 h0 = __floats2half2_rn(a, b);
  const float2 f0 = __half22float2(h0);
  const float ra = fa ? a - f0.x : 0.0f, rb = fb ? b - f0.y : 0.0f;
  __half2 h1 = __floats2half2_rn(ra, rb);
  p0 = *reinterpret_cast<uint32_t*>(&h0);
  p1 = *reinterpret_cast<uint32_t*>(&h1);
}

// Exponent e of the per-token power-of-two scale of a K range whose largest finite |x| is m:
// m * 2^e lies in [2^14, 2^15), below the f16 maximum 65504.
__device__ __forceinline__ int x_scale_exp(float m) {
  int e = 0;
  if (m > 0.0f) {
    e = 14 - ilogbf(m);
    e = e > 126 ? 126 : (e < -126 ? -126 : e);
  }
  return e;
}

template <typename Args>
__device__ __forceinline__ void write_out(const Args& a, int o, int b, double y, double y2, bool dual) {
  const int64_t idx = static_cast<int64_t>(b) * a.ld_out + o;
  if (!dual) {
    float pre = static_cast<float>(y);
    double v = static_cast<double>(pre);
    if (a.bias != nullptr && o < a.bias_len) {
      v += a.bias[o];
      pre = static_cast<float>(v);
    }
    a.pre[idx] = pre;
    const float post = static_cast<float>(activate(a.act, v));
    a.post[idx] = post;
#pragma unroll
    for (int i = 0; i < kMaxPeerOut; ++i)  // static indices: the parameter stays in registers
      if (i < a.peers.n) a.peers.post[i][idx] = post;
  } else {
    const float gate_pre = static_cast<float>(y);
    const float up_post = static_cast<float>(y2);
    const float g = static_cast<float>(activate(1, static_cast<double>(gate_pre)));
    a.pre[idx] = static_cast<float>(static_cast<double>(g) * static_cast<double>(up_post));
  }
}

// Layers of one grouped launch (same shape and dtype): blockIdx.z picks the layer.
template <int kL>
struct GroupArgs {
  KArgs a;
  GemvGroupLayer layer[kL];
};

// Warps of a CTA: kWarps K slices, each split into two halves of the 64-row set (two row groups
// per warp) for 9..16 tokens, whose accumulators would not fit four row groups per warp.
template <int kB>
__host__ __device__ constexpr int halves_of() { return kB > 8 ? 2 : 1; }
template <int kB>
__host__ __device__ constexpr int threads_of() { return kWarps * 32 * halves_of<kB>(); }

template <int kDt, int kB, bool kDual, int kL>
__global__ void __launch_bounds__(threads_of<kB>(), kDual ? 2 : (kB > 8 ? 1 : (kB > 4 ? 3 : 4)))
    k_gemv_tc(const __grid_constant__ GroupArgs<kL> ga) {
  KArgs a = ga.a;
  if constexpr (kL > 1) {
    const GemvGroupLayer& L = ga.layer[blockIdx.z];
    a.Wt = L.Wt;
    a.x = L.x;
    a.pre = L.pre;
    a.post = L.post;
    a.bias = L.bias;
    a.bias_len = L.bias_len;
    a.act = L.act;
    a.scale = L.scale;
    a.frags = static_cast<const uint2*>(L.prep);
    a.fscale = L.prep ? reinterpret_cast<const float*>(a.frags + static_cast<int64_t>(a.csize) * a.nkb_cta * 8 * kB)
                      : nullptr;
  }
  constexpr int KBPU = kDt == 16 ? 4 : 2;       // K blocks of 16 per unit
  constexpr int CK = 2 * KBPU * 16;             // K elements per chunk
  constexpr int NCOL = 2 * kB;                  // B columns in use: n = 2 * token + plane
  constexpr int NT = (NCOL + 7) / 8;            // n8 tiles per A fragment (tokens 4 nt .. 4 nt + 3)
  constexpr int kHalves = halves_of<kB>();
  constexpr int kRGW = kRG / kHalves;            // row groups per warp
  constexpr int kThreads = threads_of<kB>();
  constexpr bool kPrepared = kL > 1 || kB > 8;   // B fragments prepared by k_prep_x
  __shared__ double red[kWarps][kRowsPerSet][kDual ? 2 : 1][kB];
  __shared__ double cta_part[kRowsPerSet][kDual ? 2 : 1][kB];
  __shared__ float smax[kWarps * kHalves][kB];
  extern __shared__ uint2 frag[];                // [nkb_cta][NCOL][4]

  asm volatile("griddepcontrol.launch_dependents;");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ks = warp % kWarps;                 // the warp's K slice
  const int half = warp / kWarps;               // its half of the row set (9..16 tokens)
  const int g = lane >> 2, t = lane & 3;
  const int rank = blockIdx.x;                  // K split = rank in the cluster
  // Row sets of this CTA: blockIdx.y, blockIdx.y + gridDim.y, ... (one per CTA unless a
  // grouped launch gives each CTA several, which then share the x slice and B fragments).
  int64_t rs = blockIdx.y;
  // The CTA's chunks [cta_c0, c1) are dealt to its warps in turn (warp w: cta_c0 + w,
  // + kWarps, ...), so the four warps advance through one contiguous run of the mirror.
  const int64_t cta_c0 = static_cast<int64_t>(rank) * kWarps * a.cpw;
  const int64_t c0 = cta_c0 + ks;
  int64_t c1 = cta_c0 + static_cast<int64_t>(kWarps) * a.cpw;
  if (c1 > a.chunks) c1 = a.chunks;
  constexpr int CS = kWarps;  // chunk stride of a warp

  auto load_chunk = [&](int64_t rg0, int64_t c, uint4 (&buf)[2][kRGW], uint4 (&buf2)[2][kRGW]) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t unit = 2 * c + u;
#pragma unroll
      for (int r = 0; r < kRGW; ++r) {
        const int rr = half * kRGW + r;  // row group within the set
        const bool ok = unit < a.units_k && rg0 + rr < a.row_groups;
        const int64_t off = (((rg0 / kRG) * a.units_k + unit) * kRG + rr) * 512 + lane * 16;
        buf[u][r] = ok ? ld_stream(a.Wt + off) : make_uint4(0, 0, 0, 0);
        if (kDual) buf2[u][r] = ok ? ld_stream(a.Wt2 + off) : make_uint4(0, 0, 0, 0);
      }
    }
  };

  uint4 bufA[2][kRGW], bufA2[2][kRGW];
  uint4 bufB[2][kRGW], bufB2[2][kRGW];
  // The first two chunks' weights are requested before waiting on the previous kernel:
  // they do not depend on it.
  if (c0 < c1) load_chunk(rs * kRG, c0, bufA, bufA2);
  if (c0 + CS < c1) load_chunk(rs * kRG, c0 + CS, bufB, bufB2);
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // B fragments of this CTA's K range, in shared memory: a grouped launch has them prepared
  // once per layer and each warp copies its own K quarter (one round of 16-byte loads from
  // L2); one layer per launch builds them here from the CTA's x slice
  float sinv[kB];
  if constexpr (kPrepared) {
#pragma unroll
    for (int b = 0; b < kB; ++b) sinv[b] = ld_dep(a.fscale + rank * kB + b);
    if (cta_c0 < c1) {
      const int64_t nkb = (c1 - cta_c0) * 2 * KBPU;
      const uint4* src = reinterpret_cast<const uint4*>(a.frags + rank * a.nkb_cta * NCOL * 4);
      uint4* dst = reinterpret_cast<uint4*>(frag);
      const int n16 = static_cast<int>(nkb * NCOL * 2);  // NCOL * 4 uint2 per K block
      for (int i = tid; i < n16; i += kThreads) dst[i] = ld_dep4u(src + i);
    }
    __syncthreads();
  } else {
  // ---- the CTA's x slice, read from global memory once into shared memory (zero past
  //      `cols`), with the per-token maximum taken on the way
  const int64_t klo = cta_c0 * CK;
  const int kspan = a.nkb_cta * 16;
  int64_t khi = klo + kspan;
  if (khi > a.cols) khi = a.cols;
  float* xs = reinterpret_cast<float*>(frag + a.nkb_cta * NCOL * 4);  // [kB][kspan], 16-byte aligned
  // klo and kspan are multiples of 64: 16-byte vectors whenever x's rows are 16-byte aligned
  const bool xvec = ((reinterpret_cast<uintptr_t>(a.x) | (static_cast<uintptr_t>(a.x_ld) * 4)) & 15) == 0;
#pragma unroll
  for (int b = 0; b < kB; ++b) {
    float m = 0.0f;
    const float* xb = a.x + b * a.x_ld;
    if (xvec) {
      for (int i = 4 * tid; i < kspan; i += 4 * kThreads) {
        const int64_t k = klo + i;
        float4 v;
        if (k + 3 < khi) {
          v = ld_dep4(xb + k);
        } else {
          v.x = k < khi ? ld_dep(xb + k) : 0.0f;
          v.y = k + 1 < khi ? ld_dep(xb + k + 1) : 0.0f;
          v.z = k + 2 < khi ? ld_dep(xb + k + 2) : 0.0f;
          v.w = 0.0f;
        }
        *reinterpret_cast<float4*>(xs + b * kspan + i) = v;
        const float a4[4] = {fabsf(v.x), fabsf(v.y), fabsf(v.z), fabsf(v.w)};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (a4[q] > m && a4[q] <= 3.402823466e+38f) m = a4[q];
      }
    } else {
      for (int i = tid; i < kspan; i += kThreads) {
        const int64_t k = klo + i;
        const float v = k < khi ? ld_dep(xb + k) : 0.0f;
        xs[b * kspan + i] = v;
        const float av = fabsf(v);
        if (av > m && av <= 3.402823466e+38f) m = av;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) smax[warp][b] = m;
  }
  __syncthreads();
  float sc[kB];
#pragma unroll
  for (int b = 0; b < kB; ++b) {
    const int e = x_scale_exp(fmaxf(fmaxf(smax[0][b], smax[1][b]), fmaxf(smax[2][b], smax[3][b])));
    sc[b] = ldexpf(1.0f, e);
    sinv[b] = ldexpf(1.0f, -e);
  }

  // ---- B fragments of the CTA's K range, built once by all 128 threads: entry (kbl, n, tt)
  //      holds x[k], x[k+1] (k = 16 kbl + 2 tt) and x[k+8], x[k+9] of column n = 2 token + plane;
  //      one thread makes both planes of one (kbl, token, tt)
  const int nent = a.nkb_cta * kB * 4;
  for (int e = tid; e < nent; e += kThreads) {
    const int kbl = e / (kB * 4);
    const int rem = e - kbl * (kB * 4);
    const int b = rem >> 2, tt = rem & 3;
    const float* xr = xs + b * kspan + kbl * 16 + 2 * tt;
    const float2 lo = *reinterpret_cast<const float2*>(xr), hi = *reinterpret_cast<const float2*>(xr + 8);
    float s = sc[0];
#pragma unroll
    for (int q = 1; q < kB; ++q)
      if (b == q) s = sc[q];
    uint32_t l0, l1, h0, h1;
    x_planes(lo.x, lo.y, s, l0, l1);
    x_planes(hi.x, hi.y, s, h0, h1);
    uint2* dst = frag + (kbl * NCOL + 2 * b) * 4 + tt;
    dst[0] = make_uint2(l0, h0);  // plane 0
    dst[4] = make_uint2(l1, h1);  // plane 1
  }
  __syncthreads();
  }

  // thread (g, t) holds, in n tile nt, both planes of token 4 nt + t for rows g and g + 8
  float sinv_t[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    sinv_t[nt] = 0.0f;
#pragma unroll
    for (int b = 0; b < kB; ++b)
      if (4 * nt + t == b) sinv_t[nt] = sinv[b];
  }

  double acc[kRGW][2][NT], acc2[kRGW][2][NT];

  auto compute_chunk = [&](int64_t c, const uint4 (&buf)[2][kRGW], const uint4 (&buf2)[2][kRGW]) {
    float d[kRGW][NT][4], d2[kRGW][NT][4];
#pragma unroll
    for (int r = 0; r < kRGW; ++r)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) d[r][nt][i] = d2[r][nt][i] = 0.0f;
    const int kb_base = static_cast<int>(c - cta_c0) * 2 * KBPU;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
#pragma unroll
      for (int j = 0; j < KBPU; ++j) {
        uint2 bf[NT];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int col = 8 * nt + g;
          const int fi = ((kb_base + u * KBPU + j) * NCOL + col) * 4 + t;
          bf[nt] = col < NCOL ? frag[fi] : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int r = 0; r < kRGW; ++r) {
          uint32_t af[4];
          a_frag<kDt>(buf[u][r], j, af);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma16816(d[r][nt], af, bf[nt].x, bf[nt].y);
          if (kDual) {
            a_frag<kDt>(buf2[u][r], j, af);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma16816(d2[r][nt], af, bf[nt].x, bf[nt].y);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kRGW; ++r)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        acc[r][0][nt] += (static_cast<double>(d[r][nt][0]) + static_cast<double>(d[r][nt][1])) * sinv_t[nt];
        acc[r][1][nt] += (static_cast<double>(d[r][nt][2]) + static_cast<double>(d[r][nt][3])) * sinv_t[nt];
        if (kDual) {
          acc2[r][0][nt] += (static_cast<double>(d2[r][nt][0]) + static_cast<double>(d2[r][nt][1])) * sinv_t[nt];
          acc2[r][1][nt] += (static_cast<double>(d2[r][nt][2]) + static_cast<double>(d2[r][nt][3])) * sinv_t[nt];
        }
      }
  };

  namespace cg = cooperative_groups;
  constexpr int M = kDual ? 2 : 1;
  const int64_t nrs = (a.row_groups + kRG - 1) / kRG;
  for (; rs < nrs; rs += gridDim.y) {
    const int64_t rg0 = rs * kRG;
#pragma unroll
    for (int r = 0; r < kRGW; ++r)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[r][0][nt] = acc[r][1][nt] = acc2[r][0][nt] = acc2[r][1][nt] = 0.0;
  // the warp's chunks alternate between bufA and bufB; the chunk two ahead is requested as
  // soon as its buffer is free.
  for (int64_t c = c0; c < c1; c += 2 * CS) {
    compute_chunk(c, bufA, bufA2);
    if (c + 2 * CS < c1) load_chunk(rg0, c + 2 * CS, bufA, bufA2);
    if (c + CS < c1) {
      compute_chunk(c + CS, bufB, bufB2);
      if (c + 3 * CS < c1) load_chunk(rg0, c + 3 * CS, bufB, bufB2);
    }
  }
  // the next row set's first two chunks stream in while this one is reduced and written
  if (rs + gridDim.y < nrs) {
    if (c0 < c1) load_chunk((rs + gridDim.y) * kRG, c0, bufA, bufA2);
    if (c0 + CS < c1) load_chunk((rs + gridDim.y) * kRG, c0 + CS, bufB, bufB2);
  }

  // ---- CTA reduction over its 4 K slices (fixed order)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int tok = 4 * nt + t;
    if (tok < kB) {
#pragma unroll
      for (int r = 0; r < kRGW; ++r) {
        const int row = (half * kRGW + r) * 16 + g;
        red[ks][row][0][tok] = acc[r][0][nt];
        red[ks][row + 8][0][tok] = acc[r][1][nt];
        if (kDual) {
          red[ks][row][kDual ? 1 : 0][tok] = acc2[r][0][nt];
          red[ks][row + 8][kDual ? 1 : 0][tok] = acc2[r][1][nt];
        }
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < kRowsPerSet * M * kB; i += kThreads) {
    const int row = i / (M * kB), rem = i - row * M * kB, m = rem / kB, b = rem - m * kB;
    double y = 0.0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) y += red[w][row][m][b];
    cta_part[row][m][b] = y;
  }

  // ---- cluster reduction over the K splits through distributed shared memory
  if (a.csize > 1) cg::this_cluster().sync();
  else __syncthreads();
  if (rank == 0) {
    for (int i = tid; i < kRowsPerSet * kB; i += kThreads) {
      const int row = i / kB, b = i - row * kB;
      const int o = static_cast<int>(rs * kRowsPerSet + row);
      if (b >= a.nb) continue;  // tokens past the launch's batch (kB rounds it up)
      double y = 0.0, y2 = 0.0;
      for (int r = 0; r < a.csize; ++r) {
        const double (*part)[M][kB] = cta_part;
        if (a.csize > 1) part = cg::this_cluster().map_shared_rank(cta_part, r);
        y += part[row][0][b];
        if (kDual) y2 += part[row][M - 1][b];
      }
      if (o >= a.rows) continue;
      if (kDt == 9) { y *= static_cast<double>(a.scale); y2 *= static_cast<double>(a.scale2); }
      write_out(a, o, b, y, y2, kDual);
    }
  }
  if (a.csize > 1) cg::this_cluster().sync();  // keep every rank's shared memory alive for rank 0
  }
}

// One thread per output byte of the tiled mirror.
template <int kDt>
__global__ void k_build_tiled(const uint8_t* __restrict__ native, int rows, int cols, int64_t units_k,
                              int64_t total, uint8_t* __restrict__ out) {
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t unit_idx = t >> 9;  // (row set * units_k + unit) * 4 + row group in the set
    const int within = static_cast<int>(t & 511);
    const int lane = within >> 4;
    const int g = lane >> 2, tt = lane & 3;
    const int64_t q = unit_idx / TiledGeom::kSetGroups;
    const int64_t set = q / units_k, unit = q - set * units_k;
    const int64_t rg = set * TiledGeom::kSetGroups + (unit_idx - q * TiledGeom::kSetGroups);
    uint32_t byte = 0;
    if (kDt == 16) {
      const int j = (within >> 2) & 3;        // K block within the unit
      const int pair = within & 3;            // fragment elements 2*pair, 2*pair+1
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i = 2 * pair + h;
        const int64_t row = rg * 16 + g + 8 * ((i >> 1) & 1);
        const int64_t k = unit * 64 + j * 16 + 2 * tt + (i & 1) + 8 * (i >> 2);
        uint32_t code = 0;
        if (row < rows && k < cols) {
          const int64_t f = row * cols + k;
          code = (native[f >> 1] >> ((f & 1) * 4)) & 0xF;
        }
        byte |= code << (4 * h);
      }
    } else {
      const int j = (within >> 3) & 1;
      const int i = within & 7;
      const int64_t row = rg * 16 + g + 8 * ((i >> 1) & 1);
      const int64_t k = unit * 32 + j * 16 + 2 * tt + (i & 1) + 8 * (i >> 2);
      if (row < rows && k < cols) {
        const uint32_t c = native[row * cols + k];
        byte = kDt == 4 ? canon_e4m3(c) : (kDt == 5 ? canon_e5m2(c) : c);
      }
    }
    out[t] = static_cast<uint8_t>(byte);
  }
}

// Prepares the x of grouped layers once per layer: the kPrepSub blocks (seg * kPrepSub + sub,
// layer) of K segment seg each take the largest finite |x| of the segment per token and its
// power-of-two scale, and write their share of the segment's f16 B fragments in the layout
// the GEMV's CTAs use -- exactly what each CTA of that segment would build itself.
template <int kL>
struct PrepArgs {
  int cols = 0, nkb_cta = 0;
  int nb = 0;  // tokens present (<= kB): tokens past it are zero
  int64_t x_ld = 0;
  const float* x[kL] = {};
  uint2* frags[kL] = {};
  float* fscale[kL] = {};
};

constexpr int kPrepThreads = 256;
// Blocks per K segment: each takes the segment's scale itself (the segment is at most 8192
// floats per token, read from L2 with every load of a thread in flight at once) and writes
// its share of the fragments. One block per segment issued its loads one after another and
// took ~6 us per launch at 8192 x 16384; the dependent GEMV waits for it.
constexpr int kPrepSub = 8;

template <int kB, int kL>
__global__ void __launch_bounds__(kPrepThreads) k_prep_x(const __grid_constant__ PrepArgs<kL> pa) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // x may be the previous kernel's output
  constexpr int NCOL = 2 * kB;
  constexpr int kU = 8;  // loads in flight per thread in the scale pass
  __shared__ float smax[kPrepThreads / 32][kB];
  __shared__ float ssc[kB];
  const int seg = blockIdx.x / kPrepSub, sub = blockIdx.x % kPrepSub, layer = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* x = pa.x[layer];
  const int kspan = pa.nkb_cta * 16;
  const int64_t klo = static_cast<int64_t>(seg) * kspan;
  const int64_t khi = klo + kspan < pa.cols ? klo + kspan : pa.cols;
#pragma unroll 1
  for (int b = 0; b < kB; ++b) {
    float m = 0.0f;
    if (b < pa.nb) {
      const float* xb = x + b * pa.x_ld;
      // klo is a multiple of 64: 16-byte vectors whenever the token's row is 16-byte aligned
      if ((reinterpret_cast<uintptr_t>(xb) & 15) == 0) {
        for (int64_t k0 = klo + 4 * tid; k0 < khi; k0 += 4 * kPrepThreads * kU) {
          float4 v[kU];
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            const int64_t k = k0 + static_cast<int64_t>(u) * 4 * kPrepThreads;
            v[u] = k + 3 < khi ? ld_dep4(xb + k) : make_float4(0.f, 0.f, 0.f, 0.f);
            if (k < khi && k + 3 >= khi) {  // the segment's ragged end, element by element
              v[u].x = ld_dep(xb + k);
              if (k + 1 < khi) v[u].y = ld_dep(xb + k + 1);
              if (k + 2 < khi) v[u].z = ld_dep(xb + k + 2);
            }
          }
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            for (float av : {fabsf(v[u].x), fabsf(v[u].y), fabsf(v[u].z), fabsf(v[u].w)})
              if (av > m && av <= 3.402823466e+38f) m = av;
          }
        }
      } else {
        for (int64_t k0 = klo + tid; k0 < khi; k0 += kPrepThreads * kU) {
          float v[kU];
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            const int64_t k = k0 + static_cast<int64_t>(u) * kPrepThreads;
            v[u] = k < khi ? ld_dep(xb + k) : 0.0f;
          }
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            const float av = fabsf(v[u]);
            if (av > m && av <= 3.402823466e+38f) m = av;
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) smax[warp][b] = m;
  }
  __syncthreads();
  if (tid < kB) {
    float m = smax[0][tid];
#pragma unroll
    for (int w = 1; w < kPrepThreads / 32; ++w) m = fmaxf(m, smax[w][tid]);
    const int e = x_scale_exp(m);
    ssc[tid] = ldexpf(1.0f, e);
    if (sub == 0) pa.fscale[layer][seg * kB + tid] = ldexpf(1.0f, -e);
  }
  __syncthreads();
  uint2* fr = pa.frags[layer] + static_cast<int64_t>(seg) * pa.nkb_cta * NCOL * 4;
  const int nent = pa.nkb_cta * kB * 4;
  const int per = (nent + kPrepSub - 1) / kPrepSub;
  const int e_end = (sub + 1) * per < nent ? (sub + 1) * per : nent;
  for (int e = sub * per + tid; e < e_end; e += kPrepThreads) {
    const int kbl = e / (kB * 4);
    const int rem = e - kbl * (kB * 4);
    const int b = rem >> 2, tt = rem & 3;
    const int64_t k = klo + kbl * 16 + 2 * tt;
    const float* xb = x + b * pa.x_ld;
    const bool in = b < pa.nb;
    const float v0 = in && k < khi ? ld_dep(xb + k) : 0.0f, v1 = in && k + 1 < khi ? ld_dep(xb + k + 1) : 0.0f;
    const float v8 = in && k + 8 < khi ? ld_dep(xb + k + 8) : 0.0f, v9 = in && k + 9 < khi ? ld_dep(xb + k + 9) : 0.0f;
    uint32_t l0, l1, h0, h1;
    x_planes(v0, v1, ssc[b], l0, l1);
    x_planes(v8, v9, ssc[b], h0, h1);
    uint2* dst = fr + (kbl * NCOL + 2 * b) * 4 + tt;
    dst[0] = make_uint2(l0, h0);  // plane 0
    dst[4] = make_uint2(l1, h1);  // plane 1
  }
}

template <int kL>
Status launch_prep(const PrepArgs<kL>& pa, int csize, int nl, int batch, cudaStream_t st, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(csize * kPrepSub), static_cast<unsigned>(nl), 1);
  cfg.blockDim = dim3(kPrepThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  switch (batch) {
  case 1: return cuda_status(cudaLaunchKernelEx(&cfg, k_prep_x<1, kL>, pa), "gemv_tc prep launch");
  case 2: return cuda_status(cudaLaunchKernelEx(&cfg, k_prep_x<2, kL>, pa), "gemv_tc prep launch");
  case 3: return cuda_status(cudaLaunchKernelEx(&cfg, k_prep_x<3, kL>, pa), "gemv_tc prep launch");
  case 4: return cuda_status(cudaLaunchKernelEx(&cfg, k_prep_x<4, kL>, pa), "gemv_tc prep launch");
  default:
    if constexpr (kL == 1) {
      if (batch == 12) return cuda_status(cudaLaunchKernelEx(&cfg, k_prep_x<12, 1>, pa), "gemv_tc prep launch");
      if (batch == 16) return cuda_status(cudaLaunchKernelEx(&cfg, k_prep_x<16, 1>, pa), "gemv_tc prep launch");
    }
    return Status::Internal("gemv_tc prep: batch must be 1..4 (12 or 16 for one layer)");
  }
}

// The 48 KB default covers static + dynamic shared memory together, so every launch opts in
// to its dynamic size (the reduction arrays are static). One driver call per kernel, device
// and size, cached.
Status allow_dynamic_smem(const void* kern, size_t bytes) {
  static std::mutex mu;
  static std::vector<std::tuple<const void*, int, size_t>> done;
  int dev = 0;
  WB_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& d : done)
    if (std::get<0>(d) == kern && std::get<1>(d) == dev && std::get<2>(d) >= bytes) return Status::Ok();
  WB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)));
  for (auto& d : done)
    if (std::get<0>(d) == kern && std::get<1>(d) == dev) {
      std::get<2>(d) = bytes;
      return Status::Ok();
    }
  done.emplace_back(kern, dev, bytes);
  return Status::Ok();
}

template <int kDt, int kB, bool kDual, int kL>
Status launch_t(const GroupArgs<kL>& k, int nl, const Plan& pl, cudaStream_t st, bool pdl, bool prepared) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(pl.csize), static_cast<unsigned>(pl.grid_y), static_cast<unsigned>(nl));
  cfg.blockDim = dim3(threads_of<kB>());
  // B fragments [nkb_cta][2 kB][4] uint2, then the x slice [kB][16 nkb_cta] float (not when
  // the fragments are prepared)
  cfg.dynamicSmemBytes = static_cast<size_t>(pl.nkb_cta) * 2 * kB * 4 * sizeof(uint2) +
                         (prepared ? 0 : static_cast<size_t>(pl.nkb_cta) * 16 * kB * sizeof(float));
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = static_cast<unsigned>(pl.csize);
  attr[n].val.clusterDim.y = 1;
  attr[n].val.clusterDim.z = 1;
  ++n;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  auto kern = k_gemv_tc<kDt, kB, kDual, kL>;
  WB_TRY(allow_dynamic_smem(reinterpret_cast<const void*>(kern), cfg.dynamicSmemBytes));
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, k), "gemv_tc launch");
}

template <int kDt, bool kDual, int kL>
Status launch_b(const GroupArgs<kL>& k, int nl, const Plan& pl, int batch, cudaStream_t st, bool pdl,
                bool prepared) {
  switch (batch) {
  case 1: return launch_t<kDt, 1, kDual, kL>(k, nl, pl, st, pdl, prepared);
  case 2: return launch_t<kDt, 2, kDual, kL>(k, nl, pl, st, pdl, prepared);
  case 3: return launch_t<kDt, 3, kDual, kL>(k, nl, pl, st, pdl, prepared);
  case 4: return launch_t<kDt, 4, kDual, kL>(k, nl, pl, st, pdl, prepared);
  default:
    if constexpr (!kDual && kL == 1) {
      switch (batch) {
      case 5: return launch_t<kDt, 5, false, 1>(k, nl, pl, st, pdl, prepared);
      case 6: return launch_t<kDt, 6, false, 1>(k, nl, pl, st, pdl, prepared);
      case 7: return launch_t<kDt, 7, false, 1>(k, nl, pl, st, pdl, prepared);
      case 8: return launch_t<kDt, 8, false, 1>(k, nl, pl, st, pdl, prepared);
      default:
        if (batch >= 9 && batch <= 12) return launch_t<kDt, 12, false, 1>(k, nl, pl, st, pdl, true);
        if (batch >= 13 && batch <= 16) return launch_t<kDt, 16, false, 1>(k, nl, pl, st, pdl, true);
        break;
      }
    }
    return Status::Internal("gemv_tc: batch must be 1..16 (1..4 for the fused Gate/Up and grouped launches)");
  }
}

template <bool kDual, int kL>
Status launch_d(DType dt, const GroupArgs<kL>& k, int nl, const Plan& pl, int batch, cudaStream_t st, bool pdl,
                bool prepared = false) {
  switch (dt) {
  case DType::FP4: return launch_b<16, kDual, kL>(k, nl, pl, batch, st, pdl, prepared);
  case DType::FP8E4M3: return launch_b<4, kDual, kL>(k, nl, pl, batch, st, pdl, prepared);
  case DType::FP8E5M2: return launch_b<5, kDual, kL>(k, nl, pl, batch, st, pdl, prepared);
  case DType::Int8: return launch_b<9, kDual, kL>(k, nl, pl, batch, st, pdl, prepared);
  default: return Status::Unsupported("gemv_tc: dtype");
  }
}


} // namespace

bool gemv_tc_supported(DType dt) {
  return dt == DType::FP4 || dt == DType::FP8E4M3 || dt == DType::FP8E5M2 || dt == DType::Int8;
}

TiledGeom tiled_geom(DType dt, int rows, int cols) {
  TiledGeom g;
  g.unit_k = dt == DType::FP4 ? 64 : 32;
  g.row_groups = (rows + 15) / 16;
  g.units_k = (cols + g.unit_k - 1) / g.unit_k;
  return g;
}

Status build_tiled_mirror(DType dt, const uint8_t* native, int rows, int cols, uint8_t* tiled, cudaStream_t st) {
  const TiledGeom g = tiled_geom(dt, rows, cols);
  const int64_t total = g.bytes();
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 64) blocks = 148 * 64;
  const unsigned gb = static_cast<unsigned>(blocks);
  switch (dt) {
  case DType::FP4: k_build_tiled<16><<<gb, 256, 0, st>>>(native, rows, cols, g.units_k, total, tiled); break;
  case DType::FP8E4M3: k_build_tiled<4><<<gb, 256, 0, st>>>(native, rows, cols, g.units_k, total, tiled); break;
  case DType::FP8E5M2: k_build_tiled<5><<<gb, 256, 0, st>>>(native, rows, cols, g.units_k, total, tiled); break;
  case DType::Int8: k_build_tiled<9><<<gb, 256, 0, st>>>(native, rows, cols, g.units_k, total, tiled); break;
  default: return Status::Unsupported("tiled mirror: dtype");
  }
  return cuda_status(cudaGetLastError(), "tiled mirror launch");
}

Status launch_gemv_tc(const GemvTcArgs& a, cudaStream_t st, bool pdl) {
  if (!gemv_tc_supported(a.dtype)) return Status::Unsupported("gemv_tc: dtype");
  if (a.rows <= 0 || a.cols <= 0 || a.batch < 1 || a.batch > (a.Wt2 ? 4 : kGemvMaxBatch))
    return Status::Invalid("gemv_tc: bad dims");
  const Plan pl = make_plan(a.dtype, a.rows, a.cols, false, a.batch, a.Wt2 != nullptr);
  KArgs k{};
  k.Wt = a.Wt;
  k.Wt2 = a.Wt2;
  k.rows = a.rows;
  k.cols = a.cols;
  k.units_k = pl.g.units_k;
  k.row_groups = pl.g.row_groups;
  k.chunks = pl.chunks;
  k.cpw = pl.cpw;
  k.csize = pl.csize;
  k.nkb_cta = pl.nkb_cta;
  k.scale = a.scale;
  k.scale2 = a.scale2;
  k.x = a.x;
  k.x_ld = a.x_ld;
  k.pre = a.pre;
  k.post = a.post;
  k.ld_out = a.ld_out;
  k.bias = a.bias;
  k.bias_len = a.bias_len;
  k.act = a.act;
  k.peers = a.peers;
  k.nb = a.batch;
  if (a.batch > 8) {
    // 9..16 tokens: x is prepared once (f16 B fragments of 12 or 16 tokens per K segment)
    // by a small kernel, then the GEMV copies its segment's fragments into shared memory.
    if (a.Wt2) return Status::Invalid("gemv_tc: the fused Gate/Up form takes 1..4 tokens");
    if (!a.prep) return Status::Internal("gemv_tc: 9..16 tokens need prepared-fragment scratch");
    if (!gemv_tc_fits(a.dtype, a.rows, a.cols, a.batch))
      return Status::Invalid("gemv_tc: K too long for 9..16 tokens (the batched GEMM takes it)");
    const int kb = a.batch <= 12 ? 12 : 16;
    PrepArgs<1> pa;
    pa.cols = a.cols;
    pa.nkb_cta = pl.nkb_cta;
    pa.nb = a.batch;
    pa.x_ld = a.x_ld;
    pa.x[0] = a.x;
    pa.frags[0] = static_cast<uint2*>(a.prep);
    pa.fscale[0] = reinterpret_cast<float*>(pa.frags[0] + static_cast<int64_t>(pl.csize) * pl.nkb_cta * 8 * kb);
    WB_TRY(launch_prep(pa, pl.csize, 1, kb, st, pdl));
    k.frags = pa.frags[0];
    k.fscale = pa.fscale[0];
    pdl = true;  // the GEMV's weight loads start while the preparation runs
  }
  GroupArgs<1> g{};
  g.a = k;
  return a.Wt2 ? launch_d<true, 1>(a.dtype, g, 1, pl, a.batch, st, pdl)
               : launch_d<false, 1>(a.dtype, g, 1, pl, a.batch, st, pdl);
}

bool gemv_tc_fits(DType dt, int rows, int cols, int batch) {
  if (!gemv_tc_supported(dt) || rows <= 0 || cols <= 0 || batch < 1 || batch > kGemvMaxBatch) return false;
  if (batch <= 8) return true;
  const Plan pl = make_plan(dt, rows, cols, false, batch);
  if (pl.csize > kMaxCluster) return false;
  const int kb = batch <= 12 ? 12 : 16;
  // prepared fragments in shared memory next to the static reduction arrays (~40 KB at 16)
  return static_cast<size_t>(pl.nkb_cta) * 2 * kb * 4 * sizeof(uint2) <= 176u * 1024u;
}

size_t gemv_prep_bytes(DType dt, int rows, int cols, int batch) {
  if (batch <= 4) return gemv_group_prep_bytes(dt, rows, cols, batch);
  if (batch <= 8 || !gemv_tc_fits(dt, rows, cols, batch)) return 0;
  const Plan pl = make_plan(dt, rows, cols, false, batch);
  const int kb = batch <= 12 ? 12 : 16;
  return static_cast<size_t>(pl.csize) * pl.nkb_cta * 8 * kb * sizeof(uint2) +
         static_cast<size_t>(pl.csize) * kb * sizeof(float);
}

bool gemv_prefers_prepared(DType dt, int rows, int cols, int batch) {
  if (!gemv_tc_supported(dt) || rows <= 0 || cols <= 0 || batch < 1 || batch > 4) return false;
  if (const char* env = std::getenv("WELVET_B200_GEMV_PREP")) {
    if (env[0] == '1') return true;
    if (env[0] == '0') return false;
  }
  // measured: layers of 8192 rows and more stream faster with x prepared once (65536 x 16384
  // FP4: 147 -> 120 us, 14336 x 4096: 24.6 -> 19.5 us); 4096-row layers slower (12.4 -> 17.4)
  const Plan pl = make_plan(dt, rows, cols, true);
  return pl.row_sets >= 128;
}

Status launch_gemv_tc_group(DType dt, int rows, int cols, int batch, int64_t x_ld, int64_t ld_out,
                            const GemvGroupLayer* layers, int n, cudaStream_t st, bool pdl, const PeerOut* peers) {
  if (!gemv_tc_supported(dt)) return Status::Unsupported("gemv_tc: dtype");
  if (rows <= 0 || cols <= 0 || batch < 1 || batch > 4 || n < 0 || (n > 0 && !layers))
    return Status::Invalid("gemv_tc group: bad arguments");
  for (int i = 0; i < n; ++i) {
    const GemvGroupLayer& L = layers[i];
    if (!L.Wt || !L.x || !L.pre || !L.post || !L.prep) return Status::Invalid("gemv_tc group: null layer pointer");
  }
  Plan pl = make_plan(dt, rows, cols, true);
  // one 64-row set per CTA: many short CTAs balance over the SMs better than fewer long
  // ones (measured: 3 row sets per CTA left a partial second wave)
  pl.grid_y = pl.row_sets;
  // The layers are independent: every layer's x is prepared first (one small launch per 32
  // layers), then the GEMV launches follow as programmatic dependents, so each one's CTAs
  // start streaming weights while the launch before it drains.
  const int64_t nfr = static_cast<int64_t>(pl.csize) * pl.nkb_cta * 8 * batch;
  for (int l0 = 0; l0 < n; l0 += kGemvGroupMax) {
    const int nl = n - l0 < kGemvGroupMax ? n - l0 : kGemvGroupMax;
    PrepArgs<kGemvGroupMax> pa;
    pa.cols = cols;
    pa.nkb_cta = pl.nkb_cta;
    pa.nb = batch;
    pa.x_ld = x_ld;
    for (int i = 0; i < nl; ++i) {
      pa.x[i] = layers[l0 + i].x;
      pa.frags[i] = static_cast<uint2*>(layers[l0 + i].prep);
      pa.fscale[i] = reinterpret_cast<float*>(pa.frags[i] + nfr);
    }
    WB_TRY(launch_prep(pa, pl.csize, nl, batch, st, pdl || l0 > 0));
  }
  for (int l0 = 0; l0 < n; l0 += kGemvGroupMax) {
    const int nl = n - l0 < kGemvGroupMax ? n - l0 : kGemvGroupMax;
    GroupArgs<kGemvGroupMax> g{};
    KArgs& k = g.a;
    k.rows = rows;
    k.cols = cols;
    k.units_k = pl.g.units_k;
    k.row_groups = pl.g.row_groups;
    k.chunks = pl.chunks;
    k.cpw = pl.cpw;
    k.csize = pl.csize;
    k.nkb_cta = pl.nkb_cta;
    k.x_ld = x_ld;
    k.ld_out = ld_out;
    k.nb = batch;
    if (peers) k.peers = *peers;
    for (int i = 0; i < nl; ++i) g.layer[i] = layers[l0 + i];
    WB_TRY((launch_d<false, kGemvGroupMax>(dt, g, nl, pl, batch, st, true, true)));
  }
  return Status::Ok();
}

size_t gemv_group_prep_bytes(DType dt, int rows, int cols, int batch) {
  if (!gemv_tc_supported(dt) || rows <= 0 || cols <= 0 || batch < 1 || batch > 4) return 0;
  const Plan pl = make_plan(dt, rows, cols, true);
  return static_cast<size_t>(pl.csize) * pl.nkb_cta * 8 * batch * sizeof(uint2) +
         static_cast<size_t>(pl.csize) * batch * sizeof(float);
}

} // namespace wb
