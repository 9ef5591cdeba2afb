// gemm_tc.cu -- batched dequant GEMM on sm_100a tensor cores (tcgen05.mma kind::f16, TMEM).
//
// Replaces, for batches above 8 tokens (SwiGLU cells: above 4), the reference's per-output fp64 loop
// (src/cuda/kernels.cu:130-145) over a host-decoded fp64 W. Two kernels:
//
//   k_gemm_tm (default)  the dequantised weight tile is the MMA's A operand in TMEM: converter
//                        warps read the packed codes (one row per thread) from a deep ring of
//                        raw W tiles (bulk copies of the GEMM mirror), convert with the
//                        hardware e2m1/e4m3/e5m2 -> f16x2 converters (Int8 via an exact f16
//                        bias trick) and write them with tcgen05.st; the x planes are the B
//                        operand, TMA-loaded into shared memory. See the comment above it.
//   k_gemm_tc            the same GEMM with A in shared memory (WELVET_B200_GEMM=smem), kept
//                        for comparison.
//
// x is split per token into f16 planes after a power-of-two scale (x * 2^e = p0 + p1 [+ p2],
// k_split_x; two planes by default, three on request, one for a token whose values are exact
// in f16); the planes ride in the N dimension of the MMAs. FP8/FP4/Int8 codes are exact in
// f16, so every product is exact and the tensor core accumulates in fp32; planes are
// combined in fp64 in the epilogue, which then applies the per-token 2^-e, the Int8 scale,
// and bias / activation exactly as the reference's dense_bias_act (kernels.cu:147-161).
//
// Every mbarrier wait is bounded by %globaltimer (2 s); on expiry the kernel records an error
// word and winds down, it never spins forever. Every tensor load has one destination CTA.
#include "gemm_tc.hpp"
#include "codec.cuh"
#include "pipeline.cuh"
#include "rmsnorm.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <tuple>
#include <type_traits>
#include <utility>
#include <vector>

namespace wb {
namespace {
using namespace pipe;

constexpr int kBM = 128;      // output rows per tile (MMA M)
constexpr int kBK = 64;       // k per stage (128 bytes of f16)
constexpr int kThreads = 192; // 6 warps

struct KParams {
  int rows, cols, M, T, N, xsplit;
  int nkb_total, kb_per_split, splits;
  int Mp;
  int kbb;                     // packed bytes per row per stage
  uint32_t idesc;
  uint32_t tmem_cols;
  uint32_t stage_bytes, a_off, b_off, w_off;
  int stages;
  const float* scale_inv;      // [Mp]
  float w_scale;
  float* pre;
  float* post;
  int64_t ld_out;
  const double* bias;
  int bias_len;
  int act;
  double* partial;             // [splits][M][rows] when splits > 1
  int* err;
  int pair;                    // SwiGLU Gate/Up pair reduce (see TmParams)
  float* h;
  int64_t ld_h;
  PeerOut peers;               // further destinations of post (column-sharded layers)
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);   // start address
  d |= static_cast<uint64_t>(1) << 16;                 // leading byte offset (unused, K-major SW128)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;         // stride byte offset: 8-row groups 1024 B apart
  d |= static_cast<uint64_t>(1) << 46;                 // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                 // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// 8 packed codes of one row -> 8 f16 (16 bytes) for the A tile.
template <int kDt>
__device__ __forceinline__ uint4 codes_to_f16x8(const uint8_t* raw_row, int j) {
  uint4 o;
  if constexpr (kDt == 16) {
    const uint32_t w = reinterpret_cast<const uint32_t*>(raw_row)[j];  // 8 nibbles, low first
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
        : "=r"(o.x), "=r"(o.y), "=r"(o.z), "=r"(o.w)
        : "r"(w));
  } else {
    const uint2 w = reinterpret_cast<const uint2*>(raw_row)[j];  // 8 bytes
    if constexpr (kDt == 4 || kDt == 5) {
      if constexpr (kDt == 4) {
        asm("{\n\t.reg .b16 l0, h0, l1, h1;\n\t"
            "mov.b32 {l0, h0}, %4;\n\t"
            "mov.b32 {l1, h1}, %5;\n\t"
            "cvt.rn.f16x2.e4m3x2 %0, l0;\n\t"
            "cvt.rn.f16x2.e4m3x2 %1, h0;\n\t"
            "cvt.rn.f16x2.e4m3x2 %2, l1;\n\t"
            "cvt.rn.f16x2.e4m3x2 %3, h1;\n\t}"
            : "=r"(o.x), "=r"(o.y), "=r"(o.z), "=r"(o.w)
            : "r"(w.x), "r"(w.y));
      } else {
        asm("{\n\t.reg .b16 l0, h0, l1, h1;\n\t"
            "mov.b32 {l0, h0}, %4;\n\t"
            "mov.b32 {l1, h1}, %5;\n\t"
            "cvt.rn.f16x2.e5m2x2 %0, l0;\n\t"
            "cvt.rn.f16x2.e5m2x2 %1, h0;\n\t"
            "cvt.rn.f16x2.e5m2x2 %2, l1;\n\t"
            "cvt.rn.f16x2.e5m2x2 %3, h1;\n\t}"
            : "=r"(o.x), "=r"(o.y), "=r"(o.z), "=r"(o.w)
            : "r"(w.x), "r"(w.y));
      }
    } else {  // Int8: f16 bits 0x6400 | (q ^ 0x80) = 1024 + q + 128, minus 1152 -> q exactly
      const uint32_t ux = w.x ^ 0x80808080u, uy = w.y ^ 0x80808080u;
      const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
      uint32_t p0 = __byte_perm(ux, 0x64646464u, 0x4140), p1 = __byte_perm(ux, 0x64646464u, 0x4342);
      uint32_t p2 = __byte_perm(uy, 0x64646464u, 0x4140), p3 = __byte_perm(uy, 0x64646464u, 0x4342);
      __half2 h0 = __hsub2(*reinterpret_cast<__half2*>(&p0), bias);
      __half2 h1 = __hsub2(*reinterpret_cast<__half2*>(&p1), bias);
      __half2 h2 = __hsub2(*reinterpret_cast<__half2*>(&p2), bias);
      __half2 h3 = __hsub2(*reinterpret_cast<__half2*>(&p3), bias);
      o.x = *reinterpret_cast<uint32_t*>(&h0);
      o.y = *reinterpret_cast<uint32_t*>(&h1);
      o.z = *reinterpret_cast<uint32_t*>(&h2);
      o.w = *reinterpret_cast<uint32_t*>(&h3);
    }
  }
  return o;
}

// The reference epilogue (src/cuda/kernels.cu:147-161): pre = float(y); with bias
// v = double(pre) + bias and pre = float(v); post = float(act(v)).
// SwiGLU product of one Gate/Up pair (src/cuda/kernels.cu:296-305 with the Dense
// epilogues of Linear Gate and Up before it): gate_pre = float(y_gate), up = float(y_up),
// h = float(double(float(SiLU(double(gate_pre)))) * double(up)).
template <typename Params>
__device__ __forceinline__ void write_pair(const Params& p, int t, int i, double y_gate, double y_up) {
  const float gate_pre = static_cast<float>(y_gate);
  const float up = static_cast<float>(y_up);
  const float g = static_cast<float>(activate(1, static_cast<double>(gate_pre)));
  p.h[static_cast<int64_t>(t) * p.ld_h + i] = static_cast<float>(static_cast<double>(g) * static_cast<double>(up));
}

// The values write_out / write_pair store, for an epilogue that stages them first.
template <typename Params>
__device__ __forceinline__ void out_values(const Params& p, int o, double y, float& pre, float& post) {
  pre = static_cast<float>(y);
  double v = static_cast<double>(pre);
  if (p.bias != nullptr && o < p.bias_len) {
    v += p.bias[o];
    pre = static_cast<float>(v);
  }
  post = static_cast<float>(activate(p.act, v));
}

// The SwiGLU product of one Gate/Up pair from the floats the reference rounds Gate and Up to
// (src/cuda/kernels.cu:296-305), SiLU in fp64 with its exp inline so that the GEMM epilogue
// overlaps a few of them.
__device__ __forceinline__ float pair_value_inline(float gate_pre, float up) {
  const double x = static_cast<double>(gate_pre);
  const float g = static_cast<float>(x / (1.0 + exp(-x)));
  return static_cast<float>(static_cast<double>(g) * static_cast<double>(up));
}

// The same product with SiLU in fp32 (expf, IEEE division): SiLU within a few ulp of the
// fp64 form; the product rounds as the reference's (the fp64 product of two floats is exact,
// so its rounding to float is the fp32 product). For x below -88, expf(-x) overflows and the
// SiLU is -0 where the fp64 form gives a float of magnitude below 1e-37.
__device__ __forceinline__ float pair_value_f32(float gate_pre, float up) {
  const float g = gate_pre / (1.0f + expf(-gate_pre));
  return g * up;
}


template <typename Params>
__device__ __forceinline__ void write_out(const Params& p, int t, int o, double y) {
  const int64_t idx = static_cast<int64_t>(t) * p.ld_out + o;
  float pre = static_cast<float>(y);
  double v = static_cast<double>(pre);
  if (p.bias != nullptr && o < p.bias_len) {
    v += p.bias[o];
    pre = static_cast<float>(v);
  }
  p.pre[idx] = pre;
  const float post = static_cast<float>(activate(p.act, v));
  p.post[idx] = post;
#pragma unroll
  for (int i = 0; i < kMaxPeerOut; ++i)  // static indices: the parameter stays in registers
    if (i < p.peers.n) p.peers.post[i][idx] = post;
}

template <int kDt>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x, const KParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * p.stage_bytes);
  uint64_t* tma_full = bars;
  uint64_t* a_full = bars + S;
  uint64_t* empty = bars + 2 * S;
  uint64_t* done = bars + 3 * S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile_m = blockIdx.x;        // output-row tile
  const int tile_t = blockIdx.y;        // token tile
  const int split = blockIdx.z;
  const int kb0 = split * p.kb_per_split;
  int nkb = p.nkb_total - kb0;
  if (nkb > p.kb_per_split) nkb = p.kb_per_split;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&tma_full[s], 1);
      mbar_init(&a_full[s], 128);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t tx = static_cast<uint32_t>(kBM * p.kbb + p.xsplit * p.T * 128);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, p.err, 1)) break;
        uint8_t* st = smem + s * p.stage_bytes;
        mbar_expect_tx(&tma_full[s], tx);
        const int kb = kb0 + i;
        tma_load_2d(st + p.w_off, &tm_w, kb * p.kbb, tile_m * kBM, &tma_full[s]);
        for (int q = 0; q < p.xsplit; ++q)
          tma_load_2d(st + p.b_off + q * p.T * 128, &tm_x, kb * kBK, q * p.Mp + tile_t * p.T, &tma_full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(&a_full[s], ph, p.err, 2)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        uint8_t* st = smem + s * p.stage_bytes;
        const uint64_t ad = desc_sw128(smem_u32(st + p.a_off));
        const uint64_t bd = desc_sw128(smem_u32(st + p.b_off));
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)  // 32 bytes of K per MMA: +2 in 16-byte units
          mma_f16(tmem, ad + 2 * k, bd + 2 * k, p.idesc, (i > 0 || k > 0) ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      mma_commit(done);
    }
  } else {
    // ---------------------------------------------------------------- converters
    const int r = threadIdx.x - 64;  // 0..127: A row
    for (int i = 0; i < nkb; ++i) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1;
      if (!mbar_wait(&tma_full[s], ph, p.err, 3)) break;
      uint8_t* st = smem + s * p.stage_bytes;
      const uint8_t* raw = st + p.w_off + r * p.kbb;
      uint8_t* arow = st + p.a_off + r * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 v = codes_to_f16x8<kDt>(raw, j);
        *reinterpret_cast<uint4*>(arow + ((j ^ (r & 7)) << 4)) = v;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&a_full[s]);
    }
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;              // TMEM lane quarter of this warp
    const int row = q * 32 + lane;
    const int o = tile_m * kBM + row;
    if (mbar_wait(done, 0, p.err, 4)) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      for (int tc = 0; tc < p.T; tc += 16) {
        uint32_t v[3][16];
#pragma unroll
        for (int pl = 0; pl < 3; ++pl) {
          if (pl < p.xsplit) {
            tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(pl * p.T + tc), v[pl]);
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) v[pl][e] = 0u;
          }
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int t = tile_t * p.T + tc + e;
          if (t >= p.M || o >= p.rows) continue;
          double y = static_cast<double>(__uint_as_float(v[0][e]));
          y += static_cast<double>(__uint_as_float(v[1][e]));
          y += static_cast<double>(__uint_as_float(v[2][e]));
          y *= static_cast<double>(p.scale_inv[t]);
          if (kDt == 9) y *= static_cast<double>(p.w_scale);
          if (p.splits > 1) {
            p.partial[(static_cast<int64_t>(split) * p.M + t) * p.rows + o] = y;
          } else {
            write_out(p, t, o, y);
          }
        }
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols) : "memory");
  }
}

// ---------------------------------------------------------------------------------------
// A in tensor memory (the default batched kernel).
//
// The dequantised weight tile is the MMA's A operand and lives in TMEM, not shared memory:
// each converter thread owns one weight row (one TMEM lane), reads that row's packed codes
// from the TMA-loaded raw tile, converts them in registers and writes them with tcgen05.st.
// Shared memory then carries only the packed bytes (0.5 or 1 B per weight) and the x
// planes, instead of packed bytes + the f16 tile written by the converters + the f16 tile
// read by the tensor core. The raw tile is loaded with the 32-byte (FP4) or 64-byte (8-bit)
// swizzle so that 32 threads reading 32 rows hit 32 distinct banks.
//
// x planes: the split kernel records per token how many planes are non-zero; a CTA runs
// with the largest count P over its token block (so an x that is exact in f16 after the
// per-token power of two costs one plane, and the sums equal the three-plane sums since the
// skipped planes are exactly zero). A pass covers T = min(block, 384 / P) tokens: all P x T
// accumulator columns live in TMEM at once (one or two MMAs of N <= 256 per K step), so each
// weight stage is converted once per pass and a block of up to 384 / P tokens streams its
// weights once.
//
// TMEM columns: accumulators [0, 384) at most, then the A stages (32 columns = 64 f16 per
// row each) up to column 512.
//
// Three rings decouple the pipeline: raw W tiles (deep, so that many DRAM reads are in flight;
// a slot is free again as soon as the converters have read it), x-plane tiles (freed by the
// MMA) and TMEM A stages (freed by the MMA).
//
// Warps: 0 W producer, 1 MMA issuer, 2 x producer, 3..10 converters in two groups of four (one
// warp per TMEM lane quarter in each group) taking alternate stages, then all eight run the
// epilogue.
constexpr int kTmThreads = 352;
constexpr uint32_t kTmemCols = 512;
constexpr int kTmAccMax = 384;

struct TmParams {
  const uint8_t* Wg;           // GEMM mirror: [rows/128][nkb_total][128][kbb]
  int rows, cols, M, xsplit;
  int TB;                      // tokens per CTA block (multiple of 16, <= 256)
  int tpass[3];                // tokens per pass for 1, 2, 3 planes
  int nkb_total, kb_per_split, splits;
  int kbb;                     // packed bytes per row per stage (FP4 32, 8-bit 64)
  uint32_t x_bytes, w_bytes;    // one x-ring slot (P x T x 128 B at most), one W-ring slot (wg x 128 x kbb)
  uint32_t a_col;              // first A stage column (after the accumulators)
  int nacc[3];                 // independent accumulators for 1, 2, 3 planes
  int sx, sw;                  // stages (x slot + TMEM A slot each) and W-ring slots
  int wg;                      // pipeline stages per W-ring slot (one bulk copy each; w_bytes = wg stages)
  int w_evict_first;           // 1 when no other CTA reads this CTA's weight rows
  const float* scale_inv;      // [Mp]
  const int* pcnt;             // [Mp] planes needed per token
  float w_scale;
  float* pre;
  float* post;
  int64_t ld_out;
  const double* bias;
  int bias_len;
  int act;
  double* partial;             // [splits][M][rows] when splits > 1
  int* err;
  int pair;                    // SwiGLU Gate/Up pair: rows 2i / 2i+1, epilogue writes h
  int silu_exact;              // pair: SiLU in fp64 as the reference (else fp32, a few ulp)
  float w_scale2;              // Up's Int8 scale (pair mode)
  float* h;
  int64_t ld_h;
  int tma_out;                 // last pass stores through shared memory with bulk tensor stores
  int tma_post;                // ... and post has its own map (post != pre)
  // Tail schedule (tail_first >= 0): whole tiles for items below tail_first, then each of the
  // last tiles' K range cut tail_s ways, writing fp64 partials [tail tile][split][TB][128]
  // to `partial`.
  int tiles_t, tail_first, tail_s, tail_kbps;
  int tiles, n_items;           // work items: tiles (x splits), or whole tiles then tail slices
  uint32_t acc_buf;             // columns of one accumulator buffer when there are two, else 0
  PeerOut peers;                // further destinations of post (direct stores)
  int n_peer_maps;              // staged stores: peer maps in PeerMaps (post's layout)
  // Failure-path check (WELVET_B200_TEST_WAIT_TIMEOUT=1): each CTA first waits 1 ms on a
  // barrier that nothing arrives on, before any copy, TMEM allocation or cluster exchange;
  // the wait runs out, records code 30 in the error word, and the CTA returns.
  int probe_wait;
};

// Tensor maps of the peers' post buffers (column-sharded layers): a staged chunk's post values
// are also bulk-stored through each of them, straight into the other ranks' memory.
struct PeerMaps {
  CUtensorMap m[kMaxPeerOut];
};

// Token blocks whose plane counts a CTA keeps in shared memory (more blocks: every block runs
// with xsplit planes).
constexpr int kTmMaxBlocks = 1024;

// One work item of the persistent GEMM: a tile (128 weight rows x TB tokens) or one K slice
// of it. The roles of a CTA take items blockIdx.x, + gridDim.x, ... in the same order.
struct TmItem {
  int tb, tile_m, t_begin, t_count, kb0, nkb, split, tail_idx;
  bool tail, part;
  int P, T, npass, ntot, nacc;  // filled in by the kernel from the block's plane count
  int PA, acols;                // accumulator planes and columns (pairs: planes 1 and 2 share one)
};

__device__ __forceinline__ TmItem decode_item(const TmParams& p, int q) {
  TmItem it{};
  int tile;
  if (p.tail_first >= 0 && q >= p.tail_first) {
    const int j = q - p.tail_first;
    it.tail_idx = j / p.tail_s;
    it.split = j - it.tail_idx * p.tail_s;
    tile = p.tail_first + it.tail_idx;
    it.kb0 = it.split * p.tail_kbps;
    it.nkb = min(p.tail_kbps, p.nkb_total - it.kb0);
    it.tail = true;
  } else if (p.splits > 1) {
    it.split = q / p.tiles;
    tile = q - it.split * p.tiles;
    it.kb0 = it.split * p.kb_per_split;
    it.nkb = min(p.kb_per_split, p.nkb_total - it.kb0);
  } else {
    tile = q;
    it.nkb = p.nkb_total;
  }
  it.part = it.tail || p.splits > 1;
  it.tb = tile % p.tiles_t;  // token block varies fastest: items sharing weight rows run together
  it.tile_m = tile / p.tiles_t;
  it.t_begin = it.tb * p.TB;
  it.t_count = min(p.TB, p.M - it.t_begin);
  return it;
}

// Epilogue staging of one converter group (4 warps, 128 rows): {pre, post} x 16 tokens x 128
// rows of fp32 (h: 16 x 64) for the chunk a bulk tensor store writes out; a dedicated area
// after the rings holds both groups' buffers.
constexpr uint32_t kStageBuf = 16 * 128 * 4;
constexpr uint32_t kStageGroup = 2 * kStageBuf;
constexpr uint32_t kStageArea = 2 * kStageGroup;

__device__ __forceinline__ void named_bar(uint32_t id, uint32_t n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Outputs are written once and not read again by the GEMM: evict-first in L2, so that they
// do not push out the x planes every row tile re-reads.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tm, const void* src, int x, int y, uint64_t pol) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%1, %2}], [%3], %4;"
               ::"l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(src)), "l"(pol)
               : "memory");
}

__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* tm, int x, int y, int z,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)),
        "l"(policy)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16, fp32 accumulate.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                           uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// ---- CTA-pair forms (cta_group::2): one thread of the even CTA issues an M = 256 MMA whose
// A rows 0..127 are that CTA's TMEM and rows 128..255 the odd CTA's (same TMEM address), and
// whose B columns 0..N/2-1 are the even CTA's shared memory and N/2..N-1 the odd CTA's (same
// shared-memory offset); each CTA's TMEM receives its 128 rows x N of D.

__device__ __forceinline__ void mma_f16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                                uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// The barrier at `bar`'s offset in both CTAs of the pair tracks the MMAs issued so far: one
// commit per CTA, each naming that CTA's barrier by its cluster address.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(cluster_addr(bar, 0)) : "memory");
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(cluster_addr(bar, 1)) : "memory");
}

// x box into this CTA's shared memory, its bytes counted on the even CTA's barrier `bar`
// (a cluster address). A plain (single-destination) tensor load.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* tm, int x, int y, int z, uint32_t bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
        "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
        "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// One row's 64 codes of a stage -> 32 f16x2 words (k ascending, low half = even k).
// `tile` is the stage's raw tile, row r at r * kbb with the TMA swizzle applied.
template <int kDt>
__device__ __forceinline__ void convert_row(const uint8_t* tile, int r, uint32_t (&v)[32]) {
  if constexpr (kDt == 16) {
    // 32-byte rows, SWIZZLE_32B: 16-byte chunk j sits at j ^ ((r >> 2) & 1)
    const int sw = (r >> 2) & 1;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint4 c = *reinterpret_cast<const uint4*>(tile + r * 32 + ((j ^ sw) << 4));
      const uint32_t w4[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
            "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
            "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
            "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
            "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
            "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
            : "=r"(v[j * 16 + q * 4 + 0]), "=r"(v[j * 16 + q * 4 + 1]), "=r"(v[j * 16 + q * 4 + 2]),
              "=r"(v[j * 16 + q * 4 + 3])
            : "r"(w4[q]));
      }
    }
  } else {
    // 64-byte rows, SWIZZLE_64B: 16-byte chunk j sits at j ^ ((r >> 1) & 3)
    const int sw = (r >> 1) & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 c = *reinterpret_cast<const uint4*>(tile + r * 64 + ((j ^ sw) << 4));
      const uint32_t w4[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t* o = &v[j * 8 + q * 2];
        if constexpr (kDt == 4) {
          asm("{\n\t.reg .b16 l, h;\n\t"
              "mov.b32 {l, h}, %2;\n\t"
              "cvt.rn.f16x2.e4m3x2 %0, l;\n\t"
              "cvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
              : "=r"(o[0]), "=r"(o[1])
              : "r"(w4[q]));
        } else if constexpr (kDt == 5) {
          asm("{\n\t.reg .b16 l, h;\n\t"
              "mov.b32 {l, h}, %2;\n\t"
              "cvt.rn.f16x2.e5m2x2 %0, l;\n\t"
              "cvt.rn.f16x2.e5m2x2 %1, h;\n\t}"
              : "=r"(o[0]), "=r"(o[1])
              : "r"(w4[q]));
        } else {  // Int8: f16 bits 0x6400 | (q ^ 0x80) = 1152 + q, minus 1152 -> q exactly
          const uint32_t u = w4[q] ^ 0x80808080u;
          const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
          uint32_t p0 = __byte_perm(u, 0x64646464u, 0x4140), p1 = __byte_perm(u, 0x64646464u, 0x4342);
          __half2 h0 = __hsub2(*reinterpret_cast<__half2*>(&p0), bias);
          __half2 h1 = __hsub2(*reinterpret_cast<__half2*>(&p1), bias);
          o[0] = *reinterpret_cast<uint32_t*>(&h0);
          o[1] = *reinterpret_cast<uint32_t*>(&h1);
        }
      }
    }
  }
}

// kPair: clusters of 2 CTAs (a CTA pair) share each M = 256 MMA. A work item's tile is then
// 256 weight rows; CTA v (its rank in the pair) converts rows 128 v .. 128 v + 127 into its own
// TMEM, loads half of each x stage and writes the epilogue of its rows. Only the even CTA
// issues MMAs: the odd CTA's converters, x loads and epilogue report to the even CTA's
// barriers, and the even CTA's MMA thread releases stages and accumulators in both.
template <int kDt, bool kPair>
__global__ void __launch_bounds__(kTmThreads, 1)
    k_gemm_tm(const __grid_constant__ CUtensorMap tm_x1, const __grid_constant__ CUtensorMap tm_x2,
              const __grid_constant__ CUtensorMap tm_x3, const __grid_constant__ CUtensorMap tm_o1,
              const __grid_constant__ CUtensorMap tm_o2, const __grid_constant__ PeerMaps pm, const TmParams p) {
  // A programmatic dependent of k_split_x: every thread waits for it (and, through its own
  // wait, for everything before it) before any global access other than the packed weights,
  // which no kernel of the forward writes (the W producer starts on them before its wait);
  // the reduce that follows may launch at once and waits for this grid in turn.
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.sx, Sw = p.sw;
  uint8_t* xring = smem;                                   // S x p.x_bytes
  uint8_t* wring = smem + S * p.x_bytes;                   // Sw x p.w_bytes
  uint8_t* stage_area = wring + Sw * p.w_bytes;             // kStageArea
  uint64_t* bars = reinterpret_cast<uint64_t*>(stage_area + kStageArea);
  uint64_t* w_full = bars;                 // W producer -> converters (tx)
  uint64_t* w_empty = w_full + Sw;         // converter warps (4) -> W producer
  uint64_t* s_full = w_empty + Sw;         // x producer (1 + tx) and converter warps (4) -> MMA
  uint64_t* s_free = s_full + S;           // MMA commit -> x producer and converters
  uint64_t* acc_full = s_free + S;         // MMA commit -> epilogue, per accumulator buffer
  uint64_t* acc_empty = acc_full + 2;      // epilogue warps (8) -> MMA, per accumulator buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* s_pblk = reinterpret_cast<int*>(tmem_slot + 1);  // planes needed per token block

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t v = kPair ? cluster_ctarank() : 0u;  // rank in the pair (0 issues the MMAs)

  if (p.probe_wait) {  // uniform over the grid: every thread of every CTA returns here
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (threadIdx.x == 0) {
      mbar_init(&w_full[0], 1);
      mbar_wait_for(&w_full[0], 0, p.err, 30, 1000000ull);
    }
    __syncthreads();
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < Sw; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 4 * p.wg);  // 4 converter warps per stage of the slot
    }
    // pair: s_full and acc_empty of the even CTA count both CTAs' warps
    for (int s = 0; s < S; ++s) {
      mbar_init(&s_full[s], kPair ? 9 : 5);
      mbar_init(&s_free[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kPair ? 16 : 8);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // The W producer (this thread) fills the ring's slots with the first item's first stages
  // before the wait: its tile and K range are launch parameters, and a fresh slot needs no
  // w_empty wait. Its loop below skips what was issued here.
  const int first_item = static_cast<int>(kPair ? blockIdx.x >> 1 : blockIdx.x);
  const int item_step = static_cast<int>(kPair ? gridDim.x >> 1 : gridDim.x);
  Ring w_ring;
  int w_issued = 0, w_pre = 0;
  uint64_t w_pol = 0;
  if (threadIdx.x == 0) {
    if (p.w_evict_first)
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(w_pol));
    else
      asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(w_pol));
    if (first_item < p.n_items) {
      const TmItem it = decode_item(p, first_item);
      const uint32_t sb = p.w_bytes / static_cast<uint32_t>(p.wg);
      const int mt = kPair ? 2 * it.tile_m + static_cast<int>(v) : it.tile_m;
      const uint8_t* wfirst = p.Wg + (static_cast<int64_t>(mt) * p.nkb_total + it.kb0) * sb;
      for (int i = 0; i < it.nkb && w_pre < Sw; i += p.wg) {
        const uint32_t n = static_cast<uint32_t>(it.nkb - i < p.wg ? it.nkb - i : p.wg);
        mbar_expect_tx(&w_full[w_ring.slot], n * sb);
        bulk_load_hint(wring + w_ring.slot * p.w_bytes, wfirst + static_cast<int64_t>(i) * sb, n * sb,
                       &w_full[w_ring.slot], w_pol);
        ++w_issued;
        ++w_pre;
        w_ring.step(Sw);
      }
    }
  }
  const bool pblk_ok = p.tiles_t <= kTmMaxBlocks;
  if (pblk_ok)
    for (int b = threadIdx.x; b < p.tiles_t; b += kTmThreads) s_pblk[b] = 1;
  if (warp == 0) {
    if constexpr (kPair) {  // both CTAs' warp 0 together: the same columns in each CTA's TMEM
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if constexpr (kPair) cluster_sync_all();  // the barriers are initialised before the other CTA arrives
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // k_split_x's planes, scales and plane counts
  if (pblk_ok)
    for (int t = threadIdx.x; t < p.M; t += kTmThreads) {
      const int n = p.pcnt[t];
      if (n > 1) atomicMax(&s_pblk[t / p.TB], n);
    }
  __syncthreads();
  const uint32_t tmem = *tmem_slot;
  // items go to CTA pairs (clusters) in pair mode (first_item, item_step above)
  // the work item q as this CTA's roles see it: tile, K range, token range, planes
  auto item = [&](int q) {
    TmItem it = decode_item(p, q);
    it.P = pblk_ok ? min(s_pblk[it.tb], p.xsplit) : p.xsplit;
    it.T = p.tpass[it.P - 1];
    it.npass = (it.t_count + it.T - 1) / it.T;
    it.ntot = it.P * it.T;
    // pairs: plane 2 (2^-22 of x and below) accumulates onto plane 1's columns, whose fp32
    // rounding is then ~2^-35 of |Wx|; plane 0 keeps its own accumulator
    it.PA = kPair && it.P == 3 ? 2 : it.P;
    it.acols = it.PA * it.T;
    it.nacc = p.nacc[it.P - 1];
    return it;
  };
  const bool plain_act = p.bias == nullptr && (p.act == -1 || p.act == 0 || p.act == 6);

  // Loops keep their ring slots and phase bits as running state (Ring), across the passes and
  // the work items of this CTA: no divisions on the single-thread critical paths.
  if (warp == 0) {
    // ------------------------------------------------------------------ W producer
    if (lane == 0) {
      const uint64_t pol = w_pol;
      const uint32_t wb = p.w_bytes;                                // one slot: wg stages
      const uint32_t sb = wb / static_cast<uint32_t>(p.wg);         // one stage
      Ring w = w_ring;
      int issued = w_issued;
      bool ok = true;
      for (int qi = first_item; qi < p.n_items && ok; qi += item_step) {
        const TmItem it = item(qi);
        const int mt = kPair ? 2 * it.tile_m + static_cast<int>(v) : it.tile_m;  // 128-row mirror tile
        const uint8_t* wfirst = p.Wg + (static_cast<int64_t>(mt) * p.nkb_total + it.kb0) * sb;
        for (int pass = 0; pass < it.npass && ok; ++pass)
          for (int i = 0; i < it.nkb; i += p.wg) {  // the stages of a tile are contiguous: one copy per slot
            if (qi == first_item && pass == 0 && i < w_pre * p.wg) continue;  // issued before the wait
            const uint32_t n = static_cast<uint32_t>(it.nkb - i < p.wg ? it.nkb - i : p.wg);
            if (!mbar_wait(&w_empty[w.slot], w.phase ^ 1u, p.err, 11)) { ok = false; break; }
            mbar_expect_tx(&w_full[w.slot], n * sb);
            bulk_load_hint(wring + w.slot * wb, wfirst + static_cast<int64_t>(i) * sb, n * sb, &w_full[w.slot], pol);
            ++issued;
            w.step(Sw);
          }
      }
      // tail: the converters released every slot this thread filled before the CTA exits
      Ring t;
      for (int k = 0; k < issued; ++k) {
        if (k >= issued - Sw) mbar_wait(&w_empty[t.slot], t.phase, p.err, 12);
        t.step(Sw);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ x producer
    if (lane == 0) {
      uint64_t pol;
      asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
      Ring r;
      int issued = 0;
      bool ok = true;
      for (int qi = first_item; qi < p.n_items && ok; qi += item_step) {
        const TmItem it = item(qi);
        const CUtensorMap* tmx = it.P == 1 ? &tm_x1 : (it.P == 2 ? &tm_x2 : &tm_x3);
        const uint32_t tx = static_cast<uint32_t>(it.ntot * 128);
        for (int pass = 0; pass < it.npass && ok; ++pass) {
          const int t0 = it.t_begin + pass * it.T;
          for (int i = 0; i < it.nkb && ok; ++i) {
            if constexpr (kPair) {
              // this CTA's half of each MMA's x rows, in boxes of T/2 tokens (box b: plane b / 2,
              // tokens from (b % 2) T/2): with 1 or 2 planes boxes vP .. vP + P - 1 in one slot
              // (one MMA over the [P][T] rows); with 3, boxes 2v and 2v + 1 (the first MMA, planes
              // 0 and 1) in one slot and box 4 + v (half of plane 2, the second MMA) in the next.
              // The even CTA's barrier of each slot counts the bytes of both halves.
              const int half = it.T >> 1;
              const int p01 = it.P < 2 ? it.P : 2;
              for (int u = 0; u < (it.P == 3 ? 2 : 1); ++u) {
                if (!mbar_wait(&s_free[r.slot], r.phase ^ 1u, p.err, 18)) { ok = false; break; }
                uint8_t* dst = xring + r.slot * p.x_bytes;
                const int nb = u == 0 ? p01 : 1;
                if (v == 0) mbar_expect_tx(&s_full[r.slot], static_cast<uint32_t>(nb * it.T * 128));
                const uint32_t bar = cluster_addr(&s_full[r.slot], 0);
                for (int j = 0; j < nb; ++j) {
                  const int b = u == 0 ? static_cast<int>(v) * p01 + j : 4 + static_cast<int>(v);
                  tma_load_3d_pair(dst + j * half * 128, tmx, (it.kb0 + i) * kBK, t0 + (b & 1) * half, b >> 1, bar,
                                   pol);
                }
                ++issued;
                r.step(S);
              }
            } else {
              if (!mbar_wait(&s_free[r.slot], r.phase ^ 1u, p.err, 18)) { ok = false; break; }
              uint8_t* dst = xring + r.slot * p.x_bytes;
              mbar_expect_tx(&s_full[r.slot], tx);
              // every plane of the stage in one box ([P][T][128 B], plane pl at pl * T * 128)
              tma_load_3d_hint(dst, tmx, (it.kb0 + i) * kBK, t0, 0, &s_full[r.slot], pol);
              ++issued;
              r.step(S);
            }
          }
        }
      }
      // tail: the MMA consumed every stage this thread filled before the CTA exits
      Ring t;
      for (int k = 0; k < issued; ++k) {
        if (k >= issued - S) mbar_wait(&s_free[t.slot], t.phase, p.err, 19);
        t.step(S);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && v == 0) {
      constexpr uint32_t kM = kPair ? 256 : 128;
      const uint64_t bd_base = desc_sw128(smem_u32(xring));
      const uint64_t bd_step = static_cast<uint64_t>(p.x_bytes >> 4);   // one x slot, in 16-byte units
      Ring r;
      Ring last;
      bool any = false;
      bool ok = true;
      uint32_t fills = 0;  // accumulator fills so far (one per pass of every item)
      uint32_t dbase = 0;  // first TMEM column of the current fill's accumulator buffer
      for (int qi = first_item; qi < p.n_items && ok; qi += item_step) {
        const TmItem it = item(qi);
        // first MMA's N; the second covers [n0, ntot) (pairs: planes 0 and 1, then plane 2)
        const int n0 = kPair ? (it.P < 2 ? it.P : 2) * it.T : (it.ntot < 256 ? it.ntot : 256);
        const uint32_t idesc0 = (1u << 4) | (static_cast<uint32_t>(n0 >> 3) << 17) | ((kM >> 4) << 24);
        const uint32_t idesc1 = (1u << 4) | (static_cast<uint32_t>((it.ntot - n0) >> 3) << 17) | ((kM >> 4) << 24);
        const uint64_t bd_n0 = static_cast<uint64_t>((n0 * 128) >> 4);  // rows [n0, ntot) of a slot
        // One pass's k stages. kTwo: a second MMA per k step (single CTA: N above 256; pairs: 3
        // planes, plane 2 from the next slot onto plane 1's accumulator). Compiled once per
        // case: a run-time branch inside this issue loop cost ~40 % of the GEMM's time.
        auto stages = [&](auto two_c) -> bool {
          constexpr bool kTwo = decltype(two_c)::value;
          int j = 0;      // accumulator of the next k step (round robin over nacc)
          int first = 0;  // k steps issued this pass (each accumulator starts fresh on its first)
          for (int i = 0; i < it.nkb; ++i) {
            if (!mbar_wait(&s_full[r.slot], r.phase, p.err, 14)) return false;
            Ring r2 = r;
            if constexpr (kPair && kTwo) {
              r2.step(S);
              if (!mbar_wait(&s_full[r2.slot], r2.phase, p.err, 14)) return false;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint64_t bd = bd_base + bd_step * static_cast<uint64_t>(r.slot);
            [[maybe_unused]] const uint64_t bd2 = bd_base + bd_step * static_cast<uint64_t>(r2.slot);
            const uint32_t a = tmem + p.a_col + 32u * static_cast<uint32_t>(r.slot);
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {  // 16 k per MMA: 8 TMEM columns of A, 32 bytes of B
              const uint32_t d = tmem + dbase + static_cast<uint32_t>(j * it.acols);
              const uint32_t acc = first >= it.nacc ? 1u : 0u;
              if constexpr (kPair) {
                mma_f16_ts_pair(d, a + 8u * k, bd + 2 * k, idesc0, acc);
                if constexpr (kTwo)
                  mma_f16_ts_pair(d + static_cast<uint32_t>(it.T), a + 8u * k, bd2 + 2 * k, idesc1, 1u);
              } else {
                mma_f16_ts(d, a + 8u * k, bd + 2 * k, idesc0, acc);
                if constexpr (kTwo)
                  mma_f16_ts(d + static_cast<uint32_t>(n0), a + 8u * k, bd + bd_n0 + 2 * k, idesc1, acc);
              }
              if (++j == it.nacc) j = 0;
              ++first;
            }
            if constexpr (kPair) {
              mma_commit_pair(&s_free[r.slot]);
              if constexpr (kTwo) mma_commit_pair(&s_free[r2.slot]);
            } else {
              mma_commit(&s_free[r.slot]);
            }
            last = r2;
            any = true;
            r = r2;
            r.step(S);
          }
          return true;
        };
        const bool two = kPair ? it.P == 3 : it.ntot > n0;
        for (int pass = 0; pass < it.npass && ok; ++pass) {
          // accumulator buffer of this fill (two alternate when p.acc_buf > 0) and its use count
          const uint32_t b = p.acc_buf ? (fills & 1u) : 0u;
          const uint32_t use = p.acc_buf ? (fills >> 1) : fills;
          dbase = b * p.acc_buf;
          if (use > 0) {  // the epilogue has read this buffer's previous fill
            if (!mbar_wait(&acc_empty[b], (use - 1) & 1u, p.err, 13)) { ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          }
          if (!(two ? stages(std::true_type{}) : stages(std::false_type{}))) ok = false;
          if (ok) {
            if constexpr (kPair) mma_commit_pair(&acc_full[b]);
            else mma_commit(&acc_full[b]);
          }
          ++fills;
        }
      }
      // drain: the last MMAs issued have completed before TMEM can be released
      if (any) mbar_wait(&s_free[last.slot], last.phase, p.err, 15);
    }
  } else if (warp >= 3) {
    // ------------------------------------------------------------------ converters, then epilogue
    const int cw = warp - 3;             // 0..7
    const int grp = cw >> 2;             // converter group: takes the stages with index % 2 == grp
    const int q = warp & 3;              // TMEM lane quarter of this warp
    const int r = q * 32 + lane;         // weight row within the tile = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    Ring w, st;
    int stage_idx = 0;
    uint32_t fills = 0;
    bool ok = true;
    for (int qi = first_item; qi < p.n_items && ok; qi += item_step) {
      const TmItem it = item(qi);
      const int tile_m = it.tile_m, t_begin = it.t_begin, t_count = it.t_count, T = it.T, P = it.P;
      const int nacc = it.nacc, acols = it.acols, PA = it.PA, npass = it.npass, split = it.split,
                tail_idx = it.tail_idx;
      const bool tail = it.tail, part = it.part;
      const int mt = kPair ? 2 * tile_m + static_cast<int>(v) : tile_m;  // 128-row tile of this CTA
      const int o = mt * 128 + r;
      // Epilogue sums that are single fp32 values (one plane, one accumulator, no Int8 scale,
      // no partials) are scaled in fp32; others are summed and scaled in fp64.
      const bool f32_sums = P == 1 && nacc == 1 && kDt != 9 && !part;
      // Tail slices whose sums are single fp32 values keep them raw in fp32 (half the bytes of
      // the fp64 partials, in the first half of the tile's region); k_tail_reduce applies the
      // scales, as the fp64 path does here, and reads which form a tile has from its flag.
      const int tail_k = kPair ? 2 * tail_idx + static_cast<int>(v) : tail_idx;  // 128-row tail part
      const bool raw32 = tail && PA == 1 && nacc == 1;
      if (tail && q == 0 && lane == 0 && grp == 0) {
        int* flags = reinterpret_cast<int*>(p.partial + static_cast<int64_t>(p.tiles - p.tail_first) *
                                                            (kPair ? 2 : 1) * p.tail_s * p.TB * 128);
        flags[tail_k] = raw32 ? 1 : 0;
      }
      const bool two = kPair && P == 3;  // pairs, 3 planes: a stage takes two ring slots
      const uint32_t sb = p.w_bytes / static_cast<uint32_t>(p.wg);  // one stage of a W slot
      for (int pass = 0; pass < npass && ok; ++pass) {
        // The W slot of stage i holds stages [w_base, w_base + wn): the W producer's copies
        // restart at the pass's first stage; every stage frees its slot once (4 warps), the
        // last stage of a short slot for the stages it does not hold as well.
        int w_base = 0;
        auto w_count = [&]() { return it.nkb - w_base < p.wg ? it.nkb - w_base : p.wg; };
        auto adv_w = [&](int i) {
          if (i + 1 - w_base == w_count()) {
            w_base = i + 1;
            w.step(Sw);
          }
        };
        for (int i = 0; i < it.nkb; adv_w(i), ++i, ++stage_idx) {
          const Ring s1 = st;  // the stage's slot (its TMEM A slot)
          Ring s2 = st;        // the slot of plane 2's x (3-plane pair stages)
          if (two) s2.step(S);
          st = s2;
          st.step(S);
          if ((stage_idx & 1) != grp) continue;
          if (!warp_wait(&w_full[w.slot], w.phase, p.err, 16)) { ok = false; break; }
          uint32_t v[32];
          const int sub = i - w_base;
          convert_row<kDt>(wring + w.slot * p.w_bytes + static_cast<uint32_t>(sub) * sb, r, v);
          __syncwarp();
          if (lane == 0) {
            const int wn = w_count();
            const int arrivals = sub == wn - 1 ? 1 + p.wg - wn : 1;
            for (int a = 0; a < arrivals; ++a) mbar_arrive(&w_empty[w.slot]);
          }
          if (!warp_wait(&s_free[s1.slot], s1.phase ^ 1u, p.err, 21)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          tmem_st32(tmem + lane_base + p.a_col + 32u * static_cast<uint32_t>(s1.slot), v);
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            if constexpr (kPair) mbar_arrive_cluster(cluster_addr(&s_full[s1.slot], 0));
            else mbar_arrive(&s_full[s1.slot]);
          }
          if (two) {  // the second slot's barrier counts these warps too; its previous use is over first
            if (!warp_wait(&s_free[s2.slot], s2.phase ^ 1u, p.err, 22)) { ok = false; break; }
            if (lane == 0) mbar_arrive_cluster(cluster_addr(&s_full[s2.slot], 0));
          }
        }
        if (!ok) break;
        // ------------------------------------------------------------ epilogue of this pass
        const uint32_t b = p.acc_buf ? (fills & 1u) : 0u;
        const uint32_t use = p.acc_buf ? (fills >> 1) : fills;
        if (!warp_wait(&acc_full[b], use & 1u, p.err, 17)) { ok = false; break; }
        ++fills;
        const uint32_t acc_base = tmem + lane_base + b * p.acc_buf;  // this fill's buffer, this warp's lanes
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int t_pass = t_begin + pass * T;
        // Outputs go through the group's staging buffer to bulk tensor stores: the epilogue
        // only reads TMEM and fills shared memory, the accumulator is released at once and the
        // writes drain while the next item's MMAs run.
        const bool staged = p.tma_out && !part;
        float* stage = reinterpret_cast<float*>(stage_area + grp * kStageGroup);
        const bool issuer = q == 0 && lane == 0;  // one thread of the group issues its stores
        int chunk = 0;
        for (int tc = grp * 16; tc < T; tc += 32, ++chunk) {
          // Chunks are 16-token aligned within the block: one that starts past the block's
          // tokens holds none of them (and may hold the next block's, which a staged store must
          // not overwrite). Uniform over the group, so its barriers stay matched.
          if (t_pass + tc >= t_begin + t_count) break;
          float* s1 = stage;
          float* s2 = stage + kStageBuf / 4;
          // phase 1 (unrolled, cheap): each sum scaled, then kept as the float the reference
          // rounds it to (pre = float(y); Gate and Up are floats before the product)
          float pf[16], uf[16];
          // The chunk's 16 per-token scales, requested before the TMEM reads so that the two
          // latencies overlap (after a tcgen05.wait the loads could not move up; inside the
          // fp64 loop each would wait behind the partial stores). scale_inv holds Mp (a
          // multiple of 16) entries.
          float scv[16];
          {
            const float4* sc4 = reinterpret_cast<const float4*>(p.scale_inv + t_pass + tc);
#pragma unroll
            for (int e4 = 0; e4 < 4; ++e4) {
              // ordered, coherent loads: k_split_x (this grid's programmatic predecessor)
              // wrote the scales
              const float4 sc = ld_dep4(reinterpret_cast<const float*>(sc4 + e4));
              scv[4 * e4] = sc.x;
              scv[4 * e4 + 1] = sc.y;
              scv[4 * e4 + 2] = sc.z;
              scv[4 * e4 + 3] = sc.w;
            }
          }
          if (f32_sums) {
            // one plane, one accumulator: the sum is one fp32 value and the scale a power of two,
            // so the fp32 product is the rounding of the exact (fp64) product
            uint32_t v[16];
            tmem_ld16(acc_base + static_cast<uint32_t>(tc), v);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const bool valid = t_pass + tc + e < t_begin + t_count && o < p.rows;
              pf[e] = valid ? __uint_as_float(v[e]) * scv[e] : 0.0f;
            }
          } else {
            double y[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) y[e] = 0.0;
            // the PA x nacc accumulator reads (plane-major, as the sums are ordered), two in
            // flight per wait: each wait costs a TMEM round trip, and small token blocks have up
            // to 8 reads per chunk (four in flight spilled registers)
            const int nld = PA * nacc;
            // rolled: one copy of the read-and-add code serves every pair of reads (the
            // epilogue runs once per item, so its instructions are fetched cold)
#pragma unroll 1
            for (int g0 = 0; g0 < nld; g0 += 2) {
              uint32_t va[16], vb[16];
              tmem_ld16(acc_base + static_cast<uint32_t>((g0 % nacc) * acols + (g0 / nacc) * T + tc), va);
              const bool two_ld = g0 + 1 < nld;
              if (two_ld)
                tmem_ld16(acc_base + static_cast<uint32_t>(((g0 + 1) % nacc) * acols + ((g0 + 1) / nacc) * T + tc),
                          vb);
              asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
              for (int e = 0; e < 16; ++e) y[e] += static_cast<double>(__uint_as_float(va[e]));
              if (two_ld) {
#pragma unroll
                for (int e = 0; e < 16; ++e) y[e] += static_cast<double>(__uint_as_float(vb[e]));
              }
            }
            // this chunk's valid tokens (0 for rows past the layer) and where its partials go:
            // element e at dst[e * dstride] (fp64) or dst32[e * dstride] (raw fp32 tail sums)
            const int nvalid = o < p.rows ? min(16, t_begin + t_count - (t_pass + tc)) : 0;
            double* dst = nullptr;
            float* dst32 = nullptr;
            int64_t dstride = 0;
            if (tail) {
              const int64_t base = static_cast<int64_t>(tail_k) * p.tail_s * p.TB * 128;
              const int64_t at = (static_cast<int64_t>(split) * p.TB + (t_pass + tc - t_begin)) * 128 + r;
              if (raw32) dst32 = reinterpret_cast<float*>(p.partial) + 2 * base + at;
              else dst = p.partial + base + at;
              dstride = 128;
            } else if (p.splits > 1) {
              dst = p.partial + (static_cast<int64_t>(split) * p.M + t_pass + tc) * p.rows + o;
              dstride = p.rows;
            }
            const double wsc =
                kDt == 9 ? static_cast<double>((p.pair && (o & 1)) ? p.w_scale2 : p.w_scale) : 1.0;
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const bool valid = e < nvalid;
              double yy = y[e] * static_cast<double>(scv[e]);
              if (kDt == 9) yy *= wsc;
              if (!valid) yy = 0.0;
              if (valid && dst) dst[e * dstride] = yy;
              if (valid && dst32) dst32[e * dstride] = static_cast<float>(y[e]);
              pf[e] = static_cast<float>(yy);
            }
          }
          if (p.pair) {
            // Up row o + 1 sits in the next lane (rows of a 128-row tile are lanes)
#pragma unroll
            for (int e = 0; e < 16; ++e) uf[e] = __shfl_xor_sync(0xffffffffu, pf[e], 1);
          }
          if (part) continue;
          if (staged) {
            // the buffer's previous store (this item's last chunk or an earlier item's) has read it
            if (issuer) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            named_bar(1 + grp, 128);
          }
          // phase 2: the outputs. pf / uf are only indexed by constants here (kept in registers);
          // the general bias / activation epilogue runs on a copy one output per iteration so
          // that its fp64 code appears once.
          if (p.pair) {
            // both lanes of a Gate/Up pair work: the Gate lane takes tokens 0..7 of the chunk,
            // the Up lane 8..15 (each lane holds its row's value and, in uf, its partner's)
            const bool up_lane = (o & 1) != 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int e = (up_lane ? 8 : 0) + k;
              const int t = t_pass + tc + e;
              const bool valid = t < t_begin + t_count && o < p.rows;
              const float gv = up_lane ? uf[8 + k] : pf[k];
              const float uv = up_lane ? pf[8 + k] : uf[k];
              const float h = p.silu_exact ? pair_value_inline(gv, uv) : pair_value_f32(gv, uv);
              if (staged) s1[e * 64 + (r >> 1)] = h;
              else if (valid) p.h[static_cast<int64_t>(t) * p.ld_h + (o >> 1)] = h;
            }
          } else if (plain_act) {
            // Linear / ReLU / ReLU2 without bias: the float results of the fp64 reference
            // expressions (x < 0 ? 0 : x; x * x of a float is exact in fp64)
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float a = pf[e];
              const float b = p.act == -1 ? a : (a < 0.0f ? 0.0f : (p.act == 0 ? a : a * a));
              if (staged) {
                s1[e * 128 + r] = a;
                if (p.tma_post) s2[e * 128 + r] = b;
              } else if (t_pass + tc + e < t_begin + t_count && o < p.rows) {
                const int64_t idx = static_cast<int64_t>(t_pass + tc + e) * p.ld_out + o;
                p.pre[idx] = a;
                p.post[idx] = b;
#pragma unroll
                for (int i = 0; i < kMaxPeerOut; ++i)  // static indices: the parameter stays in registers
                  if (i < p.peers.n) p.peers.post[i][idx] = b;
              }
            }
          } else {
            float pg[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) pg[e] = pf[e];
#pragma unroll 1
            for (int e = 0; e < 16; ++e) {
              const int t = t_pass + tc + e;
              const bool valid = t < t_begin + t_count && o < p.rows;
              float a = 0.0f, b = 0.0f;
              if (valid) out_values(p, o, pg[e], a, b);
              if (staged) {
                s1[e * 128 + r] = a;
                s2[e * 128 + r] = b;
              } else if (valid) {
                const int64_t idx = static_cast<int64_t>(t) * p.ld_out + o;
                p.pre[idx] = a;
                p.post[idx] = b;
#pragma unroll
                for (int i = 0; i < kMaxPeerOut; ++i)  // static indices: the parameter stays in registers
                  if (i < p.peers.n) p.peers.post[i][idx] = b;
              }
            }
          }
          if (staged) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            named_bar(1 + grp, 128);
            if (issuer) {
              const int ty = t_pass + tc;
              uint64_t pol;
              asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
              if (p.pair) {
                tma_store_2d(&tm_o1, s1, mt * 64, ty, pol);
              } else {
                tma_store_2d(&tm_o1, s1, mt * 128, ty, pol);
                if (p.tma_post) tma_store_2d(&tm_o2, s2, mt * 128, ty, pol);
                // column-sharded layers: the same post values into every other rank's buffer
                for (int i = 0; i < p.n_peer_maps; ++i) tma_store_2d(&pm.m[i], p.tma_post ? s2 : s1, mt * 128, ty, pol);
              }
              asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            }
          }
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          if constexpr (kPair) mbar_arrive_cluster(cluster_addr(&acc_empty[b], 0));
          else mbar_arrive(&acc_empty[b]);
        }
      }
    }
    // the staging buffers stay valid until the last stores have read them; stores into other
    // ranks' memory are waited for in full, so that they are complete when the grid is
    if (q == 0 && lane == 0) {
      if (p.n_peer_maps > 0) {
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        asm volatile("fence.proxy.async.global;" ::: "memory");
      } else {
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  // pair: neither CTA frees its TMEM or exits while the other may still signal its barriers
  if constexpr (kPair) cluster_sync_all();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if constexpr (kPair)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Sum of the split-K partials in a fixed order, then the reference epilogue.
__global__ void k_splitk_reduce(const KParams p) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the GEMM's partials
  const int64_t n = static_cast<int64_t>(p.M) * p.rows;
  if (p.pair) {  // one thread per (token, Gate/Up pair)
    const int half = p.rows / 2;
    const int64_t np = static_cast<int64_t>(p.M) * half;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < np;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int t = static_cast<int>(i / half), j = static_cast<int>(i % half);
      const int64_t base = static_cast<int64_t>(t) * p.rows + 2 * j;
      double yg = 0.0, yu = 0.0;
      for (int s = 0; s < p.splits; ++s) {
        yg += p.partial[s * n + base];
        yu += p.partial[s * n + base + 1];
      }
      write_pair(p, t, j, yg, yu);
    }
    return;
  }
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    double y = 0.0;
    for (int s = 0; s < p.splits; ++s) y += p.partial[s * n + i];
    write_out(p, static_cast<int>(i / p.rows), static_cast<int>(i % p.rows), y);
  }
}

// Sum of the tail tiles' K-slice partials ([tail tile][split][TB][128] fp64) in split order,
// then the epilogue of write_out / write_pair. One thread per (tail tile, token, row) -- per
// Gate/Up pair in pair mode.
struct TailParams {
  int rows, M, TB, tiles_t, tail_first, tail_s, ntail;
  int sub;                     // 128-row parts per tile: 2 for CTA-pair tiles, else 1
  const float* scale_inv;      // per-token 2^-e (parts kept raw in fp32)
  int int8;                    // Int8 weights: w_scale (Up rows of a pair: w_scale2) as well
  float w_scale, w_scale2;
  const double* partial;
  float* pre;
  float* post;
  int64_t ld_out;
  const double* bias;
  int bias_len;
  int act;
  int pair;
  float* h;
  int64_t ld_h;
  PeerOut peers;
};

__global__ void k_tail_reduce(const TailParams p) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the GEMM's partials
  const int per_tile = p.TB * (p.pair ? 64 : 128);
  const int64_t n = static_cast<int64_t>(p.ntail) * p.sub * per_tile;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(i / per_tile);  // 128-row part: tail tile k / sub, part k % sub
    const int rem = static_cast<int>(i - static_cast<int64_t>(k) * per_tile);
    const int tile = p.tail_first + k / p.sub;
    const int t = (tile % p.tiles_t) * p.TB + rem / (p.pair ? 64 : 128);
    const int r = p.pair ? 2 * (rem % 64) : rem % 128;
    const int o = ((tile / p.tiles_t) * p.sub + k % p.sub) * 128 + r;
    if (t >= p.M || o >= p.rows) continue;
    const int64_t region = static_cast<int64_t>(k) * p.tail_s * p.TB * 128;  // this part's partials
    const int64_t at = static_cast<int64_t>(t % p.TB) * 128 + r;
    const int64_t stride = static_cast<int64_t>(p.TB) * 128;
    const int* flags = reinterpret_cast<const int*>(p.partial + static_cast<int64_t>(p.ntail) * p.sub * p.tail_s * stride);
    double y = 0.0, y2 = 0.0;
    if (flags[k]) {  // raw fp32 sums: scaled here as the GEMM's fp64 path scales them
      const float* base = reinterpret_cast<const float*>(p.partial) + 2 * region + at;
      const double sc = static_cast<double>(p.scale_inv[t]);
      for (int sp = 0; sp < p.tail_s; ++sp) {
        double a = static_cast<double>(base[sp * stride]) * sc;
        if (p.int8) a *= static_cast<double>((p.pair && (o & 1)) ? p.w_scale2 : p.w_scale);
        y += a;
        if (p.pair) {
          double b = static_cast<double>(base[sp * stride + 1]) * sc;
          if (p.int8) b *= static_cast<double>(p.w_scale2);
          y2 += b;
        }
      }
    } else {
      const double* base = p.partial + region + at;
      for (int sp = 0; sp < p.tail_s; ++sp) {
        y += base[sp * stride];
        if (p.pair) y2 += base[sp * stride + 1];
      }
    }
    if (p.pair) write_pair(p, t, o >> 1, y, y2);
    else write_out(p, t, o, y);
  }
}

// x [M][x_ld] f32 -> planes [xsplit][Mp][Kp] f16 (x * 2^e = p0 + p1 + p2) and 2^-e per token;
// pcnt[t] (when given) = planes that hold a non-zero value for token t, at most xsplit.
// One 512-thread block per token row (grid = Mp); rows >= M and columns >= K are zero. A row
// whose start is 16-byte aligned is read in 16-byte vectors, every load of a thread in flight
// at once (Kp is a multiple of 64). With nrm.gamma set, x is an RMSNorm layer's input: the
// kernel is that layer (its pre / post, [M][K], are written here) and splits post.
constexpr int kSplitThreads = 512;
static_assert(kSplitThreads == kNormThreads, "the RMSNorm prologue sums squares in k_rmsnorm's order");

// One element's planes: x * s = h0 + h1 + h2 (h0 alone for a non-finite x).
__device__ __forceinline__ void split3(float v, float s, __half& h0, __half& h1, __half& h2) {
  h1 = __float2half_rn(0.0f);
  h2 = __float2half_rn(0.0f);
  if (isfinite(v)) {
    const float vs = v * s;
    h0 = __float2half_rn(vs);
    const float r1 = vs - __half2float(h0);
    h1 = __float2half_rn(r1);
    const float r2 = r1 - __half2float(h1);
    h2 = __float2half_rn(r2);
  } else {
    h0 = __float2half_rn(v);
  }
}

__global__ void __launch_bounds__(kSplitThreads)
    k_split_x(const float* x, int64_t x_ld, int M, int K, int Mp, int Kp, int xsplit,
              __half* __restrict__ planes, float* __restrict__ scale_inv, int* __restrict__ pcnt,
              SplitNorm nrm) {
  // x may be the previous kernel's output: ordered loads after the wait (ld_dep), never
  // non-coherent ones, which may be hoisted above it
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float s_max[kSplitThreads / 32];
  __shared__ double s_part[kSplitThreads / 32];
  __shared__ int s_nz;
  const int t = blockIdx.x;
  if (t >= Mp) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* xr = x + static_cast<int64_t>(t) * x_ld;
  const bool live = t < M;
  const bool vec = (reinterpret_cast<uintptr_t>(xr) & 15) == 0;
  // x[t][k..k+3], zeros past K (16-byte loads when the row start is aligned)
  auto load4 = [&](int k) -> float4 {
    if (vec && k + 3 < K) return ld_dep4(xr + k);
    float4 v;
    v.x = k < K ? ld_dep(xr + k) : 0.0f;
    v.y = k + 1 < K ? ld_dep(xr + k + 1) : 0.0f;
    v.z = k + 2 < K ? ld_dep(xr + k + 2) : 0.0f;
    v.w = k + 3 < K ? ld_dep(xr + k + 3) : 0.0f;
    return v;
  };
  const bool norm = nrm.gamma != nullptr;
  double inv = 0.0;
  if (norm) inv = rms_inv(rms_block_ss(load4, live ? K : 0, s_part), K, nrm.eps);
  // The values this row splits, k..k+3: x, or its RMSNorm post (rms_apply4, as k_rmsnorm),
  // whose pre / post the first pass also stores.
  float* npre = norm ? nrm.pre + static_cast<int64_t>(t) * K : nullptr;
  float* npost = norm ? nrm.post + static_cast<int64_t>(t) * K : nullptr;
  const bool vec_out = norm && ((reinterpret_cast<uintptr_t>(npre) | reinterpret_cast<uintptr_t>(npost)) & 15) == 0;
  auto value4 = [&](int k, bool store) -> float4 {
    const float4 v = load4(k);
    return norm ? rms_apply4(v, k, K, inv, nrm.gamma, npre, npost, store, vec_out) : v;
  };
  float amax = 0.0f;
  if (live) {
#pragma unroll 4
    for (int k = 4 * tid; k < K; k += 4 * kSplitThreads) {
      const float4 v = value4(k, true);
      for (float a : {fabsf(v.x), fabsf(v.y), fabsf(v.z), fabsf(v.w)})
        if (a > amax && a <= 3.402823466e+38f) amax = a;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  if (lane == 0) s_max[warp] = amax;
  if (tid == 0) s_nz = 0;
  __syncthreads();
  amax = s_max[0];
#pragma unroll
  for (int w = 1; w < kSplitThreads / 32; ++w) amax = fmaxf(amax, s_max[w]);
  int e = 0;
  if (amax > 0.0f) {
    e = 13 - ilogbf(amax);  // amax * 2^e in [2^13, 2^14)
    if (e > 126) e = 126;
    if (e < -126) e = -126;
  }
  const float s = ldexpf(1.0f, e);
  if (tid == 0) scale_inv[t] = ldexpf(1.0f, -e);
  const int64_t plane = static_cast<int64_t>(Mp) * Kp;
  __half* p0 = planes + static_cast<int64_t>(t) * Kp;
  bool nz1 = false, nz2 = false;
  // four elements per thread and step; Kp is a multiple of 64, so a step is all inside
#pragma unroll 2
  for (int k = 4 * tid; k < Kp; k += 4 * kSplitThreads) {
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (live && k < K) {
      const float4 q = value4(k, false);
      v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
    }
    __half h0[4], h1[4], h2[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      split3(v[j], s, h0[j], h1[j], h2[j]);
      nz1 |= (__half_as_ushort(h1[j]) & 0x7fff) != 0;
      nz2 |= (__half_as_ushort(h2[j]) & 0x7fff) != 0;
    }
    // 8-byte stores: the plane rows start 8-byte aligned (Kp is a multiple of 64)
    *reinterpret_cast<uint2*>(p0 + k) = *reinterpret_cast<const uint2*>(h0);
    if (xsplit > 1) *reinterpret_cast<uint2*>(p0 + plane + k) = *reinterpret_cast<const uint2*>(h1);
    if (xsplit > 2) *reinterpret_cast<uint2*>(p0 + 2 * plane + k) = *reinterpret_cast<const uint2*>(h2);
  }
  if (pcnt) {
    const int f = (nz1 ? 1 : 0) | (nz2 ? 2 : 0);
    if (f) atomicOr(&s_nz, f);
    __syncthreads();
    if (tid == 0) {
      int n = (s_nz & 2) ? 3 : ((s_nz & 1) ? 2 : 1);
      if (n > xsplit) n = xsplit;
      pcnt[t] = n;
    }
  }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

Status make_map_2d(CUtensorMap* tm, CUtensorMapDataType dt, void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  auto enc = tensor_map_encoder();
  if (!enc) return Status::Internal("cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return Status::Internal("cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
  return Status::Ok();
}

// [planes][Mp][Kp] f16 planes of x: box {64 k, T tokens, 1 plane}, SWIZZLE_128B; tokens past
// Mp read as zero.
// x planes [planes][Mp][Kp] f16; a box is 64 k x T tokens x box_planes planes (one request
// brings every plane of a stage: small token blocks are bound by the number of copies an SM
// issues, not by their bytes).
Status make_map_planes(CUtensorMap* tm, void* base, uint64_t Kp, uint64_t Mp, uint64_t planes, uint32_t T,
                       uint32_t box_planes = 1) {
  auto enc = tensor_map_encoder();
  if (!enc) return Status::Internal("cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {Kp, Mp, planes};
  cuuint64_t strides[2] = {Kp * 2, Kp * Mp * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK), T, box_planes};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return Status::Internal("cuTensorMapEncodeTiled (planes) failed: " + std::to_string(static_cast<int>(r)));
  return Status::Ok();
}

struct Plan {
  int T, N, Mp, Kp, nkb, splits, kb_per_split, stages, kbb;
  uint32_t stage_bytes, a_off, b_off, w_off, tmem_cols;
  size_t planes_bytes, scale_bytes, partial_bytes;
};

Plan make_plan(int M, int cols, int rows, int xsplit, DType dt) {
  Plan pl{};
  pl.T = gemm_token_tile(M, xsplit);
  pl.N = xsplit * pl.T;
  pl.Mp = static_cast<int>(round_up(M, pl.T));
  pl.Kp = static_cast<int>(round_up(cols, kBK));
  pl.nkb = pl.Kp / kBK;
  pl.kbb = dt == DType::FP4 ? kBK / 2 : kBK;
  const int tiles = static_cast<int>(((rows + kBM - 1) / kBM) * static_cast<int64_t>((M + pl.T - 1) / pl.T));
  int splits = 1;
  if (tiles < 148) {
    splits = 296 / tiles;
    if (splits > pl.nkb / 4) splits = pl.nkb / 4;
    if (splits > 16) splits = 16;
    if (splits < 1) splits = 1;
  }
  pl.kb_per_split = (pl.nkb + splits - 1) / splits;
  pl.splits = (pl.nkb + pl.kb_per_split - 1) / pl.kb_per_split;
  pl.a_off = 0;
  pl.b_off = kBM * 128;
  pl.w_off = pl.b_off + static_cast<uint32_t>(pl.N) * 128;
  pl.stage_bytes = static_cast<uint32_t>(round_up(pl.w_off + kBM * pl.kbb, 1024));
  const int budget = 227 * 1024 - 1024 - 256;
  pl.stages = budget / static_cast<int>(pl.stage_bytes);
  if (pl.stages > 6) pl.stages = 6;
  pl.tmem_cols = 32;
  while (pl.tmem_cols < static_cast<uint32_t>(pl.N)) pl.tmem_cols <<= 1;
  pl.planes_bytes = static_cast<size_t>(round_up(static_cast<int64_t>(xsplit) * pl.Mp * pl.Kp * 2, 1024));
  pl.scale_bytes = static_cast<size_t>(round_up(static_cast<int64_t>(pl.Mp) * 4, 1024));
  pl.partial_bytes = pl.splits > 1 ? static_cast<size_t>(pl.splits) * M * rows * 8 : 0;
  return pl;
}

struct TmPlan {
  bool pair;                                           // CTA pairs: 256-row tiles, M = 256 MMAs
  int TB, tpass[3], nacc[3], Mp, Kp, nkb, splits, kb_per_split, kbb, acc_cols;
  int tiles_t, tiles, tail_first, tail_s, tail_kbps;  // tail schedule (tail_first < 0: none)
  int pblk_bytes;                                      // per-token-block plane counts (shared memory)
  int sx, sw, wg;
  uint32_t x_bytes, w_bytes, a_col;
  uint32_t acc_buf;  // columns of one accumulator buffer when there are two, else 0
  size_t smem;
  size_t planes_bytes, scale_bytes, pcnt_bytes, partial_bytes;
};

// Split-K count (1..8) for `tiles` items of `nkb` k-blocks on `units` CTAs (or CTA pairs)
// at once, from a time model: a 64-k stage costs ~0.7 us (measured per-stage period of
// k_gemm_tm), so the GEMM takes waves(s) * 0.7 us * nkb / s; with s > 1 the fp64 partials
// (s x M x rows x 8 B) are written and read back once (at the measured HBM rate) and the
// reduce launch costs ~5 us.
int tm_splits(int tiles, int nkb, int M, int rows, int units) {
  const double stage_us = 0.7, hbm_bytes_per_us = 6.5e6, reduce_us = 5.0;
  int best = 1;
  double best_t = 0.0;
  for (int s = 1; s <= 8 && s <= nkb; ++s) {
    const int ctas = tiles * s;
    const int waves = (ctas + units - 1) / units;
    const int stages = (nkb + s - 1) / s;
    double t = waves * stage_us * stages;
    if (s > 1) t += 2.0 * s * static_cast<double>(M) * rows * 8.0 / hbm_bytes_per_us + reduce_us;
    if (s == 1 || t < best_t * 0.97) {
      best_t = t;
      best = s;
    }
  }
  return best;
}

// CTA pairs halve the x bytes each SM loads per MMA (each CTA of the pair holds half of the
// stage's x rows). Opt-in (WELVET_B200_GEMM_PAIR=1): single CTAs measured as fast or faster
// on B200 except at 1024+ tokens of one-plane x. Possible when the rows make whole 256-row
// tiles (an even number of 128-row mirror tiles) and a token block fills half an MMA.
bool tm_pair_wanted(int M, int rows) {
  const char* e = std::getenv("WELVET_B200_GEMM_PAIR");
  if (!e) return false;
  // "1": blocks of 128 tokens and more; "all": every batch the GEMM takes (tuning; a block
  // of fewer than 32 tokens is padded to 32)
  const int min_m = std::strcmp(e, "1") == 0 ? 128 : (std::strcmp(e, "all") == 0 ? 1 : 1 << 30);
  return M >= min_m && ((rows + kBM - 1) / kBM) % 2 == 0;
}

TmPlan make_tm_plan(int M, int cols, int rows, int xsplit, DType dt, bool allow_tail = true, bool allow_pair = true,
                    int max_tb = 0) {
  TmPlan pl{};
  pl.pair = allow_pair && tm_pair_wanted(M, rows);
  const int units = pl.pair ? 74 : 148;  // CTAs (CTA pairs) running at once on 148 SMs
  const int m16 = static_cast<int>(round_up(M, 16));
  // pair MMAs take N in multiples of 32 (16 x rows in each CTA)
  const int mb = pl.pair ? static_cast<int>(round_up(M, 32)) : m16;
  // Two accumulator buffers, so that the epilogue of one fill overlaps the MMAs of the next,
  // when WELVET_B200_GEMM_DBUF = columns per buffer (64..192, single CTAs; tuning): token
  // blocks and passes are then sized so that a fill takes at most that many columns, and two
  // buffers leave 128 TMEM columns for 4 A stages.
  int bw = 0;
  if (const char* e = std::getenv("WELVET_B200_GEMM_DBUF")) bw = std::atoi(e) & ~15;
  if (pl.pair || bw < 64 || bw > 192) bw = 0;
  pl.TB = mb < 256 ? mb : 256;
  if (bw && pl.TB > bw) pl.TB = bw;
  // a caller's cap on tokens per block, and WELVET_B200_GEMM_TB (tuning)
  int cap_tb = max_tb & ~31;
  if (const char* e = std::getenv("WELVET_B200_GEMM_TB")) cap_tb = std::atoi(e) & ~31;
  if (cap_tb >= 32 && cap_tb < pl.TB) pl.TB = cap_tb;
  pl.acc_cols = 0;
  int xrows = 0;
  for (int P = 1; P <= 3; ++P) {
    // pairs: 256, 128, 128 tokens (3 planes: planes 1 and 2 share an accumulator); otherwise
    // up to two MMAs of 384 accumulator columns (384, 192, 128), or one buffer's columns
    const int cap = pl.pair ? (P == 1 ? 256 : 128) : (bw ? (bw / P) & ~15 : (kTmAccMax / P) & ~15);
    int T = pl.TB < cap ? pl.TB : cap;
    if (T < pl.TB) {  // passes of equal size (256 tokens at 2 planes: 128 + 128, not 192 + 64)
      const int npass = (pl.TB + cap - 1) / cap;
      T = static_cast<int>(round_up((pl.TB + npass - 1) / npass, pl.pair ? 32 : 16));
    }
    pl.tpass[P - 1] = T;
    const int ntot = P * pl.tpass[P - 1];
    const int acols = (pl.pair && P == 3 ? 2 : P) * pl.tpass[P - 1];
    // independent accumulators so that short MMAs do not wait on each other's results
    pl.nacc[P - 1] = acols <= 64 ? 4 : (acols <= 128 ? 2 : 1);
    while (bw && pl.nacc[P - 1] > 1 && pl.nacc[P - 1] * acols > bw) --pl.nacc[P - 1];
    if (P <= xsplit) {
      pl.acc_cols = std::max(pl.acc_cols, pl.nacc[P - 1] * acols);
      // pairs: a 3-plane stage puts plane 2 in a second slot
      xrows = std::max(xrows, pl.pair && P == 3 ? 2 * pl.tpass[P - 1] : ntot);
    }
  }
  pl.Mp = m16;
  pl.Kp = static_cast<int>(round_up(cols, kBK));
  pl.nkb = pl.Kp / kBK;
  pl.kbb = dt == DType::FP4 ? kBK / 2 : kBK;
  // W stages per bulk copy: one by default; WELVET_B200_GEMM_WG = 2, 4 or 8 groups that many
  // stages of a tile per copy (tuning: 4 per copy measured 1.5 % slower on the 32-layer
  // 4096-wide volume at 64 tokens, 0.815 against 0.802 ms).
  pl.wg = 1;
  if (const char* e = std::getenv("WELVET_B200_GEMM_WG")) {
    const int g = std::atoi(e);
    if (g == 1 || g == 2 || g == 4 || g == 8) pl.wg = g;
  }
  pl.x_bytes = static_cast<uint32_t>(round_up(static_cast<int64_t>(xrows) * (pl.pair ? 64 : 128), 1024));
  pl.w_bytes = static_cast<uint32_t>(kBM * pl.kbb * pl.wg);
  pl.acc_buf = bw ? static_cast<uint32_t>(round_up(pl.acc_cols, 32)) : 0u;
  pl.a_col = bw ? 2 * pl.acc_buf : static_cast<uint32_t>(round_up(pl.acc_cols, 32));
  // stages (an x slot + a TMEM A slot each): as many as TMEM allows (up to 8) while the raw W
  // ring keeps 64 KB (and at least 4 slots), but no fewer than 3; then the W ring takes the
  // rest (up to 32). Measured with 32 KB x slots (FP8, 16384^2 and the SwiGLU cell): 4 x
  // stages with 8 W slots beat 5 with 4 by 5-8 %, and 3 with 10 by 2-4 %. 1 KB aligns the
  // base, 1 KB holds the barriers (at most 2*32 + 2*8 + 2 of them); the epilogue staging and
  // the per-token-block plane counts take their own space. WELVET_B200_GEMM_XSLOTS caps the
  // x stages (tuning).
  const int tiles_t_plan = (M + pl.TB - 1) / pl.TB;
  pl.pblk_bytes = static_cast<int>(round_up(static_cast<int64_t>(std::min(tiles_t_plan, kTmMaxBlocks)) * 4, 16));
  const int64_t budget = 227 * 1024 - 2048 - pl.pblk_bytes - kStageArea;
  pl.sx = (static_cast<int>(kTmemCols) - static_cast<int>(pl.a_col)) / 32;
  if (pl.sx > 8) pl.sx = 8;
  if (const char* e = std::getenv("WELVET_B200_GEMM_XSLOTS")) {
    const int n = std::atoi(e);
    if (n >= 2 && n < pl.sx) pl.sx = n;
  }
  const int64_t xb = pl.x_bytes, wb = pl.w_bytes;
  const int64_t w_keep = std::max<int64_t>(4 * wb, 64 * 1024);
  while (pl.sx > 3 && pl.sx * xb + w_keep > budget) --pl.sx;
  while (pl.sx > 2 && pl.sx * xb + 4 * wb > budget) --pl.sx;
  pl.sw = static_cast<int>((budget - pl.sx * static_cast<int64_t>(pl.x_bytes)) / pl.w_bytes);
  if (pl.sw > 32) pl.sw = 32;
  pl.smem = static_cast<size_t>(pl.sx) * pl.x_bytes + static_cast<size_t>(pl.sw) * pl.w_bytes + 2048 + pl.pblk_bytes +
            kStageArea;
  // At least half the SM's shared memory, so that one CTA (and its 512 TMEM columns) runs per
  // SM: a second CTA on the SM would only stall in tcgen05.alloc.
  if (pl.smem < 116 * 1024) pl.smem = 116 * 1024;
  const int sub = pl.pair ? 2 : 1;
  const int tiles =
      static_cast<int>(((rows + kBM - 1) / kBM / sub) * static_cast<int64_t>((M + pl.TB - 1) / pl.TB));
  int splits = tm_splits(tiles, pl.nkb, M, rows, units);
  if (const char* e = std::getenv("WELVET_B200_GEMM_SPLITS")) {  // tuning override (1..8)
    const int n = std::atoi(e);
    if (n >= 1 && n <= 8 && n <= pl.nkb) splits = n;
  }
  pl.kb_per_split = (pl.nkb + splits - 1) / splits;
  pl.splits = (pl.nkb + pl.kb_per_split - 1) / pl.kb_per_split;
  pl.planes_bytes = static_cast<size_t>(round_up(static_cast<int64_t>(xsplit) * pl.Mp * pl.Kp * 2, 1024));
  pl.scale_bytes = static_cast<size_t>(round_up(static_cast<int64_t>(pl.Mp) * 4, 1024));
  pl.pcnt_bytes = pl.scale_bytes;
  pl.partial_bytes = pl.splits > 1 ? static_cast<size_t>(pl.splits) * M * rows * 8 : 0;
  // A last, partly filled wave of whole tiles (up to half the units) costs as long as a full
  // one: those tiles are cut along K instead (into at most 8 slices, one wave of items in
  // all), and their fp64 partials summed by a small reduce launch.
  pl.tiles_t = (M + pl.TB - 1) / pl.TB;
  pl.tiles = tiles;
  pl.tail_first = -1;
  pl.tail_s = 1;
  pl.tail_kbps = pl.nkb;
  const int ntail = tiles % units;
  if (allow_tail && pl.splits == 1 && tiles > units && ntail > 0 && ntail <= units / 2 && pl.nkb >= 2) {
    int s = units / ntail;
    if (s > 8) s = 8;
    if (s > pl.nkb) s = pl.nkb;
    if (s >= 2) {
      pl.tail_kbps = (pl.nkb + s - 1) / s;
      pl.tail_s = (pl.nkb + pl.tail_kbps - 1) / pl.tail_kbps;  // every slice non-empty
      pl.tail_first = tiles - ntail;
      // fp64 (or raw fp32) partials, then one flag per 128-row part
      pl.partial_bytes = static_cast<size_t>(ntail) * sub * pl.tail_s * pl.TB * 128 * 8 +
                         static_cast<size_t>(round_up(static_cast<int64_t>(ntail) * sub * 4, 16));
    }
  }
  return pl;
}

// SwiGLU pair epilogue: SiLU in fp64 exactly as the reference when WELVET_B200_SILU=fp64,
// else in fp32.
bool silu_exact() {
  const char* e = std::getenv("WELVET_B200_SILU");
  return e && std::strcmp(e, "fp64") == 0;
}

// Which batched kernel runs: A in TMEM (default) or A in shared memory
// (WELVET_B200_GEMM=smem, kept for comparison).
bool gemm_a_in_smem() {
  const char* e = std::getenv("WELVET_B200_GEMM");
  return e && std::strcmp(e, "smem") == 0;
}

} // namespace

namespace {
// One thread per 16-byte chunk of the GEMM mirror; see build_gemm_mirror.
// W2 != nullptr: pair mirror, destination row 2i from W row i, 2i+1 from W2 row i (`rows`
// counts the destination rows).
__global__ void k_build_gemm_mirror(const uint8_t* __restrict__ W, const uint8_t* __restrict__ W2,
                                    int64_t row_stride, int rows, int nkb, int kbb, int64_t nchunks,
                                    uint8_t* __restrict__ Wg) {
  const int cpr = kbb >> 4;  // chunks per row per stage
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nchunks;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(i % cpr);
    int64_t rest = i / cpr;
    const int r = static_cast<int>(rest % 128);
    rest /= 128;
    const int kb = static_cast<int>(rest % nkb);
    const int64_t tile = rest / nkb;
    const int64_t row = tile * 128 + r;
    const int64_t src = static_cast<int64_t>(kb) * kbb + j * 16;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < rows && src + 16 <= row_stride) {
      const uint8_t* base = W2 ? ((row & 1) ? W2 : W) + (row >> 1) * row_stride : W + row * row_stride;
      v = *reinterpret_cast<const uint4*>(base + src);
    }
    const int sw = kbb == 32 ? ((r >> 2) & 1) : ((r >> 1) & 3);
    *reinterpret_cast<uint4*>(Wg + ((tile * nkb + kb) * 128 + r) * kbb + ((j ^ sw) << 4)) = v;
  }
}
} // namespace

size_t gemm_mirror_bytes(DType dt, int rows, int cols) {
  const int64_t tiles = (rows + kBM - 1) / kBM;
  const int64_t nkb = (cols + kBK - 1) / kBK;
  const int64_t kbb = dt == DType::FP4 ? kBK / 2 : kBK;
  return static_cast<size_t>(tiles * nkb * kBM * kbb);
}

Status build_gemm_mirror(DType dt, const uint8_t* W, int rows, int64_t row_stride, int cols, uint8_t* Wg,
                         cudaStream_t st) {
  if (!gemm_supported(dt)) return Status::Unsupported("gemm mirror: dtype");
  if (!W || !Wg || row_stride % 16 != 0) return Status::Internal("gemm mirror: bad arguments");
  const int nkb = (cols + kBK - 1) / kBK;
  const int kbb = dt == DType::FP4 ? kBK / 2 : kBK;
  const int64_t nchunks = static_cast<int64_t>(gemm_mirror_bytes(dt, rows, cols) / 16);
  int64_t blocks = (nchunks + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  k_build_gemm_mirror<<<static_cast<unsigned>(blocks), 256, 0, st>>>(W, nullptr, row_stride, rows, nkb, kbb, nchunks,
                                                                      Wg);
  return cuda_status(cudaGetLastError(), "gemm mirror build");
}

Status build_gemm_pair_mirror(DType dt, const uint8_t* Wgate, const uint8_t* Wup, int inter, int64_t row_stride,
                              int cols, uint8_t* Wg, cudaStream_t st) {
  if (!gemm_supported(dt)) return Status::Unsupported("gemm pair mirror: dtype");
  if (!Wgate || !Wup || !Wg || row_stride % 16 != 0 || inter <= 0) return Status::Internal("gemm pair mirror: bad arguments");
  const int rows = 2 * inter;
  const int nkb = (cols + kBK - 1) / kBK;
  const int kbb = dt == DType::FP4 ? kBK / 2 : kBK;
  const int64_t nchunks = static_cast<int64_t>(gemm_mirror_bytes(dt, rows, cols) / 16);
  int64_t blocks = (nchunks + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  k_build_gemm_mirror<<<static_cast<unsigned>(blocks), 256, 0, st>>>(Wgate, Wup, row_stride, rows, nkb, kbb, nchunks,
                                                                      Wg);
  return cuda_status(cudaGetLastError(), "gemm pair mirror build");
}

bool gemm_uses_tmem() { return !gemm_a_in_smem(); }

bool gemm_supported(DType dt) {
  return dt == DType::FP4 || dt == DType::FP8E4M3 || dt == DType::FP8E5M2 || dt == DType::Int8;
}

int gemm_token_tile(int M, int xsplit) {
  const int tmax = xsplit == 3 ? 64 : (xsplit == 2 ? 112 : 224);
  int t = static_cast<int>(round_up(M, 16));
  if (t > tmax) t = tmax;
  return t;
}

int gemm_plan_values(int M, int cols, int rows, int xsplit, DType dt, int max_tb, int64_t* out, int n) {
  const TmPlan pl = make_tm_plan(M, cols, rows, xsplit, dt, true, true, max_tb);
  const int64_t n_items = pl.tail_first >= 0
                              ? pl.tail_first + static_cast<int64_t>(pl.tiles - pl.tail_first) * pl.tail_s
                              : static_cast<int64_t>(pl.tiles) * pl.splits;
  const int64_t v[] = {pl.pair ? 1 : 0, pl.TB, pl.tpass[0], pl.tpass[1], pl.tpass[2], pl.nacc[0], pl.nacc[1],
                       pl.nacc[2], pl.acc_cols, pl.acc_buf, pl.a_col, pl.sx, pl.sw, pl.x_bytes, pl.w_bytes,
                       static_cast<int64_t>(pl.smem), pl.nkb, pl.splits, pl.kb_per_split, pl.tiles_t, pl.tiles,
                       pl.tail_first, pl.tail_s, pl.tail_kbps, n_items, pl.wg};
  const int cnt = static_cast<int>(sizeof(v) / sizeof(v[0]));
  for (int i = 0; i < cnt && i < n; ++i) out[i] = v[i];
  return cnt;
}

size_t gemm_scratch_bytes(int M, int cols, int rows, int xsplit, bool tail, int max_tb) {
  size_t need = 0;
  for (DType dt : {DType::FP8E4M3, DType::FP4}) {
    const Plan pl = make_plan(M, cols, rows, xsplit, dt);
    need = std::max(need, pl.planes_bytes + pl.scale_bytes + pl.partial_bytes);
    for (bool pair : {true, false}) {  // CTA pairs, and single CTAs when no pair can run
      const TmPlan tp = make_tm_plan(M, cols, rows, xsplit, dt, tail, pair, max_tb);
      need = std::max(need, tp.planes_bytes + tp.scale_bytes + tp.pcnt_bytes + tp.partial_bytes);
    }
  }
  return need;
}

namespace {

// cudaFuncSetAttribute is a driver call on every use; do it once per kernel, device and size.
Status set_max_smem(const void* kern, size_t bytes) {
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

using TmKernel = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, PeerMaps, TmParams);

TmKernel tm_kernel(DType dt, bool pair) {
  switch (dt) {
  case DType::FP4: return pair ? k_gemm_tm<16, true> : k_gemm_tm<16, false>;
  case DType::FP8E4M3: return pair ? k_gemm_tm<4, true> : k_gemm_tm<4, false>;
  case DType::FP8E5M2: return pair ? k_gemm_tm<5, true> : k_gemm_tm<5, false>;
  case DType::Int8: return pair ? k_gemm_tm<9, true> : k_gemm_tm<9, false>;
  default: return nullptr;
  }
}

// A launch with programmatic stream serialization (when `pdl`).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

cudaLaunchConfig_t pair_config(unsigned pairs, size_t smem, cudaStream_t st, cudaLaunchAttribute* at) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kTmThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  return cfg;
}

// CTA pairs of `kern` that can be resident at once with `smem` bytes of shared memory each
// (asked once per kernel, device and size); 0 when none can.
int tm_max_pairs(TmKernel kern, size_t smem) {
  static std::mutex mu;
  static std::vector<std::tuple<const void*, int, size_t, int>> known;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const void* key = reinterpret_cast<const void*>(kern);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& k : known)
      if (std::get<0>(k) == key && std::get<1>(k) == dev && std::get<2>(k) == smem) return std::get<3>(k);
  }
  int n = 0;
  if (set_max_smem(key, smem).ok()) {
    cudaLaunchAttribute at[2];
    const cudaLaunchConfig_t cfg = pair_config(74, smem, nullptr, at);
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      n = 0;
    }
  }
  std::lock_guard<std::mutex> lock(mu);
  known.emplace_back(key, dev, smem, n);
  return n;
}

Status launch_tm(const GemmArgs& a, cudaStream_t st) {
  if (!a.Wg || (reinterpret_cast<uintptr_t>(a.Wg) & 15) != 0)
    return Status::Internal("gemm_tc: the layer has no GEMM mirror (16-byte aligned)");
  TmPlan pl = make_tm_plan(a.M, a.cols, a.rows, a.xsplit, a.dtype, true, true, a.max_tb);
  int pairs = 0;
  if (pl.pair) {
    const TmKernel k = tm_kernel(a.dtype, true);
    pairs = k ? tm_max_pairs(k, pl.smem) : 0;
    if (pairs < 1) pl = make_tm_plan(a.M, a.cols, a.rows, a.xsplit, a.dtype, true, false, a.max_tb);
  }
  if (pl.sw < 2 || pl.sx < 2 || pl.a_col + 32u * pl.sx > kTmemCols)
    return Status::Internal("gemm_tc: pipeline does not fit on the SM");
  size_t need = pl.planes_bytes + pl.scale_bytes + pl.pcnt_bytes + pl.partial_bytes;
  if (pl.tail_first >= 0 && a.scratch_bytes < need) {  // no room for the tail partials
    pl = make_tm_plan(a.M, a.cols, a.rows, a.xsplit, a.dtype, false, pl.pair, a.max_tb);
    need = pl.planes_bytes + pl.scale_bytes + pl.pcnt_bytes + pl.partial_bytes;
  }
  if (!a.scratch || a.scratch_bytes < need) return Status::Internal("gemm_tc: scratch too small");
  uint8_t* scr = static_cast<uint8_t*>(a.scratch);
  __half* planes = reinterpret_cast<__half*>(scr);
  float* scale_inv = reinterpret_cast<float*>(scr + pl.planes_bytes);
  int* pcnt = reinterpret_cast<int*>(scr + pl.planes_bytes + pl.scale_bytes);
  double* partial = pl.splits > 1 || pl.tail_first >= 0
                        ? reinterpret_cast<double*>(scr + pl.planes_bytes + pl.scale_bytes + pl.pcnt_bytes)
                        : nullptr;

  WB_CUDA(launch_pdl(k_split_x, dim3(static_cast<unsigned>(pl.Mp)), dim3(kSplitThreads), 0, st, a.pdl, a.x, a.x_ld,
                     a.M, a.cols, pl.Mp, pl.Kp, a.xsplit, planes, scale_inv, pcnt, a.norm));

  CUtensorMap tm_x[3];
  for (int P = 1; P <= 3; ++P) {
    const int q = P <= a.xsplit ? P : 1;  // maps for plane counts above xsplit are never used
    // a CTA of a pair loads boxes of half a pass's tokens, one plane each; a single CTA one box
    // of all q planes per stage
    const int box = pl.pair ? pl.tpass[q - 1] / 2 : pl.tpass[q - 1];
    WB_TRY(make_map_planes(&tm_x[P - 1], planes, static_cast<uint64_t>(pl.Kp), static_cast<uint64_t>(pl.Mp),
                           static_cast<uint64_t>(a.xsplit), static_cast<uint32_t>(box),
                           pl.pair ? 1u : static_cast<uint32_t>(q)));
  }

  TmParams p{};
  p.Wg = a.Wg;
  p.rows = a.rows; p.cols = a.cols; p.M = a.M; p.xsplit = a.xsplit;
  p.TB = pl.TB;
  for (int i = 0; i < 3; ++i) p.tpass[i] = pl.tpass[i];
  p.nkb_total = pl.nkb; p.kb_per_split = pl.kb_per_split; p.splits = pl.splits; p.kbb = pl.kbb;
  p.x_bytes = pl.x_bytes; p.w_bytes = pl.w_bytes; p.a_col = pl.a_col; p.acc_buf = pl.acc_buf;
  p.sx = pl.sx; p.sw = pl.sw; p.wg = pl.wg;
  for (int i = 0; i < 3; ++i) p.nacc[i] = pl.nacc[i];
  p.w_evict_first = (a.M + pl.TB - 1) / pl.TB == 1 ? 1 : 0;
  p.scale_inv = scale_inv; p.pcnt = pcnt; p.w_scale = a.scale;
  p.pre = a.pre; p.post = a.post; p.ld_out = a.ld_out;
  p.bias = a.bias; p.bias_len = a.bias_len; p.act = a.act;
  p.partial = partial; p.err = a.err;
  if (const char* e = std::getenv("WELVET_B200_TEST_WAIT_TIMEOUT")) p.probe_wait = e[0] == '1' ? 1 : 0;
  p.pair = a.pair ? 1 : 0; p.w_scale2 = a.scale2; p.h = a.h; p.ld_h = a.ld_h;
  p.silu_exact = silu_exact() ? 1 : 0;
  p.tiles_t = pl.tiles_t; p.tail_first = pl.tail_first; p.tail_s = pl.tail_s; p.tail_kbps = pl.tail_kbps;
  p.tiles = pl.tiles;
  p.n_items = pl.tail_first >= 0 ? pl.tail_first + (pl.tiles - pl.tail_first) * pl.tail_s : pl.tiles * pl.splits;

  // Outputs through bulk tensor stores (the epilogue stages them in its own shared memory):
  // fp32 rows whose pitch is a multiple of 16 bytes at 16-byte aligned bases.
  CUtensorMap tm_o[2] = {tm_x[0], tm_x[0]};  // placeholders when the epilogue stores directly
  {
    auto aligned = [](const void* ptr, int64_t ld) {
      return ptr != nullptr && (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && (ld * 4) % 16 == 0;
    };
    bool ok = true;
    if (ok && a.pair) {
      ok = aligned(a.h, a.ld_h) &&
           make_map_2d(&tm_o[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.h, static_cast<uint64_t>(a.rows / 2),
                       static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.ld_h) * 4, kBM / 2, 16,
                       CU_TENSOR_MAP_SWIZZLE_NONE).ok();
    } else if (ok) {
      ok = aligned(a.pre, a.ld_out) && aligned(a.post, a.ld_out) &&
           make_map_2d(&tm_o[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.pre, static_cast<uint64_t>(a.rows),
                       static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.ld_out) * 4, kBM, 16,
                       CU_TENSOR_MAP_SWIZZLE_NONE).ok();
      p.tma_post = ok && a.post != a.pre;
      if (p.tma_post)
        ok = make_map_2d(&tm_o[1], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.post, static_cast<uint64_t>(a.rows),
                         static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.ld_out) * 4, kBM, 16,
                         CU_TENSOR_MAP_SWIZZLE_NONE).ok();
    }
    p.tma_out = ok ? 1 : 0;
    if (!ok) p.tma_post = 0;
  }
  // Column-sharded layers: post also goes to the peers -- through bulk tensor stores of the
  // staged chunks (one map per peer, post's layout) and direct stores everywhere else. If a
  // map cannot be made, every output takes the direct-store path.
  PeerMaps pm{};
  p.peers = a.peers;
  p.n_peer_maps = 0;
  if (p.tma_out && a.peers.n > 0) {
    bool ok = !a.pair;
    for (int i = 0; ok && i < a.peers.n; ++i)
      ok = (reinterpret_cast<uintptr_t>(a.peers.post[i]) & 15) == 0 &&
           make_map_2d(&pm.m[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.peers.post[i], static_cast<uint64_t>(a.rows),
                       static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.ld_out) * 4, kBM, 16,
                       CU_TENSOR_MAP_SWIZZLE_NONE).ok();
    if (ok) {
      p.n_peer_maps = a.peers.n;
    } else {
      p.tma_out = 0;
      p.tma_post = 0;
    }
  }

  const size_t smem = pl.smem;
  // persistent: one CTA per SM (or per item when there are fewer), each looping over items
  int sms = 148;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms < 1) sms = 148;
  }
  const TmKernel kern = tm_kernel(a.dtype, pl.pair);
  if (!kern) return Status::Unsupported("gemm_tc: dtype");
  WB_TRY(set_max_smem(reinterpret_cast<const void*>(kern), smem));
  if (pl.pair) {
    // clusters of 2, one pair per item up to the pairs that fit at once
    cudaLaunchAttribute at[2];
    const cudaLaunchConfig_t cfg =
        pair_config(static_cast<unsigned>(p.n_items < pairs ? p.n_items : pairs), smem, st, at);
    WB_CUDA(cudaLaunchKernelEx(&cfg, kern, tm_x[0], tm_x[1], tm_x[2], tm_o[0], tm_o[1], pm, p));
  } else {
    const dim3 grid(static_cast<unsigned>(p.n_items < sms ? p.n_items : sms), 1, 1);
    WB_TRY(cuda_status(launch_pdl(kern, grid, dim3(kTmThreads), smem, st, true, tm_x[0], tm_x[1], tm_x[2], tm_o[0],
                                  tm_o[1], pm, p),
                       "gemm_tc (tmem) launch"));
  }
  if (pl.tail_first >= 0) {
    const int ntail = pl.tiles - pl.tail_first;
    TailParams r{};
    r.rows = a.rows; r.M = a.M; r.TB = pl.TB; r.tiles_t = pl.tiles_t; r.tail_first = pl.tail_first;
    r.tail_s = pl.tail_s; r.ntail = ntail; r.sub = pl.pair ? 2 : 1; r.partial = partial;
    r.scale_inv = scale_inv; r.int8 = a.dtype == DType::Int8 ? 1 : 0; r.w_scale = a.scale; r.w_scale2 = a.scale2;
    r.pre = a.pre; r.post = a.post; r.ld_out = a.ld_out; r.bias = a.bias; r.bias_len = a.bias_len; r.act = a.act;
    r.pair = a.pair ? 1 : 0; r.h = a.h; r.ld_h = a.ld_h;
    r.peers = a.peers;
    const int64_t n = static_cast<int64_t>(ntail) * r.sub * pl.TB * (a.pair ? 64 : 128);
    WB_CUDA(launch_pdl(k_tail_reduce, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, st, true, r));
  }
  if (pl.splits > 1) {
    KParams r{};
    r.rows = a.rows; r.M = a.M; r.splits = pl.splits; r.partial = partial;
    r.pre = a.pre; r.post = a.post; r.ld_out = a.ld_out; r.bias = a.bias; r.bias_len = a.bias_len; r.act = a.act;
    r.pair = a.pair ? 1 : 0; r.h = a.h; r.ld_h = a.ld_h;
    r.peers = a.peers;
    const int64_t n = static_cast<int64_t>(a.M) * a.rows;
    int blocks = static_cast<int>((n + 255) / 256);
    if (blocks > 148 * 16) blocks = 148 * 16;
    WB_CUDA(launch_pdl(k_splitk_reduce, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st, true, r));
  }
  return Status::Ok();
}

Status launch_smem(const GemmArgs& a, cudaStream_t st) {
  const Plan pl = make_plan(a.M, a.cols, a.rows, a.xsplit, a.dtype);
  if (pl.stages < 2) return Status::Internal("gemm_tc: stage does not fit in shared memory");
  const size_t need = pl.planes_bytes + pl.scale_bytes + pl.partial_bytes;
  if (!a.scratch || a.scratch_bytes < need) return Status::Internal("gemm_tc: scratch too small");
  uint8_t* scr = static_cast<uint8_t*>(a.scratch);
  __half* planes = reinterpret_cast<__half*>(scr);
  float* scale_inv = reinterpret_cast<float*>(scr + pl.planes_bytes);
  double* partial = pl.splits > 1 ? reinterpret_cast<double*>(scr + pl.planes_bytes + pl.scale_bytes) : nullptr;

  {
    const int warps = pl.Mp;
    k_split_x<<<warps, kSplitThreads, 0, st>>>(a.x, a.x_ld, a.M, a.cols, pl.Mp, pl.Kp, a.xsplit, planes, scale_inv,
                                               nullptr, a.norm);
    WB_CUDA(cudaGetLastError());
  }

  CUtensorMap tm_w, tm_x;
  WB_TRY(make_map_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, const_cast<uint8_t*>(a.W),
                     static_cast<uint64_t>(a.row_stride), static_cast<uint64_t>(a.rows),
                     static_cast<uint64_t>(a.row_stride), static_cast<uint32_t>(pl.kbb), kBM,
                     CU_TENSOR_MAP_SWIZZLE_NONE));
  WB_TRY(make_map_2d(&tm_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, planes, static_cast<uint64_t>(pl.Kp),
                     static_cast<uint64_t>(a.xsplit) * pl.Mp, static_cast<uint64_t>(pl.Kp) * 2, kBK,
                     static_cast<uint32_t>(pl.T), CU_TENSOR_MAP_SWIZZLE_128B));

  KParams p{};
  p.rows = a.rows; p.cols = a.cols; p.M = a.M; p.T = pl.T; p.N = pl.N; p.xsplit = a.xsplit;
  p.nkb_total = pl.nkb; p.kb_per_split = pl.kb_per_split; p.splits = pl.splits; p.Mp = pl.Mp; p.kbb = pl.kbb;
  // instruction descriptor: D f32, A/B f16, both K-major, N>>3 at bit 17, M>>4 at bit 24
  p.idesc = (1u << 4) | (static_cast<uint32_t>(pl.N >> 3) << 17) | (static_cast<uint32_t>(kBM >> 4) << 24);
  p.tmem_cols = pl.tmem_cols;
  p.stage_bytes = pl.stage_bytes; p.a_off = pl.a_off; p.b_off = pl.b_off; p.w_off = pl.w_off;
  p.stages = pl.stages;
  p.scale_inv = scale_inv;
  p.w_scale = a.scale;
  p.peers = a.peers;
  p.pre = a.pre; p.post = a.post; p.ld_out = a.ld_out;
  p.bias = a.bias; p.bias_len = a.bias_len; p.act = a.act;
  p.partial = partial;
  p.err = a.err;

  const size_t smem = static_cast<size_t>(pl.stages) * pl.stage_bytes + 1024 + 256;
  dim3 grid(static_cast<unsigned>((a.rows + kBM - 1) / kBM), static_cast<unsigned>((a.M + pl.T - 1) / pl.T),
            static_cast<unsigned>(pl.splits));
  auto launch = [&](auto kern) -> Status {
    WB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    kern<<<grid, kThreads, smem, st>>>(tm_w, tm_x, p);
    return cuda_status(cudaGetLastError(), "gemm_tc launch");
  };
  switch (a.dtype) {
  case DType::FP4: WB_TRY(launch(k_gemm_tc<16>)); break;
  case DType::FP8E4M3: WB_TRY(launch(k_gemm_tc<4>)); break;
  case DType::FP8E5M2: WB_TRY(launch(k_gemm_tc<5>)); break;
  case DType::Int8: WB_TRY(launch(k_gemm_tc<9>)); break;
  default: return Status::Unsupported("gemm_tc: dtype");
  }
  if (pl.splits > 1) {
    const int64_t n = static_cast<int64_t>(a.M) * a.rows;
    int blocks = static_cast<int>((n + 255) / 256);
    if (blocks > 148 * 16) blocks = 148 * 16;
    k_splitk_reduce<<<blocks, 256, 0, st>>>(p);
    WB_CUDA(cudaGetLastError());
  }
  return Status::Ok();
}

} // namespace

Status launch_gemm_tc(const GemmArgs& a, cudaStream_t st) {
  if (!gemm_supported(a.dtype)) return Status::Unsupported("gemm_tc: dtype");
  if (a.M <= 0 || a.rows <= 0 || a.cols <= 0) return Status::Invalid("gemm_tc: bad dims");
  if (a.xsplit < 1 || a.xsplit > 3) return Status::Invalid("gemm_tc: xsplit must be 1..3");
  if (a.pair && (gemm_a_in_smem() || !a.h || a.rows % 2 != 0 || a.ld_h < a.rows / 2))
    return Status::Invalid("gemm_tc: the Gate/Up pair mode needs the TMEM kernel, an h buffer and even rows");
  if (a.norm.gamma && (!a.norm.pre || !a.norm.post)) return Status::Invalid("gemm_tc: RMSNorm prologue without outputs");
  if ((reinterpret_cast<uintptr_t>(a.norm.gamma) & 15) != 0) return Status::Invalid("gemm_tc: RMSNorm gamma not 16-byte aligned");
  return gemm_a_in_smem() ? launch_smem(a, st) : launch_tm(a, st);
}

// ---------------------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot call cudaMalloc when they run a forward: a serving loop that must
// never stall on an allocation (cudaMalloc can synchronize the device), or a framework or
// plugin host that owns all device memory up front and forbids other allocations once it runs. For them launch_gemm_tc_static runs the same
// tcgen05 GEMM with its scratch (the f16 planes of x, the per-token scales and the split-K
// partials) in one array that lives in this file for the life of the process.
//
// The array is kStaticScratchBytes (32 MiB) on every GPU that loads the library, held until
// the process exits. All calls share it: two calls whose kernels overlap on a GPU (different
// streams, or different host threads on one device) race on it and must be serialized by
// the caller. A call keeps the previous call's contents; nothing in it has to start at zero
// (each launch writes every plane, scale and partial before reading it).
constexpr size_t kStaticScratchBytes = static_cast<size_t>(32) << 20;
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
// Per device: the array's device address and the context it was looked up in. A device reset
// (cudaDeviceReset) or a context re-created by the host application reloads the module and
// moves the array, so the address is looked up again whenever the current context differs.
void* g_static_ptr[kMaxDevices] = {};
CUcontext g_static_ctx[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}
} // namespace

size_t gemm_static_scratch_bytes() { return kStaticScratchBytes; }

Status launch_gemm_tc_static(const GemmArgs& a_in, cudaStream_t st) {
  const size_t need = gemm_scratch_bytes(a_in.M, a_in.cols, a_in.rows, a_in.xsplit, false, a_in.max_tb);
  if (need > kStaticScratchBytes)
    return Status::Invalid("allocation-free forward: needs " + std::to_string(need) +
                           " bytes of scratch, the static array holds " + std::to_string(kStaticScratchBytes) +
                           " (fewer tokens per call, or the allocating entry point)");
  int dev = 0;
  WB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return Status::Internal("allocation-free forward: device index out of range");
  void* ptr = nullptr;
  {
    // Once per device (and context), with that device current: the array's device address.
    // The host-side symbol is only a stand-in and must never reach a kernel.
    CUcontext ctx = nullptr;  // current since the session's mount ran on this device
    auto get_ctx = ctx_get_current();
    if (!get_ctx || get_ctx(&ctx) != CUDA_SUCCESS || !ctx)
      return Status::Internal("allocation-free forward: no current CUDA context");
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_ptr[dev] || g_static_ctx[dev] != ctx) {
      void* p = nullptr;
      WB_CUDA(cudaGetSymbolAddress(&p, g_static_scratch));
      g_static_ptr[dev] = p;
      g_static_ctx[dev] = ctx;
    }
    ptr = g_static_ptr[dev];
  }
  GemmArgs a = a_in;
  a.scratch = ptr;
  a.scratch_bytes = kStaticScratchBytes;
  return launch_gemm_tc(a, st);
}

} // namespace wb
