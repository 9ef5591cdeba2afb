// gemm_tc.cu -- batched dequant GEMM on sm_100a tensor cores (tcgen05.mma kind::f16, TMEM).
//
// Replaces, for batch >= 8 tokens, the reference's per-output fp64 loop
// (src/cuda/kernels.cu:130-145) over a host-decoded fp64 W. The packed mirror is read once
// per token tile:
//
//   warp 0      TMA producer: the raw packed W tile (128 rows x 64 k) and the activation
//               tile of every x plane (T tokens x 64 k, f16, SWIZZLE_128B) per stage; also
//               allocates / frees the TMEM accumulator.
//   warp 1      MMA issuer (one thread): 4 x tcgen05.mma (K = 16 each) per stage, A and B from
//               shared memory, fp32 accumulation in TMEM; tcgen05.commit frees the stage.
//   warps 2..5  converters: raw codes -> f16 (hardware e2m1/e4m3/e5m2 -> f16x2 converters,
//               Int8 via an exact f16 bias trick) written in the UMMA K-major SWIZZLE_128B
//               layout; then the epilogue: tcgen05.ld of the accumulator, the planes of each
//               token combined in fp64, per-token 2^-e and Int8 scale applied, then bias /
//               activation exactly as the reference's dense_bias_act (kernels.cu:147-161).
//
// The x planes ride in the N dimension of one MMA ([plane][token] rows of B), so each A tile
// is read from shared memory once per K step. Every mbarrier wait is bounded by
// %globaltimer (2 s); on expiry the kernel records an error word and winds down, it never
// spins forever. No TMA multicast is used.
#include "gemm_tc.hpp"
#include "codec.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace wb {
namespace {

constexpr int kBM = 128;      // output rows per tile (MMA M)
constexpr int kBK = 64;       // k per stage (128 bytes of f16)
constexpr int kThreads = 192; // 6 warps
constexpr uint64_t kWaitNs = 2000000000ull;

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
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false (and the error word set) once kWaitNs of wall time has passed.
__device__ __noinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitNs) {
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
}

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

__device__ __forceinline__ void write_out(const KParams& p, int t, int o, double y) {
  const int64_t idx = static_cast<int64_t>(t) * p.ld_out + o;
  float pre = static_cast<float>(y);
  double v = static_cast<double>(pre);
  if (p.bias != nullptr && o < p.bias_len) {
    v += p.bias[o];
    pre = static_cast<float>(v);
  }
  p.pre[idx] = pre;
  p.post[idx] = static_cast<float>(activate(p.act, v));
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

// Sum of the split-K partials in a fixed order, then the reference epilogue.
__global__ void k_splitk_reduce(const KParams p) {
  const int64_t n = static_cast<int64_t>(p.M) * p.rows;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    double y = 0.0;
    for (int s = 0; s < p.splits; ++s) y += p.partial[s * n + i];
    write_out(p, static_cast<int>(i / p.rows), static_cast<int>(i % p.rows), y);
  }
}

// x [M][x_ld] f32 -> planes [xsplit][Mp][Kp] f16 (x * 2^e = p0 + p1 + p2) and 2^-e per token.
// One warp per token row; rows >= M and columns >= K are zero.
__global__ void k_split_x(const float* __restrict__ x, int64_t x_ld, int M, int K, int Mp, int Kp, int xsplit,
                          __half* __restrict__ planes, float* __restrict__ scale_inv) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= Mp) return;
  const float* xr = x + static_cast<int64_t>(t) * x_ld;
  float amax = 0.0f;
  if (t < M)
    for (int k = lane; k < K; k += 32) {
      const float a = fabsf(xr[k]);
      if (a > amax && a <= 3.402823466e+38f) amax = a;
    }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  int e = 0;
  if (amax > 0.0f) {
    e = 13 - ilogbf(amax);  // amax * 2^e in [2^13, 2^14)
    if (e > 126) e = 126;
    if (e < -126) e = -126;
  }
  const float s = ldexpf(1.0f, e);
  if (lane == 0) scale_inv[t] = ldexpf(1.0f, -e);
  const int64_t plane = static_cast<int64_t>(Mp) * Kp;
  __half* p0 = planes + static_cast<int64_t>(t) * Kp;
  for (int k = lane; k < Kp; k += 32) {
    const float v = (t < M && k < K) ? xr[k] : 0.0f;
    __half h0, h1 = __float2half_rn(0.0f), h2 = __float2half_rn(0.0f);
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
    p0[k] = h0;
    if (xsplit > 1) p0[plane + k] = h1;
    if (xsplit > 2) p0[2 * plane + k] = h2;
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

} // namespace

bool gemm_supported(DType dt) {
  return dt == DType::FP4 || dt == DType::FP8E4M3 || dt == DType::FP8E5M2 || dt == DType::Int8;
}

int gemm_token_tile(int M, int xsplit) {
  const int tmax = xsplit == 3 ? 64 : (xsplit == 2 ? 112 : 224);
  int t = static_cast<int>(round_up(M, 16));
  if (t > tmax) t = tmax;
  return t;
}

size_t gemm_scratch_bytes(int M, int cols, int rows, int xsplit) {
  const Plan pl = make_plan(M, cols, rows, xsplit, DType::FP8E4M3);
  const Plan p4 = make_plan(M, cols, rows, xsplit, DType::FP4);
  const size_t a = pl.planes_bytes + pl.scale_bytes + pl.partial_bytes;
  const size_t b = p4.planes_bytes + p4.scale_bytes + p4.partial_bytes;
  return a > b ? a : b;
}

Status launch_gemm_tc(const GemmArgs& a, cudaStream_t st) {
  if (!gemm_supported(a.dtype)) return Status::Unsupported("gemm_tc: dtype");
  if (a.M <= 0 || a.rows <= 0 || a.cols <= 0) return Status::Invalid("gemm_tc: bad dims");
  if (a.xsplit < 1 || a.xsplit > 3) return Status::Invalid("gemm_tc: xsplit must be 1..3");
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
    k_split_x<<<(warps + 7) / 8, 256, 0, st>>>(a.x, a.x_ld, a.M, a.cols, pl.Mp, pl.Kp, a.xsplit, planes, scale_inv);
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

// ---------------------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot call cudaMalloc when they run a forward: a serving loop that must
// never stall on an allocation (cudaMalloc can synchronize the device), code running while
// a CUDA graph is being captured, or a framework that owns all device memory up front and
// forbids other allocations once it runs. For them launch_gemm_tc_static runs the same
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
void* g_static_ptr[kMaxDevices] = {};
} // namespace

size_t gemm_static_scratch_bytes() { return kStaticScratchBytes; }

Status launch_gemm_tc_static(const GemmArgs& a_in, cudaStream_t st) {
  const size_t need = gemm_scratch_bytes(a_in.M, a_in.cols, a_in.rows, a_in.xsplit);
  if (need > kStaticScratchBytes)
    return Status::Invalid("allocation-free forward: needs " + std::to_string(need) +
                           " bytes of scratch, the static array holds " + std::to_string(kStaticScratchBytes) +
                           " (fewer tokens per call, or the allocating entry point)");
  int dev = 0;
  WB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return Status::Internal("allocation-free forward: device index out of range");
  void* ptr = nullptr;
  {
    // Once per device, with that device current: the array's device address. The host-side
    // symbol is only a stand-in and must never reach a kernel.
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_ptr[dev]) {
      void* p = nullptr;
      WB_CUDA(cudaGetSymbolAddress(&p, g_static_scratch));
      g_static_ptr[dev] = p;
    }
    ptr = g_static_ptr[dev];
  }
  GemmArgs a = a_in;
  a.scratch = ptr;
  a.scratch_bytes = kStaticScratchBytes;
  return launch_gemm_tc(a, st);
}

} // namespace wb
