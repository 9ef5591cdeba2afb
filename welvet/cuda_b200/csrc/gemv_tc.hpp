// gemv_tc.hpp -- small-batch (1..8 tokens) dequant GEMV on the tensor cores' register path.
#pragma once

#include "common.hpp"

namespace wb {

// Fragment-tiled weight mirror: rows in groups of 16, K in units of 64 (FP4) or 32 (FP8 /
// Int8) elements; each 512-byte unit holds, for every lane of a warp, the codes of its
// mma.m16n8k16 A fragments for 4 (FP4) or 2 (FP8 / Int8) consecutive 16-wide K blocks.
// Units are ordered [row set of 4 row groups][K unit][row group in the set]: a warp that
// streams a K range of one 64-row set reads one contiguous run of bytes (DRAM rows are
// opened once per 2 KB instead of once per 512-byte unit). Row groups are padded to a
// multiple of 4 with zero codes.
struct TiledGeom {
  static constexpr int kSetGroups = 4;
  int64_t row_groups = 0;   // ceil(rows / 16)
  int64_t units_k = 0;      // K units per row group
  int unit_k = 0;           // elements of K per unit (64 or 32)
  int64_t row_sets() const { return (row_groups + kSetGroups - 1) / kSetGroups; }
  int64_t bytes() const { return row_sets() * kSetGroups * units_k * 512; }
};

TiledGeom tiled_geom(DType dt, int rows, int cols);
bool gemv_tc_supported(DType dt);

// Build the tiled mirror from reference-layout native bytes (FP8 codes canonicalised).
Status build_tiled_mirror(DType dt, const uint8_t* native, int rows, int cols, uint8_t* tiled, cudaStream_t st);

// Tokens per launch: up to 16 for one layer (5..8: two n8 tiles of x per A fragment; 9..16:
// four, with x prepared once per K segment by a small kernel and two row groups per warp), up
// to 4 for the fused Gate/Up (SwiGLU) form and for grouped launches.
constexpr int kGemvMaxBatch = 16;
// Whether the tensor GEMV takes `batch` tokens of this layer (9..16 tokens: the prepared
// fragments of a CTA's K range must fit in shared memory, which bounds K).
bool gemv_tc_fits(DType dt, int rows, int cols, int batch);
// Device scratch a session of this batch gives the GEMV for prepared x fragments (0: none).
size_t gemv_prep_bytes(DType dt, int rows, int cols, int batch);

struct GemvTcArgs {
  DType dtype = DType::FP4;
  const uint8_t* Wt = nullptr;   // tiled mirror
  const uint8_t* Wt2 = nullptr;  // SwiGLU Up (same geometry) or nullptr
  int rows = 0, cols = 0;
  float scale = 1.0f, scale2 = 1.0f;  // Int8 per-tensor scales
  const float* x = nullptr;      // [batch][x_ld], any alignment
  int64_t x_ld = 0;
  int batch = 1;                 // 1..8 (1..4 with Wt2)
  float* pre = nullptr;          // [batch][ld_out]  (SwiGLU: h)
  float* post = nullptr;
  int64_t ld_out = 0;
  const double* bias = nullptr;
  int bias_len = 0;
  int act = -1;
  PeerOut peers;                 // further destinations of post (column-sharded layers)
  void* prep = nullptr;          // gemv_prep_bytes of device scratch (required for 9..16 tokens)
};

// Launches on `st` with a thread-block cluster per 64-row set (split-K reduced in
// distributed shared memory); with pdl=true it may overlap the previous kernel (weights are
// prefetched before griddepcontrol.wait; x is read and outputs written after it).
Status launch_gemv_tc(const GemvTcArgs& a, cudaStream_t st, bool pdl);

// Independent layers of one shape and dtype in one launch (blockIdx.z = layer): the same
// kernel over a grid that fills the GPU, for several forwards that do not depend on each
// other (parallel projections, layers of different sequences). Launches of at most
// kGemvGroupMax layers each; every layer reads its own x and writes its own outputs.
struct GemvGroupLayer {
  const uint8_t* Wt = nullptr;   // tiled mirror
  const float* x = nullptr;      // [batch][x_ld]
  float* pre = nullptr;          // [batch][ld_out]
  float* post = nullptr;
  const double* bias = nullptr;
  int bias_len = 0;
  int act = -1;
  float scale = 1.0f;            // Int8 per-tensor scale
  void* prep = nullptr;          // gemv_group_prep_bytes of device scratch (required)
};
constexpr int kGemvGroupMax = 32;
// Device bytes a grouped layer needs to have its x prepared once: its f16 B fragments and
// per-K-segment scales. A grouped launch first runs a small kernel that prepares each
// layer's x, then the GEMV, whose CTAs (one per 64 rows) read the fragments instead of each
// staging x and building them.
size_t gemv_group_prep_bytes(DType dt, int rows, int cols, int batch);
// `peers` (may be nullptr): further destinations of post, applied to every layer of the launch
// (used with one layer, by column-sharded layers).
Status launch_gemv_tc_group(DType dt, int rows, int cols, int batch, int64_t x_ld, int64_t ld_out,
                            const GemvGroupLayer* layers, int n, cudaStream_t st, bool pdl,
                            const PeerOut* peers = nullptr);
// Whether one layer runs faster as a one-layer grouped launch (x prepared once by a small kernel,
// longer K ranges per CTA) than with the single-layer plan: layers whose grouped plan still fills
// the GPU with CTAs (WELVET_B200_GEMV_PREP=1 / 0 forces the choice). Batches of 1..4.
bool gemv_prefers_prepared(DType dt, int rows, int cols, int batch);

} // namespace wb
