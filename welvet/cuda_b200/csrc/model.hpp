// model.hpp -- persistent model sessions over a stored model descriptor (WMN1).
//
// Reference interface mirrored: welvet_model_mount / welvet_model_forward /
// welvet_model_release (src/interop/model_session.cpp:317-410), the descriptor layout of
// include/welvet/interop/child_wire.hpp (children) and model_wire.hpp:195-263 (controls), and
// the store section read_store (model_session.cpp:135-153). Served here: Stack (root 0) and
// Grid (root 2) models whose children are Dense, RMSNorm, SwiGLU and MHA, mounted from the
// stores' native bytes into a device-resident volume (volume.hpp); other roots and child
// kinds are gaps (status 3), dtypes off the quantized forward path unsupported (status 2).
#pragma once

#include "volume.hpp"

#include <mutex>
#include <vector>

namespace wb {

struct ModelSession {
  std::mutex mu;          // one forward at a time, as the reference's per-session lock
  int root = 0;           // 0 Stack, 2 Grid
  Volume* vol = nullptr;
  std::vector<int> mha;   // flat indices of MHA cells: tokens per sequence follow the input
  bool dense = false;     // an enabled Dense cell: inputs must be [batch, in]
  int max_width = 0;      // widest cell output (forward output buffer)
  float* x_dev = nullptr;
  float* y_dev = nullptr;
  size_t x_cap = 0, y_cap = 0;  // floats
  ~ModelSession();
};

// The descriptor bytes are read during the call; nothing is retained.
Status model_mount(const uint8_t* desc, size_t size, ModelSession** out);
// input: a tensor record (int32 rank 1..5, int32 dims, float32 data); `out` receives the output
// tensor record of the last executed cell.
Status model_forward(ModelSession* s, const uint8_t* input, size_t size, std::vector<uint8_t>* out);

} // namespace wb
