#pragma once
// welvet/cuda/matvec.hpp -- a Dense layer's device state. The reference keeps an fp64 mirror
// here (include/welvet/cuda/matvec.hpp:14-25); this library keeps the packed codes in its own
// session, so the struct is an opaque handle with the same name and the same role.

#ifndef WELVET_CXX_API
#define WELVET_CXX_API __attribute__((visibility("default")))
#endif

namespace welvet::cuda {

struct ResidentDense {
  void* session = nullptr;  // the layer's Dense session (packed device mirror, staging, graphs)
  void* cell = nullptr;     // a fused SwiGLU / MHA cell over this layer and its siblings
  int cell_kind = 0;        // 1 SwiGLU (held by Gate), 2 MHA (held by Q)
};

// Frees the device state (safe on an empty handle).
WELVET_CXX_API void resident_release(ResidentDense* r);

} // namespace welvet::cuda
