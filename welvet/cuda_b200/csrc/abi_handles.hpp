// abi_handles.hpp -- the opaque handle types of include/welvet_b200.h, shared by the ABI files.
#pragma once

#include "../../../include/welvet_b200.h"

#include "comm.hpp"
#include "sharded.hpp"
#include "volume.hpp"

struct welvet_b200_volume {
  wb::Volume* v;
};
struct welvet_b200_comm {
  wb::Comm* c;
};
struct welvet_b200_sharded_dense {
  wb::ShardedDense* s;
};
