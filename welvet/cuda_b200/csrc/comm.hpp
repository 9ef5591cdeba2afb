// comm.hpp -- the library's multi-GPU plumbing: one process per GPU, an NCCL communicator over
// the ranks of one box, and peer memory (CUDA IPC over NVLink) for kernels that write straight
// into other ranks' buffers.
//
// The reference has no multi-GPU code (device 0 is hard-coded, src/cuda/device.cpp:40-61); this
// is new capability behind additive welvet_b200_comm_* entry points. NCCL is loaded at run time
// (dlopen of libnccl.so.2, or WELVET_B200_NCCL): a process that already holds an NCCL (a host
// application that loaded torch, for instance) shares that copy, and the library still loads
// where no NCCL is installed (comm calls then return status 2).
#pragma once

#include "common.hpp"

#include <nccl.h>

#include <vector>

namespace wb {

struct Comm {
  int nranks = 1;
  int rank = 0;
  int device = 0;
  ncclComm_t nccl = nullptr;
  cudaStream_t stream = nullptr;  // the library's own stream for bootstrap exchanges
  ~Comm();
};

// ncclGetUniqueId: 128 bytes that rank 0 creates and every rank passes to comm_create.
Status comm_unique_id(uint8_t* id128);
// A communicator of `nranks` processes, this one being `rank` on CUDA device `device`
// (collective: every rank calls it with the same id).
Status comm_create(const uint8_t* id128, int nranks, int rank, int device, Comm** out);

// All-gather of `n` bytes per rank through the communicator (host buffers, synchronous):
// recv holds nranks * n bytes, rank r's at r * n.
Status comm_allgather_host(Comm* c, const void* send, size_t n, void* recv);

// Device all-gather of `count` floats per rank on `st` (rank-major in `recv`).
Status comm_allgather_f32(Comm* c, const float* send, float* recv, size_t count, cudaStream_t st);
// Point-to-point float transfers on `st`.
Status comm_send_f32(Comm* c, const float* buf, size_t count, int peer, cudaStream_t st);
Status comm_recv_f32(Comm* c, float* buf, size_t count, int peer, cudaStream_t st);
Status comm_broadcast_f32(Comm* c, float* buf, size_t count, int root, cudaStream_t st);

// Device memory whose address every rank knows: `local` is this rank's cudaMalloc'd buffer,
// `ptr[r]` the address under which this process reaches rank r's buffer (ptr[rank] == local),
// opened through CUDA IPC (peer access over NVLink). Collective over the communicator.
struct PeerBuffer {
  int device = 0;
  size_t bytes = 0;
  void* local = nullptr;
  std::vector<void*> ptr;
  void release();
  ~PeerBuffer() { release(); }
};
Status peer_buffer_create(Comm* c, size_t bytes, PeerBuffer* out);

// True when NCCL could be loaded into this process.
bool nccl_available();

} // namespace wb
