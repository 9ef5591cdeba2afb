// sharded.hpp -- a Dense layer split by output rows over the GPUs of one box (one process per
// GPU), its output all-gathered on every rank.
//
// The reference runs every Dense on device 0 (src/cuda/device.cpp:40-61) through
// dense::forward_f32 (src/layers/dense/dense.cpp:58-86); a layer larger than one GPU has no
// counterpart there. Here rank r holds the rows shard_rows(out, N, r) of the layer (whole
// 128-row blocks, so GEMM tiles never straddle two ranks) and computes its columns of
// y[batch][out] with the same kernels as a one-GPU layer. Two ways to gather:
//
//  * fused (default): the kernels' epilogues store each output of this rank's columns into
//    the gathered buffer of every rank at once -- their own, and the others' through CUDA IPC
//    peer memory over NVLink (bulk tensor stores of staged tiles, direct stores elsewhere) --
//    so the transfer overlaps the math tile by tile; a small kernel then exchanges one flag
//    per rank (release / acquire at system scope, bounded wait) so that every rank holds the
//    whole output when its stream passes it. Outputs alternate between two buffers by call
//    parity: a rank starts writing call i + 1 into the buffer of call i - 1 only after every
//    rank has passed call i's flag exchange, by which point each rank's stream has finished
//    whatever read call i - 1's output before call i. The exchange number is kept on the
//    device, so two consecutive calls captured in a CUDA graph (one per buffer) replay
//    correctly.
//  * nccl: the local forward into a [batch][rows of the shard] buffer, then ncclAllGather
//    (rank-major, shards padded to the largest) and a permute into [batch][out]: the library
//    baseline the fused form is measured against.
//
// pre equals post for a Linear layer without bias (the whole output then comes back as
// both); otherwise pre holds this rank's columns only (others zero) and post is gathered.
#pragma once

#include "comm.hpp"
#include "dense.hpp"

namespace wb {

// Rows [begin, end) of rank `rank` among `nranks`: whole 128-row blocks dealt as evenly as
// possible in rank order (ranks may get none when the layer has fewer blocks than ranks).
void shard_rows(int rows, int nranks, int rank, int* begin, int* end);

enum class GatherMode : int32_t { Fused = 0, Nccl = 1 };

struct ShardedDense {
  Comm* comm = nullptr;  // not owned
  int device = 0;
  int batch = 0, in = 0, out = 0, act = -1;
  int row_begin = 0, row_end = 0;  // this rank's rows
  int shard_max = 0;               // rows of the largest shard (NCCL padding)
  GatherMode mode = GatherMode::Fused;
  bool pre_is_post = false;        // Linear without bias
  cudaStream_t stream = nullptr;   // host-buffer execute
  WeightStore store;
  DeviceDense dev;
  DenseIO io;
  // fused
  PeerBuffer outbuf[2];            // gathered post [batch][out], by call parity
  PeerBuffer flags;                // uint32 [nranks], slot s written by rank s
  float* pre_local = nullptr;      // [batch][out], this rank's columns (when pre differs)
  uint32_t epoch = 0;              // calls so far (host): picks the output buffer
  int* err = nullptr;              // [0] flag-exchange timeout word, [1] = count
  uint32_t* count = nullptr;       // device: flag exchanges so far (graph replays count too)
  // nccl
  float* shard_post = nullptr;     // [batch][shard_max]
  float* shard_pre = nullptr;
  float* gathered = nullptr;       // [nranks][batch][shard_max]
  float* out_nccl = nullptr;       // [batch][out]
  // host-buffer execute staging
  float* x_dev = nullptr;          // [batch][in]
  ~ShardedDense();
};

Status sharded_mount(Comm* comm, int batch, int in, int out, int act, DType dt, const float* W_rows, bool w_dev,
                     const double* bias, size_t bias_len, GatherMode mode, ShardedDense** s_out);
// One forward of x (device, [batch][in], the same on every rank) on `st`: *post receives the
// device address of the whole output [batch][out] on this rank, *pre that of pre (see above).
// Collective: every rank makes the same calls in the same order.
Status sharded_execute_device(ShardedDense* s, const float* x, cudaStream_t st, const float** post,
                              const float** pre);
// Host buffers, synchronous: x [batch][in] in, pre / post [batch][out] out (may be nullptr).
Status sharded_execute(ShardedDense* s, const float* x, float* pre, float* post);
// Synchronizes `st` and reports (then clears) a flag exchange or pipeline wait that timed out.
Status sharded_check_error(ShardedDense* s, cudaStream_t st);

// The cell-per-GPU pipeline over a volume: this rank runs hops [hop_begin, hop_end) of
// `v` on micro-batches of `micro` rows; rank 0 reads x, every other rank receives its input
// rows from the rank before it and sends its output to the rank after it (NCCL point-to-point),
// the last rank's output is broadcast so that every rank gets out [rows][out_width].
struct Volume;
Status volume_pipeline_forward(Volume* v, Comm* comm, int hop_begin, int hop_end, int rows, const float* x,
                               int stage_in_width, int micro, float* out, int out_width, cudaStream_t st);
// Hop range of `rank`: whole cells, contiguous in hop order, split as evenly as possible.
void stage_plan(int cells, int layers_per_cell, int nranks, int rank, int* hop_begin, int* hop_end);

} // namespace wb
