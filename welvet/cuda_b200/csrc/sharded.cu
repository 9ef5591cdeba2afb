// sharded.cu -- column-sharded Dense over the GPUs of a box, and the cell-per-GPU volume
// pipeline (see sharded.hpp).
#include "sharded.hpp"

#include "volume.hpp"

#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace wb {

namespace {

constexpr int kMaxRanks = kMaxPeerOut + 1;

struct FlagPtrs {
  uint32_t* p[kMaxRanks];
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The flag exchange that closes a fused sharded forward (one warp). The exchange number lives
// in device memory (*count, this rank's exchanges so far), so that a captured CUDA graph of the
// call counts correctly on every replay. Thread s (s != rank) publishes the new number in rank
// s's flag slot `rank` -- after a system-scope fence, so that every store this rank's forward
// made into rank s's buffers (the kernels before this one on the stream) is visible there
// first -- and then waits until rank s has published the same number here. The wait is
// bounded: past `limit_ns` it records bit 0 in *err and gives up. Launched as a programmatic
// dependent of the forward's last kernel: it is resident early and starts the moment that
// kernel's grid has completed and its stores are visible (griddepcontrol.wait). It lets its
// own dependents launch at once: the next call's kernels start streaming their weights while
// this exchange waits, and wait themselves for its completion before touching any output.
__global__ void k_flag_exchange(FlagPtrs peers, const uint32_t* mine, uint32_t* count, int nranks, int rank,
                                int* err, unsigned long long limit_ns) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int s = threadIdx.x;
  const uint32_t epoch = *count + 1u;  // read by every lane before lane 0 updates it below
  if (s < nranks && s != rank) {
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peers.p[s] + rank), "r"(epoch) : "memory");
    const uint64_t t0 = global_ns();
    while (true) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine + s) : "memory");
      if (static_cast<int32_t>(v - epoch) >= 0) break;
      if (global_ns() - t0 > limit_ns) {
        atomicOr(err, 1);
        break;
      }
      __nanosleep(128);
    }
  }
  __syncwarp();
  if (s == 0) *count = epoch;
}

struct ShardGeom {
  int begin[kMaxRanks];
  int len[kMaxRanks];
};

// NCCL mode: the rank-major gathered shards [nranks][batch][smax] -> [batch][out].
__global__ void k_unshard(const float* __restrict__ g, float* __restrict__ out, int nranks, int batch, int smax,
                          int cols, ShardGeom geo) {
  const int64_t total = static_cast<int64_t>(nranks) * batch * smax;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t per = static_cast<int64_t>(batch) * smax;
    const int r = static_cast<int>(i / per);
    const int64_t rem = i - r * per;
    const int b = static_cast<int>(rem / smax);
    const int j = static_cast<int>(rem - static_cast<int64_t>(b) * smax);
    if (j < geo.len[r]) out[static_cast<int64_t>(b) * cols + geo.begin[r] + j] = g[i];
  }
}

unsigned long long wait_limit_ns() {
  const char* env = std::getenv("WELVET_B200_SHARD_WAIT_MS");
  long ms = env && *env ? std::atol(env) : 5000;
  if (ms < 1) ms = 1;
  return static_cast<unsigned long long>(ms) * 1000000ull;
}

template <typename T>
void free_dev(T*& p) {
  if (p) cudaFree(p);
  p = nullptr;
}

} // namespace

void shard_rows(int rows, int nranks, int rank, int* begin, int* end) {
  if (rows <= 0 || nranks <= 0 || rank < 0 || rank >= nranks) {
    *begin = *end = 0;
    return;
  }
  const int64_t blocks = (static_cast<int64_t>(rows) + 127) / 128;
  const int64_t b0 = blocks * rank / nranks, b1 = blocks * (rank + 1) / nranks;
  const int64_t r0 = b0 * 128, r1 = b1 * 128 < rows ? b1 * 128 : rows;
  *begin = static_cast<int>(r0 < rows ? r0 : rows);
  *end = static_cast<int>(r1);
}

void stage_plan(int cells, int lpc, int nranks, int rank, int* hop_begin, int* hop_end) {
  if (cells <= 0 || lpc <= 0 || nranks <= 0 || rank < 0 || rank >= nranks) {
    *hop_begin = *hop_end = 0;
    return;
  }
  int c0, c1;
  if (nranks <= cells) {
    c0 = static_cast<int>(static_cast<int64_t>(cells) * rank / nranks);
    c1 = static_cast<int>(static_cast<int64_t>(cells) * (rank + 1) / nranks);
  } else {
    c0 = rank < cells ? rank : cells;
    c1 = rank + 1 < cells ? rank + 1 : cells;
  }
  *hop_begin = c0 * lpc;
  *hop_end = c1 * lpc;
}

ShardedDense::~ShardedDense() {
  cudaSetDevice(device);
  if (stream) cudaStreamSynchronize(stream);
  cudaDeviceSynchronize();
  outbuf[0].release();
  outbuf[1].release();
  flags.release();
  free_dev(pre_local);
  free_dev(err);
  free_dev(shard_post);
  free_dev(shard_pre);
  free_dev(gathered);
  free_dev(out_nccl);
  free_dev(x_dev);
  io.release();
  dev.release();
  if (stream) cudaStreamDestroy(stream);
}

Status sharded_mount(Comm* comm, int batch, int in, int out, int act, DType dt, const float* W_rows, bool w_dev,
                     const double* bias, size_t bias_len, GatherMode mode, ShardedDense** s_out) {
  if (!comm || !s_out) return Status::Invalid("null sharded mount args");
  if (batch <= 0 || in <= 0 || out <= 0) return Status::Invalid("sharded dense: bad dims");
  if (!dtype_on_path(static_cast<int32_t>(dt)))
    return Status::Unsupported(std::string("sharded dense: unsupported dtype id ") +
                               std::to_string(static_cast<int32_t>(dt)));
  if (!activation_valid(act)) return Status::Invalid("sharded dense: bad activation");
  if (mode != GatherMode::Fused && mode != GatherMode::Nccl) return Status::Invalid("sharded dense: bad mode");
  if (comm->nranks > kMaxRanks) return Status::Unsupported("sharded dense: at most 8 ranks");
  WB_CUDA(cudaSetDevice(comm->device));
  auto* s = new ShardedDense();
  s->comm = comm;
  s->device = comm->device;
  s->batch = batch;
  s->in = in;
  s->out = out;
  s->act = act;
  s->mode = mode;
  shard_rows(out, comm->nranks, comm->rank, &s->row_begin, &s->row_end);
  for (int r = 0; r < comm->nranks; ++r) {
    int b, e;
    shard_rows(out, comm->nranks, r, &b, &e);
    if (e - b > s->shard_max) s->shard_max = e - b;
  }
  s->pre_is_post = act == -1 && (bias == nullptr || bias_len == 0);
  const int rows = s->row_end - s->row_begin;
  auto fail = [&](Status st) {
    delete s;
    return st;
  };
  Status st = cuda_status(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "stream");
  if (!st.ok()) return fail(st);
  if (rows > 0) {
    if (!W_rows) return fail(Status::Invalid("sharded dense: null weights"));
    // the layer's bias applies to rows o < bias_len (src/cuda/kernels.cu:152-160): this
    // shard's part of it, in local row numbers
    const double* lb = nullptr;
    size_t lbl = 0;
    if (bias && bias_len > static_cast<size_t>(s->row_begin)) {
      lb = bias + s->row_begin;
      lbl = bias_len - static_cast<size_t>(s->row_begin);
      if (lbl > static_cast<size_t>(rows)) lbl = static_cast<size_t>(rows);
    }
    st = mount_dense(s->device, rows, in, dt, act, W_rows, w_dev, lb, lbl, &s->store, &s->dev, s->stream, batch);
    if (st.ok()) st = alloc_io(s->dev, batch, &s->io, s->stream);
    if (!st.ok()) return fail(st);
  }
  const size_t ybytes = static_cast<size_t>(batch) * static_cast<size_t>(out) * 4;
  if (mode == GatherMode::Fused) {
    for (auto& b : s->outbuf) {
      st = peer_buffer_create(comm, ybytes, &b);
      if (!st.ok()) return fail(st);
    }
    st = peer_buffer_create(comm, static_cast<size_t>(comm->nranks) * sizeof(uint32_t), &s->flags);
    if (!st.ok()) return fail(st);
    if (!s->pre_is_post) {
      st = cuda_status(cudaMalloc(&s->pre_local, ybytes), "cudaMalloc");
      if (st.ok()) st = cuda_status(cudaMemset(s->pre_local, 0, ybytes), "cudaMemset");
      if (!st.ok()) return fail(st);
    }
  } else {
    const size_t sb = static_cast<size_t>(batch) * static_cast<size_t>(s->shard_max) * 4;
    st = cuda_status(cudaMalloc(&s->shard_post, sb), "cudaMalloc");
    if (st.ok()) st = cuda_status(cudaMalloc(&s->shard_pre, sb), "cudaMalloc");
    if (st.ok()) st = cuda_status(cudaMemset(s->shard_post, 0, sb), "cudaMemset");
    if (st.ok()) st = cuda_status(cudaMalloc(&s->gathered, sb * static_cast<size_t>(comm->nranks)), "cudaMalloc");
    if (st.ok()) st = cuda_status(cudaMalloc(&s->out_nccl, ybytes), "cudaMalloc");
    if (st.ok() && !s->pre_is_post) {
      st = cuda_status(cudaMalloc(&s->pre_local, ybytes), "cudaMalloc");
      if (st.ok()) st = cuda_status(cudaMemset(s->pre_local, 0, ybytes), "cudaMemset");
    }
    if (!st.ok()) return fail(st);
  }
  st = cuda_status(cudaMalloc(&s->err, 2 * sizeof(int)), "cudaMalloc");
  if (st.ok()) st = cuda_status(cudaMemset(s->err, 0, 2 * sizeof(int)), "cudaMemset");
  s->count = reinterpret_cast<uint32_t*>(s->err + 1);
  if (st.ok())
    st = cuda_status(cudaMalloc(&s->x_dev, static_cast<size_t>(batch) * static_cast<size_t>(in) * 4), "cudaMalloc");
  if (st.ok()) st = cuda_status(cudaDeviceSynchronize(), "mount sync");
  if (!st.ok()) return fail(st);
  *s_out = s;
  return Status::Ok();
}

Status sharded_execute_device(ShardedDense* s, const float* x, cudaStream_t st, const float** post,
                              const float** pre) {
  if (!s || !x) return Status::Invalid("null sharded execute args");
  WB_CUDA(cudaSetDevice(s->device));
  Comm* c = s->comm;
  const int rows = s->row_end - s->row_begin;
  if (s->mode == GatherMode::Fused) {
    const int parity = static_cast<int>(s->epoch & 1u);
    PeerBuffer& ob = s->outbuf[parity];
    float* y = static_cast<float*>(ob.local);
    float* ypre = s->pre_is_post ? y : s->pre_local;
    if (rows > 0) {
      PeerOut peers;
      for (int r = 0; r < c->nranks; ++r)
        if (r != c->rank) peers.post[peers.n++] = static_cast<float*>(ob.ptr[static_cast<size_t>(r)]) + s->row_begin;
      // a programmatic dependent of whatever precedes it on the stream (the previous call's
      // flag exchange): its first kernel waits for that kernel's completion before reading x
      WB_TRY(forward_device(s->dev, s->batch, x, s->in, ypre + s->row_begin, y + s->row_begin, &s->io, st, true,
                            s->out, &peers));
    }
    ++s->epoch;
    if (c->nranks > 1) {
      FlagPtrs fp{};
      for (int r = 0; r < c->nranks; ++r) fp.p[r] = static_cast<uint32_t*>(s->flags.ptr[static_cast<size_t>(r)]);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1);
      cfg.blockDim = dim3(32);
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = rows > 0 ? 1 : 0;
      WB_CUDA(cudaLaunchKernelEx(&cfg, k_flag_exchange, fp, static_cast<const uint32_t*>(s->flags.local), s->count,
                                 c->nranks, c->rank, s->err, wait_limit_ns()));
    }
    if (post) *post = y;
    if (pre) *pre = ypre;
    return Status::Ok();
  }
  // NCCL baseline: local forward into [batch][shard_max], all-gather, permute
  if (rows > 0)
    WB_TRY(forward_device(s->dev, s->batch, x, s->in, s->shard_pre, s->shard_post, &s->io, st, false, s->shard_max));
  WB_TRY(comm_allgather_f32(c, s->shard_post, s->gathered,
                            static_cast<size_t>(s->batch) * static_cast<size_t>(s->shard_max), st));
  ShardGeom geo{};
  for (int r = 0; r < c->nranks; ++r) {
    int b, e;
    shard_rows(s->out, c->nranks, r, &b, &e);
    geo.begin[r] = b;
    geo.len[r] = e - b;
  }
  const int64_t total = static_cast<int64_t>(c->nranks) * s->batch * s->shard_max;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  k_unshard<<<static_cast<unsigned>(blocks), 256, 0, st>>>(s->gathered, s->out_nccl, c->nranks, s->batch,
                                                           s->shard_max, s->out, geo);
  WB_CUDA(cudaGetLastError());
  if (!s->pre_is_post && rows > 0)
    WB_CUDA(cudaMemcpy2DAsync(s->pre_local + s->row_begin, static_cast<size_t>(s->out) * 4, s->shard_pre,
                              static_cast<size_t>(s->shard_max) * 4, static_cast<size_t>(rows) * 4,
                              static_cast<size_t>(s->batch), cudaMemcpyDeviceToDevice, st));
  if (post) *post = s->out_nccl;
  if (pre) *pre = s->pre_is_post ? s->out_nccl : s->pre_local;
  return Status::Ok();
}

Status sharded_check_error(ShardedDense* s, cudaStream_t st) {
  if (!s) return Status::Invalid("null sharded session");
  WB_CUDA(cudaSetDevice(s->device));
  int e = 0;
  WB_CUDA(cudaMemcpyAsync(&e, s->err, sizeof(int), cudaMemcpyDeviceToHost, st));
  WB_CUDA(cudaStreamSynchronize(st));
  if (e != 0) {
    WB_CUDA(cudaMemsetAsync(s->err, 0, sizeof(int), st));
    WB_CUDA(cudaStreamSynchronize(st));
    return Status::Internal("sharded dense: a rank did not reach the output exchange in time");
  }
  if (s->row_end > s->row_begin) return check_pipeline_error(s->io, st);
  return Status::Ok();
}

Status sharded_execute(ShardedDense* s, const float* x, float* pre, float* post) {
  if (!s || !x) return Status::Invalid("null sharded execute args");
  WB_CUDA(cudaSetDevice(s->device));
  const size_t xb = static_cast<size_t>(s->batch) * static_cast<size_t>(s->in) * 4;
  const size_t yb = static_cast<size_t>(s->batch) * static_cast<size_t>(s->out) * 4;
  WB_CUDA(cudaMemcpyAsync(s->x_dev, x, xb, cudaMemcpyHostToDevice, s->stream));
  const float *yd = nullptr, *pd = nullptr;
  WB_TRY(sharded_execute_device(s, s->x_dev, s->stream, &yd, &pd));
  if (post) WB_CUDA(cudaMemcpyAsync(post, yd, yb, cudaMemcpyDeviceToHost, s->stream));
  if (pre) WB_CUDA(cudaMemcpyAsync(pre, pd, yb, cudaMemcpyDeviceToHost, s->stream));
  return sharded_check_error(s, s->stream);
}

Status volume_pipeline_forward(Volume* v, Comm* comm, int hop_begin, int hop_end, int rows, const float* x,
                               int stage_in_width, int micro, float* out, int out_width, cudaStream_t st) {
  if (!v || !comm) return Status::Invalid("null pipeline args");
  if (rows <= 0 || micro <= 0 || stage_in_width <= 0 || out_width <= 0 || !out)
    return Status::Invalid("pipeline: bad sizes");
  if (comm->rank == 0 && !x) return Status::Invalid("pipeline: rank 0 needs the input");
  const int hops = volume_hops(*v);
  if (hop_begin < 0 || hop_end > hops || hop_begin > hop_end) return Status::Invalid("pipeline: bad hop range");
  // every remote link of this range must target a cell of the same range (its activation
  // lives on this GPU)
  for (int h = hop_begin; h < hop_end; ++h) {
    const VolumeCell& c = v->cells[static_cast<size_t>(h)];
    if (!c.disabled && c.remote && (c.target < hop_begin || c.target >= hop_end))
      return Status::Invalid("pipeline: remote link across GPUs at hop " + std::to_string(h));
  }
  WB_CUDA(cudaSetDevice(comm->device));
  const int rank = comm->rank, n = comm->nranks;
  // the receive buffer of this stage's input micro-batches
  float* recv = nullptr;
  if (rank > 0)
    WB_CUDA(cudaMallocAsync(&recv, static_cast<size_t>(micro) * static_cast<size_t>(stage_in_width) * 4, st));
  Status status = Status::Ok();
  for (int r0 = 0; r0 < rows && status.ok(); r0 += micro) {
    const int m = rows - r0 < micro ? rows - r0 : micro;
    const float* xin = rank == 0 ? x + static_cast<int64_t>(r0) * stage_in_width : recv;
    if (rank > 0) {
      status = comm_recv_f32(comm, recv, static_cast<size_t>(m) * stage_in_width, rank - 1, st);
      if (!status.ok()) break;
    }
    const float* y = xin;
    int yw = stage_in_width;
    if (hop_begin < hop_end) {
      status = volume_forward_range(v, m, xin, stage_in_width, hop_begin, hop_end, nullptr, &yw, st, true, &y);
      if (!status.ok()) break;
    }
    if (rank < n - 1) {
      status = comm_send_f32(comm, y, static_cast<size_t>(m) * yw, rank + 1, st);
    } else {
      if (yw != out_width) {
        status = Status::Invalid("pipeline: the last stage's width differs from out_width");
        break;
      }
      status = cuda_status(cudaMemcpyAsync(out + static_cast<int64_t>(r0) * out_width, y,
                                           static_cast<size_t>(m) * out_width * 4, cudaMemcpyDeviceToDevice, st),
                           "pipeline output copy");
    }
  }
  if (status.ok() && n > 1)
    status = comm_broadcast_f32(comm, out, static_cast<size_t>(rows) * out_width, n - 1, st);
  if (recv) cudaFreeAsync(recv, st);
  return status;
}

} // namespace wb
