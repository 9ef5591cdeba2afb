// comm.cpp -- NCCL communicator (loaded at run time) and CUDA-IPC peer buffers.
#include "comm.hpp"

#include <dlfcn.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>

namespace wb {

namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclBroadcast) broadcast = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
};

const NcclApi& nccl_api() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* env = std::getenv("WELVET_B200_NCCL");
    const char* name = env && *env ? env : "libnccl.so.2";
    void* h = dlopen(name, RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      const char* e = dlerror();
      api.why = std::string("cannot load ") + name + (e ? std::string(": ") + e : std::string());
      return;
    }
    bool all = true;
    auto sym = [&](auto& fn, const char* s) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, s));
      if (!fn) {
        all = false;
        api.why = std::string("NCCL lacks ") + s;
      }
    };
    sym(api.get_unique_id, "ncclGetUniqueId");
    sym(api.init_rank, "ncclCommInitRank");
    sym(api.destroy, "ncclCommDestroy");
    sym(api.all_gather, "ncclAllGather");
    sym(api.broadcast, "ncclBroadcast");
    sym(api.send, "ncclSend");
    sym(api.recv, "ncclRecv");
    sym(api.group_start, "ncclGroupStart");
    sym(api.group_end, "ncclGroupEnd");
    sym(api.error_string, "ncclGetErrorString");
    api.ok = all;
  });
  return api;
}

Status nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return Status::Ok();
  const NcclApi& a = nccl_api();
  return Status::Internal(std::string(what) + ": " + (a.error_string ? a.error_string(r) : "NCCL error"));
}

Status need_nccl() {
  const NcclApi& a = nccl_api();
  if (!a.ok) return Status::Unsupported("multi-GPU needs NCCL: " + a.why);
  return Status::Ok();
}

Status check_comm(Comm* c) {
  if (!c) return Status::Invalid("null communicator");
  WB_TRY(need_nccl());
  return cuda_status(cudaSetDevice(c->device), "cudaSetDevice");
}

} // namespace

bool nccl_available() { return nccl_api().ok; }

Comm::~Comm() {
  cudaSetDevice(device);
  if (stream) cudaStreamSynchronize(stream);
  if (nccl && nccl_available()) nccl_api().destroy(nccl);
  if (stream) cudaStreamDestroy(stream);
}

Status comm_unique_id(uint8_t* id128) {
  if (!id128) return Status::Invalid("null unique id buffer");
  WB_TRY(need_nccl());
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  ncclUniqueId id;
  WB_TRY(nccl_status(nccl_api().get_unique_id(&id), "ncclGetUniqueId"));
  std::memcpy(id128, &id, sizeof(id));
  return Status::Ok();
}

Status comm_create(const uint8_t* id128, int nranks, int rank, int device, Comm** out) {
  if (!id128 || !out) return Status::Invalid("null communicator arguments");
  if (nranks < 1 || rank < 0 || rank >= nranks) return Status::Invalid("communicator: rank out of range");
  WB_TRY(need_nccl());
  int count = 0;
  WB_CUDA(cudaGetDeviceCount(&count));
  if (device < 0 || device >= count) return Status::Invalid("communicator: device out of range");
  WB_CUDA(cudaSetDevice(device));
  auto* c = new Comm();
  c->nranks = nranks;
  c->rank = rank;
  c->device = device;
  Status st = cuda_status(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream");
  if (st.ok()) {
    ncclUniqueId id;
    std::memcpy(&id, id128, sizeof(id));
    st = nccl_status(nccl_api().init_rank(&c->nccl, nranks, id, rank), "ncclCommInitRank");
    if (!st.ok()) c->nccl = nullptr;
  }
  if (!st.ok()) {
    delete c;
    return st;
  }
  *out = c;
  return Status::Ok();
}

Status comm_allgather_host(Comm* c, const void* send, size_t n, void* recv) {
  WB_TRY(check_comm(c));
  if (n == 0) return Status::Ok();
  if (!send || !recv) return Status::Invalid("null all-gather buffers");
  uint8_t* d = nullptr;
  const size_t total = n * static_cast<size_t>(c->nranks);
  WB_CUDA(cudaMalloc(&d, total + n));
  Status st = cuda_status(cudaMemcpyAsync(d + total, send, n, cudaMemcpyHostToDevice, c->stream), "H2D");
  if (st.ok()) st = nccl_status(nccl_api().all_gather(d + total, d, n, ncclUint8, c->nccl, c->stream), "ncclAllGather");
  if (st.ok()) st = cuda_status(cudaMemcpyAsync(recv, d, total, cudaMemcpyDeviceToHost, c->stream), "D2H");
  if (st.ok()) st = cuda_status(cudaStreamSynchronize(c->stream), "all-gather sync");
  cudaFree(d);
  return st;
}

Status comm_allgather_f32(Comm* c, const float* send, float* recv, size_t count, cudaStream_t st) {
  WB_TRY(check_comm(c));
  return nccl_status(nccl_api().all_gather(send, recv, count, ncclFloat32, c->nccl, st), "ncclAllGather");
}

Status comm_send_f32(Comm* c, const float* buf, size_t count, int peer, cudaStream_t st) {
  WB_TRY(check_comm(c));
  return nccl_status(nccl_api().send(buf, count, ncclFloat32, peer, c->nccl, st), "ncclSend");
}

Status comm_recv_f32(Comm* c, float* buf, size_t count, int peer, cudaStream_t st) {
  WB_TRY(check_comm(c));
  return nccl_status(nccl_api().recv(buf, count, ncclFloat32, peer, c->nccl, st), "ncclRecv");
}

Status comm_broadcast_f32(Comm* c, float* buf, size_t count, int root, cudaStream_t st) {
  WB_TRY(check_comm(c));
  return nccl_status(nccl_api().broadcast(buf, buf, count, ncclFloat32, root, c->nccl, st), "ncclBroadcast");
}

void PeerBuffer::release() {
  if (ptr.empty() && !local) return;
  cudaSetDevice(device);
  cudaDeviceSynchronize();
  for (size_t r = 0; r < ptr.size(); ++r)
    if (ptr[r] && ptr[r] != local) cudaIpcCloseMemHandle(ptr[r]);
  if (local) cudaFree(local);
  local = nullptr;
  ptr.clear();
  bytes = 0;
}

Status peer_buffer_create(Comm* c, size_t bytes, PeerBuffer* out) {
  WB_TRY(check_comm(c));
  if (!out || bytes == 0) return Status::Invalid("peer buffer: bad arguments");
  out->release();
  out->device = c->device;
  out->bytes = bytes;
  WB_CUDA(cudaMalloc(&out->local, bytes));
  WB_CUDA(cudaMemset(out->local, 0, bytes));
  out->ptr.assign(static_cast<size_t>(c->nranks), nullptr);
  out->ptr[static_cast<size_t>(c->rank)] = out->local;
  if (c->nranks == 1) return Status::Ok();
  cudaIpcMemHandle_t mine;
  WB_CUDA(cudaIpcGetMemHandle(&mine, out->local));
  std::vector<cudaIpcMemHandle_t> all(static_cast<size_t>(c->nranks));
  WB_TRY(comm_allgather_host(c, &mine, sizeof(mine), all.data()));
  for (int r = 0; r < c->nranks; ++r) {
    if (r == c->rank) continue;
    void* p = nullptr;
    WB_CUDA(cudaIpcOpenMemHandle(&p, all[static_cast<size_t>(r)], cudaIpcMemLazyEnablePeerAccess));
    out->ptr[static_cast<size_t>(r)] = p;
  }
  return Status::Ok();
}

} // namespace wb
