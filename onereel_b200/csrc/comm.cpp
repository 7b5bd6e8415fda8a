// NCCL wrappers of the C ABI: the collectives of the multi-GPU scene path (K/V exchange, broadcast of rows every peer
// reads, Ulysses all-to-all, all-reduce) on a caller-given CUDA stream, with a timeout-aware wait.
//
// Replaces the torch.distributed calls of the reference's src/onereel/parallel/comm.py (HaloExchange 126-201:
// batch_isend_irecv of K then V per interval and peer; a2a_heads / a2a_tokens 276-295: all_to_all_single;
// dist.all_reduce of the text rows) for callers that drive the path from C / C++ without a Python process group.
// NCCL is loaded at the first call with dlopen("libnccl.so.2"): a process that already loaded NCCL (PyTorch does)
// shares that copy, and the library itself links without NCCL. Every function returns an ORL_* status; no NCCL or
// CUDA error crosses the ABI as anything else.
//
// Waiting: orl_comm_wait polls the stream (cudaStreamQuery) and the communicator's asynchronous error
// (ncclCommGetAsyncError) until the stream is idle, an error appears or timeout_ns passes; on an error or a timeout
// it aborts the communicator (ncclCommAbort ends the communicator's in-flight operations) and returns ORL_ERR_COMM /
// ORL_ERR_TIMEOUT, so a rank whose peer died does not wait forever.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <new>
#include <thread>

#include "orl_common.h"

namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclCommAbort) abort = nullptr;
  decltype(&ncclCommGetAsyncError) async_error = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  decltype(&ncclBroadcast) broadcast = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) return;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      return fn != nullptr;
    };
    api.ok = sym(api.get_unique_id, "ncclGetUniqueId") && sym(api.init_rank, "ncclCommInitRank") &&
             sym(api.destroy, "ncclCommDestroy") && sym(api.abort, "ncclCommAbort") &&
             sym(api.async_error, "ncclCommGetAsyncError") && sym(api.group_start, "ncclGroupStart") &&
             sym(api.group_end, "ncclGroupEnd") && sym(api.send, "ncclSend") && sym(api.recv, "ncclRecv") &&
             sym(api.broadcast, "ncclBroadcast") && sym(api.all_reduce, "ncclAllReduce");
  });
  return api;
}

}  // namespace

struct orl_comm {
  ncclComm_t nc = nullptr;
  int world = 0, rank = 0, device = 0;
  bool aborted = false;
};

static int comm_usable(const orl_comm* c) {
  if (c == nullptr || c->nc == nullptr) return ORL_ERR_ARG;
  if (c->aborted) return ORL_ERR_COMM;
  return nccl().ok ? ORL_OK : ORL_ERR_DRIVER;
}

extern "C" int orl_comm_available(void) { return nccl().ok ? 1 : 0; }

extern "C" int orl_comm_unique_id(uint8_t* id_out) {
  if (id_out == nullptr) return ORL_ERR_ARG;
  const NcclApi& api = nccl();
  if (!api.ok) return ORL_ERR_DRIVER;
  ncclUniqueId id;
  if (api.get_unique_id(&id) != ncclSuccess) return ORL_ERR_COMM;
  std::memcpy(id_out, id.internal, NCCL_UNIQUE_ID_BYTES);
  return ORL_OK;
}

extern "C" int orl_comm_init(orl_comm** out, const uint8_t* id, int world, int rank, int device) {
  if (out == nullptr || id == nullptr || world <= 0 || rank < 0 || rank >= world || device < 0) return ORL_ERR_ARG;
  *out = nullptr;
  const NcclApi& api = nccl();
  if (!api.ok) return ORL_ERR_DRIVER;
  if (cudaSetDevice(device) != cudaSuccess) return ORL_ERR_LAUNCH;
  ncclUniqueId uid;
  std::memcpy(uid.internal, id, NCCL_UNIQUE_ID_BYTES);
  auto* c = new (std::nothrow) orl_comm;
  if (c == nullptr) return ORL_ERR_CAPACITY;
  if (api.init_rank(&c->nc, world, uid, rank) != ncclSuccess) {
    delete c;
    return ORL_ERR_COMM;
  }
  c->world = world;
  c->rank = rank;
  c->device = device;
  *out = c;
  return ORL_OK;
}

extern "C" int orl_comm_destroy(orl_comm* c) {
  if (c == nullptr) return ORL_ERR_ARG;
  int rc = ORL_OK;
  if (c->nc != nullptr && nccl().ok && !c->aborted)
    rc = nccl().destroy(c->nc) == ncclSuccess ? ORL_OK : ORL_ERR_COMM;
  delete c;
  return rc;
}

extern "C" int orl_comm_exchange(orl_comm* c, const orl_p2p* sends, int n_send, const orl_p2p* recvs, int n_recv,
                                 void* stream_ptr) {
  int rc = comm_usable(c);
  if (rc != ORL_OK) return rc;
  if (n_send < 0 || n_recv < 0 || (n_send > 0 && sends == nullptr) || (n_recv > 0 && recvs == nullptr))
    return ORL_ERR_ARG;
  for (int i = 0; i < n_send + n_recv; ++i) {
    const orl_p2p& p = i < n_send ? sends[i] : recvs[i - n_send];
    if (p.peer < 0 || p.peer >= c->world || p.peer == c->rank || p.bytes < 0 || (p.bytes > 0 && p.ptr == nullptr))
      return ORL_ERR_ARG;
  }
  const NcclApi& api = nccl();
  cudaStream_t s = static_cast<cudaStream_t>(stream_ptr);
  // one NCCL group: per peer, the operations keep their list order on both sides (K then V of each interval)
  if (api.group_start() != ncclSuccess) return ORL_ERR_COMM;
  bool bad = false;
  for (int i = 0; i < n_send && !bad; ++i)
    if (sends[i].bytes > 0)
      bad = api.send(sends[i].ptr, static_cast<size_t>(sends[i].bytes), ncclUint8, sends[i].peer, c->nc, s) !=
            ncclSuccess;
  for (int i = 0; i < n_recv && !bad; ++i)
    if (recvs[i].bytes > 0)
      bad = api.recv(recvs[i].ptr, static_cast<size_t>(recvs[i].bytes), ncclUint8, recvs[i].peer, c->nc, s) !=
            ncclSuccess;
  const bool end_bad = api.group_end() != ncclSuccess;
  return (bad || end_bad) ? ORL_ERR_COMM : ORL_OK;
}

extern "C" int orl_comm_broadcast(orl_comm* c, void* buf, long long bytes, int root, void* stream_ptr) {
  int rc = comm_usable(c);
  if (rc != ORL_OK) return rc;
  if (bytes < 0 || (bytes > 0 && buf == nullptr) || root < 0 || root >= c->world) return ORL_ERR_ARG;
  if (bytes == 0) return ORL_OK;
  return nccl().broadcast(buf, buf, static_cast<size_t>(bytes), ncclUint8, root, c->nc,
                          static_cast<cudaStream_t>(stream_ptr)) == ncclSuccess
             ? ORL_OK
             : ORL_ERR_COMM;
}

extern "C" int orl_comm_all_to_all(orl_comm* c, const void* send, void* recv, long long bytes_per_peer,
                                   void* stream_ptr) {
  int rc = comm_usable(c);
  if (rc != ORL_OK) return rc;
  if (bytes_per_peer < 0 || (bytes_per_peer > 0 && (send == nullptr || recv == nullptr))) return ORL_ERR_ARG;
  if (bytes_per_peer == 0) return ORL_OK;
  const NcclApi& api = nccl();
  cudaStream_t s = static_cast<cudaStream_t>(stream_ptr);
  const size_t n = static_cast<size_t>(bytes_per_peer);
  // block p of send goes to rank p, block p of recv comes from rank p (all_to_all_single with equal splits); the
  // rank's own block is copied on the stream
  if (cudaMemcpyAsync(static_cast<uint8_t*>(recv) + c->rank * n, static_cast<const uint8_t*>(send) + c->rank * n, n,
                      cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return ORL_ERR_LAUNCH;
  if (api.group_start() != ncclSuccess) return ORL_ERR_COMM;
  bool bad = false;
  for (int p = 0; p < c->world && !bad; ++p) {
    if (p == c->rank) continue;
    bad = api.send(static_cast<const uint8_t*>(send) + p * n, n, ncclUint8, p, c->nc, s) != ncclSuccess ||
          api.recv(static_cast<uint8_t*>(recv) + p * n, n, ncclUint8, p, c->nc, s) != ncclSuccess;
  }
  const bool end_bad = api.group_end() != ncclSuccess;
  return (bad || end_bad) ? ORL_ERR_COMM : ORL_OK;
}

extern "C" int orl_comm_all_reduce_f32(orl_comm* c, float* buf, long long n, void* stream_ptr) {
  int rc = comm_usable(c);
  if (rc != ORL_OK) return rc;
  if (n < 0 || (n > 0 && buf == nullptr)) return ORL_ERR_ARG;
  if (n == 0) return ORL_OK;
  return nccl().all_reduce(buf, buf, static_cast<size_t>(n), ncclFloat32, ncclSum, c->nc,
                           static_cast<cudaStream_t>(stream_ptr)) == ncclSuccess
             ? ORL_OK
             : ORL_ERR_COMM;
}

extern "C" int orl_comm_wait(orl_comm* c, void* stream_ptr, unsigned long long timeout_ns) {
  int rc = comm_usable(c);
  if (rc != ORL_OK) return rc;
  const NcclApi& api = nccl();
  cudaStream_t s = static_cast<cudaStream_t>(stream_ptr);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) return ORL_OK;
    if (q != cudaErrorNotReady) return ORL_ERR_LAUNCH;
    ncclResult_t async = ncclSuccess;
    if (api.async_error(c->nc, &async) != ncclSuccess || (async != ncclSuccess && async != ncclInProgress)) {
      api.abort(c->nc);
      c->aborted = true;
      return ORL_ERR_COMM;
    }
    const auto waited = std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0);
    if (static_cast<unsigned long long>(waited.count()) > timeout_ns) {
      api.abort(c->nc);             // ends the communicator's in-flight operations; the stream then drains
      c->aborted = true;
      return ORL_ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}
