// ulysses.cu -- the sequence-parallel (Ulysses) exchange of the long-video DiT over NCCL, and
// the communicator management around it: non-blocking initialisation with a host deadline,
// asynchronous-error polling, and abort.
//
// The reference runs Wan on one device and has no collectives (crates/sketchpad-dit/src/wan.rs
// :489-573); splitting its 75,600-token sequence over P GPUs needs one exchange step around
// each self-attention: an all-to-all that turns [S/P tokens, H heads] into [S tokens, H/P
// heads] and back.  sp_ulysses_a2a is that all-to-all as grouped point-to-point transfers
// (chunk p of the send buffer goes to rank p, chunk p of the receive buffer comes from rank
// p), so a Rust or C++ host can run the sequence-parallel block without Python.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2; a copy already loaded into the process,
// e.g. by torch, is the one used), so the library links and loads on machines without it.
// NCCL only: no peer-memory library kernels and no TMA multicast take part in the exchange.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "common.cuh"

namespace sp {
namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*CommCount)(const ncclComm_t, int*) = nullptr;
  ncclResult_t (*CommUserRank)(const ncclComm_t, int*) = nullptr;
};

template <typename F>
bool bind(void* h, const char* name, F& fn) {
  fn = reinterpret_cast<F>(dlsym(h, name));
  return fn != nullptr;
}

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    // RTLD_NOLOAD first: reuse the NCCL the process already has (torch's), else load one
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      api.why = "libnccl.so.2 could not be loaded";
      return;
    }
    bool ok = bind(h, "ncclGetUniqueId", api.GetUniqueId) &&
              bind(h, "ncclCommInitRankConfig", api.CommInitRankConfig) &&
              bind(h, "ncclCommGetAsyncError", api.CommGetAsyncError) &&
              bind(h, "ncclCommAbort", api.CommAbort) &&
              bind(h, "ncclCommDestroy", api.CommDestroy) &&
              bind(h, "ncclCommFinalize", api.CommFinalize) &&
              bind(h, "ncclGroupStart", api.GroupStart) && bind(h, "ncclGroupEnd", api.GroupEnd) &&
              bind(h, "ncclSend", api.Send) && bind(h, "ncclRecv", api.Recv) &&
              bind(h, "ncclAllGather", api.AllGather) &&
              bind(h, "ncclGetErrorString", api.GetErrorString) &&
              bind(h, "ncclCommCount", api.CommCount) &&
              bind(h, "ncclCommUserRank", api.CommUserRank);
    if (!ok) {
      api.why = "libnccl.so.2 lacks a symbol this library needs (NCCL >= 2.18 required)";
      return;
    }
    api.ok = true;
  });
  return api;
}

int need_nccl() {
  const NcclApi& a = nccl();
  if (!a.ok) return set_error(SP_ERR_COMM, "NCCL unavailable: %s", a.why.c_str());
  return SP_OK;
}

bool nccl_dtype(int dt, ncclDataType_t* out) {
  switch (dt) {
    case SP_F32: *out = ncclFloat32; return true;
    case SP_F16: *out = ncclFloat16; return true;
    case SP_BF16: *out = ncclBfloat16; return true;
    default: return false;
  }
}

using Clock = std::chrono::steady_clock;

Clock::time_point deadline_after(double seconds) {
  return Clock::now() + std::chrono::microseconds((int64_t)(seconds * 1e6));
}

// Polls the communicator's asynchronous state until it leaves ncclInProgress or the deadline
// passes.  On an error or an expired deadline the communicator is aborted (every NCCL kernel
// and proxy thread of it stops) and SP_ERR_COMM is returned with `what` in the message.
int settle(ncclComm_t comm, Clock::time_point deadline, const char* what) {
  const NcclApi& a = nccl();
  ncclResult_t st = ncclInProgress;
  for (;;) {
    if (a.CommGetAsyncError(comm, &st) != ncclSuccess) st = ncclInternalError;
    if (st != ncclInProgress) break;
    if (Clock::now() > deadline) {
      a.CommAbort(comm);
      return set_error(SP_ERR_COMM, "%s: not complete by the deadline; communicator aborted", what);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
  if (st != ncclSuccess) {
    const char* msg = a.GetErrorString(st);
    a.CommAbort(comm);
    return set_error(SP_ERR_COMM, "%s: NCCL error %d (%s); communicator aborted", what, (int)st,
                     msg ? msg : "?");
  }
  return SP_OK;
}

}  // namespace
}  // namespace sp

extern "C" {

int sp_nccl_unique_id(void* id_out, size_t id_bytes) {
  using namespace sp;
  clear_error();
  if (!id_out || id_bytes < sizeof(ncclUniqueId))
    return set_error(SP_ERR_INVALID_ARG, "nccl unique id: need a buffer of %zu bytes",
                     sizeof(ncclUniqueId));
  if (int rc = need_nccl()) return rc;
  ncclUniqueId id;
  const ncclResult_t r = nccl().GetUniqueId(&id);
  if (r != ncclSuccess)
    return set_error(SP_ERR_COMM, "ncclGetUniqueId failed: %s", nccl().GetErrorString(r));
  std::memcpy(id_out, &id, sizeof(id));
  return SP_OK;
}

size_t sp_nccl_unique_id_bytes(void) { return sizeof(ncclUniqueId); }

int sp_nccl_comm_init(void** comm_out, int nranks, int rank, const void* id, double timeout_s) {
  using namespace sp;
  clear_error();
  if (!comm_out || !id || nranks < 1 || rank < 0 || rank >= nranks || !(timeout_s > 0))
    return set_error(SP_ERR_INVALID_ARG, "nccl comm init: bad arguments (nranks %d, rank %d)",
                     nranks, rank);
  *comm_out = nullptr;
  if (int rc = need_nccl()) return rc;
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // init and every call return at once; progress is polled below
  ncclComm_t comm = nullptr;
  const auto deadline = deadline_after(timeout_s);
  const ncclResult_t r = nccl().CommInitRankConfig(&comm, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (comm) nccl().CommAbort(comm);
    return set_error(SP_ERR_COMM, "ncclCommInitRankConfig failed: %s", nccl().GetErrorString(r));
  }
  if (int rc = settle(comm, deadline, "communicator initialisation")) return rc;
  *comm_out = comm;
  return SP_OK;
}

int sp_nccl_comm_poll(void* comm, int* nccl_status_out) {
  using namespace sp;
  clear_error();
  if (!comm || !nccl_status_out) return set_error(SP_ERR_INVALID_ARG, "nccl poll: bad arguments");
  if (int rc = need_nccl()) return rc;
  ncclResult_t st = ncclSuccess;
  if (nccl().CommGetAsyncError(static_cast<ncclComm_t>(comm), &st) != ncclSuccess)
    return set_error(SP_ERR_COMM, "ncclCommGetAsyncError failed");
  *nccl_status_out = (int)st;
  return SP_OK;
}

int sp_nccl_wait(void* comm, void* stream, double timeout_s) {
  using namespace sp;
  clear_error();
  if (!comm || !(timeout_s > 0)) return set_error(SP_ERR_INVALID_ARG, "nccl wait: bad arguments");
  if (int rc = need_nccl()) return rc;
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  const auto deadline = deadline_after(timeout_s);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (;;) {
    ncclResult_t st = ncclSuccess;
    nccl().CommGetAsyncError(c, &st);
    if (st != ncclSuccess && st != ncclInProgress) {
      nccl().CommAbort(c);
      return set_error(SP_ERR_COMM, "nccl wait: NCCL error %d (%s); communicator aborted",
                       (int)st, nccl().GetErrorString(st));
    }
    const cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) return SP_OK;
    if (q != cudaErrorNotReady)
      return set_error(SP_ERR_LAUNCH, "nccl wait: stream error %s", cudaGetErrorString(q));
    if (Clock::now() > deadline) {
      nccl().CommAbort(c);
      return set_error(SP_ERR_COMM, "nccl wait: stream not done by the deadline; communicator "
                                    "aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int sp_nccl_comm_abort(void* comm) {
  using namespace sp;
  clear_error();
  if (!comm) return set_error(SP_ERR_INVALID_ARG, "nccl abort: null communicator");
  if (int rc = need_nccl()) return rc;
  nccl().CommAbort(static_cast<ncclComm_t>(comm));
  return SP_OK;
}

int sp_nccl_comm_destroy(void* comm, double timeout_s) {
  using namespace sp;
  clear_error();
  if (!comm || !(timeout_s > 0)) return set_error(SP_ERR_INVALID_ARG, "nccl destroy: bad arguments");
  if (int rc = need_nccl()) return rc;
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  const auto deadline = deadline_after(timeout_s);
  ncclResult_t r = nccl().CommFinalize(c);
  if (r != ncclSuccess && r != ncclInProgress) {
    nccl().CommAbort(c);
    return set_error(SP_ERR_COMM, "ncclCommFinalize failed: %s; communicator aborted",
                     nccl().GetErrorString(r));
  }
  if (int rc = settle(c, deadline, "communicator finalisation")) return rc;
  nccl().CommDestroy(c);
  return SP_OK;
}

int sp_ulysses_a2a(const void* send, void* recv, int64_t count, int dtype, void* comm,
                   void* stream, double timeout_s) {
  using namespace sp;
  clear_error();
  ncclDataType_t dt;
  if (!send || !recv || !comm || count <= 0 || !(timeout_s > 0))
    return set_error(SP_ERR_INVALID_ARG, "ulysses all-to-all: bad arguments");
  if (!nccl_dtype(dtype, &dt)) return set_error(SP_ERR_DTYPE, "ulysses all-to-all: bad dtype");
  if (send == recv)
    return set_error(SP_ERR_INVALID_ARG, "ulysses all-to-all: send and recv must not alias");
  if (int rc = need_nccl()) return rc;
  const NcclApi& a = nccl();
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  int P = 0, me = 0;
  if (a.CommCount(c, &P) != ncclSuccess || a.CommUserRank(c, &me) != ncclSuccess || P < 1)
    return set_error(SP_ERR_COMM, "ulysses all-to-all: communicator not usable");
  const size_t es = (size_t)dtype_size(dtype);
  const size_t chunk = (size_t)count * es;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto deadline = deadline_after(timeout_s);
  // the rank's own chunk stays on the device: a plain copy, no NCCL traffic
  if (cudaMemcpyAsync(static_cast<char*>(recv) + me * chunk,
                      static_cast<const char*>(send) + me * chunk, chunk,
                      cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
    cudaGetLastError();
    return set_error(SP_ERR_LAUNCH, "ulysses all-to-all: local chunk copy failed");
  }
  if (P == 1) return SP_OK;
  ncclResult_t r = a.GroupStart();
  for (int p = 0; p < P && (r == ncclSuccess || r == ncclInProgress); ++p) {
    if (p == me) continue;
    r = a.Send(static_cast<const char*>(send) + p * chunk, (size_t)count, dt, p, c, s);
    if (r != ncclSuccess && r != ncclInProgress) break;
    r = a.Recv(static_cast<char*>(recv) + p * chunk, (size_t)count, dt, p, c, s);
  }
  const ncclResult_t e = a.GroupEnd();
  if ((r != ncclSuccess && r != ncclInProgress) || (e != ncclSuccess && e != ncclInProgress)) {
    a.CommAbort(c);
    return set_error(SP_ERR_COMM, "ulysses all-to-all: enqueue failed (%s); communicator aborted",
                     a.GetErrorString(r != ncclSuccess && r != ncclInProgress ? r : e));
  }
  // non-blocking communicator: wait (bounded) until the transfers are enqueued on `stream`
  return settle(c, deadline, "ulysses all-to-all enqueue");
}

int sp_nccl_all_gather(const void* send, void* recv, int64_t count, int dtype, void* comm,
                       void* stream, double timeout_s) {
  using namespace sp;
  clear_error();
  ncclDataType_t dt;
  if (!send || !recv || !comm || count <= 0 || !(timeout_s > 0))
    return set_error(SP_ERR_INVALID_ARG, "all-gather: bad arguments");
  if (!nccl_dtype(dtype, &dt)) return set_error(SP_ERR_DTYPE, "all-gather: bad dtype");
  if (int rc = need_nccl()) return rc;
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  const auto deadline = deadline_after(timeout_s);
  const ncclResult_t r =
      nccl().AllGather(send, recv, (size_t)count, dt, c, static_cast<cudaStream_t>(stream));
  if (r != ncclSuccess && r != ncclInProgress) {
    nccl().CommAbort(c);
    return set_error(SP_ERR_COMM, "all-gather: enqueue failed (%s); communicator aborted",
                     nccl().GetErrorString(r));
  }
  return settle(c, deadline, "all-gather enqueue");
}

}  // extern "C"
