// Stage hand-off over NCCL behind the C ABI (include/dial_cuda.h,
// dial_stage_comm_*).
//
// Replaces the reference's worker/client hand-off of the hidden state: the
// master serialises a tensor to bytes (RawTensor::from_tensor / to_tensor,
// dial-core/src/spm/proto/message.rs:147-165), frames it (:366-408) and sends it
// over TCP to the worker that owns the next layers (Client::forward_batch
// spm/client.rs:389-452, worker loop spm/worker.rs:645-765), with a D2H and an
// H2D copy at every stage boundary.  Here each pipeline link (stage s -> s+1,
// and the token ring from the last stage back to stage 0) is a two-rank NCCL
// communicator, and the hidden state moves device to device, enqueued on the
// caller's stream.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, reusing a copy the
// process already loaded), so the library loads on hosts without NCCL and
// returns DIAL_ERR_NCCL from these entry points there.  Communicators are
// created non-blocking: initialisation, the first transfer on a link (NCCL's
// connection set-up, which needs the peer's matching call) and teardown are
// polled against a host deadline and end in DIAL_ERR_TIMEOUT, with the
// communicator aborted, instead of hanging.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "common.cuh"

struct dial_stage_comm {
  ncclComm_t comm;
  int rank, nranks, device;
  double timeout_s;
  bool broken;  // aborted after an error or a timeout
};

namespace dial {
namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommFinalize)(ncclComm_t);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
  bool ok;
};

const NcclApi& nccl() {
  static NcclApi api = [] {
    NcclApi a{};
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the copy torch loaded, if any
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
    if (!h) return a;
    bool all = true;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      all = all && fn != nullptr;
    };
    sym(a.GetUniqueId, "ncclGetUniqueId");
    sym(a.CommInitRankConfig, "ncclCommInitRankConfig");
    sym(a.CommGetAsyncError, "ncclCommGetAsyncError");
    sym(a.CommAbort, "ncclCommAbort");
    sym(a.CommFinalize, "ncclCommFinalize");
    sym(a.CommDestroy, "ncclCommDestroy");
    sym(a.Send, "ncclSend");
    sym(a.Recv, "ncclRecv");
    sym(a.GetErrorString, "ncclGetErrorString");
    a.ok = all;
    return a;
  }();
  return api;
}

dial_status nccl_fail(ncclResult_t r, const char* what) {
  const NcclApi& n = nccl();
  return fail(DIAL_ERR_NCCL, "%s: %s", what, n.ok ? n.GetErrorString(r) : "NCCL unavailable");
}

using Clock = std::chrono::steady_clock;

// Polls the communicator until its pending operation has settled (ncclSuccess),
// failed, or the deadline passed; aborts it on failure or timeout.
dial_status settle(dial_stage_comm* c, Clock::time_point deadline, const char* what) {
  const NcclApi& n = nccl();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t r = n.CommGetAsyncError(c->comm, &st);
    if (r != ncclSuccess) st = r;
    if (st == ncclSuccess) return DIAL_OK;
    if (st != ncclInProgress) {
      n.CommAbort(c->comm);
      c->broken = true;
      return nccl_fail(st, what);
    }
    if (Clock::now() > deadline) {
      n.CommAbort(c->comm);
      c->broken = true;
      return fail(DIAL_ERR_TIMEOUT, "%s: no progress within %.1f s (peer missing?)", what, c->timeout_s);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

Clock::time_point deadline_of(const dial_stage_comm* c) {
  return Clock::now() + std::chrono::microseconds((int64_t)(c->timeout_s * 1e6));
}

dial_status check_comm(const dial_stage_comm* c, int peer) {
  if (!c) return fail(DIAL_ERR_INVALID_ARG, "null communicator");
  if (c->broken) return fail(DIAL_ERR_NCCL, "communicator was aborted after an earlier failure");
  if (peer < 0 || peer >= c->nranks) return fail(DIAL_ERR_INVALID_ARG, "peer %d out of range", peer);
  return DIAL_OK;
}

}  // namespace
}  // namespace dial

using namespace dial;

extern "C" {

dial_status dial_stage_comm_unique_id(uint8_t* id_out) {
  clear_error();
  if (!id_out) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  const NcclApi& n = nccl();
  if (!n.ok) return fail(DIAL_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  const ncclResult_t r = n.GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  static_assert(sizeof(id.internal) == DIAL_STAGE_COMM_ID_BYTES, "NCCL unique id size");
  std::memcpy(id_out, id.internal, DIAL_STAGE_COMM_ID_BYTES);
  return DIAL_OK;
}

dial_status dial_stage_comm_init(const uint8_t* unique_id, int rank, int nranks, int device,
                                 double timeout_s, dial_stage_comm** out) {
  clear_error();
  if (!unique_id || !out) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  *out = nullptr;
  if (nranks <= 0 || rank < 0 || rank >= nranks)
    return fail(DIAL_ERR_INVALID_ARG, "rank %d of %d is out of range", rank, nranks);
  if (!(timeout_s > 0.0)) return fail(DIAL_ERR_INVALID_ARG, "timeout_s must be positive");
  const NcclApi& n = nccl();
  if (!n.ok) return fail(DIAL_ERR_NCCL, "libnccl.so.2 could not be loaded");
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  ncclUniqueId id;
  std::memcpy(id.internal, unique_id, DIAL_STAGE_COMM_ID_BYTES);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // every wait below is polled against the deadline
  auto* c = new dial_stage_comm{nullptr, rank, nranks, device, timeout_s, false};
  const ncclResult_t r = n.CommInitRankConfig(&c->comm, nranks, id, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (c->comm) n.CommAbort(c->comm);
    delete c;
    return nccl_fail(r, "ncclCommInitRankConfig");
  }
  const dial_status s = settle(c, deadline_of(c), "ncclCommInitRankConfig");
  if (s != DIAL_OK) {
    delete c;
    return s;
  }
  *out = c;
  return DIAL_OK;
}

dial_status dial_stage_comm_send(dial_stage_comm* c, const void* buf, size_t bytes, int peer,
                                 dial_stream stream) {
  clear_error();
  dial_status s = check_comm(c, peer);
  if (s != DIAL_OK) return s;
  if (!buf && bytes) return fail(DIAL_ERR_INVALID_ARG, "null buffer");
  const NcclApi& n = nccl();
  const ncclResult_t r = n.Send(buf, bytes, ncclUint8, peer, c->comm, as_stream(stream));
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclSend");
  return settle(c, deadline_of(c), "ncclSend");  // the first transfer on a link connects it
}

dial_status dial_stage_comm_recv(dial_stage_comm* c, void* buf, size_t bytes, int peer,
                                 dial_stream stream) {
  clear_error();
  dial_status s = check_comm(c, peer);
  if (s != DIAL_OK) return s;
  if (!buf && bytes) return fail(DIAL_ERR_INVALID_ARG, "null buffer");
  const NcclApi& n = nccl();
  const ncclResult_t r = n.Recv(buf, bytes, ncclUint8, peer, c->comm, as_stream(stream));
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclRecv");
  return settle(c, deadline_of(c), "ncclRecv");
}

dial_status dial_stage_comm_wait(dial_stage_comm* c, dial_stream stream) {
  clear_error();
  dial_status s = check_comm(c, 0);
  if (s != DIAL_OK) return s;
  const auto deadline = deadline_of(c);
  for (;;) {
    const cudaError_t e = cudaStreamQuery(as_stream(stream));
    if (e == cudaSuccess) return settle(c, deadline, "stream wait");
    if (e != cudaErrorNotReady) return cuda_fail(e, "cudaStreamQuery");
    ncclResult_t st = ncclSuccess;
    nccl().CommGetAsyncError(c->comm, &st);
    if (st != ncclSuccess && st != ncclInProgress) {
      nccl().CommAbort(c->comm);
      c->broken = true;
      return nccl_fail(st, "stage transfer");
    }
    if (Clock::now() > deadline) {
      nccl().CommAbort(c->comm);
      c->broken = true;
      return fail(DIAL_ERR_TIMEOUT, "stage transfer did not complete within %.1f s", c->timeout_s);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

dial_status dial_stage_comm_destroy(dial_stage_comm* c) {
  clear_error();
  if (!c) return DIAL_OK;
  const NcclApi& n = nccl();
  dial_status s = DIAL_OK;
  if (!c->broken) {
    const ncclResult_t r = n.CommFinalize(c->comm);
    if (r != ncclSuccess && r != ncclInProgress) s = nccl_fail(r, "ncclCommFinalize");
    else s = settle(c, deadline_of(c), "ncclCommFinalize");
  }
  if (!c->broken) n.CommDestroy(c->comm);  // after an abort the communicator is already gone
  delete c;
  return s;
}

}  // extern "C"
