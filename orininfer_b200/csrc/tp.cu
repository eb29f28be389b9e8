// tp.cu — tensor parallelism over NCCL (NVLink / NVSwitch on one node).
//
// Column-parallel projections (q/k/v, gate/up, LM head) need no exchange:
// each rank runs orin_linear on its weight shard.  Row-parallel projections
// (o_proj, down_proj, sharded along K) produce fp32 partial sums that are
// all-reduced in fp32 and then rounded once, with the residual added after
// the sum: the result equals the single-GPU round16(x + round16(acc)) up to
// fp32 summation order.  The reference is single-GPU (include/kv_cache.h:7)
// and has no counterpart for this file.
//
// Communicators are created non-blocking; every wait on NCCL or on the stream
// is bounded by the communicator's timeout, after which it is aborted and the
// call returns ORIN_ERR_TIMEOUT.
#include "orin_b200.h"
#include "orin_internal.h"

#include <chrono>
#include <nccl.h>
#include <string.h>
#include <thread>

using namespace orin;

namespace {

struct TpComm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, device = 0;
  double timeout_s = 30.0;
  bool aborted = false;
};

static_assert(sizeof(ncclUniqueId) == ORIN_TP_UNIQUE_ID_BYTES, "NCCL unique id size changed");

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

orin_status abort_comm(TpComm* c, const char* what) {
  if (c->comm && !c->aborted) {
    ncclCommAbort(c->comm);
    c->aborted = true;
  }
  set_error("%s: timed out after %.1f s; communicator aborted", what, c->timeout_s);
  return ORIN_ERR_TIMEOUT;
}

// Wait until the communicator has no operation in progress on the host side.
orin_status settle(TpComm* c, ncclResult_t r, const char* what) {
  if (r != ncclSuccess && r != ncclInProgress) {
    set_error("%s: %s", what, ncclGetErrorString(r));
    return ORIN_ERR_NCCL;
  }
  const double t0 = now_s();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t q = ncclCommGetAsyncError(c->comm, &st);
    if (q != ncclSuccess) {
      set_error("%s: ncclCommGetAsyncError: %s", what, ncclGetErrorString(q));
      return ORIN_ERR_NCCL;
    }
    if (st == ncclSuccess) return ORIN_OK;
    if (st != ncclInProgress) {
      set_error("%s: %s", what, ncclGetErrorString(st));
      return ORIN_ERR_NCCL;
    }
    if (now_s() - t0 > c->timeout_s) return abort_comm(c, what);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace

extern "C" {

orin_status orin_tp_unique_id(void* id_out) {
  if (!id_out) {
    set_error("orin_tp_unique_id: null output");
    return ORIN_ERR_INVALID_ARG;
  }
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) {
    set_error("ncclGetUniqueId: %s", ncclGetErrorString(r));
    return ORIN_ERR_NCCL;
  }
  memcpy(id_out, &id, sizeof(id));
  return ORIN_OK;
}

orin_status orin_tp_init(void** comm_out, const void* id, int rank, int world_size, int device,
                         double timeout_s) {
  if (!comm_out || !id || world_size < 1 || rank < 0 || rank >= world_size || device < 0 ||
      !(timeout_s > 0)) {
    set_error("orin_tp_init: bad arguments (rank %d of %d, device %d, timeout %g)", rank,
              world_size, device, timeout_s);
    return ORIN_ERR_INVALID_ARG;
  }
  *comm_out = nullptr;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    set_error("orin_tp_init: cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
    return ORIN_ERR_CUDA;
  }
  TpComm* c = new TpComm;
  c->rank = rank;
  c->world = world_size;
  c->device = device;
  c->timeout_s = timeout_s;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = ncclCommInitRankConfig(&c->comm, world_size, uid, rank, &cfg);
  orin_status st = settle(c, r, "orin_tp_init");
  if (st != ORIN_OK) {
    if (c->comm && !c->aborted) ncclCommAbort(c->comm);
    delete c;
    return st;
  }
  *comm_out = c;
  return ORIN_OK;
}

orin_status orin_tp_allreduce_f32(void* comm, float* buf, long long n, void* stream) {
  TpComm* c = static_cast<TpComm*>(comm);
  if (!c || !buf || n < 0) {
    set_error("orin_tp_allreduce_f32: bad arguments");
    return ORIN_ERR_INVALID_ARG;
  }
  if (c->aborted) {
    set_error("orin_tp_allreduce_f32: communicator was aborted");
    return ORIN_ERR_NCCL;
  }
  if (n == 0) return ORIN_OK;
  ncclResult_t r = ncclAllReduce(buf, buf, static_cast<size_t>(n), ncclFloat32, ncclSum, c->comm,
                                 static_cast<cudaStream_t>(stream));
  return settle(c, r, "ncclAllReduce");
}

orin_status orin_tp_linear_row(void* comm, void* C, const void* A_shard, const void* W_shard,
                               int M, int N, int K_shard, int dtype, const void* residual,
                               float* partial_f32, void* stream) {
  TpComm* c = static_cast<TpComm*>(comm);
  if (!c || !C || !partial_f32) {
    set_error("orin_tp_linear_row: null communicator, output or partial buffer");
    return ORIN_ERR_INVALID_ARG;
  }
  orin_status st = orin_linear(partial_f32, A_shard, W_shard, M, N, K_shard, dtype,
                               ORIN_EPI_F32_PARTIAL, nullptr, stream);
  if (st != ORIN_OK) return st;
  st = orin_tp_allreduce_f32(comm, partial_f32, static_cast<long long>(M) * N, stream);
  if (st != ORIN_OK) return st;
  cudaError_t e = launch_finish_rows(C, partial_f32, residual, static_cast<long long>(M) * N,
                                     dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("orin_tp_linear_row: finish kernel: %s", cudaGetErrorString(e));
    return ORIN_ERR_CUDA;
  }
  return ORIN_OK;
}

orin_status orin_tp_wait(void* comm, void* stream) {
  TpComm* c = static_cast<TpComm*>(comm);
  if (!c) {
    set_error("orin_tp_wait: null communicator");
    return ORIN_ERR_INVALID_ARG;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const double t0 = now_s();
  for (;;) {
    cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) return ORIN_OK;
    if (q != cudaErrorNotReady) {
      set_error("orin_tp_wait: %s", cudaGetErrorString(q));
      return ORIN_ERR_CUDA;
    }
    ncclResult_t st = ncclSuccess;
    ncclCommGetAsyncError(c->comm, &st);
    if (st != ncclSuccess && st != ncclInProgress) {
      set_error("orin_tp_wait: NCCL async error: %s", ncclGetErrorString(st));
      ncclCommAbort(c->comm);
      c->aborted = true;
      return ORIN_ERR_NCCL;
    }
    if (now_s() - t0 > c->timeout_s) return abort_comm(c, "orin_tp_wait");
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

orin_status orin_tp_destroy(void* comm) {
  TpComm* c = static_cast<TpComm*>(comm);
  if (!c) return ORIN_OK;
  orin_status st = ORIN_OK;
  if (c->comm && !c->aborted) {
    ncclResult_t r = ncclCommFinalize(c->comm);
    st = settle(c, r, "ncclCommFinalize");
    if (!c->aborted) ncclCommDestroy(c->comm);
  }
  delete c;
  return st;
}

}  // extern "C"
