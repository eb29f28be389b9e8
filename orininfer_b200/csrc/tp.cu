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
//
// orin_tp_enable_p2p gives a communicator a peer-memory region (one
// cudaMalloc per rank, mapped by every peer through CUDA IPC; the handles
// travel over the communicator itself): row-parallel calls that fit then
// reduce with the kernel of tp_p2p.cu instead of ncclAllReduce.
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
  // peer-memory reduction (orin_tp_enable_p2p)
  bool p2p = false;
  long long p2p_cap = 0;               // partial-sum elements the region holds
  char* region = nullptr;              // flags | fp32 partial | 16-bit result
  char* peer_region[kP2PMaxRanks] = {};
  int* state = nullptr;                // per-block epochs (kP2PMaxBlocks ints)
};

constexpr long long align256(long long b) { return (b + 255) & ~255LL; }
long long p2p_partial_off() { return kP2PFlagBytes; }
long long p2p_result_off(long long cap) { return kP2PFlagBytes + align256(cap * 4); }

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

int orin::tp_comm_device(const void* comm) { return static_cast<const TpComm*>(comm)->device; }

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
  if (!c || !C || M < 1 || N < 1) {
    set_error("orin_tp_linear_row: null communicator or output, or non-positive size");
    return ORIN_ERR_INVALID_ARG;
  }
  const bool aligned = (reinterpret_cast<uintptr_t>(C) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(residual) % 16 == 0);
  if (c->p2p && static_cast<long long>(M) * N <= c->p2p_cap && N % 8 == 0 && aligned) {
    float* part = reinterpret_cast<float*>(c->region + p2p_partial_off());
    orin_status st = orin_linear(part, A_shard, W_shard, M, N, K_shard, dtype,
                                 ORIN_EPI_F32_PARTIAL, nullptr, stream);
    if (st != ORIN_OK) return st;
    cudaError_t e = cudaSuccess;
    DeviceCtx* ctx = device_ctx(c->device, &e);
    if (!ctx) {
      set_error("orin_tp_linear_row: device set-up: %s", cudaGetErrorString(e));
      return ORIN_ERR_CUDA;
    }
    P2PView v = {};
    v.rank = c->rank;
    v.world = c->world;
    v.N = N;
    for (int r = 0; r <= c->world; ++r)
      v.row0[r] = static_cast<long long>(r) * M / c->world;
    for (int r = 0; r < c->world; ++r) {
      char* base = (r == c->rank) ? c->region : c->peer_region[r];
      v.partial[r] = reinterpret_cast<const float*>(base + p2p_partial_off());
      v.result[r] = base + p2p_result_off(c->p2p_cap);
      v.flags[r] = reinterpret_cast<int*>(base);
    }
    v.local_flags = reinterpret_cast<int*>(c->region);
    v.result_local = c->region + p2p_result_off(c->p2p_cap);
    v.C = C;
    v.R = residual;
    v.epoch = c->state;
    v.err = ctx->err;
    e = launch_p2p_reduce(v, dtype, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
      set_error("orin_tp_linear_row: peer-memory reduction: %s", cudaGetErrorString(e));
      return ORIN_ERR_CUDA;
    }
    return ORIN_OK;
  }
  if (!partial_f32) {
    set_error("orin_tp_linear_row: null partial buffer (needed unless the peer-memory "
              "reduction is enabled and the problem fits it)");
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

orin_status orin_tp_lm_head_argmax(void* comm, int* token, const void* h, const void* W_shard,
                                   int M, int V_shard, int v_offset, int K, int dtype,
                                   unsigned long long* keys, void* stream) {
  TpComm* c = static_cast<TpComm*>(comm);
  if (!c || !token || !h || !W_shard || !keys || M < 1 || V_shard < 1 || K < 1 || v_offset < 0 ||
      (dtype != ORIN_F16 && dtype != ORIN_BF16)) {
    set_error("orin_tp_lm_head_argmax: bad arguments");
    return ORIN_ERR_INVALID_ARG;
  }
  if (static_cast<long long>(v_offset) + V_shard > 0x7fffffffLL) {
    set_error("orin_tp_lm_head_argmax: vocabulary positions beyond 2^31");
    return ORIN_ERR_UNSUPPORTED;
  }
  if (K % 8 != 0 || reinterpret_cast<uintptr_t>(h) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(W_shard) % 16 != 0) {
    set_error("orin_tp_lm_head_argmax: needs K %% 8 == 0 and 16-byte aligned h and W_shard");
    return ORIN_ERR_UNSUPPORTED;
  }
  if (c->aborted) {
    set_error("orin_tp_lm_head_argmax: communicator was aborted");
    return ORIN_ERR_NCCL;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_argmax_keys(keys, h, W_shard, M, V_shard, K, dtype, v_offset, s);
  if (e != cudaSuccess) {
    set_error("orin_tp_lm_head_argmax: %s", cudaGetErrorString(e));
    return ORIN_ERR_CUDA;
  }
  // the keys order (value, tie-break) globally: the best of the ranks' bests
  ncclResult_t r = ncclAllReduce(keys, keys, static_cast<size_t>(M), ncclUint64, ncclMax, c->comm,
                                 s);
  orin_status st = settle(c, r, "orin_tp_lm_head_argmax: ncclAllReduce");
  if (st != ORIN_OK) return st;
  e = launch_argmax_decode(token, keys, M, s);
  if (e != cudaSuccess) {
    set_error("orin_tp_lm_head_argmax: %s", cudaGetErrorString(e));
    return ORIN_ERR_CUDA;
  }
  return ORIN_OK;
}

orin_status orin_p2p_watchdog_selftest(void* stream) {
  // A two-rank view on one GPU whose "peer" is a plain buffer: the reduction
  // kernel signals into it and waits on a local flag that nothing sets, so
  // its bounded wait must give up and record DEVERR_TIMEOUT_PEER.
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  DeviceCtx* ctx = (e == cudaSuccess) ? device_ctx(dev, &e) : nullptr;
  if (!ctx) {
    set_error("orin_p2p_watchdog_selftest: device set-up: %s", cudaGetErrorString(e));
    return ORIN_ERR_CUDA;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  constexpr int M = 2, N = 8;
  char* buf = nullptr;
  const size_t flags_b = kP2PFlagBytes, part_b = 256, epoch_b = kP2PMaxBlocks * sizeof(int);
  const size_t total = 2 * flags_b + 4 * part_b + epoch_b;
  if ((e = cudaMalloc(&buf, total)) != cudaSuccess) {
    set_error("orin_p2p_watchdog_selftest: cudaMalloc: %s", cudaGetErrorString(e));
    return ORIN_ERR_CUDA;
  }
  cudaMemset(buf, 0, total);
  P2PView v = {};
  v.rank = 0;
  v.world = 2;
  v.N = N;
  v.row0[0] = 0;
  v.row0[1] = 1;
  v.row0[2] = M;
  char* p = buf;
  v.flags[0] = reinterpret_cast<int*>(p);      // this rank's flags: nothing writes them
  v.local_flags = v.flags[0];
  p += flags_b;
  v.flags[1] = reinterpret_cast<int*>(p);      // the "peer": receives our signal only
  p += flags_b;
  v.partial[0] = reinterpret_cast<const float*>(p);
  v.partial[1] = reinterpret_cast<const float*>(p + part_b);
  v.result[0] = p + 2 * part_b;
  v.result[1] = p + 2 * part_b;
  v.result_local = p + 2 * part_b;
  v.C = p + 3 * part_b;
  v.R = nullptr;
  p += 4 * part_b;
  v.epoch = reinterpret_cast<int*>(p);
  v.err = ctx->err;
  e = launch_p2p_reduce(v, ORIN_F16, s);
  cudaError_t e2 = cudaStreamSynchronize(s);
  cudaFree(buf);
  if (e != cudaSuccess || e2 != cudaSuccess) {
    set_error("orin_p2p_watchdog_selftest: %s",
              cudaGetErrorString(e != cudaSuccess ? e : e2));
    return ORIN_ERR_CUDA;
  }
  return ORIN_OK;
}

orin_status orin_tp_enable_p2p(void* comm, long long max_elems, void* stream) {
  TpComm* c = static_cast<TpComm*>(comm);
  if (!c || max_elems < 8) {
    set_error("orin_tp_enable_p2p: null communicator or max_elems < 8");
    return ORIN_ERR_INVALID_ARG;
  }
  if (c->aborted) {
    set_error("orin_tp_enable_p2p: communicator was aborted");
    return ORIN_ERR_NCCL;
  }
  if (c->p2p) {
    if (max_elems <= c->p2p_cap) return ORIN_OK;
    set_error("orin_tp_enable_p2p: already enabled for %lld elements", c->p2p_cap);
    return ORIN_ERR_UNSUPPORTED;
  }
  if (c->world > kP2PMaxRanks) {
    set_error("orin_tp_enable_p2p: %d ranks; at most %d", c->world, kP2PMaxRanks);
    return ORIN_ERR_UNSUPPORTED;
  }
  cudaError_t e = cudaSetDevice(c->device);
  const long long bytes = p2p_result_off(max_elems) + align256(max_elems * 2);
  char* region = nullptr;
  int* state = nullptr;
  char* dbuf = nullptr;
  cudaIpcMemHandle_t handles[kP2PMaxRanks];
  orin_status st = ORIN_OK;
  auto fail = [&](orin_status code, const char* what) {
    set_error("orin_tp_enable_p2p: %s: %s", what, cudaGetErrorString(e));
    st = code;
  };
  if (e != cudaSuccess) fail(ORIN_ERR_CUDA, "cudaSetDevice");
  if (st == ORIN_OK && (e = cudaMalloc(&region, bytes)) != cudaSuccess) fail(ORIN_ERR_CUDA, "cudaMalloc");
  if (st == ORIN_OK && (e = cudaMalloc(&state, kP2PMaxBlocks * sizeof(int))) != cudaSuccess)
    fail(ORIN_ERR_CUDA, "cudaMalloc");
  if (st == ORIN_OK) {
    // flags and counters are zero before any peer can learn where they are
    cudaMemset(region, 0, kP2PFlagBytes);
    cudaMemset(state, 0, kP2PMaxBlocks * sizeof(int));
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) fail(ORIN_ERR_CUDA, "zeroing the flags");
  }
  if (st == ORIN_OK && (e = cudaIpcGetMemHandle(&handles[c->rank], region)) != cudaSuccess)
    fail(ORIN_ERR_UNSUPPORTED, "cudaIpcGetMemHandle");
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  if (st == ORIN_OK && (e = cudaMalloc(&dbuf, hb * c->world)) != cudaSuccess)
    fail(ORIN_ERR_CUDA, "cudaMalloc");
  if (st == ORIN_OK &&
      (e = cudaMemcpy(dbuf + hb * c->rank, &handles[c->rank], hb, cudaMemcpyHostToDevice)) !=
          cudaSuccess)
    fail(ORIN_ERR_CUDA, "cudaMemcpy");
  if (st == ORIN_OK) {
    ncclResult_t r = ncclAllGather(dbuf + hb * c->rank, dbuf, hb, ncclUint8, c->comm,
                                   static_cast<cudaStream_t>(stream));
    st = settle(c, r, "orin_tp_enable_p2p: handle exchange");
    if (st == ORIN_OK) st = orin_tp_wait(c, stream);
  }
  if (st == ORIN_OK &&
      (e = cudaMemcpy(handles, dbuf, hb * c->world, cudaMemcpyDeviceToHost)) != cudaSuccess)
    fail(ORIN_ERR_CUDA, "cudaMemcpy");
  for (int p = 0; st == ORIN_OK && p < c->world; ++p) {
    if (p == c->rank) continue;
    void* ptr = nullptr;
    e = cudaIpcOpenMemHandle(&ptr, handles[p], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      fail(ORIN_ERR_UNSUPPORTED, "cudaIpcOpenMemHandle (no peer access between these GPUs?)");
      break;
    }
    c->peer_region[p] = static_cast<char*>(ptr);
  }
  if (dbuf) cudaFree(dbuf);
  if (st != ORIN_OK) {
    for (int p = 0; p < c->world; ++p)
      if (c->peer_region[p]) cudaIpcCloseMemHandle(c->peer_region[p]), c->peer_region[p] = nullptr;
    if (region) cudaFree(region);
    if (state) cudaFree(state);
    return st;
  }
  c->region = region;
  c->state = state;
  c->p2p_cap = max_elems;
  c->p2p = true;
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
  if (c->p2p) {
    cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    // no peer may still read this rank's region: one collective step first
    if (!c->aborted) {
      int* one = nullptr;
      if (cudaMalloc(&one, sizeof(int)) == cudaSuccess) {
        cudaMemset(one, 0, sizeof(int));
        ncclResult_t r = ncclAllReduce(one, one, 1, ncclInt32, ncclSum, c->comm, nullptr);
        if (settle(c, r, "orin_tp_destroy barrier") == ORIN_OK) orin_tp_wait(c, nullptr);
        cudaFree(one);
      }
    }
    for (int p = 0; p < c->world; ++p)
      if (c->peer_region[p]) cudaIpcCloseMemHandle(c->peer_region[p]);
    cudaFree(c->region);
    cudaFree(c->state);
    c->p2p = false;
  }
  if (c->comm && !c->aborted) {
    ncclResult_t r = ncclCommFinalize(c->comm);
    st = settle(c, r, "ncclCommFinalize");
    if (!c->aborted) ncclCommDestroy(c->comm);
  }
  delete c;
  return st;
}

}  // extern "C"
