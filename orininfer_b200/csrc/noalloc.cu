// noalloc.cu — orin_tp_linear_row_static: the row-parallel linear of tp.cu
// with its fp32 partial-sum scratch in a file-scope device array instead of a
// caller buffer, so a caller that must not allocate device memory (nor keep a
// scratch buffer of its own) can still run the row-parallel path.
//
// The array is part of this translation unit's module: the driver places one
// copy on every device that loads the module.  Its device address is looked
// up with cudaGetSymbolAddress once per device, on the first call there
// (under a mutex); nothing here calls cudaMalloc, cudaFree or any library
// function that allocates.  Problems whose M*N partial sums exceed the array
// are rejected with ORIN_ERR_UNSUPPORTED before any device work.
//
// Races: the array is one per device, shared by every call on that device.
// Two calls whose kernels can overlap on one device (different streams, or
// different communicators, without an ordering between them) write the same
// scratch and corrupt each other's sums; calls on one device must be ordered,
// e.g. issued on a single stream.  The first call on a device performs the
// look-up (it may load the module) and must happen outside stream capture; a
// first call made under capture is refused with ORIN_ERR_INVALID_ARG.  The
// array used is the one of the communicator's device, which must be the
// current device (the kernels run there).
#include "orin_b200.h"
#include "orin_internal.h"

#include <mutex>

using namespace orin;

namespace {

// 16 Mi floats = 64 MiB: M*N up to 16,777,216 (e.g. 4096 tokens x 4096 features).
constexpr long long kStaticPartialFloats = 16ll << 20;
static __device__ __align__(256) float g_tp_partial[kStaticPartialFloats];

constexpr int kMaxDevices = 64;
float* g_partial_addr[kMaxDevices] = {};
std::mutex g_partial_mutex;

// This device's address of g_tp_partial (looked up once per device, with the
// device current).  A look-up under stream capture is refused: it may load the
// module, which would invalidate the capture.
float* static_partial(int device, cudaStream_t s, orin_status* st, const char** why) {
  *st = ORIN_ERR_CUDA;
  if (device < 0 || device >= kMaxDevices) {
    *why = "device ordinal out of range";
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_partial_mutex);
  if (!g_partial_addr[device]) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone) {
      *st = ORIN_ERR_INVALID_ARG;
      *why = "the first call on a device looks the array up and must not be stream-captured; "
             "make one uncaptured call first";
      return nullptr;
    }
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_tp_partial);
    if (e != cudaSuccess) {
      *why = cudaGetErrorString(e);
      return nullptr;
    }
    g_partial_addr[device] = static_cast<float*>(p);
  }
  return g_partial_addr[device];
}

}  // namespace

long long orin_tp_static_partial_capacity(void) { return kStaticPartialFloats; }

orin_status orin_tp_linear_row_static(void* comm, void* C, const void* A_shard,
                                      const void* W_shard, int M, int N, int K_shard, int dtype,
                                      const void* residual, void* stream) {
  if (!comm || !C || !A_shard || !W_shard) {
    set_error("orin_tp_linear_row_static: null communicator or operand");
    return ORIN_ERR_INVALID_ARG;
  }
  if (M <= 0 || N <= 0 || K_shard <= 0) {
    set_error("orin_tp_linear_row_static: M, N and K_shard must be positive");
    return ORIN_ERR_INVALID_ARG;
  }
  if (static_cast<long long>(M) * N > kStaticPartialFloats) {
    set_error("orin_tp_linear_row_static: M*N = %lld partial sums exceed the static scratch "
              "of %lld floats; use orin_tp_linear_row with a caller buffer",
              static_cast<long long>(M) * N, kStaticPartialFloats);
    return ORIN_ERR_UNSUPPORTED;
  }
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) {
    set_error("orin_tp_linear_row_static: cudaGetDevice: %s", cudaGetErrorString(e));
    return ORIN_ERR_CUDA;
  }
  const int comm_device = tp_comm_device(comm);
  if (device != comm_device) {
    set_error("orin_tp_linear_row_static: the current device (%d) is not the communicator's "
              "(%d); make the communicator's device current", device, comm_device);
    return ORIN_ERR_INVALID_ARG;
  }
  const char* why = "";
  orin_status st = ORIN_OK;
  float* partial = static_partial(device, static_cast<cudaStream_t>(stream), &st, &why);
  if (!partial) {
    set_error("orin_tp_linear_row_static: static scratch look-up failed: %s", why);
    return st;
  }
  return orin_tp_linear_row(comm, C, A_shard, W_shard, M, N, K_shard, dtype, residual, partial,
                            stream);
}
