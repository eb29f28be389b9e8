// api.cu — the C ABI (include/orin_b200.h): argument checks, kernel choice,
// per-device set-up and the elementwise entry points.
#include "orin_b200.h"
#include "orin_common.cuh"
#include "orin_internal.h"

#include <mutex>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

namespace orin {

namespace {
thread_local char g_err[512] = "";
std::mutex g_ctx_mu;
DeviceCtx g_ctx[64];
}  // namespace

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

// The device error word: kernels that give up a bounded wait record a code
// here (one copy per device; host code reaches it through its address).
__device__ int g_device_error_word;

bool device_ctx_ready(int device) {
  if (device < 0 || device >= 64) return false;
  std::lock_guard<std::mutex> lock(g_ctx_mu);
  return g_ctx[device].device == device;
}

DeviceCtx* device_ctx(int device, cudaError_t* e) {
  *e = cudaSuccess;
  if (device < 0 || device >= 64) {
    *e = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_ctx_mu);
  DeviceCtx& c = g_ctx[device];
  if (c.device == device) return &c;
  int sms = 0;
  if ((*e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
    return nullptr;
  int major = 0;
  if ((*e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device)) !=
      cudaSuccess)
    return nullptr;
  if (major != 10) {
    *e = cudaErrorNoKernelImageForDevice;
    return nullptr;
  }
  void* addr = nullptr;
  if ((*e = cudaGetSymbolAddress(&addr, g_device_error_word)) != cudaSuccess) return nullptr;
  c.sm_count = sms;
  c.err = static_cast<int*>(addr);
  c.device = device;
  return &c;
}

}  // namespace orin

using namespace orin;

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

orin_status cuda_fail(cudaError_t e, const char* what) {
  set_error("%s: %s", what, cudaGetErrorString(e));
  return ORIN_ERR_CUDA;
}

orin_status check_common(int dtype, int epi) {
  if (dtype != ORIN_F16 && dtype != ORIN_BF16) {
    set_error("dtype %d is not ORIN_F16 or ORIN_BF16", dtype);
    return ORIN_ERR_INVALID_ARG;
  }
  if (epi < ORIN_EPI_NONE || epi > ORIN_EPI_F32_PARTIAL) {
    set_error("epilogue %d is not an orin_epilogue", epi);
    return ORIN_ERR_INVALID_ARG;
  }
  return ORIN_OK;
}

// Which kernel serves this call.
// Tokens up to which AUTO takes the decode weight stream (csrc/gemv.cu).
// Measured on the 22-layer decode path: M=8 0.59 ms (skinny tcgen05 tiles
// 1.09); M=32 1.30 ms against 1.22 for the skinny tiles, whose tensor-core
// operands reuse each token fragment across 128 weight rows.
constexpr int kGemvAutoTokens = 16;

int choose_algo(int req, const void* A, const void* W, int M, int K) {
  const bool tma_ok = (K % 8 == 0) && aligned16(A) && aligned16(W);
  if (req == ORIN_ALGO_SIMT) return 3;
  if (!tma_ok) return (req == ORIN_ALGO_AUTO) ? 3 : -1;
  if (req == ORIN_ALGO_TC_WIDE) return 1;
  if (req == ORIN_ALGO_TC_SKINNY) return (M <= 64) ? 2 : -1;
  if (req == ORIN_ALGO_GEMV) return (M <= kGemvMaxTokens) ? 4 : -1;
  if (M <= kGemvAutoTokens) return 4;
  return (M <= 64) ? 2 : 1;
}

orin_status linear_impl(void* C, const void* A, const void* W, int M, int N, int K, int dtype,
                        int epilogue, const void* residual, int algo, void* workspace,
                        size_t workspace_bytes, void* stream);

}  // namespace

extern "C" {

int orin_version(void) { return 100; }

const char* orin_last_error(void) { return g_err; }

orin_status orin_linear_ex(void* C, const void* A, const void* W, int M, int N, int K, int dtype,
                           int epilogue, const void* residual, int algo, void* stream) {
  return linear_impl(C, A, W, M, N, K, dtype, epilogue, residual, algo, nullptr, 0, stream);
}

orin_status orin_linear_ws(void* C, const void* A, const void* W, int M, int N, int K, int dtype,
                           int epilogue, const void* residual, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (workspace && !aligned16(workspace)) {
    set_error("orin_linear_ws: the workspace must be 16-byte aligned");
    return ORIN_ERR_UNSUPPORTED;
  }
  return linear_impl(C, A, W, M, N, K, dtype, epilogue, residual, ORIN_ALGO_AUTO, workspace,
                     workspace ? workspace_bytes : 0, stream);
}

orin_status orin_linear_workspace_bytes(size_t* bytes) {
  if (!bytes) {
    set_error("orin_linear_workspace_bytes: null output");
    return ORIN_ERR_INVALID_ARG;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  *bytes = sk_workspace_max_bytes(sms);
  return ORIN_OK;
}

}  // extern "C"

namespace {

orin_status linear_impl(void* C, const void* A, const void* W, int M, int N, int K, int dtype,
                        int epilogue, const void* residual, int algo, void* workspace,
                        size_t workspace_bytes, void* stream) {
  orin_status st = check_common(dtype, epilogue);
  if (st != ORIN_OK) return st;
  if (!C || !A || !W) {
    set_error("orin_linear: null C, A or W");
    return ORIN_ERR_INVALID_ARG;
  }
  if (M < 1 || N < 1 || K < 1) {
    set_error("orin_linear: M=%d N=%d K=%d must all be >= 1", M, N, K);
    return ORIN_ERR_INVALID_ARG;
  }
  if (epilogue == ORIN_EPI_RESIDUAL && !residual) {
    set_error("orin_linear: RESIDUAL epilogue needs a residual pointer");
    return ORIN_ERR_INVALID_ARG;
  }
  if (epilogue == ORIN_EPI_SWIGLU && N % 64 != 0) {
    set_error("orin_linear: SWIGLU needs the intermediate size N=%d to be a multiple of 64", N);
    return ORIN_ERR_UNSUPPORTED;
  }
  if (algo < ORIN_ALGO_AUTO || algo > ORIN_ALGO_GEMV) {
    set_error("orin_linear: algo %d is not an orin_algo", algo);
    return ORIN_ERR_INVALID_ARG;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int a = choose_algo(algo, A, W, M, K);
  if (a < 0) {
    set_error("orin_linear: algo %d can't take M=%d K=%d (needs K%%8==0, 16-byte aligned "
              "A and W%s)", algo, M, K,
              algo == ORIN_ALGO_TC_SKINNY ? ", M<=64" : algo == ORIN_ALGO_GEMV ? ", M<=32" : "");
    return ORIN_ERR_UNSUPPORTED;
  }
  if (a == 3) {
    cudaError_t e = launch_simt(C, A, W, M, N, K, dtype, epilogue, residual, s);
    if (e != cudaSuccess) return cuda_fail(e, "orin_linear (simt)");
    return ORIN_OK;
  }
  if (a == 4) {
    cudaError_t e = launch_gemv(C, A, W, M, N, K, dtype, epilogue, residual, s);
    if (e != cudaSuccess) return cuda_fail(e, "orin_linear (gemv)");
    return ORIN_OK;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (!device_ctx_ready(dev)) {
    // The first call on a device loads its set-up; keep it out of capture.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone) {
      set_error("orin_linear: the first call on device %d sets the device up and must not be "
                "stream-captured; make one uncaptured call first", dev);
      return ORIN_ERR_INVALID_ARG;
    }
  }
  DeviceCtx* ctx = device_ctx(dev, &e);
  if (!ctx) {
    if (e == cudaErrorNoKernelImageForDevice) {
      set_error("orin_linear: device %d is not an sm_100 GPU", dev);
      return ORIN_ERR_NO_DEVICE;
    }
    return cuda_fail(e, "orin_linear: device set-up");
  }
  Plan pl;
  plan_tc(pl, M, N, K, epilogue, a, ctx->sm_count, workspace_bytes);
  const size_t esz = (epilogue == ORIN_EPI_F32_OUT || epilogue == ORIN_EPI_F32_PARTIAL) ? 4 : 2;
  pl.p.C = C;
  pl.p.ldc = N;
  pl.p.R = residual;
  pl.p.ldr = N;
  pl.p.vec_ok = aligned16(C) && ((N * esz) % 16 == 0) &&
                (!residual || (aligned16(residual) && (N * 2) % 16 == 0));
  const char* why = nullptr;
  e = launch_tc(pl, dtype, epilogue, A, W, ctx->err, s, &why, workspace);
  if (e != cudaSuccess) {
    if (why) {
      set_error("orin_linear: %s", why);
      return ORIN_ERR_UNSUPPORTED;
    }
    return cuda_fail(e, "orin_linear (tcgen05 launch)");
  }
  return ORIN_OK;
}

}  // namespace

extern "C" {

orin_status orin_linear_rmsnorm(void* C, const void* A, const void* W, const void* norm_w,
                                float eps, int M, int N, int K, int dtype, int epilogue,
                                void* stream) {
  orin_status st = check_common(dtype, epilogue);
  if (st != ORIN_OK) return st;
  if (!C || !A || !W || !norm_w || M < 1 || N < 1 || K < 1) {
    set_error("orin_linear_rmsnorm: null pointer or non-positive size (M=%d N=%d K=%d)", M, N,
              K);
    return ORIN_ERR_INVALID_ARG;
  }
  if (epilogue != ORIN_EPI_NONE && epilogue != ORIN_EPI_SWIGLU) {
    set_error("orin_linear_rmsnorm: epilogue %d (NONE and SWIGLU follow a norm)", epilogue);
    return ORIN_ERR_UNSUPPORTED;
  }
  if (epilogue == ORIN_EPI_SWIGLU && N % 64 != 0) {
    set_error("orin_linear_rmsnorm: SWIGLU needs N=%d to be a multiple of 64", N);
    return ORIN_ERR_UNSUPPORTED;
  }
  if (M > kGemvMaxTokens || K % 8 != 0 || !aligned16(A) || !aligned16(W) || !aligned16(norm_w)) {
    set_error("orin_linear_rmsnorm: the folded norm runs on the decode weight stream: needs "
              "M <= %d, K %% 8 == 0 and 16-byte aligned A, W and norm_w (M=%d K=%d); use "
              "orin_rmsnorm + orin_linear otherwise",
              kGemvMaxTokens, M, K);
    return ORIN_ERR_UNSUPPORTED;
  }
  cudaError_t e = launch_gemv(C, A, W, M, N, K, dtype, epilogue, nullptr,
                              static_cast<cudaStream_t>(stream), 0, norm_w, eps);
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_linear_rmsnorm");
}

orin_status orin_lm_head_argmax_rmsnorm(int* token, const void* h, const void* W,
                                        const void* norm_w, float eps, int M, int V, int K,
                                        int dtype, unsigned long long* keys, void* stream) {
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  if (!token || !h || !W || !norm_w || !keys || M < 1 || V < 1 || K < 1) {
    set_error("orin_lm_head_argmax_rmsnorm: null pointer or non-positive size");
    return ORIN_ERR_INVALID_ARG;
  }
  if (K % 8 != 0 || !aligned16(h) || !aligned16(W) || !aligned16(norm_w)) {
    set_error("orin_lm_head_argmax_rmsnorm: needs K %% 8 == 0 and 16-byte aligned h, W and "
              "norm_w (K=%d)", K);
    return ORIN_ERR_UNSUPPORTED;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_argmax_keys(keys, h, W, M, V, K, dtype, 0, s, norm_w, eps);
  if (e == cudaSuccess) e = launch_argmax_decode(token, keys, M, s);
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_lm_head_argmax_rmsnorm");
}

orin_status orin_plan_info(int M, int N, int K, int dtype, int epilogue, int algo, int info[6]) {
  int full[7];
  orin_status st = orin_plan_info_ws(M, N, K, dtype, epilogue, algo, 0, full);
  if (st == ORIN_OK)
    for (int i = 0; i < 6; ++i) info[i] = full[i];
  return st;
}

orin_status orin_plan_info_ws(int M, int N, int K, int dtype, int epilogue, int algo,
                              size_t workspace_bytes, int info[7]) {
  orin_status st = check_common(dtype, epilogue);
  if (st != ORIN_OK) return st;
  if (!info || M < 1 || N < 1 || K < 1) {
    set_error("orin_plan_info: bad arguments");
    return ORIN_ERR_INVALID_ARG;
  }
  static const char probe[16] __attribute__((aligned(16))) = {0};
  const int a = choose_algo(algo, probe, probe, M, K);
  if (a < 0) {
    set_error("orin_plan_info: algo %d can't take M=%d K=%d", algo, M, K);
    return ORIN_ERR_UNSUPPORTED;
  }
  for (int i = 0; i < 7; ++i) info[i] = 0;
  info[0] = a;
  if (a == 3) return ORIN_OK;
  if (a == 4) {
    info[1] = (M <= 8) ? 8 : (M <= 16) ? 16 : 32;
    info[3] = 1;
    info[4] = gemv_grid(N);
    info[5] = info[4];
    return ORIN_OK;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  DeviceCtx* ctx = device_ctx(dev, &e);
  if (!ctx) return cuda_fail(e, "orin_plan_info: device set-up");
  Plan pl;
  plan_tc(pl, M, N, K, epilogue, a, ctx->sm_count, workspace_bytes);
  info[1] = pl.bn;
  info[2] = pl.pair;
  info[3] = pl.p.split;
  info[4] = pl.grid;
  info[5] = pl.p.tiles_p * pl.p.tiles_q;
  info[6] = pl.p.sk;
  return ORIN_OK;
}

orin_status orin_lm_head_argmax(int* token, const void* h, const void* W, int M, int V, int K,
                                int dtype, unsigned long long* keys, void* stream) {
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  if (!token || !h || !W || !keys || M < 1 || V < 1 || K < 1) {
    set_error("orin_lm_head_argmax: null pointer or non-positive size");
    return ORIN_ERR_INVALID_ARG;
  }
  if (K % 8 != 0 || !aligned16(h) || !aligned16(W)) {
    set_error("orin_lm_head_argmax: needs K %% 8 == 0 and 16-byte aligned h and W (K=%d)", K);
    return ORIN_ERR_UNSUPPORTED;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_argmax_keys(keys, h, W, M, V, K, dtype, 0, s);
  if (e == cudaSuccess) e = launch_argmax_decode(token, keys, M, s);
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_lm_head_argmax");
}

orin_status orin_linear(void* C, const void* A, const void* W, int M, int N, int K, int dtype,
                        int epilogue, const void* residual, void* stream) {
  return orin_linear_ex(C, A, W, M, N, K, dtype, epilogue, residual, ORIN_ALGO_AUTO, stream);
}

orin_status orin_pack_gate_up(void* w_packed, const void* w_gate, const void* w_up, int IM, int K,
                              int dtype, void* stream) {
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  if (!w_packed || !w_gate || !w_up || IM < 1 || K < 1) {
    set_error("orin_pack_gate_up: null pointer or non-positive size");
    return ORIN_ERR_INVALID_ARG;
  }
  if (IM % 64 != 0) {
    set_error("orin_pack_gate_up: IM=%d must be a multiple of 64", IM);
    return ORIN_ERR_UNSUPPORTED;
  }
  cudaError_t e =
      launch_pack_gate_up(w_packed, w_gate, w_up, IM, K, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_pack_gate_up");
}

orin_status orin_silu_mul(void* out, const void* gate, const void* up, long long n, int dtype,
                          void* stream) {
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  if (n < 0 || (n > 0 && (!out || !gate || !up))) {
    set_error("orin_silu_mul: null pointer or negative n");
    return ORIN_ERR_INVALID_ARG;
  }
  cudaError_t e = launch_silu_mul(out, gate, up, n, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_silu_mul");
}

orin_status orin_add(void* x, const void* y, long long n, int dtype, void* stream) {
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  if (n < 0 || (n > 0 && (!x || !y))) {
    set_error("orin_add: null pointer or negative n");
    return ORIN_ERR_INVALID_ARG;
  }
  cudaError_t e = launch_add(x, y, n, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_add");
}

orin_status orin_widen_f32(float* out, const void* in, long long n, int dtype, void* stream) {
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  if (n < 0 || (n > 0 && (!out || !in))) {
    set_error("orin_widen_f32: null pointer or negative n");
    return ORIN_ERR_INVALID_ARG;
  }
  cudaError_t e = launch_widen(out, in, n, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_widen_f32");
}

namespace {

// Shared argument checks of the attention entry points.
orin_status check_attention(const char* fn, int seq_len, int cache_len, int num_heads,
                            int num_kv_heads, int head_dim, int n_sink, int window) {
  if (seq_len < 0 || cache_len < seq_len || num_heads < 1 || num_kv_heads < 1 ||
      num_heads % num_kv_heads != 0 || n_sink < 0 || window < 1) {
    set_error("%s: needs 0 <= seq_len <= cache_len, num_heads a multiple of num_kv_heads, "
              "n_sink >= 0, window_size >= 1 (seq_len=%d cache_len=%d heads=%d/%d n_sink=%d "
              "window=%d)",
              fn, seq_len, cache_len, num_heads, num_kv_heads, n_sink, window);
    return ORIN_ERR_INVALID_ARG;
  }
  if (head_dim != 64 && head_dim != 128) {
    set_error("%s: head_dim %d (64 and 128 are built)", fn, head_dim);
    return ORIN_ERR_UNSUPPORTED;
  }
  if (static_cast<long long>(n_sink) + window > 0x7fffffffLL / 2) {
    set_error("%s: n_sink + window_size too large", fn);
    return ORIN_ERR_INVALID_ARG;
  }
  return ORIN_OK;
}

// The current device's error word once its set-up has run (a linear call or
// orin_device_check), else null: a kernel's bounded waits still give up and
// return, without recording a code.
int* error_word_if_ready() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || !device_ctx_ready(dev)) return nullptr;
  cudaError_t e = cudaSuccess;
  DeviceCtx* ctx = device_ctx(dev, &e);
  return ctx ? ctx->err : nullptr;
}

}  // namespace

orin_status orin_attention_workspace_bytes(size_t* bytes, int seq_len, int cache_len,
                                           int num_heads, int num_kv_heads, int head_dim,
                                           int n_sink, int window_size) {
  if (!bytes) {
    set_error("orin_attention_workspace_bytes: null output");
    return ORIN_ERR_INVALID_ARG;
  }
  orin_status st = check_attention("orin_attention_workspace_bytes", seq_len, cache_len,
                                   num_heads, num_kv_heads, head_dim, n_sink, window_size);
  if (st != ORIN_OK) return st;
  *bytes = seq_len == 0 ? 0
                        : plan_attention(seq_len, cache_len, num_heads, num_kv_heads, head_dim,
                                         n_sink, window_size, ~static_cast<size_t>(0))
                              .workspace_bytes;
  return ORIN_OK;
}

orin_status orin_attention(void* out, const void* q, const void* k_pool, const void* v_pool,
                           int seq_len, int cache_len, int num_heads, int num_kv_heads,
                           int head_dim, float scale, int n_sink, int window_size, int dtype,
                           void* workspace, size_t workspace_bytes, void* stream) {
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  st = check_attention("orin_attention", seq_len, cache_len, num_heads, num_kv_heads, head_dim,
                       n_sink, window_size);
  if (st != ORIN_OK) return st;
  if (seq_len == 0) return ORIN_OK;
  if (!out || !q || !k_pool || !v_pool) {
    set_error("orin_attention: null pointer");
    return ORIN_ERR_INVALID_ARG;
  }
  if (!aligned16(out) || !aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) ||
      (workspace && !aligned16(workspace))) {
    set_error("orin_attention: out, q, the pools and the workspace must be 16-byte aligned");
    return ORIN_ERR_UNSUPPORTED;
  }
  cudaError_t e = launch_attention(out, q, k_pool, v_pool, seq_len, cache_len, num_heads,
                                   num_kv_heads, head_dim, scale, n_sink, window_size, dtype,
                                   workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                                   1, 0, error_word_if_ready());
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_attention");
}

orin_status orin_attention_batch(void* out, const void* q, const void* k_pool, const void* v_pool,
                                 int batch, long long pool_stride, int seq_len, int cache_len,
                                 int num_heads, int num_kv_heads, int head_dim, float scale,
                                 int n_sink, int window_size, int dtype, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  return orin_attention_batch_ex(out, q, k_pool, v_pool, batch, pool_stride, seq_len, cache_len,
                                 num_heads, num_kv_heads, head_dim, scale, n_sink, window_size,
                                 dtype, workspace, workspace_bytes, 0, stream);
}

orin_status orin_attention_batch_ex(void* out, const void* q, const void* k_pool,
                                    const void* v_pool, int batch, long long pool_stride,
                                    int seq_len, int cache_len, int num_heads, int num_kv_heads,
                                    int head_dim, float scale, int n_sink, int window_size,
                                    int dtype, void* workspace, size_t workspace_bytes,
                                    unsigned flags, void* stream) {
  if (flags & ~static_cast<unsigned>(ORIN_ATTN_OWN_SLOTS_ONLY)) {
    set_error("orin_attention_batch_ex: unknown flags 0x%x", flags);
    return ORIN_ERR_INVALID_ARG;
  }
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  st = check_attention("orin_attention_batch", seq_len, cache_len, num_heads, num_kv_heads,
                       head_dim, n_sink, window_size);
  if (st != ORIN_OK) return st;
  const long long pool_elems =
      (static_cast<long long>(n_sink) + window_size) * num_kv_heads * head_dim;
  if (batch < 0 || (batch > 1 && pool_stride < pool_elems)) {
    set_error("orin_attention_batch: batch %d, pool_stride %lld (at least one pool, %lld "
              "elements, apart)", batch, pool_stride, pool_elems);
    return ORIN_ERR_INVALID_ARG;
  }
  if (seq_len == 0 || batch == 0) return ORIN_OK;
  if (!out || !q || !k_pool || !v_pool) {
    set_error("orin_attention_batch: null pointer");
    return ORIN_ERR_INVALID_ARG;
  }
  if (!aligned16(out) || !aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) ||
      (workspace && !aligned16(workspace)) || (pool_stride * 2) % 16 != 0) {
    set_error("orin_attention_batch: out, q, the pools, the pool stride and the workspace must "
              "be 16-byte aligned");
    return ORIN_ERR_UNSUPPORTED;
  }
  if (static_cast<long long>(num_kv_heads) * batch > 65535) {
    set_error("orin_attention_batch: batch * num_kv_heads above 65535");
    return ORIN_ERR_UNSUPPORTED;
  }
  cudaError_t e = launch_attention(out, q, k_pool, v_pool, seq_len, cache_len, num_heads,
                                   num_kv_heads, head_dim, scale, n_sink, window_size, dtype,
                                   workspace, workspace_bytes, static_cast<cudaStream_t>(stream),
                                   batch, pool_stride, error_word_if_ready(),
                                   (flags & ORIN_ATTN_OWN_SLOTS_ONLY) ? kAttnOwnSlotsOnly : 0);
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_attention_batch");
}

orin_status orin_kv_append(void* k_pool, void* v_pool, const void* k_src, const void* v_src,
                           int seq_len, int start_pos, int n_sink, int window_size, int kv_dim,
                           int dtype, void* stream) {
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  if (seq_len < 0 || start_pos < 0 || n_sink < 0 || window_size < 1 || kv_dim < 1 ||
      (seq_len > 0 && (!k_pool || !v_pool || !k_src || !v_src))) {
    set_error("orin_kv_append: null pointer or bad size (seq_len=%d start_pos=%d n_sink=%d "
              "window=%d kv_dim=%d)",
              seq_len, start_pos, n_sink, window_size, kv_dim);
    return ORIN_ERR_INVALID_ARG;
  }
  if (static_cast<long long>(seq_len) > static_cast<long long>(n_sink) + window_size) {
    // the reference's precondition (src/kv_cache.cu:99-103)
    set_error("orin_kv_append: seq_len %d exceeds n_sink + window_size (%d)", seq_len,
              n_sink + window_size);
    return ORIN_ERR_INVALID_ARG;
  }
  if (static_cast<long long>(start_pos) + seq_len > 0x7fffffffLL) {
    set_error("orin_kv_append: positions past 2^31");
    return ORIN_ERR_INVALID_ARG;
  }
  cudaError_t e = launch_kv_scatter(k_pool, v_pool, k_src, v_src, seq_len, start_pos, n_sink,
                                    window_size, kv_dim, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_kv_append");
}

orin_status orin_embedding(void* out, const void* table, const int* token_ids, int seq_len,
                           int hidden, int vocab_size, void* stream) {
  if (seq_len < 0 || hidden < 1 || vocab_size < 1 ||
      (seq_len > 0 && (!out || !table || !token_ids))) {
    set_error("orin_embedding: null pointer or bad size (seq_len=%d hidden=%d vocab=%d)", seq_len,
              hidden, vocab_size);
    return ORIN_ERR_INVALID_ARG;
  }
  cudaError_t e = launch_embedding(out, table, token_ids, seq_len, hidden, vocab_size,
                                   static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_embedding");
}

orin_status orin_rmsnorm(void* out, const void* x, const void* weight, int rows, int dim,
                         float eps, int dtype, void* stream) {
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  if (rows < 0 || dim < 1 || (rows > 0 && (!out || !x || !weight))) {
    set_error("orin_rmsnorm: null pointer or bad size (rows=%d dim=%d)", rows, dim);
    return ORIN_ERR_INVALID_ARG;
  }
  cudaError_t e = launch_rmsnorm(out, x, weight, rows, dim, eps, dtype,
                                 static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_rmsnorm");
}

orin_status orin_rope(void* q, void* k, int seq_len, int num_heads, int num_kv_heads,
                      int head_dim, int start_pos, float theta, int dtype, void* stream) {
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  if (seq_len < 0 || num_heads < 1 || num_kv_heads < 0 || head_dim < 2 || head_dim % 2 != 0 ||
      start_pos < 0 || (seq_len > 0 && (!q || (num_kv_heads > 0 && !k)))) {
    set_error("orin_rope: null pointer or bad size (seq_len=%d heads=%d/%d head_dim=%d "
              "start_pos=%d)",
              seq_len, num_heads, num_kv_heads, head_dim, start_pos);
    return ORIN_ERR_INVALID_ARG;
  }
  cudaError_t e = launch_rope(q, k, seq_len, num_heads, num_kv_heads, head_dim, start_pos, theta,
                              dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_rope");
}

orin_status orin_qkv_rope_append(void* q_out, const void* qkv, const void* q_norm,
                                 const void* k_norm, void* k_pool, void* v_pool, int seq_len,
                                 int start_pos, int num_heads, int num_kv_heads, int head_dim,
                                 float eps, float theta, int n_sink, int window_size, int dtype,
                                 void* stream) {
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  if (seq_len < 0 || start_pos < 0 || num_heads < 1 || num_kv_heads < 1 ||
      num_heads % num_kv_heads != 0 || n_sink < 0 || window_size < 1 ||
      (seq_len > 0 && (!q_out || !qkv || !k_pool || !v_pool)) ||
      (q_norm == nullptr) != (k_norm == nullptr)) {
    set_error("orin_qkv_rope_append: null pointer or bad size (seq_len=%d start_pos=%d "
              "heads=%d/%d n_sink=%d window=%d; q_norm and k_norm both or neither)",
              seq_len, start_pos, num_heads, num_kv_heads, n_sink, window_size);
    return ORIN_ERR_INVALID_ARG;
  }
  if (static_cast<long long>(seq_len) > static_cast<long long>(n_sink) + window_size ||
      static_cast<long long>(start_pos) + seq_len > 0x7fffffffLL) {
    set_error("orin_qkv_rope_append: seq_len %d exceeds n_sink + window_size, or positions "
              "past 2^31",
              seq_len);
    return ORIN_ERR_INVALID_ARG;
  }
  if (head_dim != 64 && head_dim != 128) {
    set_error("orin_qkv_rope_append: head_dim %d (64 and 128 are built)", head_dim);
    return ORIN_ERR_UNSUPPORTED;
  }
  cudaError_t e = launch_qkv_rope_append(q_out, qkv, q_norm, k_norm, k_pool, v_pool, seq_len,
                                         start_pos, num_heads, num_kv_heads, head_dim, eps, theta,
                                         n_sink, window_size, dtype,
                                         static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_qkv_rope_append");
}

orin_status orin_qkv_rope_append_batch(void* q_out, const void* qkv, const void* q_norm,
                                       const void* k_norm, void* k_pool, void* v_pool, int batch,
                                       long long pool_stride, int seq_len, int start_pos,
                                       int num_heads, int num_kv_heads, int head_dim, float eps,
                                       float theta, int n_sink, int window_size, int dtype,
                                       void* stream) {
  const long long pool_elems =
      (static_cast<long long>(n_sink) + window_size) * num_kv_heads * head_dim;
  if (batch < 0 || (batch > 1 && pool_stride < pool_elems)) {
    set_error("orin_qkv_rope_append_batch: batch %d, pool_stride %lld (at least one pool, %lld "
              "elements, apart)", batch, pool_stride, pool_elems);
    return ORIN_ERR_INVALID_ARG;
  }
  if (batch == 0) return ORIN_OK;
  if (batch == 1)
    return orin_qkv_rope_append(q_out, qkv, q_norm, k_norm, k_pool, v_pool, seq_len, start_pos,
                                num_heads, num_kv_heads, head_dim, eps, theta, n_sink,
                                window_size, dtype, stream);
  // the single-sequence checks hold for every sequence of the batch
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  if (seq_len < 0 || start_pos < 0 || num_heads < 1 || num_kv_heads < 1 ||
      num_heads % num_kv_heads != 0 || n_sink < 0 || window_size < 1 ||
      (seq_len > 0 && (!q_out || !qkv || !k_pool || !v_pool)) ||
      (q_norm == nullptr) != (k_norm == nullptr)) {
    set_error("orin_qkv_rope_append_batch: null pointer or bad size (seq_len=%d start_pos=%d "
              "heads=%d/%d n_sink=%d window=%d; q_norm and k_norm both or neither)",
              seq_len, start_pos, num_heads, num_kv_heads, n_sink, window_size);
    return ORIN_ERR_INVALID_ARG;
  }
  if (static_cast<long long>(seq_len) > static_cast<long long>(n_sink) + window_size ||
      static_cast<long long>(start_pos) + seq_len > 0x7fffffffLL) {
    set_error("orin_qkv_rope_append_batch: seq_len %d exceeds n_sink + window_size, or "
              "positions past 2^31", seq_len);
    return ORIN_ERR_INVALID_ARG;
  }
  if (head_dim != 64 && head_dim != 128) {
    set_error("orin_qkv_rope_append_batch: head_dim %d (64 and 128 are built)", head_dim);
    return ORIN_ERR_UNSUPPORTED;
  }
  cudaError_t e = launch_qkv_rope_append(q_out, qkv, q_norm, k_norm, k_pool, v_pool, seq_len,
                                         start_pos, num_heads, num_kv_heads, head_dim, eps, theta,
                                         n_sink, window_size, dtype,
                                         static_cast<cudaStream_t>(stream), batch, pool_stride);
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_qkv_rope_append_batch");
}

orin_status orin_linear_rope_append(void* q_out, const void* x, const void* w_qkv, void* k_pool,
                                    void* v_pool, int batch, long long pool_stride, int seq_len,
                                    int start_pos, int hidden, int num_heads, int num_kv_heads,
                                    int head_dim, float theta, int n_sink, int window_size,
                                    int dtype, void* stream) {
  orin_status st = check_common(dtype, ORIN_EPI_NONE);
  if (st != ORIN_OK) return st;
  const long long pool_elems =
      (static_cast<long long>(n_sink) + window_size) * num_kv_heads * head_dim;
  if (!q_out || !x || !w_qkv || !k_pool || !v_pool || batch < 1 || seq_len < 1 ||
      start_pos < 0 || hidden < 1 || num_heads < 1 || num_kv_heads < 1 ||
      num_heads % num_kv_heads != 0 || n_sink < 0 || window_size < 1 ||
      (batch > 1 && pool_stride < pool_elems) ||
      static_cast<long long>(seq_len) > static_cast<long long>(n_sink) + window_size ||
      static_cast<long long>(start_pos) + seq_len > 0x7fffffffLL) {
    set_error("orin_linear_rope_append: null pointer or bad size (batch=%d seq_len=%d "
              "start_pos=%d hidden=%d heads=%d/%d n_sink=%d window=%d pool_stride=%lld)",
              batch, seq_len, start_pos, hidden, num_heads, num_kv_heads, n_sink, window_size,
              pool_stride);
    return ORIN_ERR_INVALID_ARG;
  }
  const long long M = static_cast<long long>(batch) * seq_len;
  if (M > kGemvMaxTokens || hidden % 8 != 0 || !aligned16(x) || !aligned16(w_qkv) ||
      (head_dim != 64 && head_dim != 128)) {
    set_error("orin_linear_rope_append: runs on the decode weight stream: needs batch * "
              "seq_len <= %d, hidden %% 8 == 0, 16-byte aligned x and w_qkv and head_dim 64 or "
              "128 (M=%lld hidden=%d head_dim=%d); use orin_linear + "
              "orin_qkv_rope_append_batch otherwise",
              kGemvMaxTokens, M, hidden, head_dim);
    return ORIN_ERR_UNSUPPORTED;
  }
  cudaError_t e = launch_gemv_rope(q_out, x, w_qkv, static_cast<int>(M), hidden, dtype,
                                   num_heads, num_kv_heads, head_dim, seq_len, start_pos, theta,
                                   n_sink, window_size, k_pool, v_pool, pool_stride,
                                   static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ORIN_OK : cuda_fail(e, "orin_linear_rope_append");
}

orin_status orin_device_check(void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "orin_device_check: stream synchronize");
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "orin_device_check: pending launch error");
  int dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  DeviceCtx* ctx = device_ctx(dev, &e);
  if (!ctx) return cuda_fail(e, "orin_device_check: device set-up");
  int word = 0;
  if ((e = cudaMemcpy(&word, ctx->err, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
    return cuda_fail(e, "orin_device_check: read error word");
  if (word != 0) {
    cudaMemset(ctx->err, 0, sizeof(int));
    cudaDeviceSynchronize();
    set_error("orin_device_check: a kernel gave up waiting (device error code %d)", word);
    return ORIN_ERR_TIMEOUT;
  }
  return ORIN_OK;
}

}  // extern "C"
