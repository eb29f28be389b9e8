// ref_entry.cu — C entry points into the reference's own GEMM-path kernels.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's unmodified sources (kernels/matmul.cu, kernels/gemm_cute.cu,
// kernels/fused_swiglu.cu, kernels/softmax.cu, kernels/attention.cu,
// kernels/rmsnorm.cu, kernels/rope.cu, kernels/embedding.cu) into oracle/_ref/.  The tests
// use it to pin the CPU oracle to what the reference computes; nothing in the
// product links it.
#include <cuda_runtime.h>

#include "kernels.h"  // the reference's include/kernels.h

extern bool launch_gemm_cute(__nv_bfloat16* C, const __nv_bfloat16* A, const __nv_bfloat16* B,
                             int M, int N, int K);

extern "C" {

// kernels::matmul: M == 1 -> gemv_kernel; M > 1 -> cuBLAS (USE_CUBLAS build) or
// CuTe / per-row GEMV (the other build).
int ref_matmul(void* C, const void* A, const void* B, int M, int N, int K) {
  kernels::matmul(static_cast<__nv_bfloat16*>(C), static_cast<const __nv_bfloat16*>(A),
                  static_cast<const __nv_bfloat16*>(B), M, N, K);
  return static_cast<int>(cudaGetLastError());
}

// The CuTe sm80 kernel alone; returns 1 if it launched (tile-aligned shapes).
int ref_gemm_cute(void* C, const void* A, const void* B, int M, int N, int K) {
  return launch_gemm_cute(static_cast<__nv_bfloat16*>(C), static_cast<const __nv_bfloat16*>(A),
                          static_cast<const __nv_bfloat16*>(B), M, N, K)
             ? 1
             : 0;
}

int ref_fused_silu_mul(void* out, const void* gate, const void* up, int seq, int im) {
  kernels::fused_silu_mul(static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(gate),
                          static_cast<const __nv_bfloat16*>(up), seq, im);
  return static_cast<int>(cudaGetLastError());
}

int ref_add(void* x, const void* y, int n) {
  kernels::add(static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(y), n);
  return static_cast<int>(cudaGetLastError());
}

int ref_bf16_to_fp32(float* out, const void* in, int n) {
  kernels::bf16_to_fp32(out, static_cast<const __nv_bfloat16*>(in), n);
  return static_cast<int>(cudaGetLastError());
}

// kernels::attention: sink + sliding-window GQA attention over the ring pool
// (one CTA of 128 threads per query token and head).
int ref_attention(void* out, const void* q, const void* k_pool, const void* v_pool, int seq_len,
                  int cache_len, int num_heads, int num_kv_heads, int head_dim, float scale,
                  int n_sink, int window_size) {
  kernels::attention(static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(q),
                     static_cast<const __nv_bfloat16*>(k_pool),
                     static_cast<const __nv_bfloat16*>(v_pool), seq_len, cache_len, num_heads,
                     num_kv_heads, head_dim, scale, n_sink, window_size);
  return static_cast<int>(cudaGetLastError());
}

int ref_rmsnorm(void* out, const void* x, const void* w, int rows, int dim, float eps) {
  kernels::rmsnorm(static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(x),
                   static_cast<const __nv_bfloat16*>(w), rows, dim, eps);
  return static_cast<int>(cudaGetLastError());
}

int ref_rope(void* q, void* k, int seq_len, int num_heads, int num_kv_heads, int head_dim,
             int start_pos, float theta) {
  kernels::rope(static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k), seq_len,
                num_heads, num_kv_heads, head_dim, start_pos, theta);
  return static_cast<int>(cudaGetLastError());
}

int ref_embedding(void* out, const void* table, const int* ids, int seq_len, int hidden) {
  kernels::embedding(static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(table),
                     ids, seq_len, hidden);
  return static_cast<int>(cudaGetLastError());
}

int ref_sync(void) { return static_cast<int>(cudaDeviceSynchronize()); }

}  // extern "C"
