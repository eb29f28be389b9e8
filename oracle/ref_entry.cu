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

extern "C" {

// Returned instead of launching when a call of the build without USE_CUBLAS would
// reach the reference's CuTe kernel.
#define REF_REFUSED_CUTE (-2)

// kernels::matmul: M == 1 -> gemv_kernel; M > 1 -> cuBLAS (USE_CUBLAS build) or
// the per-row GEMV fallback (the other build).
//
// Without USE_CUBLAS, kernels::matmul sends tile-aligned shapes (M % 128, N % 128,
// K % 32 all zero; kernels/gemm_cute.cu:302) to gemm_multi_stage.  That kernel
// made an illegal address access on a B200: its copy layouts cover 128 threads
// (kernels/gemm_cute.cu:211-249) while the block has 256, so the upper half reads
// past A and writes past the C tile on the last k-tile.  Those shapes are refused
// here before anything is launched; only the per-row GEMV fallback stays callable.
int ref_matmul(void* C, const void* A, const void* B, int M, int N, int K) {
#ifndef USE_CUBLAS
  if (M > 1 && M % 128 == 0 && N % 128 == 0 && K % 32 == 0) return REF_REFUSED_CUTE;
#endif
  kernels::matmul(static_cast<__nv_bfloat16*>(C), static_cast<const __nv_bfloat16*>(A),
                  static_cast<const __nv_bfloat16*>(B), M, N, K);
  return static_cast<int>(cudaGetLastError());
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

// kernels::argmax: the greedy sampler (one CTA of 512 threads, kernels/softmax.cu:52-73).
int ref_argmax(int* out, const float* logits, int n) {
  kernels::argmax(reinterpret_cast<int32_t*>(out), logits, n);
  return static_cast<int>(cudaGetLastError());
}

int ref_sync(void) { return static_cast<int>(cudaDeviceSynchronize()); }

}  // extern "C"
