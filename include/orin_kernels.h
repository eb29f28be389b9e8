/*
 * orin_kernels.h — C++ link-compatible replacements for the reference's
 * entry points of the linear-layer path and of the attention around it,
 * implemented by liborin_b200.so on top of the C ABI in orin_b200.h.  A
 * program compiled against the reference's include/kernels.h links these
 * instead of kernels/matmul.cu, kernels/fused_swiglu.cu, kernels/embedding.cu,
 * kernels/rmsnorm.cu, kernels/rope.cu, kernels/attention.cu and the add /
 * bf16_to_fp32 part of kernels/softmax.cu.
 *
 * Like the originals they take raw bf16 device pointers, run on the legacy
 * default stream and return nothing.  A failure is recorded (read it with
 * orin_last_error()) instead of being silently dropped.
 */
#ifndef ORIN_KERNELS_H
#define ORIN_KERNELS_H

#include <cuda_bf16.h>
#include <stdint.h>

namespace kernels {

/* C[M,N] = A[M,K] · B[N,K]^T.  Reference: include/kernels.h:51-56,
 * kernels/matmul.cu:47-81 (M==1 GEMV, M>1 cuBLAS or CuTe). */
void matmul(__nv_bfloat16* C, const __nv_bfloat16* A, const __nv_bfloat16* B,
            int M, int N, int K);

/* out = silu(gate) * up over seq_len*intermediate_size elements.
 * Reference: include/kernels.h:88-94, kernels/fused_swiglu.cu:19-26. */
void fused_silu_mul(__nv_bfloat16* out, const __nv_bfloat16* gate,
                    const __nv_bfloat16* up, int seq_len,
                    int intermediate_size);

/* x += y elementwise.  Reference: include/kernels.h:97-101,
 * kernels/softmax.cu:112-115. */
void add(__nv_bfloat16* x, const __nv_bfloat16* y, int n);

/* out = float(in).  Reference: include/kernels.h:104-108,
 * kernels/softmax.cu:117-120. */
void bf16_to_fp32(float* out, const __nv_bfloat16* in, int n);

/* out[t] = table[token_ids[t]] (orin_embedding).  Reference:
 * include/kernels.h:12-19, kernels/embedding.cu:14-21. */
void embedding(__nv_bfloat16* out, const __nv_bfloat16* table,
               const int32_t* token_ids, int seq_len, int hidden_size);

/* out = rmsnorm(x) per row (orin_rmsnorm).  Reference: include/kernels.h:22-31,
 * kernels/rmsnorm.cu:7-41. */
void rmsnorm(__nv_bfloat16* out, const __nv_bfloat16* x,
             const __nv_bfloat16* weight, int seq_len, int dim, float eps);

/* Rotary embedding in place on q and k (orin_rope).  Reference:
 * include/kernels.h:33-45, kernels/rope.cu:7-60. */
void rope(__nv_bfloat16* q, __nv_bfloat16* k, int seq_len, int num_heads,
          int num_kv_heads, int head_dim, int start_pos, float theta);

/* Sink + sliding-window GQA attention over the ring KV pool (orin_attention).
 * Reference: include/kernels.h:58-80, kernels/attention.cu:140-175.  Split-key
 * partials of few-token calls use a 4 MB static device array. */
void attention(__nv_bfloat16* out, const __nv_bfloat16* q,
               const __nv_bfloat16* k_pool, const __nv_bfloat16* v_pool,
               int seq_len, int cache_len, int num_heads, int num_kv_heads,
               int head_dim, float scale, int n_sink, int window_size);

}  // namespace kernels

/* Reference: kernels/gemm_cute.cu:295-324 (declared at kernels/matmul.cu:9-12).
 * The original returns false unless M%128 == N%128 == K%32 == 0.  This one
 * launches for every shape orin_linear accepts and returns false only when
 * the arguments are invalid or the launch failed. */
bool launch_gemm_cute(__nv_bfloat16* C, const __nv_bfloat16* A,
                      const __nv_bfloat16* B, int M, int N, int K);

#endif /* ORIN_KERNELS_H */
