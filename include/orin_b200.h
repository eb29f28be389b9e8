/*
 * orin_b200.h — C ABI of the B200 (sm_100a) linear-layer hot path.
 *
 * Every entry point takes plain device pointers, element counts and an opaque
 * CUDA stream (cudaStream_t passed as void*; NULL = legacy default stream).
 * The GEMM entry points allocate no workspace: split-K partial sums stay on
 * chip (thread-block clusters combine them through distributed shared memory).
 * The library does own a few file-scope device arrays, present on every
 * device that loads it until exit: a 4-byte error word per device, the 4 MB
 * split-key array behind the kernels::attention drop-in, and the 64 MiB
 * partial-sum array of orin_tp_linear_row_static.  orin_attention and
 * orin_tp_linear_row take their workspace from the caller.  The tensor-parallel
 * set-up allocates: orin_tp_enable_p2p the peer-memory region it maps (freed by
 * orin_tp_destroy, which also uses a 4-byte buffer for its closing barrier),
 * orin_p2p_watchdog_selftest a small buffer for the duration of the call.  The first GEMM
 * call on a device does a one-time set-up (device attributes, the device
 * error word); it must not be inside CUDA stream capture, later calls may be
 * captured into graphs.
 * Weights read ahead: the projection and RMSNorm entry points are launched
 * with programmatic dependent launch and start streaming their weights (W,
 * the norm weight) before the kernels issued before them on the same stream
 * have finished (this library's kernels let the next one start early, so
 * more than one can still be running), so no such kernel may write those
 * weights: write them before a synchronisation point, an ordinary (non-PDL)
 * launch, or with orin_pack_gate_up (which ends with one).  Activations,
 * residuals and pools are read only after the previous kernel has finished
 * (pools: unless the caller passes ORIN_ATTN_OWN_SLOTS_ONLY to
 * orin_attention_batch_ex).
 * No C++ exception crosses this boundary: every function returns orin_status,
 * and orin_last_error() gives a thread-local message for the last failure.
 *
 * Semantics shared by every GEMM entry point (the reference's, restated):
 *   C[m, n] = round16( sum_k f32(A[m, k]) * f32(W[n, k]) )
 * with A row-major [M, K] (activations), W row-major [N, K] (HF weight layout,
 * "B stored transposed"), fp32 accumulation and exactly one rounding of the
 * result to the 16-bit type.  Reference: kernels/matmul.cu:25-44 (GEMV),
 * kernels/matmul.cu:59-68 (cublasGemmEx, CUBLAS_COMPUTE_32F),
 * kernels/gemm_cute.cu:147,176-178 (CuTe mma.sync, fp32 accumulator).
 */
#ifndef ORIN_B200_H
#define ORIN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum orin_status {
    ORIN_OK = 0,
    ORIN_ERR_INVALID_ARG = 1, /* null pointer, negative size, bad enum      */
    ORIN_ERR_UNSUPPORTED = 2, /* shape/alignment this entry point can't do  */
    ORIN_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed          */
    ORIN_ERR_NCCL = 4,        /* an NCCL call failed                        */
    ORIN_ERR_TIMEOUT = 5,     /* a bounded wait expired (device or host)    */
    ORIN_ERR_NO_DEVICE = 6    /* no sm_100 device visible                   */
} orin_status;

typedef enum orin_dtype {
    ORIN_F16 = 0,
    ORIN_BF16 = 1
} orin_dtype;

/* What happens to the fp32 accumulator before it is stored. */
typedef enum orin_epilogue {
    /* C = round16(acc)                                    (kernels/matmul.cu:43) */
    ORIN_EPI_NONE = 0,
    /* W holds 2N rows, gate and up interleaved in 64-row groups (see
     * orin_pack_gate_up); C[M, N] = round16(silu(round16(g)) * round16(u)).
     * Folds kernels/fused_swiglu.cu:7-16 into the gate/up GEMM. */
    ORIN_EPI_SWIGLU = 1,
    /* C = round16(f32(R) + f32(round16(acc))); C may alias R.
     * Folds kernels/softmax.cu:78-83 (add) into the O / down GEMM. */
    ORIN_EPI_RESIDUAL = 2,
    /* C is float: C = f32(round16(acc)).
     * Folds kernels/softmax.cu:87-90 (bf16_to_fp32) into the LM head. */
    ORIN_EPI_F32_OUT = 3,
    /* C is float: C = acc, unrounded (tensor-parallel partial sums). */
    ORIN_EPI_F32_PARTIAL = 4
} orin_epilogue;

/* Kernel selection; AUTO is what every production caller should pass. */
typedef enum orin_algo {
    ORIN_ALGO_AUTO = 0,
    ORIN_ALGO_TC_WIDE = 1,   /* tcgen05, 128 tokens x 256 features per tile  */
    ORIN_ALGO_TC_SKINNY = 2, /* tcgen05, 128 features x <=64 tokens (M<=64)  */
    ORIN_ALGO_SIMT = 3,      /* CUDA-core kernel for unaligned shapes        */
    ORIN_ALGO_GEMV = 4       /* decode weight stream, M <= 32 tokens         */
} orin_algo;

/* Library version (major*10000 + minor*100 + patch). */
int orin_version(void);

/* Thread-local description of the last non-OK status returned on this thread. */
const char* orin_last_error(void);

/*
 * C = epilogue(A · W^T).  Replaces kernels::matmul (include/kernels.h:51-56,
 * kernels/matmul.cu:47-81) and, through the epilogue argument, the pairs
 * matmul+fused_silu_mul (src/model.cu:100-104), matmul+add (src/model.cu:87-90,
 * 107-110) and matmul+bf16_to_fp32 (src/model.cu:125-130).
 *   C         [M, N] 16-bit, or float for F32_OUT / F32_PARTIAL
 *   A         [M, K] 16-bit
 *   W         [N, K] 16-bit ([2N, K] packed gate/up for SWIGLU)
 *   residual  [M, N] 16-bit for RESIDUAL, else NULL
 * Any M, N >= 1 and K >= 1 are accepted.  K % 8 == 0 with 16-byte aligned
 * A, W (and C rows) takes the decode weight stream for M <= 16 (up to 32
 * on request) and the tcgen05 path above; other shapes take the SIMT path.
 */
orin_status orin_linear(void* C, const void* A, const void* W,
                        int M, int N, int K, int dtype, int epilogue,
                        const void* residual, void* stream);

/*
 * orin_linear with an explicit kernel choice (orin_algo).  ORIN_ALGO_AUTO is
 * what orin_linear passes; the others exist for tests and tuning and return
 * ORIN_ERR_UNSUPPORTED for shapes they can't take.
 */
orin_status orin_linear_ex(void* C, const void* A, const void* W,
                           int M, int N, int K, int dtype, int epilogue,
                           const void* residual, int algo, void* stream);

/*
 * Diagnostics: the launch orin_linear_ex would make for this problem on the
 * current device.  info[0] kernel (1 tcgen05 wide tiles, 2 tcgen05 skinny
 * tiles, 3 CUDA cores, 4 decode weight stream), info[1] tile columns
 * (tokens per tile for 4), info[2] 1 if tiles run on
 * tcgen05 CTA pairs, info[3] split-K factor (cluster split), info[4] grid
 * size (CTAs), info[5] number of tiles.  Assumes 16-byte aligned operands.
 */
orin_status orin_plan_info(int M, int N, int K, int dtype, int epilogue, int algo,
                           int info[6]);

/*
 * orin_linear with a caller workspace (no counterpart in the reference, whose
 * matmul takes none).  With a workspace of at least
 * orin_linear_workspace_bytes() bytes, wide (prefill) problems may run a
 * stream-K schedule: the tiles x K work is dealt to one CTA (pair) per SM in
 * equal contiguous ranges, so no SM idles in a last partial wave; a CTA whose
 * range starts inside a tile leaves that partial fp32 accumulator in the
 * workspace and the CTA holding the tile's first k-blocks adds it (in a fixed
 * order: deterministic) before its epilogue.  Same semantics and epilogues as
 * orin_linear; without a workspace (NULL or too small) it is orin_linear.
 * The workspace: 16-byte aligned device memory whose first 4 KB (flag words)
 * are zero before its first use (cudaMemset once); every call leaves them
 * zero again.  Calls that share a workspace must be ordered (one stream);
 * after an ORIN_ERR_TIMEOUT from orin_device_check, zero it again.
 */
orin_status orin_linear_ws(void* C, const void* A, const void* W,
                           int M, int N, int K, int dtype, int epilogue,
                           const void* residual, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Workspace bytes that let orin_linear_ws choose any plan on the current
 * device (one 128 x 256 fp32 slot per SM plus 4 KB of flags: 19 MB on B200). */
orin_status orin_linear_workspace_bytes(size_t* bytes);

/* orin_plan_info for orin_linear_ws with a workspace of workspace_bytes:
 * info[0..5] as orin_plan_info, info[6] 1 for a stream-K schedule. */
orin_status orin_plan_info_ws(int M, int N, int K, int dtype, int epilogue,
                              int algo, size_t workspace_bytes, int info[7]);

/*
 * Build the packed gate/up weight the SWIGLU epilogue reads:
 * rows [128g, 128g+64) = gate rows [64g, 64g+64), rows [128g+64, 128g+128) =
 * up rows [64g, 64g+64).  w_gate, w_up [IM, K] (include/weight_store.h:17-18);
 * w_packed [2*IM, K].  Requires IM % 64 == 0.  Runs on the device, on stream,
 * and ends with an ordinary launch, so the next call may use w_packed at once
 * (see the note on weights read ahead below).
 */
orin_status orin_pack_gate_up(void* w_packed, const void* w_gate,
                              const void* w_up, int IM, int K, int dtype,
                              void* stream);

/*
 * Greedy next token of each of M rows (no separate logits pass): replaces
 * the LM head matmul + bf16_to_fp32 (src/model.cu:113-131) followed by
 * kernels::argmax (include/kernels.h:118-125, kernels/softmax.cu:52-73,
 * src/sampler.cu:24-27).  token[m] = argmax over v < V of
 * f32(round16(h[m] . W[v])), ties resolved exactly as the reference's
 * 512-thread sampler resolves them: among the positions of the maximum, the
 * one whose residue v mod 512 has the smallest 9-bit bit-reversal, then the
 * smallest v; -inf and NaN never win; if nothing counts, 0.
 *   token  [M] int32 (device)      h [M, K] 16-bit      W [V, K] 16-bit
 *   keys   caller scratch of M 64-bit words (device), overwritten
 * Needs K % 8 == 0 and 16-byte aligned h and W.  Rows go through the decode
 * weight-stream kernel 32 at a time.
 */
orin_status orin_lm_head_argmax(int* token, const void* h, const void* W,
                                int M, int V, int K, int dtype,
                                unsigned long long* keys, void* stream);

/*
 * The projection that follows an RMSNorm, with the norm folded in:
 *   C = epilogue( round16(A * r * norm_w) · W^T ),  r = rsqrtf(sum(A_row^2)/K + eps)
 * per token row of A, the normalised row rounded to 16 bits exactly as
 * orin_rmsnorm stores it (kernels/rmsnorm.cu:7-34), so the result equals
 * orin_rmsnorm followed by orin_linear.  Replaces the reference's
 * rmsnorm + matmul pairs (src/model.cu:53,59-61 and :95,100-101) at decode:
 * the decode weight stream, M <= 32 tokens, epilogue NONE or SWIGLU, K % 8 == 0,
 * 16-byte aligned A, W and norm_w; ORIN_ERR_UNSUPPORTED otherwise (use
 * orin_rmsnorm + orin_linear).
 */
orin_status orin_linear_rmsnorm(void* C, const void* A, const void* W,
                                const void* norm_w, float eps, int M, int N,
                                int K, int dtype, int epilogue, void* stream);

/* orin_lm_head_argmax of the RMS-normalised rows of h (the final norm of
 * src/model.cu:116-117 folded in, rounded as orin_rmsnorm stores it). */
orin_status orin_lm_head_argmax_rmsnorm(int* token, const void* h, const void* W,
                                        const void* norm_w, float eps, int M,
                                        int V, int K, int dtype,
                                        unsigned long long* keys, void* stream);

/* out = round16(silu(f32(gate)) * f32(up)), n elements; out may alias gate.
 * Replaces kernels::fused_silu_mul (include/kernels.h:88-94). */
orin_status orin_silu_mul(void* out, const void* gate, const void* up,
                          long long n, int dtype, void* stream);

/* x = round16(f32(x) + f32(y)), n elements.
 * Replaces kernels::add (include/kernels.h:97-101, kernels/softmax.cu:78-83). */
orin_status orin_add(void* x, const void* y, long long n, int dtype,
                     void* stream);

/* out = f32(in), n elements.
 * Replaces kernels::bf16_to_fp32 (include/kernels.h:104-108). */
orin_status orin_widen_f32(float* out, const void* in, long long n, int dtype,
                           void* stream);

/* out[t, :] = table[token_ids[t], :] (16-bit rows of hidden elements; token_ids
 * int32 on the device).  An id outside [0, vocab_size) gives a zero row.
 * Replaces kernels::embedding (include/kernels.h:12-19, kernels/embedding.cu:4-21). */
orin_status orin_embedding(void* out, const void* table, const int* token_ids,
                           int seq_len, int hidden, int vocab_size, void* stream);

/* out = round16(x * r * w) per row of dim elements, r = rsqrtf(sum(x^2)/dim + eps),
 * fp32.  out may alias x.  Replaces kernels::rmsnorm (include/kernels.h:22-31,
 * kernels/rmsnorm.cu:7-41). */
orin_status orin_rmsnorm(void* out, const void* x, const void* weight, int rows,
                         int dim, float eps, int dtype, void* stream);

/* Rotary embedding in place on q [seq_len][num_heads][head_dim] and
 * k [seq_len][num_kv_heads][head_dim]: pairs (i, i + head_dim/2) of each head
 * at position start_pos + t rotate by (start_pos + t) * powf(theta,
 * -2i/head_dim), each result rounded to 16 bits.  Replaces kernels::rope
 * (include/kernels.h:33-45, kernels/rope.cu:7-60). */
orin_status orin_rope(void* q, void* k, int seq_len, int num_heads,
                      int num_kv_heads, int head_dim, int start_pos, float theta,
                      int dtype, void* stream);

/*
 * The steps between this library's fused q/k/v projection and the attention,
 * in one launch.  qkv: token rows [q (num_heads*head_dim) | k | v
 * (num_kv_heads*head_dim each)], as orin_linear writes them with the q, k and
 * v weights stacked.  Per head: the optional RMSNorm with q_norm / k_norm
 * [head_dim] (Qwen3, src/model.cu:64-67; both NULL for Llama), the rotation of
 * orin_rope, then q -> q_out [seq_len][num_heads][head_dim] and k, v into their
 * ring slots as orin_kv_append places them (src/model.cu:70-73).  Rounding
 * points are the reference's (normed value, then each rotated value).
 * head_dim 64 or 128.
 */
orin_status orin_qkv_rope_append(void* q_out, const void* qkv, const void* q_norm,
                                 const void* k_norm, void* k_pool, void* v_pool,
                                 int seq_len, int start_pos, int num_heads,
                                 int num_kv_heads, int head_dim, float eps,
                                 float theta, int n_sink, int window_size,
                                 int dtype, void* stream);

/*
 * orin_qkv_rope_append for `batch` sequences of seq_len tokens each at the
 * same positions (batched decode; no counterpart in the single-sequence
 * reference): qkv and q_out rows are [batch][seq_len]; sequence b's K/V go
 * into the pools at k_pool / v_pool + b * pool_stride elements
 * (pool_stride >= (n_sink + window_size) * num_kv_heads * head_dim).  Each
 * sequence's results are those of its own orin_qkv_rope_append call.
 */
orin_status orin_qkv_rope_append_batch(void* q_out, const void* qkv,
                                       const void* q_norm, const void* k_norm,
                                       void* k_pool, void* v_pool, int batch,
                                       long long pool_stride, int seq_len,
                                       int start_pos, int num_heads,
                                       int num_kv_heads, int head_dim, float eps,
                                       float theta, int n_sink, int window_size,
                                       int dtype, void* stream);

/*
 * The q/k/v projection with RoPE and the K/V append in its epilogue, for
 * decode-sized calls without per-head q/k norms (Llama-family layers):
 * replaces orin_linear(qkv, x, w_qkv) followed by
 * orin_qkv_rope_append_batch(q_out, qkv, NULL, NULL, ...) (src/model.cu:
 * 59-75) with one launch of the decode weight stream, with the same results
 * bit for bit: every q/k/v sum is rounded to 16 bits as the projection
 * stores it, q and k are rotated with the reference's angle, v is copied.
 * x [batch * seq_len][hidden] (token rows of sequence b after those of
 * sequence b - 1, all at positions start_pos ..), w_qkv the stacked
 * [(num_heads + 2 num_kv_heads) * head_dim][hidden] weight, q_out
 * [batch * seq_len][num_heads][head_dim]; sequence b's K/V go to its pools
 * at k_pool / v_pool + b * pool_stride.  Needs batch * seq_len <= 32,
 * hidden % 8 == 0, 16-byte aligned x and w_qkv, and head_dim 64 or 128
 * (ORIN_ERR_UNSUPPORTED otherwise: use the two calls above).
 */
orin_status orin_linear_rope_append(void* q_out, const void* x, const void* w_qkv,
                                    void* k_pool, void* v_pool, int batch,
                                    long long pool_stride, int seq_len, int start_pos,
                                    int hidden, int num_heads, int num_kv_heads,
                                    int head_dim, float theta, int n_sink,
                                    int window_size, int dtype, void* stream);

/* ------------------------------------------------------------------------ */
/* Sink + sliding-window GQA attention over the ring KV pool (the callers of */
/* the linear layers on either side: q/k/v come from the q/k/v projection,   */
/* the output feeds o_proj).                                                 */

/*
 * The KV pool of one layer, as the reference lays it out (include/kv_cache.h:
 * 12-25, src/kv_cache.cu:21-41): K and V pools of n_sink + window_size slots,
 * each [slot][num_kv_heads][head_dim]; logical position p is stored in slot
 * p (p < n_sink) or n_sink + (p - n_sink) % window_size.
 *
 * Scatter seq_len new rows (k_src, v_src: [seq_len][kv_dim]) of positions
 * start_pos .. start_pos + seq_len - 1 into their slots.  Replaces
 * KVCache::append_kv (include/kv_cache.h:37-40, src/kv_cache.cu:95-111) with
 * the pools passed explicitly.  seq_len > n_sink + window_size is
 * ORIN_ERR_INVALID_ARG, as the reference throws.  When more than window_size
 * window positions arrive in one call, the later of two tokens sharing a
 * slot is the one stored (the reference leaves that to launch order).
 */
orin_status orin_kv_append(void* k_pool, void* v_pool, const void* k_src,
                           const void* v_src, int seq_len, int start_pos,
                           int n_sink, int window_size, int kv_dim, int dtype,
                           void* stream);

/*
 * out[t, h, :] = round16( sum_p softmax_p(scale * q[t, h] . K[p, h / G]) V[p, h / G] )
 * over the positions p query token t sees: with ap = cache_len - seq_len + t,
 * p <= ap and (p < n_sink or p >= ap + 1 - window_size), each read through
 * its pool slot.  q, out: [seq_len][num_heads][head_dim]; G = num_heads /
 * num_kv_heads; fp32 scores, softmax and sums.  Replaces kernels::attention
 * (include/kernels.h:58-80, kernels/attention.cu:27-175).
 *
 * head_dim 64 or 128 (else ORIN_ERR_UNSUPPORTED); all pointers 16-byte
 * aligned.  workspace (device, may be NULL) lets few-token calls split the
 * keys across CTAs; orin_attention_workspace_bytes gives the size that
 * unlocks every split, a smaller one splits less.  Its first 4 KB hold the
 * arrival counters the split CTAs merge through: they must be zero before
 * the first call (allocate the workspace zeroed), and every call leaves them
 * zero.  Calls that share a workspace must be ordered on one stream.
 */
orin_status orin_attention(void* out, const void* q, const void* k_pool,
                           const void* v_pool, int seq_len, int cache_len,
                           int num_heads, int num_kv_heads, int head_dim,
                           float scale, int n_sink, int window_size, int dtype,
                           void* workspace, size_t workspace_bytes,
                           void* stream);
orin_status orin_attention_workspace_bytes(size_t* bytes, int seq_len,
                                           int cache_len, int num_heads,
                                           int num_kv_heads, int head_dim,
                                           int n_sink, int window_size);

/*
 * orin_attention over `batch` independent sequences in one launch (batched
 * decode; the reference's engine is single-sequence, include/kv_cache.h:7, so
 * this has no counterpart there).  Every sequence has seq_len new tokens at
 * the same positions (cache_len); q and out hold [batch][seq_len][num_heads]
 * [head_dim]; sequence b's pools start pool_stride elements after sequence
 * b-1's (pool_stride >= (n_sink + window_size) * num_kv_heads * head_dim,
 * a multiple of 8).  Each sequence is computed exactly as its own
 * orin_attention call would be (same key splits, same summation order), so
 * its output is bit-identical to that call's; the workspace for that is batch
 * times orin_attention_workspace_bytes (a smaller one splits less).
 */
orin_status orin_attention_batch(void* out, const void* q, const void* k_pool,
                                 const void* v_pool, int batch, long long pool_stride,
                                 int seq_len, int cache_len, int num_heads,
                                 int num_kv_heads, int head_dim, float scale,
                                 int n_sink, int window_size, int dtype,
                                 void* workspace, size_t workspace_bytes,
                                 void* stream);

/*
 * orin_attention_batch with flags (batch 1 is a single sequence).
 * ORIN_ATTN_OWN_SLOTS_ONLY: the caller states that no kernel that may still
 * be running when this call starts writes a slot of these pools other than
 * those of this call's own positions (a decode step whose only pool write is
 * the new token's orin_linear_rope_append, orin_qkv_rope_append(_batch) or
 * orin_kv_append); a single-token call then loads the other slots' keys and
 * values before the previous kernel has finished.  Without the flag every
 * load waits for it.
 */
#define ORIN_ATTN_OWN_SLOTS_ONLY 1u
orin_status orin_attention_batch_ex(void* out, const void* q, const void* k_pool,
                                    const void* v_pool, int batch,
                                    long long pool_stride, int seq_len, int cache_len,
                                    int num_heads, int num_kv_heads, int head_dim,
                                    float scale, int n_sink, int window_size, int dtype,
                                    void* workspace, size_t workspace_bytes,
                                    unsigned flags, void* stream);

/*
 * Synchronise stream and report device-side failures of this library's
 * kernels: every spin-wait inside them gives up after a bounded time and
 * records an error code instead of hanging.  Returns ORIN_ERR_TIMEOUT (and
 * clears the record) if one did.
 */
orin_status orin_device_check(void* stream);

/* ------------------------------------------------------------------------ */
/* Tensor parallelism over NCCL (no counterpart in the reference, which is   */
/* single-GPU: include/kv_cache.h:7).  One process per GPU.                  */
/* ------------------------------------------------------------------------ */

#define ORIN_TP_UNIQUE_ID_BYTES 128

/* Rank 0 creates the id and shares it (e.g. through a torch.distributed
 * store); every rank then calls orin_tp_init with it. */
orin_status orin_tp_unique_id(void* id_out /* ORIN_TP_UNIQUE_ID_BYTES */);

/* Create this rank's communicator on `device`.  The NCCL communicator is
 * non-blocking; a collective that has not finished after timeout_s seconds
 * is aborted and reported as ORIN_ERR_TIMEOUT. */
orin_status orin_tp_init(void** comm_out, const void* id, int rank,
                         int world_size, int device, double timeout_s);

/* In-place fp32 sum over all ranks of buf[n] on stream. */
orin_status orin_tp_allreduce_f32(void* comm, float* buf, long long n,
                                  void* stream);

/*
 * Row-parallel linear (o_proj / down_proj sharded along K):
 *   partial = A_shard · W_shard^T  (fp32, unrounded, [M, N])
 *   sum     = all-reduce(partial)  over ranks
 *   C       = round16(f32(residual) + f32(round16(sum)))   if residual
 *           = round16(sum)                                   otherwise
 * partial_f32 is caller scratch of M*N floats (may be NULL when the call
 * takes the peer-memory reduction below).  C may alias residual.
 */
orin_status orin_tp_linear_row(void* comm, void* C, const void* A_shard,
                               const void* W_shard, int M, int N, int K_shard,
                               int dtype, const void* residual,
                               float* partial_f32, void* stream);

/*
 * orin_tp_linear_row without the caller's partial buffer (no counterpart in
 * the reference): the fp32 partial sums live in a file-scope device array of
 * orin_tp_static_partial_capacity() floats (64 MiB), one per device; the
 * entry point allocates nothing.  M*N above that capacity returns
 * ORIN_ERR_UNSUPPORTED.  The array is shared by every call on a device: calls
 * on one device must be ordered (one stream), or they corrupt each other's
 * sums.  The first call on a device looks the array up and must not be
 * inside stream capture.
 */
orin_status orin_tp_linear_row_static(void* comm, void* C, const void* A_shard,
                                      const void* W_shard, int M, int N, int K_shard,
                                      int dtype, const void* residual, void* stream);

/* Floats of the static partial-sum array behind orin_tp_linear_row_static. */
long long orin_tp_static_partial_capacity(void);

/*
 * Vocabulary-parallel LM head + greedy argmax: this rank holds rows
 * [v_offset, v_offset + V_shard) of the LM head (any split, ragged allowed);
 * every rank gets the same token[m] as orin_lm_head_argmax over the whole
 * vocabulary, tie-break included: each rank reduces its shard to one 64-bit
 * key per row (the order the tie-break defines), one ncclAllReduce(max) of
 * M keys combines them.  keys: caller scratch of M 64-bit words.
 */
orin_status orin_tp_lm_head_argmax(void* comm, int* token, const void* h,
                                   const void* W_shard, int M, int V_shard,
                                   int v_offset, int K, int dtype,
                                   unsigned long long* keys, void* stream);

/*
 * Give the communicator a peer-memory reduction for row-parallel calls
 * (no counterpart in the reference).  Collective: every rank calls it with
 * the same max_elems.  Each rank allocates one region (fp32 partials and
 * 16-bit results of max_elems elements, plus flags) and maps every peer's
 * (CUDA IPC over NVLink; the handles travel over the communicator).  From
 * then on orin_tp_linear_row with M*N <= max_elems, N % 8 == 0 and 16-byte
 * aligned C and residual reduces with one kernel of plain peer loads and
 * stores instead of ncclAllReduce: each rank sums the rows it owns over all
 * ranks in rank order (deterministic), applies residual and rounding, and
 * copies the other ranks' finished rows (blocks synchronise only with the
 * same block of each peer).  Every cross-GPU wait gives up after
 * 2 s (orin_device_check reports ORIN_ERR_TIMEOUT; destroy the communicator).
 * ORIN_ERR_UNSUPPORTED if the GPUs can't map each other's memory.
 */
orin_status orin_tp_enable_p2p(void* comm, long long max_elems, void* stream);

/*
 * Diagnostic of the cross-GPU watchdog, on one GPU: runs the peer-memory
 * reduction kernel against a "peer" that never signals (a plain buffer).
 * The kernel must give up its bounded wait after 2 s and record a timeout in
 * the device error word; the next orin_device_check then returns
 * ORIN_ERR_TIMEOUT (and clears it) while the context stays usable.  Returns
 * after the kernel has finished.
 */
orin_status orin_p2p_watchdog_selftest(void* stream);

/* Block until every collective of comm issued on stream is done or the
 * timeout passes (then the communicator is aborted). */
orin_status orin_tp_wait(void* comm, void* stream);

orin_status orin_tp_destroy(void* comm);

#ifdef __cplusplus
}
#endif

#endif /* ORIN_B200_H */
