// orin_internal.h — host-side declarations shared by the library's .cu files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace orin {

// Problem description handed to the tcgen05 kernels (by value, in the
// kernel's parameter space).  "P" is the operand whose rows fill the 128
// accumulator lanes of a tile, "Q" the operand whose rows fill its BN
// accumulator columns.  Wide tiles: P = activations, Q = weights.  Skinny
// (swap) tiles: P = weights, Q = activations.
struct TcParams {
  int P, Q, K;
  int M, N;          // logical output C[M, N] (N = output columns)
  int tiles_p, tiles_q, kb;
  int split;         // 1: persistent over tiles; S > 1: clusters of S CTAs
                     //    split each tile's K range
  int group_p;       // raster: this many P tiles walk together
  void* C;
  long long ldc;     // elements
  const void* R;     // residual (EPI_RESIDUAL)
  long long ldr;
  int* err;          // device error word
  int vec_ok;        // C / R rows are 16-byte aligned for vector stores
  int out_tma;       // wide tiles: stores (and the residual) go through TMA
  // Stream-K (wide tiles, split == 1): the tiles x K work is dealt to the
  // persistent CTA groups in equal contiguous ranges of k-block pairs, so a
  // tile's K range may be shared by consecutive groups.  A group whose range
  // starts inside a tile writes that partial accumulator to its slot of
  // sk_ws (kBM x BN floats per CTA) and raises its flag; the group that holds
  // the tile's first k-blocks adds those partials in group order and stores.
  int sk;            // 1: stream-K schedule
  float* sk_ws;      // gridDim.x slots of kBM * BN floats
  int* sk_flags;     // gridDim.x flags, zero between calls
};

struct Plan {
  int algo;          // 1 wide, 2 skinny, 3 simt, 4 gemv
  int bn;            // tile columns (Q extent)
  int pair;          // 1: tiles of 256 P rows on tcgen05 CTA pairs
  int grid;
  TcParams p;
};

// Per-device state: SM count and the device error word.
struct DeviceCtx {
  int device = -1;
  int sm_count = 0;
  int* err = nullptr;        // device address of the error word
};

DeviceCtx* device_ctx(int device, cudaError_t* e);
bool device_ctx_ready(int device);

// Fill the tiling / scheduling fields of a plan for the tcgen05 kernels.
// sk_bytes: caller workspace available for a stream-K schedule (0: none).
void plan_tc(Plan& pl, int M, int N, int K, int epi, int algo, int sm_count,
             size_t sk_bytes = 0);

// Stream-K workspace layout: kSkFlagBytes of flag words (one per CTA, grids of
// up to kSkMaxGrid CTAs, zero between calls) at the start, then one slot of
// 128 x BN floats per CTA.  The flags sit at a fixed offset whatever the plan,
// so slots written by one call never land on another call's flags.
constexpr int kSkMaxGrid = 1024;
constexpr size_t kSkFlagBytes = kSkMaxGrid * sizeof(int);
size_t sk_workspace_bytes(int grid, int bn);
// Bytes that unlock every stream-K plan on a device with sm_count SMs.
size_t sk_workspace_max_bytes(int sm_count);

// Launch the tcgen05 GEMM described by pl.
// sk_ws: the caller's workspace when pl is a stream-K plan (else unused).
cudaError_t launch_tc(const Plan& pl, int dtype, int epi, const void* A, const void* W,
                      int* err, cudaStream_t stream, const char** why, void* sk_ws = nullptr);

// Decode-time weight-streaming kernel (csrc/gemv.cu) for M <= kGemvMaxTokens,
// K % 8 == 0 and 16-byte aligned A and W.  Same epilogues and rounding.
constexpr int kGemvMaxTokens = 32;
// norm (optional): RMSNorm weight [K] applied to the rows of A first (eps);
// epilogues NONE, SWIGLU and ARGMAX only.
cudaError_t launch_gemv(void* C, const void* A, const void* W, int M, int N, int K, int dtype,
                        int epi, const void* R, cudaStream_t stream, int n_offset = 0,
                        const void* norm = nullptr, float eps = 0.f);
int gemv_grid(int N);
// The stacked q/k/v projection on the weight stream with RoPE and the K/V
// append in its epilogue (M = batch * seq_len tokens, K % 8 == 0, head_dim a
// multiple of 16): q_out [M][num_heads][head_dim], k and v into the ring
// slots of sequence m / seq_len's pools; the same values as launch_gemv then
// launch_qkv_rope_append without q/k norms.
cudaError_t launch_gemv_rope(void* q_out, const void* A, const void* W, int M, int K, int dtype,
                             int num_heads, int num_kv_heads, int head_dim, int seq_len,
                             int start_pos, float theta, int n_sink, int window, void* k_pool,
                             void* v_pool, long long pool_stride, cudaStream_t stream);
// LM head + greedy argmax per row: keys[m] = the best 64-bit argmax key of
// row m over the V vocabulary rows of W (positions v_offset + v), then
// token[m] = its position (keys: caller scratch of M words).
cudaError_t launch_argmax_keys(unsigned long long* keys, const void* A, const void* W, int M,
                               int V, int K, int dtype, int v_offset, cudaStream_t stream,
                               const void* norm = nullptr, float eps = 0.f);
cudaError_t launch_argmax_decode(int* token, const unsigned long long* keys, int M,
                                 cudaStream_t stream);

// CUDA-core GEMM for shapes the tcgen05 path can't take (K % 8 != 0,
// unaligned rows).  Same epilogues and rounding.
cudaError_t launch_simt(void* C, const void* A, const void* W, int M, int N, int K, int dtype,
                        int epi, const void* R, cudaStream_t stream);

// Elementwise kernels (the reference's unfused neighbours of matmul).
cudaError_t launch_silu_mul(void* out, const void* gate, const void* up, long long n,
                            int dtype, cudaStream_t s);
cudaError_t launch_add(void* x, const void* y, long long n, int dtype, cudaStream_t s);
cudaError_t launch_widen(float* out, const void* in, long long n, int dtype, cudaStream_t s);
cudaError_t launch_pack_gate_up(void* wp, const void* wg, const void* wu, int IM, int K,
                                int dtype, cudaStream_t s);
// C = round16(f32(R) + round16(S)) (R may be null: C = round16(S)); S fp32.
cudaError_t launch_finish_rows(void* C, const float* S, const void* R, long long n, int dtype,
                               cudaStream_t s);

// Sink + sliding-window GQA attention over the ring KV pool and the K/V
// scatter into it (csrc/attention.cu).  head_dim 64 or 128.
struct AttnPlan {
  int rw;                  // warps stacked on rows (1: decode blocks, 4: prefill)
  int hpb, tpb, hsb;       // group heads / tokens per row block; row blocks per group
  int splits;              // key splits across CTAs (1: no workspace used)
  long long row_blocks;
  size_t workspace_bytes;  // what `splits` needs
};
// A split plan's workspace starts with kAttnCounterBytes of arrival counters
// (one int per CTA row of the grid; zero before the first call, left zero by
// every call), then the split partials.
constexpr size_t kAttnCounterBytes = 4096;
// launch_attention flags: the kernel issued just before on the stream wrote
// no pool slot other than those of the call's own positions (ORIN_ATTN_OWN_SLOTS_ONLY)
constexpr int kAttnOwnSlotsOnly = 1;
AttnPlan plan_attention(int seq_len, int cache_len, int num_heads, int num_kv_heads,
                        int head_dim, int n_sink, int window, size_t workspace_bytes);
// `batch` sequences of seq_len tokens each, all at the same positions: q/out
// rows [batch][seq_len][num_heads][head_dim], sequence b's pools at
// k_pool/v_pool + b * pool_stride elements.  Every sequence gets the plan a
// single-sequence call would (the workspace is divided among them), so each
// sequence's result is bit-identical to its own batch-1 call.
cudaError_t launch_attention(void* out, const void* q, const void* k_pool, const void* v_pool,
                             int seq_len, int cache_len, int num_heads, int num_kv_heads,
                             int head_dim, float scale, int n_sink, int window, int dtype,
                             void* workspace, size_t workspace_bytes, cudaStream_t s,
                             int batch = 1, long long pool_stride = 0, int* err = nullptr,
                             int flags = 0);
// The tensor-core prefill kernel (csrc/attention_tc.cu): one sequence, head
// dim 64 or 128, a GQA group that divides 128 (or a multiple of 128), at
// least 128 query rows.  launch_attention picks it for calls with 32 or more
// 128-row blocks; the ORIN_ATTN_KERNEL tuning override ("mma", "tc", "tc1"
// or "tc2", read once per process) forces one kernel where both apply.
// pairing: 0 lets the launcher choose between one query tile per CTA and two
// (head dim 64), 1 forces one, 2 forces two where the head dim allows.
bool attention_tc_supported(int seq_len, int num_heads, int num_kv_heads, int head_dim,
                            int n_sink, int window);
cudaError_t launch_attention_tc(void* out, const void* q, const void* k_pool, const void* v_pool,
                                int seq_len, int cache_len, int num_heads, int num_kv_heads,
                                int head_dim, float scale, int n_sink, int window, int dtype,
                                int* err, cudaStream_t s, int pairing = 0);
// A row-major [rows, cols] 16-bit (type 0 f16, 1 bf16) or fp32 (type 2)
// matrix as a TMA map with box_cols x box_rows boxes, 128-byte swizzle
// (box_cols * element size = 128), zero fill (csrc/gemm_tc.cu).
bool encode_tmap_2d(CUtensorMap* out, const void* ptr, int type, unsigned long long rows,
                    unsigned long long cols, int box_cols, int box_rows);
cudaError_t launch_kv_scatter(void* k_pool, void* v_pool, const void* k_src, const void* v_src,
                              int seq_len, int start_pos, int n_sink, int window, int kv_dim,
                              cudaStream_t s);

// RMSNorm over rows, rotary embedding, and the fused per-head norm + rotation
// + K/V scatter that follows this library's q/k/v projection (csrc/norm_rope.cu).
cudaError_t launch_embedding(void* out, const void* table, const int* ids, int seq_len,
                             int hidden, int vocab, cudaStream_t s);
cudaError_t launch_rmsnorm(void* out, const void* x, const void* w, int rows, int dim, float eps,
                           int dtype, cudaStream_t s);
cudaError_t launch_rope(void* q, void* k, int seq_len, int num_heads, int num_kv_heads,
                        int head_dim, int start_pos, float theta, int dtype, cudaStream_t s);
cudaError_t launch_qkv_rope_append(void* q_out, const void* qkv, const void* q_norm,
                                   const void* k_norm, void* k_pool, void* v_pool, int seq_len,
                                   int start_pos, int num_heads, int num_kv_heads, int head_dim,
                                   float eps, float theta, int n_sink, int window, int dtype,
                                   cudaStream_t s, int batch = 1, long long pool_stride = 0);

// Row-parallel reduction over peer memory (csrc/tp_p2p.cu).  Each rank's
// shared region starts with a flag block of ints written by the peers, one
// per (block, rank): "partial ready" at kP2PArrive + b * kP2PMaxRanks + rank,
// "rows done" at kP2PDone + b * kP2PMaxRanks + rank.
constexpr int kP2PMaxRanks = 8;
constexpr int kP2PMaxBlocks = 1024;
constexpr int kP2PArrive = 0;
constexpr int kP2PDone = kP2PMaxBlocks * kP2PMaxRanks;
constexpr int kP2PFlagBytes = 2 * kP2PMaxBlocks * kP2PMaxRanks * 4;
struct P2PView {
  int rank, world, N;
  long long row0[kP2PMaxRanks + 1];  // rank r owns rows [row0[r], row0[r+1])
  const float* partial[kP2PMaxRanks];
  const void* result[kP2PMaxRanks];
  int* flags[kP2PMaxRanks];
  int* local_flags;
  void* result_local;
  void* C;
  const void* R;
  int* epoch;  // kP2PMaxBlocks per-block epochs (this rank's memory)
  int* err;
};
cudaError_t launch_p2p_reduce(const P2PView& v, int dtype, cudaStream_t s);

// Launch `kern` with programmatic dependent launch allowed (it may start while
// the previous kernel on the stream finishes; it orders itself with
// griddepcontrol.wait) and `smem` bytes of dynamic shared memory.
template <class... KArgs, class... Args>
cudaError_t launch_pdl_smem(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Record a failure message for orin_last_error().
void set_error(const char* fmt, ...);

// The CUDA device ordinal a tensor-parallel communicator (orin_tp_init's
// handle) was created on (csrc/tp.cu).
int tp_comm_device(const void* comm);

}  // namespace orin
