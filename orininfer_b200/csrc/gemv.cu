// gemv.cu — decode-time linear layers (M <= 32 tokens) as a weight stream.
//
// At decode the weight matrix is read once per step and the token count is
// tiny, so the kernel is bound by how early and how deeply it can keep HBM
// busy.  Design:
//
// * One CTA (8 warps) per group of 16 output features: its 16 weight rows
//   (32 for SwiGLU: 16 gate rows and the 16 matching up rows of the packed
//   layout), over the whole of K, split evenly across the 8 warps.
// * Every lane streams two weight rows (g and g + 8, g = lane / 4) with
//   128-bit non-caching loads: lanes 4g .. 4g+3 cover 64 contiguous bytes of a
//   row per 32-element k-block.  The loads of a batch of k-blocks are all in
//   flight at once (registers, not shared memory, hold them).
// * The products run on mma.sync.m16n8k16 (fp32 accumulate): weight rows are
//   the MMA's M, tokens its N (8 per tile).  Within a 32-element k-block the
//   two MMAs use a fixed permutation of k, the same for weights and tokens:
//   lane (g, q) holds k = 8q .. 8q+7 of its rows and of token g, words 0-1 for
//   the first MMA and 2-3 for the second.  A permutation of the k-sum leaves
//   the dot product unchanged, and every 16-byte load is already a fragment.
// * The first batch of weight loads and an L2 prefetch of the rest of the
//   warp's weights are issued before griddepcontrol.wait: weights do not
//   depend on the previous kernel, so under programmatic dependent launch
//   they stream while it finishes.  Tokens and the residual are read after
//   the wait, through L2 (ld.global.cg).
// * The 8 warps' partial fragments are summed in shared memory in warp order
//   (deterministic), and warp 0 applies the epilogue with the rounding points
//   of the other kernels.
// * EPI_ROPE (the stacked q/k/v projection at decode): a CTA streams rows
//   8j + g and 8j + g + head_dim / 2 of one head instead of 16 consecutive
//   rows, so every lane holds both dims of its RoPE pairs; one warp per
//   (token tile, token parity) rounds, rotates and writes q to its buffer and
//   k / v to their ring slots (the separate RoPE/append kernel's values).
//
// The reference's decode path is kernels/matmul.cu:25-44 (one CTA per output
// row, 2-byte loads, shared-memory tree reduction); this replaces it for
// M = 1 and the skinny cuBLAS calls for M <= 32.  No spin-waits, no mbarriers.
#include "orin_common.cuh"
#include "orin_internal.h"

namespace orin {
namespace {

constexpr int kGvWarps = 8;
constexpr int kGvThreads = kGvWarps * 32;
constexpr int kGvRows = 16;    // output features per CTA (MMA M)
constexpr int kGvBlockK = 32;  // k elements per block: two m16n8k16 MMAs
// NORM's dynamic shared memory cap (the norm weight, K 16-bit values): with
// the static arrays (at most 33 KB, the SwiGLU reduction of four token tiles)
// within the 227 KB a CTA may hold
constexpr size_t kGvMaxSmem = 192 * 1024;

struct GvParams {
  const void* W;
  const void* X;
  void* C;
  const void* R;
  int M, N, K;
  int w_rows;  // rows of W: N, or 2N for the packed gate/up weight
  int n_offset;  // EPI_ARGMAX: vocabulary position of row 0 (a tensor-parallel shard)
  const void* norm;  // NORM: RMSNorm weight [K] applied to every token row of X first
  float eps;
  // EPI_ROPE: W is the stacked [q | k | v] weight of num_heads + 2 num_kv_heads
  // heads; token m is token m % seq_len of sequence m / seq_len, at position
  // start_pos + m % seq_len; C is q_out [M][num_heads][head_dim], k and v go
  // to their ring slots in sequence b's pools (pool_stride elements apart)
  void* k_pool;
  void* v_pool;
  long long pool_stride;
  int head_dim, num_heads, num_kv_heads, seq_len, start_pos, n_sink, window;
  float theta;
};

__device__ __forceinline__ uint4 ld_weights(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Written by the previous kernel: read through L2 only.
__device__ __forceinline__ uint4 ld_l2_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ unsigned short ld_l2_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ void prefetch_l2_bytes(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <int DT>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (DT == DT_F16) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// Greedy-argmax key of logit v at vocabulary position n: larger is better.
// The reference's sampler (kernels/softmax.cu:52-73, one CTA of 512 threads)
// picks, among the positions of the maximum, the one whose residue n mod 512
// has the smallest 9-bit bit-reversal (its tree keeps the lower slot on ties,
// and two tied threads meet at their lowest differing bit), then the smallest
// n; values not above -FLT_MAX never count (key 0, which decodes to token 0,
// as the reference returns when nothing counts).
__device__ __forceinline__ unsigned long long argmax_key(float v, int n) {
  if (!(v > -3.402823466e38f)) return 0ull;
  // the reference compares with '>': -0 and +0 tie
  const uint32_t b = (v == 0.f) ? 0u : __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  const uint32_t rev = __brev(static_cast<uint32_t>(n) & 511u) >> 23;
  const uint32_t lo = ~((rev << 22) | (static_cast<uint32_t>(n) >> 9));
  return (static_cast<unsigned long long>(ord) << 32) | lo;
}

template <int DT>
__device__ __forceinline__ float bits_to_f(unsigned short b) {
  if constexpr (DT == DT_F16) return __half2float(__ushort_as_half(b));
  else return __bfloat162float(__ushort_as_bfloat16(b));
}

// x * r * w for the 8 16-bit values of one fragment word set, rounded as the
// RMSNorm kernel rounds its output.
template <int DT>
__device__ __forceinline__ uint4 rmsnorm8(uint4 x, float r, uint4 w) {
  using E = Elem<DT>;
  const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 a = E::unpack2(xs[i]);
    const float2 b = E::unpack2(ws[i]);
    o[i] = E::pack2(a.x * r * b.x, a.y * r * b.y);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// NT token tiles of 8 (M <= 8 * NT; NT = 1, 2 or 4).  NORM: the token rows are
// RMS-normalised on the way in (the reference's RMSNorm before the projection,
// kernels/rmsnorm.cu:7-34): every CTA sums the squares of the rows it reads
// anyway (fp32, fixed order), then multiplies each loaded fragment by r and the
// norm weight and rounds it to 16 bits, exactly what the separate kernel
// would have stored.
template <int DT, int EPI, int NT, bool NORM = false>
__global__ void __launch_bounds__(kGvThreads, 2) gemv_kernel(const GvParams p) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int H = (EPI == EPI_SWIGLU) ? 2 : 1;  // row sets per group: gate, up
  // k-blocks per load batch (registers: U * (2H + NT) 16-byte fragments)
  constexpr int U = (NT >= 4) ? 2 : (H == 2 || NT == 2) ? 4 : 8;
  constexpr int V = H * NT * 4;                   // fragment values per lane
  __shared__ float red[kGvWarps][V][32];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int q = lane & 3;
  const int f0 = blockIdx.x * kGvRows;  // first output feature of this CTA

  // first weight row of each row set (packed gate/up: 64-row gate and up
  // groups); a lane's two rows are rstride apart: 8, or for EPI_ROPE half a
  // head, so that each lane holds both dims of its RoPE pairs (the CTA takes
  // pairs 8j .. 8j + 7 of head f0 / head_dim's rows)
  int wrow[H];
  int rstride = 8;
  if constexpr (EPI == EPI_SWIGLU) {
    wrow[0] = (f0 / 64) * 128 + (f0 % 64);
    wrow[1] = wrow[0] + 64;
  } else if constexpr (EPI == EPI_ROPE) {
    const int cph = p.head_dim / kGvRows;  // CTAs per head
    wrow[0] = (blockIdx.x / cph) * p.head_dim + 8 * (blockIdx.x % cph);
    rstride = p.head_dim / 2;
  } else {
    wrow[0] = f0;
  }
  const int nkb = (p.K + kGvBlockK - 1) / kGvBlockK;
  const int kb0 = (warp * nkb) / kGvWarps;
  const int kb1 = ((warp + 1) * nkb) / kGvWarps;
  const T* W = static_cast<const T*>(p.W);
  const T* X = static_cast<const T*>(p.X);

  const T* wp[H][2];
  bool wv[H][2];
#pragma unroll
  for (int h = 0; h < H; ++h) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int row = wrow[h] + g + rstride * r;
      wv[h][r] = row < p.w_rows;
      wp[h][r] = W + static_cast<long long>(wv[h][r] ? row : 0) * p.K + 8 * q;
    }
  }

  float acc[H][NT][4];
#pragma unroll
  for (int h = 0; h < H; ++h)
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[h][t][i] = 0.f;

  // one batch of U k-blocks of this warp's weight rows into registers
  uint4 w[U][H][2];
  auto load_w = [&](int kb) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = (kb + u) * kGvBlockK + 8 * q;
      const bool kin = (kb + u < kb1) && (k < p.K);
#pragma unroll
      for (int h = 0; h < H; ++h)
#pragma unroll
        for (int r = 0; r < 2; ++r)
          w[u][h][r] = (kin && wv[h][r]) ? ld_weights(wp[h][r] + (kb + u) * kGvBlockK)
                                         : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  // The weights do not depend on the previous kernel: the first batch goes
  // into registers and the rest of this warp's k-range into L2 before
  // griddepcontrol.wait, so the weight stream overlaps the previous kernel.
  if (kb0 < kb1) load_w(kb0);
  {
    const int rest = kb0 + U;
    if (rest < kb1 && lane < kGvRows * H) {
      const int lr = lane % kGvRows;  // local row: g = lr % 8 of row set lr / 8
      const int row = wrow[lane / kGvRows] + (lr & 7) + rstride * (lr >> 3);
      const int k_end = (kb1 * kGvBlockK < p.K) ? kb1 * kGvBlockK : p.K;
      if (row < p.w_rows)
        prefetch_l2_bytes(W + static_cast<long long>(row) * p.K + rest * kGvBlockK,
                          static_cast<uint32_t>((k_end - rest * kGvBlockK) * 2));
    }
  }
  // NORM: the norm weight does not depend on the previous kernel either; it
  // is staged in shared memory here, so the main loop's token loads go out
  // back to back with no global load between them and the normalisation
  extern __shared__ uint4 s_nw[];  // [K / 8], NORM only
  if constexpr (NORM) {
    const T* NWg = static_cast<const T*>(p.norm);
    for (int c = threadIdx.x; c < p.K / 8; c += kGvThreads) s_nw[c] = ld_weights(NWg + 8 * c);
  }
  pdl_launch_dependents();
  pdl_wait();
  // RESIDUAL: warp 0's residual values (written by the previous kernel) are
  // fetched now, while the MMAs run, instead of in the epilogue; each lane
  // reads exactly the elements it later writes, so an in-place call (C == R)
  // is unaffected.
  float res[EPI == EPI_RESIDUAL ? NT * 4 : 1];
  if constexpr (EPI == EPI_RESIDUAL) {
    if (warp == 0) {
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int n = f0 + g + 8 * (i >> 1);
          const int m = 8 * t + 2 * q + (i & 1);
          res[t * 4 + i] = (n < p.N && m < p.M)
                               ? bits_to_f<DT>(ld_l2_u16(static_cast<const T*>(p.R) +
                                                         static_cast<long long>(m) * p.N + n))
                               : 0.f;
        }
    }
  }
  __shared__ float s_r[NORM ? kGemvMaxTokens : 1];
  if constexpr (NORM) {
    // the row statistics (the token rows come from the previous kernel)
    __shared__ float s_ss[kGvWarps][kGemvMaxTokens];
    for (int m = 0; m < p.M; ++m) {
      float ss = 0.f;
      for (int c = threadIdx.x; c < p.K / 8; c += kGvThreads) {
        const uint4 v = ld_l2_v4(X + static_cast<long long>(m) * p.K + 8 * c);
        const uint32_t vs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = E::unpack2(vs[i]);
          ss += f.x * f.x + f.y * f.y;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) s_ss[warp][m] = ss;
    }
    __syncthreads();
    if (threadIdx.x < p.M) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kGvWarps; ++w) tot += s_ss[w][threadIdx.x];
      s_r[threadIdx.x] = rsqrtf(tot / static_cast<float>(p.K) + p.eps);
    }
    __syncthreads();
  }
  for (int kb = kb0; kb < kb1; kb += U) {
    if (kb != kb0) load_w(kb);
    uint4 x[U][NT];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int k = (kb + u) * kGvBlockK + 8 * q;
      const bool kin = (kb + u < kb1) && (k < p.K);
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int tok = 8 * t + g;
        x[u][t] = (kin && tok < p.M) ? ld_l2_v4(X + static_cast<long long>(tok) * p.K + k)
                                     : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    if constexpr (NORM) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int k = (kb + u) * kGvBlockK + 8 * q;
        if ((kb + u < kb1) && (k < p.K)) {
          const uint4 nw = s_nw[k / 8];
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const int tok = 8 * t + g;
            if (tok < p.M) x[u][t] = rmsnorm8<DT>(x[u][t], s_r[tok], nw);
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int h = 0; h < H; ++h)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          mma_16816<DT>(acc[h][t], w[u][h][0].x, w[u][h][1].x, w[u][h][0].y, w[u][h][1].y,
                        x[u][t].x, x[u][t].y);
          mma_16816<DT>(acc[h][t], w[u][h][0].z, w[u][h][1].z, w[u][h][0].w, w[u][h][1].w,
                        x[u][t].z, x[u][t].w);
        }
  }
#pragma unroll
  for (int h = 0; h < H; ++h)
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[warp][(h * NT + t) * 4 + i][lane] = acc[h][t][i];
  __syncthreads();
  if constexpr (EPI == EPI_ROPE) {
    // One warp per (token tile t, token parity jj): lane (g, q) sums dims i
    // and i + head_dim / 2 of head hb (values t*4 + jj and t*4 + 2 + jj, in
    // the warp order of the other epilogues) for token 8t + 2q + jj, rounds
    // each to 16 bits as the projection stores it and rotates the pair as the
    // RoPE kernel does: one angle per thread.
    using TT = typename E::T;
    if (warp >= 2 * NT) return;
    const int t = warp >> 1, jj = warp & 1;
    const int m = 8 * t + 2 * q + jj;
    if (m >= p.M) return;
    float x0 = red[0][t * 4 + jj][lane], x1 = red[0][t * 4 + 2 + jj][lane];
#pragma unroll
    for (int ww = 1; ww < kGvWarps; ++ww) {
      x0 += red[ww][t * 4 + jj][lane];
      x1 += red[ww][t * 4 + 2 + jj][lane];
    }
    x0 = E::round(x0);
    x1 = E::round(x1);
    const int cph = p.head_dim / kGvRows;
    const int hb = blockIdx.x / cph;
    const int half = p.head_dim / 2;
    const int i = 8 * (blockIdx.x % cph) + g;
    const int b = m / p.seq_len;
    const int tok = m - b * p.seq_len;
    const int pos = p.start_pos + tok;
    if (hb < p.num_heads) {
      float c, sn;
      rope_angle(pos, i, p.head_dim, p.theta, c, sn);
      TT* dst = static_cast<TT*>(p.C) + (static_cast<size_t>(m) * p.num_heads + hb) * p.head_dim;
      dst[i] = E::from_f(x0 * c - x1 * sn);
      dst[i + half] = E::from_f(x0 * sn + x1 * c);
      return;
    }
    // a later token of this call that lands in the same ring slot owns it
    if (pos >= p.n_sink && tok + p.window < p.seq_len) return;
    const size_t kv_dim = static_cast<size_t>(p.num_kv_heads) * p.head_dim;
    const size_t ring =
        static_cast<size_t>(pos < p.n_sink ? pos : p.n_sink + (pos - p.n_sink) % p.window);
    const size_t off = static_cast<size_t>(b) * p.pool_stride + ring * kv_dim;
    if (hb < p.num_heads + p.num_kv_heads) {
      float c, sn;
      rope_angle(pos, i, p.head_dim, p.theta, c, sn);
      TT* dst = static_cast<TT*>(p.k_pool) + off +
                static_cast<size_t>(hb - p.num_heads) * p.head_dim;
      dst[i] = E::from_f(x0 * c - x1 * sn);
      dst[i + half] = E::from_f(x0 * sn + x1 * c);
    } else {
      TT* dst = static_cast<TT*>(p.v_pool) + off +
                static_cast<size_t>(hb - p.num_heads - p.num_kv_heads) * p.head_dim;
      dst[i] = E::from_f(x0);
      dst[i + half] = E::from_f(x1);
    }
    return;
  }
  if (warp != 0) return;

  float s[V];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    float a = red[0][v][lane];
#pragma unroll
    for (int ww = 1; ww < kGvWarps; ++ww) a += red[ww][v][lane];
    s[v] = a;
  }
  if constexpr (EPI == EPI_ARGMAX) {
    // per token: the best key of the CTA's 16 positions (the 8 lanes of equal
    // q hold them), then one atomicMax per token
    unsigned long long* keys = static_cast<unsigned long long*>(p.C);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        unsigned long long k = 0ull;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int n = f0 + g + 8 * r;
          const unsigned long long kr =
              (n < p.N) ? argmax_key(E::round(s[t * 4 + 2 * r + j]), n + p.n_offset) : 0ull;
          k = kr > k ? kr : k;
        }
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
          k = o > k ? o : k;
        }
        const int m = 8 * t + 2 * q + j;
        if (g == 0 && m < p.M && k != 0ull) atomicMax(keys + m, k);
      }
    }
    return;
  }
  // fragment value i of tile t: row g + 8*(i/2), token 8t + 2q + (i%2)
#pragma unroll
  for (int t = 0; t < NT; ++t) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int n = f0 + g + 8 * (i >> 1);
      const int m = 8 * t + 2 * q + (i & 1);
      if (n >= p.N || m >= p.M) continue;
      const long long o = static_cast<long long>(m) * p.N + n;
      const float a = s[t * 4 + i];
      if constexpr (EPI == EPI_NONE) {
        static_cast<T*>(p.C)[o] = E::from_f(a);
      } else if constexpr (EPI == EPI_RESIDUAL) {
        static_cast<T*>(p.C)[o] = E::from_f(res[t * 4 + i] + E::round(a));
      } else if constexpr (EPI == EPI_F32_OUT) {
        static_cast<float*>(p.C)[o] = E::round(a);
      } else if constexpr (EPI == EPI_F32_PARTIAL) {
        static_cast<float*>(p.C)[o] = a;
      } else {
        const float u = s[(NT + t) * 4 + i];
        static_cast<T*>(p.C)[o] = E::from_f(silu_fast(E::round(a)) * E::round(u));
      }
    }
  }
}

template <int DT, int EPI, int NT, bool NORM = false>
cudaError_t gemv_launch(const GvParams& p, cudaStream_t s) {
  const size_t smem = NORM ? static_cast<size_t>(p.K) * 2 : 0;
  if (smem > 48 * 1024) {
    // the cap, once per device: every call's size is at most that
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
      cudaError_t e = cudaFuncSetAttribute(gemv_kernel<DT, EPI, NT, NORM>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(kGvMaxSmem));
      if (e != cudaSuccess) return e;
      if (dev >= 0 && dev < 64) configured[dev] = 1;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.N + kGvRows - 1) / kGvRows);
  cfg.blockDim = dim3(kGvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<DT, EPI, NT, NORM>, p);
}

template <int DT, int NT>
cudaError_t gemv_dispatch(const GvParams& p, int epi, cudaStream_t s) {
  if (p.norm) {  // RMSNorm folded in: the projections that follow a norm
    switch (epi) {
      case EPI_NONE: return gemv_launch<DT, EPI_NONE, NT, true>(p, s);
      case EPI_SWIGLU: return gemv_launch<DT, EPI_SWIGLU, NT, true>(p, s);
      case EPI_ARGMAX: return gemv_launch<DT, EPI_ARGMAX, NT, true>(p, s);
    }
    return cudaErrorInvalidValue;
  }
  switch (epi) {
    case EPI_NONE: return gemv_launch<DT, EPI_NONE, NT>(p, s);
    case EPI_SWIGLU: return gemv_launch<DT, EPI_SWIGLU, NT>(p, s);
    case EPI_RESIDUAL: return gemv_launch<DT, EPI_RESIDUAL, NT>(p, s);
    case EPI_F32_OUT: return gemv_launch<DT, EPI_F32_OUT, NT>(p, s);
    case EPI_F32_PARTIAL: return gemv_launch<DT, EPI_F32_PARTIAL, NT>(p, s);
    case EPI_ARGMAX: return gemv_launch<DT, EPI_ARGMAX, NT>(p, s);
    case EPI_ROPE: return gemv_launch<DT, EPI_ROPE, NT>(p, s);
  }
  return cudaErrorInvalidValue;
}

// token[m] = the vocabulary position encoded in keys[m] (0 when nothing counted).
__global__ void argmax_decode_kernel(int* token, const unsigned long long* keys, int M) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  const unsigned long long k = keys[m];
  if (k == 0ull) {
    token[m] = 0;
    return;
  }
  const uint32_t lo = ~static_cast<uint32_t>(k);
  const uint32_t residue = __brev(lo >> 22) >> 23;
  token[m] = static_cast<int>(((lo & 0x3fffffu) << 9) | residue);
}

}  // namespace

int gemv_grid(int N) { return (N + kGvRows - 1) / kGvRows; }

cudaError_t launch_argmax_keys(unsigned long long* keys, const void* A, const void* W, int M,
                               int V, int K, int dtype, int v_offset, cudaStream_t s,
                               const void* norm, float eps) {
  const size_t esz = 2;
  for (int r0 = 0; r0 < M; r0 += kGemvMaxTokens) {
    const int rows = (M - r0) < kGemvMaxTokens ? (M - r0) : kGemvMaxTokens;
    cudaError_t e = cudaMemsetAsync(keys + r0, 0, rows * sizeof(unsigned long long), s);
    if (e != cudaSuccess) return e;
    e = launch_gemv(keys + r0, static_cast<const char*>(A) + static_cast<size_t>(r0) * K * esz, W,
                    rows, V, K, dtype, EPI_ARGMAX, nullptr, s, v_offset, norm, eps);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_argmax_decode(int* token, const unsigned long long* keys, int M,
                                 cudaStream_t s) {
  argmax_decode_kernel<<<(M + 127) / 128, 128, 0, s>>>(token, keys, M);
  return cudaGetLastError();
}

cudaError_t launch_gemv_rope(void* q_out, const void* A, const void* W, int M, int K, int dtype,
                             int num_heads, int num_kv_heads, int head_dim, int seq_len,
                             int start_pos, float theta, int n_sink, int window, void* k_pool,
                             void* v_pool, long long pool_stride, cudaStream_t s) {
  if (M < 1 || M > kGemvMaxTokens || K % 8 != 0 || head_dim % kGvRows != 0 || seq_len < 1 ||
      M % seq_len != 0)
    return cudaErrorInvalidValue;
  GvParams p = {};
  p.W = W;
  p.X = A;
  p.C = q_out;
  p.M = M;
  p.N = (num_heads + 2 * num_kv_heads) * head_dim;
  p.K = K;
  p.w_rows = p.N;
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.pool_stride = pool_stride;
  p.head_dim = head_dim;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.seq_len = seq_len;
  p.start_pos = start_pos;
  p.n_sink = n_sink;
  p.window = window;
  p.theta = theta;
  if (dtype == DT_F16)
    return (M <= 8)    ? gemv_dispatch<DT_F16, 1>(p, EPI_ROPE, s)
           : (M <= 16) ? gemv_dispatch<DT_F16, 2>(p, EPI_ROPE, s)
                       : gemv_dispatch<DT_F16, 4>(p, EPI_ROPE, s);
  return (M <= 8)    ? gemv_dispatch<DT_BF16, 1>(p, EPI_ROPE, s)
         : (M <= 16) ? gemv_dispatch<DT_BF16, 2>(p, EPI_ROPE, s)
                     : gemv_dispatch<DT_BF16, 4>(p, EPI_ROPE, s);
}

cudaError_t launch_gemv(void* C, const void* A, const void* W, int M, int N, int K, int dtype,
                        int epi, const void* R, cudaStream_t s, int n_offset, const void* norm,
                        float eps) {
  if (M < 1 || M > kGemvMaxTokens) return cudaErrorInvalidValue;
  if (norm && K % 8 != 0) return cudaErrorInvalidValue;
  if (norm && static_cast<size_t>(K) * 2 > kGvMaxSmem) return cudaErrorInvalidValue;
  GvParams p = {};
  p.n_offset = n_offset;
  p.norm = norm;
  p.eps = eps;
  p.W = W;
  p.X = A;
  p.C = C;
  p.R = R;
  p.M = M;
  p.N = N;
  p.K = K;
  p.w_rows = (epi == EPI_SWIGLU) ? 2 * N : N;
  if (dtype == DT_F16)
    return (M <= 8)    ? gemv_dispatch<DT_F16, 1>(p, epi, s)
           : (M <= 16) ? gemv_dispatch<DT_F16, 2>(p, epi, s)
                       : gemv_dispatch<DT_F16, 4>(p, epi, s);
  return (M <= 8)    ? gemv_dispatch<DT_BF16, 1>(p, epi, s)
         : (M <= 16) ? gemv_dispatch<DT_BF16, 2>(p, epi, s)
                     : gemv_dispatch<DT_BF16, 4>(p, epi, s);
}

}  // namespace orin
