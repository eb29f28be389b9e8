// gemm_tc.cu — the sm_100a linear-layer kernel: C = epilogue(A · W^T).
//
// One kernel template covers both tensor-core shapes of the hot path:
//   * wide tiles (prefill, M > 64): 128 tokens x {128,256} weight rows per
//     CTA, or 256 tokens x {128,256} on a tcgen05 CTA pair (cta_group::2:
//     each CTA of the pair loads its 128 A rows and half the B rows, the
//     leader issues M=256 MMAs);
//   * skinny tiles (decode, 17-64 tokens; 1-16 go to gemv.cu): 128 weight
//     rows x {16,32,64} tokens ("swap AB": the weight matrix feeds the
//     128-lane side of the MMA).  With <= 32 token columns a CTA takes at most
//     113 KB of shared memory, so two fit on an SM and the next kernel's CTAs
//     are resident (programmatic dependent launch) while this one finishes.
//
// Per CTA, 192 threads (one CTA per SM for wide tiles):
//   warp 0    TMA producer: 2-D tiled loads, 128-byte swizzle, into a ring of
//             stage pairs guarded by mbarriers (one full/empty barrier per
//             pair).  Weight tiles of the first ring pass are issued before
//             the grid waits on the previous kernel.
//   warp 1    MMA issuer: one thread issues tcgen05.mma kind::f16 (fp16/bf16
//             in, fp32 accumulate) into a double-buffered tensor-memory
//             accumulator; tcgen05.commit frees ring slots.
//   warps 2-5 epilogue: tcgen05.ld, the fused epilogue (SwiGLU / residual /
//             fp32), stores — through 128-byte-swizzled staging and TMA stores
//             for wide tiles, per element (coalesced) for skinny tiles.
//
// Scheduling (chosen on the host per problem, gemm_tc.cu plan_tc):
//   * split 1 — persistent: CTA (pair) c takes tiles c, c+grid, ... over the
//     full K; the next tile's mainloop overlaps this tile's epilogue.  Tiles
//     are rastered in groups of P tiles so concurrent CTAs share L2 panels.
//   * split S — fewer tiles than SMs: each tile's K range is split over a
//     thread-block cluster of S CTAs (or S pairs).  Wide tiles: every CTA
//     stages the 32-column units other CTAs own in shared memory and sends
//     each owner its block with one bulk DSMEM copy; owners add them to their
//     own units in rank order.  Skinny tiles: every CTA pushes each partial
//     row straight from tensor memory into the shared memory of the CTA that
//     owns that feature; one cluster barrier, then owners sum in rank order.
//     Deterministic, no global workspace, no atomics.
//
// Every mbarrier wait is bounded (orin_common.cuh): after 2 s the CTA records
// an error code in the device error word and unwinds instead of hanging.
//
// Reference semantics (kernels/matmul.cu:32-43, kernels/gemm_cute.cu:147,
// 176-178): fp32 products and accumulation, one rounding to 16 bits.
#include "orin_common.cuh"
#include "orin_internal.h"

#include <stdio.h>
#include <stdlib.h>

namespace orin {

constexpr int kBM = 128;       // tile rows = MMA M = tensor-memory lanes
constexpr int kBK = 64;        // K per ring stage: one 128-byte row of 16-bit
constexpr int kUmmaK = 16;     // K per tcgen05.mma kind::f16
constexpr int kThreads = 192;  // 6 warps
constexpr int kEpiThreads = 128;
constexpr int kGroupP = 8;     // P tiles per raster group

// Weight/token rows (Q operand) one CTA loads per stage: a CTA pair splits
// them between its two CTAs.
__host__ __device__ constexpr int tc_qrows(int bn, bool pair) { return pair ? bn / 2 : bn; }
__host__ __device__ constexpr int tc_stage_bytes(int bn, bool pair) {
  return kBM * kBK * 2 + tc_qrows(bn, pair) * kBK * 2;
}
__host__ __device__ constexpr uint32_t tc_tmem_cols(int bn) {
  // two accumulator buffers of bn fp32 columns, rounded to a power of two >= 32
  return (2 * bn <= 32) ? 32u : (2 * bn <= 64) ? 64u : (2 * bn <= 128) ? 128u
                                               : (2 * bn <= 256) ? 256u : 512u;
}
__host__ __device__ constexpr int tc_xch_bytes(int bn, int epi, bool swap) {
  // skinny SwiGLU: up-half rows hand their rounded values to gate-half rows
  return (swap && epi == EPI_SWIGLU) ? 64 * 32 * 4 : 0;
}
// Skinny split-K: every CTA of a cluster pushes each fp32 partial row of its
// tile into the shared memory of the CTA that owns (reduces) that row.  Owners
// hold contiguous slices of the tile's output features (64 for SwiGLU, whose
// gate and up rows travel together, else 128); a slot row is [gate | up] or
// one partial row, +4 floats of padding.
__host__ __device__ constexpr int tc_push_features(int epi) { return epi == EPI_SWIGLU ? 64 : 128; }
__host__ __device__ constexpr int tc_push_pitch(int bn, int epi) {
  return (epi == EPI_SWIGLU ? 2 * bn : bn) + 4;
}
__host__ __device__ constexpr int tc_push_bytes(int bn, int epi, bool swap) {
  // S senders x ceil(F / S) rows <= F + 7 rows for S <= 8
  return swap ? (tc_push_features(epi) + 8) * tc_push_pitch(bn, epi) * 4 : 0;
}
// Shared memory a skinny CTA may use: up to 64 token columns, two CTAs per SM,
// so that the next kernel's CTAs (programmatic dependent launch) are resident
// and streaming their weights while this kernel's CTAs finish.
__host__ __device__ constexpr int tc_skinny_budget(int bn) {
  return bn <= 32 ? 113 * 1024 : 227 * 1024;
}
// Stages come in pairs: the MMA issuer waits once per pair of stages and the
// producer refills a pair per wait (one barrier wait costs about as much as
// issuing a stage's MMAs or its loads).
__host__ __device__ constexpr int tc_stages_fit(int bytes, int stage) {
  return ((bytes / stage) > 12 ? 12 : (bytes / stage)) & ~1;
}
__host__ __device__ constexpr int tc_stages(int bn, bool pair, bool swap = false, int epi = 0) {
  return swap ? tc_stages_fit(tc_skinny_budget(bn) - tc_xch_bytes(bn, epi, true) -
                                  tc_push_bytes(bn, epi, true) - 2048,
                              tc_stage_bytes(bn, false))
              : tc_stages_fit(196608, tc_stage_bytes(bn, pair));
}
// Wide tiles stage their output in two 16 KB buffers (128 rows x 128 bytes,
// 128-byte swizzle) for TMA stores.
constexpr int kOutBuf = 128 * 128;
__host__ __device__ constexpr int tc_out_bytes(bool swap) { return swap ? 0 : 2 * kOutBuf; }
__host__ __device__ constexpr int tc_smem_bytes(int bn, int epi, bool swap, bool pair) {
  return tc_stages(bn, pair, swap, epi) * tc_stage_bytes(bn, pair) + tc_xch_bytes(bn, epi, swap) +
         tc_push_bytes(bn, epi, swap) + tc_out_bytes(swap) + 1024;
}
static_assert(tc_smem_bytes(16, EPI_SWIGLU, true, false) + 1024 <= 114 * 1024, "two per SM");
static_assert(tc_smem_bytes(32, EPI_SWIGLU, true, false) + 1024 <= 114 * 1024, "two per SM");
static_assert(tc_smem_bytes(32, EPI_NONE, true, false) + 1024 <= 114 * 1024, "two per SM");
static_assert(tc_stages(16, false, true, EPI_SWIGLU) >= 4 && tc_stages(64, false, true, 0) >= 4,
              "skinny rings keep at least two stage pairs");

// ---------------------------------------------------------------------------
// Work decomposition, computed identically by every role of a CTA.  A tile is
// 128 (one CTA) or 256 (a CTA pair, tcgen05 cta_group::2) P rows by BN Q rows.
//   split == 1: persistent; CTA group g takes tiles g, g + groups, ... over
//               the full K range.
//   split == S: one cluster of S groups per tile; group j takes a range of
//               whole k-block pairs.
// The k-block count kb is rounded up to even (a trailing block past K is
// zero-filled by TMA), so stage pairs never straddle two tiles.
// ---------------------------------------------------------------------------

struct Unit {
  int tile;
  int k0, k1;  // k-block range [k0, k1)
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

template <int GROUP>
__device__ __forceinline__ int g_of_cta() {
  return static_cast<int>(blockIdx.x) / GROUP;
}

// Stream-K range of CTA group g of G over W k-block pairs: [W g / G, W (g+1) / G).
__device__ __forceinline__ long long sk_range_start(long long W, int g, int G) {
  return W * g / G;
}

struct UnitIter {
  int tile, stride, tiles, k0, k1;
  int kp;                // stream-K: k-block pairs per tile
  long long cur, hi;     // stream-K: this group's remaining range of pairs
  bool sk;
  // group: CTAs that share one tile's accumulator (2 for a CTA pair)
  __device__ __forceinline__ void init(const TcParams& p, int group) {
    const int kb = p.kb;
    tiles = p.tiles_p * p.tiles_q;
    sk = p.sk != 0;
    if (sk) {
      kp = kb / 2;
      const long long W = static_cast<long long>(tiles) * kp;
      const int G = gridDim.x / group, g = blockIdx.x / group;
      cur = sk_range_start(W, g, G);
      hi = sk_range_start(W, g + 1, G);
      tile = 0;
      stride = 0;
      k0 = k1 = 0;
    } else if (p.split == 1) {
      tile = blockIdx.x / group;
      stride = gridDim.x / group;
      k0 = 0;
      k1 = kb;
    } else {
      // k ranges are whole pairs of k-blocks (kb is even)
      const int j = static_cast<int>(cluster_rank()) / group;
      const int kp = kb / 2;
      tile = blockIdx.x / (group * p.split);
      stride = tiles;  // one unit only
      k0 = 2 * static_cast<int>((static_cast<long long>(j) * kp) / p.split);
      k1 = 2 * static_cast<int>((static_cast<long long>(j + 1) * kp) / p.split);
    }
  }
  __device__ __forceinline__ bool next(Unit& u) {
    if (sk) {
      if (cur >= hi) return false;
      const int t = static_cast<int>(cur / kp);
      const long long tile_end = static_cast<long long>(t + 1) * kp;
      const long long e = hi < tile_end ? hi : tile_end;
      u.tile = t;
      u.k0 = 2 * static_cast<int>(cur - static_cast<long long>(t) * kp);
      u.k1 = 2 * static_cast<int>(e - static_cast<long long>(t) * kp);
      cur = e;
      return true;
    }
    if (tile >= tiles) return false;
    u.tile = tile;
    u.k0 = k0;
    u.k1 = k1;
    tile += stride;
    return true;
  }
};

__device__ __forceinline__ void tile_coords(int tile, const TcParams& p, int& tp, int& tq) {
  const int per_group = kGroupP * p.tiles_q;
  const int g = tile / per_group;
  const int within = tile - g * per_group;
  const int rows_left = p.tiles_p - g * kGroupP;
  const int gp = rows_left < kGroupP ? rows_left : kGroupP;
  tp = g * kGroupP + within % gp;
  tq = within / gp;
}

// ---------------------------------------------------------------------------
// Epilogue helpers
// ---------------------------------------------------------------------------

template <int DT>
__device__ __forceinline__ void store16_row(typename Elem<DT>::T* dst, const float* v, int cnt,
                                            int valid, bool vec) {
  using E = Elem<DT>;
  if (vec && valid >= cnt) {
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      if (i < cnt) {
        uint4 u;
        u.x = E::pack2(v[i + 0], v[i + 1]);
        u.y = E::pack2(v[i + 2], v[i + 3]);
        u.z = E::pack2(v[i + 4], v[i + 5]);
        u.w = E::pack2(v[i + 6], v[i + 7]);
        *reinterpret_cast<uint4*>(dst + i) = u;
      }
    }
  } else {
    // fully unrolled so v stays in registers
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < cnt && i < valid) dst[i] = E::from_f(v[i]);
  }
}

template <int DT>
__device__ __forceinline__ void load16_row(const typename Elem<DT>::T* src, float* v, int cnt,
                                           int valid, bool vec) {
  using E = Elem<DT>;
  if (vec && valid >= cnt) {
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      if (i < cnt) {
        const uint4 u = *reinterpret_cast<const uint4*>(src + i);
        float2 f;
        f = E::unpack2(u.x); v[i + 0] = f.x; v[i + 1] = f.y;
        f = E::unpack2(u.y); v[i + 2] = f.x; v[i + 3] = f.y;
        f = E::unpack2(u.z); v[i + 4] = f.x; v[i + 5] = f.y;
        f = E::unpack2(u.w); v[i + 6] = f.x; v[i + 7] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < cnt) v[i] = (i < valid) ? E::to_f(src[i]) : 0.0f;
  }
}

__device__ __forceinline__ void store32f_row(float* dst, const float* v, int cnt, int valid,
                                             bool vec) {
  if (vec && valid >= cnt) {
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      if (i < cnt) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < cnt && i < valid) dst[i] = v[i];
  }
}

// Accumulator chunks for the direct epilogue come from tensor memory.
template <int CW>
struct TmemChunks {
  uint32_t taddr;  // lane base + accumulator buffer column
  __device__ __forceinline__ void get(int col, float* v) const {
    if constexpr (CW == 32) tmem_ld_32x32b_x32(taddr + col, v);
    else tmem_ld_32x32b_x16(taddr + col, v);
  }
};

// Apply the epilogue to one tile row held by this thread (row `lr` of the
// tile) and store it.  Chunks come from `src` CW columns at a time.
template <int DT, int BN, int EPI, bool SWAP, int CW, class Src>
__device__ __forceinline__ void emit_tile(const TcParams& p, const Src& src, int prow0,
                                          int qcol0, int lr, float* xch) {
  using E = Elem<DT>;
  using T = typename E::T;
  const bool vec = p.vec_ok != 0;
  float v[32];
  if constexpr (!SWAP) {
    const int m = prow0 + lr;
    const bool mval = m < p.M;
    if constexpr (EPI == EPI_SWIGLU) {
      // Q columns are packed [gate 64 | up 64] groups; output column of the
      // first gate column of group g is (qcol0 + 128g) / 2.
      float u[32];
#pragma unroll 1
      for (int g = 0; g < BN / 128; ++g) {
#pragma unroll 1
        for (int h = 0; h < 64; h += 32) {
          src.get(128 * g + h, v);
          src.get(128 * g + 64 + h, u);
          const int n = (qcol0 + 128 * g) / 2 + h;
          if (mval && n < p.N) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              v[j] = silu_fast(E::round(v[j])) * E::round(u[j]);
            store16_row<DT>(static_cast<T*>(p.C) + m * p.ldc + n, v, 32, p.N - n, vec);
          }
        }
      }
    } else {
#pragma unroll 1
      for (int c = 0; c < BN; c += CW) {
        src.get(c, v);
        const int n = qcol0 + c;
        if (mval && n < p.N) {
          const int valid = p.N - n;
          if constexpr (EPI == EPI_NONE) {
            store16_row<DT>(static_cast<T*>(p.C) + m * p.ldc + n, v, CW, valid, vec);
          } else if constexpr (EPI == EPI_RESIDUAL) {
            float r[32];
            load16_row<DT>(static_cast<const T*>(p.R) + m * p.ldr + n, r, CW, valid, vec);
#pragma unroll
            for (int j = 0; j < CW; ++j) v[j] = r[j] + E::round(v[j]);
            store16_row<DT>(static_cast<T*>(p.C) + m * p.ldc + n, v, CW, valid, vec);
          } else if constexpr (EPI == EPI_F32_OUT) {
#pragma unroll
            for (int j = 0; j < CW; ++j) v[j] = E::round(v[j]);
            store32f_row(static_cast<float*>(p.C) + m * p.ldc + n, v, CW, valid, vec);
          } else {
            store32f_row(static_cast<float*>(p.C) + m * p.ldc + n, v, CW, valid, vec);
          }
        }
      }
    }
  } else {
    // Skinny: this thread's row is weight row (feature) prow0 + lr; its
    // columns are tokens qcol0 + c.
    if constexpr (EPI == EPI_SWIGLU) {
      // Packed rows: lanes 0-63 gate, 64-127 up, of output features
      // prow0/2 + (lr % 64).
#pragma unroll 1
      for (int c = 0; c < BN; c += CW) {
        src.get(c, v);
        // token-major (column j of the 64 gate rows at xch[64 j ..]): a warp's
        // 32 rows land in 32 consecutive words, one bank each
        if (lr >= 64) {
#pragma unroll
          for (int j = 0; j < CW; ++j) xch[j * 64 + (lr - 64)] = E::round(v[j]);
        }
        named_bar_sync(1, kEpiThreads);
        // the gate rows compute their CW outputs; once every up value has
        // been read, they go back into the exchange buffer as 16-bit values,
        // token-major (64 features of a token contiguous), and all 128
        // threads store them as 16-byte vectors: a feature per thread would
        // take one 2-byte store per token
        T* out16 = reinterpret_cast<T*>(xch);
        float o[CW];
        if (lr < 64) {
#pragma unroll
          for (int j = 0; j < CW; ++j) o[j] = silu_fast(E::round(v[j])) * xch[j * 64 + lr];
        }
        named_bar_sync(1, kEpiThreads);
        if (lr < 64) {
#pragma unroll
          for (int j = 0; j < CW; ++j) out16[j * 64 + lr] = E::from_f(o[j]);
        }
        named_bar_sync(1, kEpiThreads);
        const int n0 = prow0 / 2;  // first output feature of the tile (a multiple of 64)
#pragma unroll 1
        for (int idx = lr; idx < CW * 8; idx += kEpiThreads) {
          const int j = idx >> 3, q = idx & 7;  // token, 8-feature group
          const int m = qcol0 + c + j;
          const int nn = n0 + 8 * q;
          if (m >= p.M || nn >= p.N) continue;
          const T* srcv = out16 + j * 64 + 8 * q;
          T* dst = static_cast<T*>(p.C) + m * p.ldc + nn;
          if (vec && nn + 8 <= p.N) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(srcv);
          } else {
            for (int t = 0; t < 8 && nn + t < p.N; ++t) dst[t] = srcv[t];
          }
        }
        named_bar_sync(1, kEpiThreads);
      }
    } else {
      const int n = prow0 + lr;
      const bool nval = n < p.N;
#pragma unroll 1
      for (int c = 0; c < BN; c += CW) {
        src.get(c, v);
        if (!nval) continue;
#pragma unroll
        for (int j = 0; j < CW; ++j) {
          const int m = qcol0 + c + j;
          if (m < p.M) {
            if constexpr (EPI == EPI_NONE) {
              static_cast<T*>(p.C)[m * p.ldc + n] = E::from_f(v[j]);
            } else if constexpr (EPI == EPI_RESIDUAL) {
              const float r = E::to_f(static_cast<const T*>(p.R)[m * p.ldr + n]);
              static_cast<T*>(p.C)[m * p.ldc + n] = E::from_f(r + E::round(v[j]));
            } else if constexpr (EPI == EPI_F32_OUT) {
              static_cast<float*>(p.C)[m * p.ldc + n] = E::round(v[j]);
            } else {
              static_cast<float*>(p.C)[m * p.ldc + n] = v[j];
            }
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Epilogue through TMA stores (wide tiles)
// ---------------------------------------------------------------------------

__device__ __forceinline__ float4 ld_smem_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_smem_f4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// Byte offset of 16-byte chunk j of row r in a 128-byte-swizzled buffer
// (the layout TMA reads and writes with CU_TENSOR_MAP_SWIZZLE_128B).
__device__ __forceinline__ uint32_t sw128(int r, int j) {
  return static_cast<uint32_t>(r * 128 + ((j ^ (r & 7)) << 4));
}

// One thread of the 128 epilogue threads waits (bounded) on `bar`; the rest
// park on a named barrier instead of polling.  Returns false on timeout, in
// every thread.
__device__ __forceinline__ bool epi_wait(uint32_t bar, uint32_t parity, int et,
                                         volatile int* abort_flag, int* err, volatile int* flag) {
  (void)flag;
  const bool ok =
      et != 0 || mbar_wait_bounded(bar, parity, abort_flag, err, DEVERR_TIMEOUT_EPILOGUE);
  return named_bar_and(1, kEpiThreads, ok);
}

// ---------------------------------------------------------------------------
// Stream-K partial accumulators
// ---------------------------------------------------------------------------

// A CTA's slot holds its kBM x BN fp32 partial accumulator as float4 columns
// groups: float4 (c4, row) at index c4 * kBM + row, so that the 32 rows of a
// warp touch 512 contiguous bytes per access (writer and reader alike).
__device__ __forceinline__ int ld_acquire_gpu(const int* f) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* f, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}

// Stream-K slots: CTA b's partial accumulator is rows [128 b, 128 b + 128) of
// an fp32 [grid * 128, BN] matrix in the workspace, moved by the TMA unit in
// boxes of 32 columns x 128 rows (16 KB, 128-byte swizzle) that use the same
// shared-memory layout as the epilogue's staging buffers (row r, 16-byte
// chunk j at sw128(r, j)).

// Orders this thread's async-proxy (TMA) global accesses against its generic
// ones: TMA stores before a flag release, a flag acquire before TMA loads.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Contributor: this CTA's partial accumulator (columns [0, BN) of its 128
// rows) into its slot: each 32-column chunk staged in one of the two output
// staging buffers and stored by TMA; once every store has completed, the
// flag, released at GPU scope.
template <int BN>
__device__ __forceinline__ void sk_write_partial(const TcParams& p, const void* tm_s,
                                                 uint32_t taddr, int lr, int et,
                                                 uint32_t outbuf) {
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    const uint32_t buf = outbuf + static_cast<uint32_t>(((c / 32) & 1) * kOutBuf);
    // the store that last read this buffer is done with it (at the first
    // chunk: every earlier store of this CTA)
    if (et == 0) {
      if (c == 0) bulk_wait_group_read<0>();
      else bulk_wait_group_read<1>();
    }
    named_bar_sync(1, kEpiThreads);
    float v[32];
    tmem_ld_32x32b_x32(taddr + c, v);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      st_smem_f4(buf + sw128(lr, j), v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    fence_proxy_async_smem();
    named_bar_sync(1, kEpiThreads);
    if (et == 0) {
      tma_store_2d(tm_s, buf, c, static_cast<int>(blockIdx.x) * kBM);
      bulk_commit_group();
    }
  }
  if (et == 0) {
    bulk_wait_group<0>();  // the slot is written, not just read out of shared memory
    fence_proxy_async_global();
    __threadfence();
    st_release_gpu(p.sk_flags + blockIdx.x, 1);
  }
}

// Finisher: add the partial accumulators of n contributor CTAs (first, first
// + stride, ...) to this CTA's tile in tensor memory, in that order, before
// the ordinary epilogue reads it.  The operand ring is idle by now (a
// finisher's unit is its group's last): one thread loads a column range of
// every slot into it by TMA (as many 32-column boxes as fit), then the 128
// epilogue threads add them to their rows: tcgen05.ld, n adds, tcgen05.st.
template <int BN>
__device__ __forceinline__ bool sk_fixup(const void* tm_s, uint32_t taddr, int lr, int et,
                                         uint32_t ring, uint32_t ring_bytes, int first, int n,
                                         int stride, uint32_t bar, uint32_t& phase,
                                         volatile int* abort_flag, int* err, volatile int* flag) {
  constexpr uint32_t kBox = 32 * kBM * 4;  // one 32-column box: 16 KB
  if (static_cast<uint32_t>(n) * kBox > ring_bytes) {
    // the planner never makes such a plan; refuse rather than overrun the ring
    if (et == 0) {
      *abort_flag = 1;
      if (err) atomicCAS(err, 0, DEVERR_TIMEOUT_EPILOGUE);
    }
    return false;
  }
  int nb = BN / 32;  // 32-column boxes per slot in one part
  while (nb > 1 && static_cast<uint32_t>(n * nb) * kBox > ring_bytes) nb >>= 1;
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32 * nb) {
    if (et == 0) {
      // the ring's last readers were the MMAs (complete) or this loop's
      // generic loads (finished at the barrier below); the flags were
      // acquired with generic loads before these async-proxy reads
      fence_proxy_async_smem();
      fence_proxy_async_global();
      mbar_arrive_expect_tx(bar, static_cast<uint32_t>(n * nb) * kBox);
      for (int j = 0; j < n; ++j)
        for (int b = 0; b < nb; ++b)
          tma_load_2d_plain(ring + static_cast<uint32_t>(j * nb + b) * kBox, tm_s, bar,
                            c0 + 32 * b, (first + j * stride) * kBM);
    }
    if (!epi_wait(bar, phase, et, abort_flag, err, flag)) return false;
    phase ^= 1u;
#pragma unroll 1
    for (int b = 0; b < nb; ++b) {
      float v[32];
      tmem_ld_32x32b_x32(taddr + c0 + 32 * b, v);
      for (int j = 0; j < n; ++j) {
        const uint32_t box = ring + static_cast<uint32_t>(j * nb + b) * kBox;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 t = ld_smem_f4(box + sw128(lr, i));
          v[4 * i + 0] += t.x;
          v[4 * i + 1] += t.y;
          v[4 * i + 2] += t.z;
          v[4 * i + 3] += t.w;
        }
      }
      tmem_st_32x32b_x32(taddr + c0 + 32 * b, v);
    }
    named_bar_sync(1, kEpiThreads);
  }
  return true;
}

// Finisher: one thread waits (bounded) for the flags of the n contributor
// CTAs first, first + stride, ...; the result reaches all 128 epilogue threads.
__device__ __forceinline__ bool sk_wait(const int* flags, int first, int n, int stride, int et,
                                        volatile int* abort_flag, int* err, volatile int* flag) {
  (void)flag;
  bool ok = true;
  if (et == 0) {
    bool good = true;
    const unsigned long long t0 = global_timer_ns();
    for (int j = 0; j < n && good; ++j) {
      while (ld_acquire_gpu(flags + first + j * stride) == 0) {
        if (*abort_flag) {
          good = false;
          break;
        }
        if (global_timer_ns() - t0 > kWaitTimeoutNs) {
          *abort_flag = 1;
          if (err) atomicCAS(err, 0, DEVERR_TIMEOUT_EPILOGUE);
          good = false;
          break;
        }
        __nanosleep(64);
      }
    }
    ok = good;
  }
  const bool all = named_bar_and(1, kEpiThreads, ok);
  __threadfence();
  return all;
}

// Store one tile held in tensor memory: for each 128-byte-wide chunk of
// output columns, every thread writes its row into a swizzled staging buffer
// and one thread issues the TMA store.  Chunks go in rounds of two, one per
// staging buffer; a round starts once every earlier store has read its
// buffer, and for RESIDUAL both chunks' residual tiles are TMA-loaded into the
// buffers at once (one barrier, one wait per round).  Rows and columns
// outside C are clipped by the TMA unit.
template <int DT, int BN, int EPI>
__device__ __forceinline__ bool emit_tile_tma(const TcParams& p, uint32_t taddr, int prow0,
                                              int qcol0, int lr, int et, uint32_t outbuf,
                                              const void* tm_c, const void* tm_r,
                                              uint32_t res_bar, uint32_t& res_phase,
                                              volatile int* abort_flag, volatile int* flag) {
  using E = Elem<DT>;
  constexpr bool F32 = (EPI == EPI_F32_OUT || EPI == EPI_F32_PARTIAL);
  constexpr int CH = F32 ? 32 : 64;  // output columns per 128-byte chunk
  constexpr int OUT_COLS = (EPI == EPI_SWIGLU) ? BN / 2 : BN;
  constexpr int NCH = OUT_COLS / CH;
  const int ocol0 = (EPI == EPI_SWIGLU) ? qcol0 / 2 : qcol0;
#pragma unroll 1
  for (int oc0 = 0; oc0 < NCH; oc0 += 2) {
    const int n_round = (NCH - oc0) < 2 ? (NCH - oc0) : 2;
    // every earlier store has read its staging buffer
    if (et == 0) bulk_wait_group_read<0>();
    if constexpr (EPI == EPI_RESIDUAL) {
      if (et == 0) {
        mbar_arrive_expect_tx(res_bar, static_cast<uint32_t>(n_round * kOutBuf));
        for (int b = 0; b < n_round; ++b)
          tma_load_2d_plain(outbuf + static_cast<uint32_t>(b * kOutBuf), tm_r, res_bar,
                            ocol0 + (oc0 + b) * CH, prow0);
      }
    }
    named_bar_sync(1, kEpiThreads);
    if constexpr (EPI == EPI_RESIDUAL) {
      if (!epi_wait(res_bar, res_phase, et, abort_flag, p.err, flag)) return false;
      res_phase ^= 1u;
    }
#pragma unroll 1
    for (int b = 0; b < n_round; ++b) {
      const int oc = oc0 + b;
      const uint32_t buf = outbuf + static_cast<uint32_t>(b * kOutBuf);
      const int ocol = ocol0 + oc * CH;
      if constexpr (F32) {
        float v[32];
        tmem_ld_32x32b_x32(taddr + oc * 32, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float o[4];
#pragma unroll
          for (int t = 0; t < 4; ++t)
            o[t] = (EPI == EPI_F32_OUT) ? E::round(v[4 * j + t]) : v[4 * j + t];
          st_smem_f4(buf + sw128(lr, j), o[0], o[1], o[2], o[3]);
        }
      } else {
        // both 32-column halves of the chunk in flight before one wait
        float vh[2][32];
        if constexpr (EPI != EPI_SWIGLU)
          tmem_ld_32x32b_x32x2(taddr + 64 * oc, taddr + 64 * oc + 32, vh[0], vh[1]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float v[32];
          if constexpr (EPI == EPI_SWIGLU) {
            // output chunk oc <- packed group oc: gate cols [128oc, 128oc+64), up +64
            float u[32];
            tmem_ld_32x32b_x32x2(taddr + 128 * oc + 32 * h, taddr + 128 * oc + 64 + 32 * h, v, u);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = silu_fast(E::round(v[j])) * E::round(u[j]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = vh[h][j];
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t a = buf + sw128(lr, 4 * h + j);
            if constexpr (EPI == EPI_RESIDUAL) {
              uint4 r;
              asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                           : "r"(a));
              float2 f;
              f = E::unpack2(r.x); v[8 * j + 0] = f.x + E::round(v[8 * j + 0]); v[8 * j + 1] = f.y + E::round(v[8 * j + 1]);
              f = E::unpack2(r.y); v[8 * j + 2] = f.x + E::round(v[8 * j + 2]); v[8 * j + 3] = f.y + E::round(v[8 * j + 3]);
              f = E::unpack2(r.z); v[8 * j + 4] = f.x + E::round(v[8 * j + 4]); v[8 * j + 5] = f.y + E::round(v[8 * j + 5]);
              f = E::unpack2(r.w); v[8 * j + 6] = f.x + E::round(v[8 * j + 6]); v[8 * j + 7] = f.y + E::round(v[8 * j + 7]);
            }
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a),
                         "r"(E::pack2(v[8 * j + 0], v[8 * j + 1])), "r"(E::pack2(v[8 * j + 2], v[8 * j + 3])),
                         "r"(E::pack2(v[8 * j + 4], v[8 * j + 5])), "r"(E::pack2(v[8 * j + 6], v[8 * j + 7]))
                         : "memory");
          }
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, kEpiThreads);
      if (et == 0) {
        tma_store_2d(tm_c, buf, ocol, prow0);
        bulk_commit_group();
      }
    }
  }
  return true;
}

// ---------------------------------------------------------------------------
// Cluster split-K for wide tiles.  The S CTAs of a tile own consecutive blocks
// of column units (unit = 32 accumulator columns; SwiGLU: a 32-column gate
// chunk with its up chunk 64 columns to the right).  Each CTA
//   1. stages the units it does not own, grouped by owner, in its own shared
//      memory (rows of 128-byte segments, 16-byte chunks XOR-swizzled by row);
//   2. after a cluster barrier, sends each owner its block with one bulk copy
//      into the owner's receive slot (DMA engine, completion counted on the
//      owner's mbarrier, armed with the expected bytes beforehand);
//   3. sums, for the units it owns, its own part (re-read from tensor memory)
//      and then the S-1 received parts in rank order (a fixed order:
//      deterministic), applies the epilogue, stores.
// Shared memory (the idle operand ring): the staging blocks first, then the
// S-1 receive slots.
// ---------------------------------------------------------------------------

template <int BN, int EPI>
__host__ __device__ constexpr int split_units() { return EPI == EPI_SWIGLU ? BN / 64 : BN / 32; }
template <int EPI>
__host__ __device__ constexpr int unit_cols() { return EPI == EPI_SWIGLU ? 64 : 32; }
// accumulator column of unit u's first half (its second half is +64 for SwiGLU)
template <int EPI>
__device__ __forceinline__ int unit_col(int u) {
  return EPI == EPI_SWIGLU ? (u / 2) * 128 + (u % 2) * 32 : u * 32;
}
__host__ __device__ constexpr int owner_first_unit(int j, int units, int S) {
  // owner of unit u is (u*S)/units; this is the first u with owner j
  return (j * units + S - 1) / S;
}
__host__ __device__ constexpr int owner_units(int j, int units, int S) {
  return owner_first_unit(j + 1, units, S) - owner_first_unit(j, units, S);
}
// Shared memory a split of S needs (bytes): staging of the units a CTA does
// not own plus S-1 receive slots, maximised over the cluster ranks.
__host__ __device__ constexpr int split_smem_bytes(int units, int ucols, int S) {
  int worst = 0;
  for (int j = 0; j < S; ++j) {
    const int own = owner_units(j, units, S);
    const int b = ((units - own) + (S - 1) * own) * 128 * ucols * 4;
    worst = b > worst ? b : worst;
  }
  return worst;
}

// 16-byte chunk c of row r in a block whose rows are `segs` 128-byte segments
__device__ __forceinline__ uint32_t blk_off(int r, int c, int segs) {
  return static_cast<uint32_t>(r * segs * 128 + ((c & ~7) << 4) + (((c & 7) ^ (r & 7)) << 4));
}

template <int DT, int BN, int EPI>
__device__ __forceinline__ void stage_unowned(uint32_t ring, uint32_t taddr, int lr, int S, int j) {
  constexpr int U = split_units<BN, EPI>();
  constexpr int UC = unit_cols<EPI>();
  uint32_t base = ring;
#pragma unroll 1
  for (int o = 0; o < S; ++o) {
    const int n_o = owner_units(o, U, S);
    if (o == j) continue;
    const int u0 = owner_first_unit(o, U, S);
    const int segs = n_o * UC / 32;  // 128-byte segments per row
#pragma unroll 1
    for (int ui = 0; ui < n_o; ++ui) {
      const int c = unit_col<EPI>(u0 + ui);
#pragma unroll
      for (int part = 0; part < UC / 32; ++part) {
        float v[32];
        tmem_ld_32x32b_x32(taddr + c + part * 64, v);
        const int chunk0 = (ui * UC + part * 32) / 4;  // first 16-byte chunk in the row
#pragma unroll
        for (int i = 0; i < 8; ++i)
          st_smem_f4(base + blk_off(lr, chunk0 + i, segs), v[4 * i], v[4 * i + 1], v[4 * i + 2],
                     v[4 * i + 3]);
      }
    }
    base += static_cast<uint32_t>(128 * n_o * UC * 4);
  }
}

// Byte offset of the receive slots in the ring of owner j.
template <int BN, int EPI>
__device__ __forceinline__ uint32_t recv_base(int S, int j) {
  constexpr int U = split_units<BN, EPI>();
  constexpr int UC = unit_cols<EPI>();
  return static_cast<uint32_t>((U - owner_units(j, U, S)) * 128 * UC * 4);
}

// One thread: send every other owner its staged block.
template <int BN, int EPI>
__device__ __forceinline__ void send_blocks(uint32_t ring, uint32_t recv_bar_local, int S, int j,
                                            int half, int group) {
  constexpr int U = split_units<BN, EPI>();
  constexpr int UC = unit_cols<EPI>();
  uint32_t src = ring;
#pragma unroll 1
  for (int o = 0; o < S; ++o) {
    const int n_o = owner_units(o, U, S);
    if (o == j) continue;
    const uint32_t bytes = static_cast<uint32_t>(128 * n_o * UC * 4);
    const int slot = (j < o) ? j : j - 1;  // my slot at owner o
    const uint32_t rank = static_cast<uint32_t>(half + o * group);
    const uint32_t dst = mapa_shared(ring + recv_base<BN, EPI>(S, o) + slot * bytes, rank);
    bulk_copy_s2cluster(dst, src, bytes, mapa_shared(recv_bar_local, rank));
    src += bytes;
  }
}

template <int DT, int BN, int EPI>
__device__ __forceinline__ void reduce_received(const TcParams& p, uint32_t ring, uint32_t taddr,
                                                int lr, int S, int j, int prow0, int qcol0) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int U = split_units<BN, EPI>();
  constexpr int UC = unit_cols<EPI>();
  const int u0 = owner_first_unit(j, U, S);
  const int n_j = owner_units(j, U, S);
  const int segs = n_j * UC / 32;
  const uint32_t slots = ring + recv_base<BN, EPI>(S, j);
  const uint32_t slot_bytes = static_cast<uint32_t>(128 * n_j * UC * 4);
  const int m = prow0 + lr;
  const bool vec = p.vec_ok != 0;
  // every owned unit's residual row segment (16-bit words) is loaded first:
  // the loads are in flight together while the tensor-memory and
  // shared-memory reads below run (an owner holds at most U/2 units)
  constexpr int MAXU = (U + 1) / 2;
  uint32_t rw[(EPI == EPI_RESIDUAL) ? MAXU : 1][16];
  if constexpr (EPI == EPI_RESIDUAL) {
#pragma unroll
    for (int ui = 0; ui < MAXU; ++ui) {
      const int n = qcol0 + unit_col<EPI>(u0 + ui);
      const int valid = p.N - n;
      const T* src = static_cast<const T*>(p.R) + m * p.ldr + n;
      if (ui < n_j && m < p.M && valid >= 32 && vec) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 t = reinterpret_cast<const uint4*>(src)[q];
          rw[ui][4 * q] = t.x; rw[ui][4 * q + 1] = t.y; rw[ui][4 * q + 2] = t.z; rw[ui][4 * q + 3] = t.w;
        }
      } else if (ui < n_j && m < p.M && valid > 0) {
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float lo = (2 * q < valid) ? E::to_f(src[2 * q]) : 0.f;
          const float hi = (2 * q + 1 < valid) ? E::to_f(src[2 * q + 1]) : 0.f;
          rw[ui][q] = E::pack2(lo, hi);
        }
      }
    }
  }
#pragma unroll
  for (int ui = 0; ui < MAXU; ++ui) {
    if (ui >= n_j) break;
    const int u = u0 + ui;
    const int c = unit_col<EPI>(u);
    float v[32], w[32];
    tmem_ld_32x32b_x32(taddr + c, v);
    if constexpr (EPI == EPI_SWIGLU) tmem_ld_32x32b_x32(taddr + c + 64, w);
#pragma unroll 1
    for (int sl = 0; sl < S - 1; ++sl) {
      const uint32_t sb = slots + sl * slot_bytes;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 a = ld_smem_f4(sb + blk_off(lr, (ui * UC) / 4 + i, segs));
        v[4 * i] += a.x; v[4 * i + 1] += a.y; v[4 * i + 2] += a.z; v[4 * i + 3] += a.w;
        if constexpr (EPI == EPI_SWIGLU) {
          const float4 b = ld_smem_f4(sb + blk_off(lr, (ui * UC + 32) / 4 + i, segs));
          w[4 * i] += b.x; w[4 * i + 1] += b.y; w[4 * i + 2] += b.z; w[4 * i + 3] += b.w;
        }
      }
    }
    if (m >= p.M) continue;
    if constexpr (EPI == EPI_SWIGLU) {
      const int n = qcol0 / 2 + (u / 2) * 64 + (u % 2) * 32;
      if (n >= p.N) continue;
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = silu_fast(E::round(v[i])) * E::round(w[i]);
      store16_row<DT>(static_cast<T*>(p.C) + m * p.ldc + n, v, 32, p.N - n, vec);
    } else {
      const int n = qcol0 + c;
      if (n >= p.N) continue;
      const int valid = p.N - n;
      if constexpr (EPI == EPI_NONE) {
        store16_row<DT>(static_cast<T*>(p.C) + m * p.ldc + n, v, 32, valid, vec);
      } else if constexpr (EPI == EPI_RESIDUAL) {
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float2 f = E::unpack2(rw[ui][q]);
          v[2 * q] = f.x + E::round(v[2 * q]);
          v[2 * q + 1] = f.y + E::round(v[2 * q + 1]);
        }
        store16_row<DT>(static_cast<T*>(p.C) + m * p.ldc + n, v, 32, valid, vec);
      } else if constexpr (EPI == EPI_F32_OUT) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = E::round(v[i]);
        store32f_row(static_cast<float*>(p.C) + m * p.ldc + n, v, 32, valid, vec);
      } else {
        store32f_row(static_cast<float*>(p.C) + m * p.ldc + n, v, 32, valid, vec);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Cluster split-K: shared-memory staging and the DSMEM reduction
// ---------------------------------------------------------------------------



// All threads of all CTAs of the cluster; release/acquire orders the shared
// memory writes before it with the remote reads after it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// Row pitch (floats) of the fp32 staging tile: +4 keeps the per-row float4
// writes of a warp (32 rows) on distinct banks.
template <int BN>
__host__ __device__ constexpr int stage_pitch() { return BN + 4; }

// Output one reduced 4-column group (row, col .. col+3) of the tile.
template <int DT, int BN, int EPI, bool SWAP>
__device__ __forceinline__ void out_group(const TcParams& p, int prow0, int qcol0, int row, int col,
                                          const float4& a, const float4* up) {
  using E = Elem<DT>;
  using T = typename E::T;
  const bool vec = p.vec_ok != 0;
  if constexpr (!SWAP) {
    const int m = prow0 + row;
    if constexpr (EPI == EPI_SWIGLU) {
      const int n = qcol0 / 2 + (col / 128) * 64 + (col % 128);
      if (m >= p.M || n >= p.N) return;
      const float4 u = *up;
      float o[4] = {silu_fast(E::round(a.x)) * E::round(u.x), silu_fast(E::round(a.y)) * E::round(u.y),
                    silu_fast(E::round(a.z)) * E::round(u.z), silu_fast(E::round(a.w)) * E::round(u.w)};
      T* dst = static_cast<T*>(p.C) + m * p.ldc + n;
      if (vec && n + 4 <= p.N) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(E::pack2(o[0], o[1]), E::pack2(o[2], o[3]));
      } else {
        for (int j = 0; j < 4; ++j)
          if (n + j < p.N) dst[j] = E::from_f(o[j]);
      }
    } else {
      const int n = qcol0 + col;
      if (m >= p.M || n >= p.N) return;
      float o[4] = {a.x, a.y, a.z, a.w};
      const bool full = vec && n + 4 <= p.N;
      if constexpr (EPI == EPI_F32_OUT || EPI == EPI_F32_PARTIAL) {
        if constexpr (EPI == EPI_F32_OUT) {
#pragma unroll
          for (int j = 0; j < 4; ++j) o[j] = E::round(o[j]);
        }
        float* dst = static_cast<float*>(p.C) + m * p.ldc + n;
        if (full) {
          *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
        } else {
          for (int j = 0; j < 4; ++j)
            if (n + j < p.N) dst[j] = o[j];
        }
      } else {
        if constexpr (EPI == EPI_RESIDUAL) {
          const T* rs = static_cast<const T*>(p.R) + m * p.ldr + n;
          if (full) {
            const uint2 rv = *reinterpret_cast<const uint2*>(rs);
            const float2 r01 = E::unpack2(rv.x), r23 = E::unpack2(rv.y);
            o[0] = r01.x + E::round(o[0]);
            o[1] = r01.y + E::round(o[1]);
            o[2] = r23.x + E::round(o[2]);
            o[3] = r23.y + E::round(o[3]);
          } else {
            for (int j = 0; j < 4; ++j)
              if (n + j < p.N) o[j] = E::to_f(rs[j]) + E::round(o[j]);
          }
        }
        T* dst = static_cast<T*>(p.C) + m * p.ldc + n;
        if (full) {
          *reinterpret_cast<uint2*>(dst) = make_uint2(E::pack2(o[0], o[1]), E::pack2(o[2], o[3]));
        } else {
          for (int j = 0; j < 4; ++j)
            if (n + j < p.N) dst[j] = E::from_f(o[j]);
        }
      }
    }
  } else {
    // skinny: rows are weight rows (features), columns tokens
    const float o[4] = {a.x, a.y, a.z, a.w};
    if constexpr (EPI == EPI_SWIGLU) {
      const int n = prow0 / 2 + row;
      if (n >= p.N) return;
      const float uo[4] = {up->x, up->y, up->z, up->w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int m = qcol0 + col + j;
        if (m < p.M)
          static_cast<T*>(p.C)[m * p.ldc + n] = E::from_f(silu_fast(E::round(o[j])) * E::round(uo[j]));
      }
    } else {
      const int n = prow0 + row;
      if (n >= p.N) return;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int m = qcol0 + col + j;
        if (m >= p.M) continue;
        if constexpr (EPI == EPI_NONE) {
          static_cast<T*>(p.C)[m * p.ldc + n] = E::from_f(o[j]);
        } else if constexpr (EPI == EPI_RESIDUAL) {
          const float r = E::to_f(static_cast<const T*>(p.R)[m * p.ldr + n]);
          static_cast<T*>(p.C)[m * p.ldc + n] = E::from_f(r + E::round(o[j]));
        } else if constexpr (EPI == EPI_F32_OUT) {
          static_cast<float*>(p.C)[m * p.ldc + n] = E::round(o[j]);
        } else {
          static_cast<float*>(p.C)[m * p.ldc + n] = o[j];
        }
      }
    }
  }
}

// Skinny split-K, owner side: sum the S partial rows pushed for each owned
// feature [f0, f1) of the tile in sender order 0..S-1 (deterministic), apply
// the epilogue and store.  Work item = one feature x one 4-token group;
// consecutive threads take consecutive features, so the stores of one token
// row coalesce.  rm = slot rows per sender.
template <int DT, int BN, int EPI, int S>
__device__ __forceinline__ void reduce_pushed_s(const TcParams& p, uint32_t pbuf, int prow0,
                                                int qcol0, int f0, int f1, int rm, int tid,
                                                int nthreads) {
  constexpr int PITCH = tc_push_pitch(BN, EPI);
  const int rows = f1 - f0;
  const int items = rows * (BN / 4);
  for (int e = tid; e < items; e += nthreads) {
    const int i = e % rows;
    const int col = 4 * (e / rows);
    float4 x[S], y[S];
#pragma unroll
    for (int r = 0; r < S; ++r) {
      const uint32_t a = pbuf + static_cast<uint32_t>(((r * rm + i) * PITCH + col) * 4);
      x[r] = ld_smem_f4(a);
      if constexpr (EPI == EPI_SWIGLU) y[r] = ld_smem_f4(a + BN * 4);
    }
    float4 a = x[0], b = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (EPI == EPI_SWIGLU) b = y[0];
#pragma unroll
    for (int r = 1; r < S; ++r) {
      a.x += x[r].x; a.y += x[r].y; a.z += x[r].z; a.w += x[r].w;
      if constexpr (EPI == EPI_SWIGLU) {
        b.x += y[r].x; b.y += y[r].y; b.z += y[r].z; b.w += y[r].w;
      }
    }
    out_group<DT, BN, EPI, true>(p, prow0, qcol0, f0 + i, col, a, &b);
  }
}

template <int DT, int BN, int EPI>
__device__ __forceinline__ void reduce_pushed(const TcParams& p, uint32_t pbuf, int S, int prow0,
                                              int qcol0, int f0, int f1, int rm, int tid,
                                              int nthreads) {
#define ORIN_REDUCE_CASE(n)                                                                   \
  case n:                                                                                     \
    reduce_pushed_s<DT, BN, EPI, n>(p, pbuf, prow0, qcol0, f0, f1, rm, tid, nthreads);        \
    break;
  switch (S) {
    ORIN_REDUCE_CASE(2)
    ORIN_REDUCE_CASE(3)
    ORIN_REDUCE_CASE(4)
    ORIN_REDUCE_CASE(5)
    ORIN_REDUCE_CASE(6)
    ORIN_REDUCE_CASE(7)
    default:
      reduce_pushed_s<DT, BN, EPI, 8>(p, pbuf, prow0, qcol0, f0, f1, rm, tid, nthreads);
      break;
  }
#undef ORIN_REDUCE_CASE
}

// ---------------------------------------------------------------------------
// The kernel
//
// PAIR (wide tiles only): the CTAs of cluster ranks 2i and 2i+1 form a
// tcgen05 CTA pair.  Each loads its own 128 A rows and half of the tile's B
// rows; both signal the leader's (even rank) full barrier.  The leader's MMA
// warp issues M=256 cta_group::2 MMAs, and its commits arrive on the empty
// and accumulator-full barriers of both CTAs (one commit per barrier).  Each
// CTA's epilogue reads its own 128 accumulator rows and releases the buffer on
// the leader's accumulator-empty barrier.
// ---------------------------------------------------------------------------

template <int DT, int BN, int EPI, bool SWAP, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    tc_linear_kernel(const __grid_constant__ CUtensorMap tm_p,
                     const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_c,
                     const __grid_constant__ CUtensorMap tm_r,
                     const __grid_constant__ CUtensorMap tm_s, const TcParams p) {
  static_assert(!(PAIR && SWAP), "CTA pairs are used for wide tiles only");
  constexpr int GROUP = PAIR ? 2 : 1;         // CTAs per tile accumulator
  constexpr int TILE_P = GROUP * kBM;         // P rows per tile
  constexpr int QR = tc_qrows(BN, PAIR);      // Q rows this CTA loads per stage
  constexpr int STAGES = tc_stages(BN, PAIR, SWAP, EPI);
  constexpr uint32_t A_BYTES = kBM * kBK * 2;
  constexpr uint32_t STAGE_BYTES = tc_stage_bytes(BN, PAIR);
  constexpr uint32_t TMEM_COLS = tc_tmem_cols(BN);
  constexpr uint32_t IDESC = instr_desc_f16(DT, TILE_P, BN);
  constexpr int CW = (BN >= 32) ? 32 : 16;
  static_assert(kBM * stage_pitch<BN>() * 4 <= STAGES * STAGE_BYTES,
                "split-K staging tile must fit in the operand ring");

  extern __shared__ uint8_t dsmem[];
  constexpr int PAIRS = STAGES / 2;
  static_assert(STAGES % 2 == 0, "stages come in pairs");
  __shared__ __align__(8) uint64_t full_bar[PAIRS];   // one per pair of stages
  __shared__ __align__(8) uint64_t empty_bar[PAIRS];  // one per pair of stages
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ __align__(8) uint64_t res_bar;
  __shared__ __align__(8) uint64_t recv_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  __shared__ volatile int epi_flag;
  __shared__ int split_coords[2];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t ring = (smem_u32(dsmem) + 1023u) & ~1023u;
  float* xch = reinterpret_cast<float*>(dsmem + (ring - smem_u32(dsmem)) + STAGES * STAGE_BYTES);
  // output staging (wide tiles): 1024-aligned, after the ring
  const uint32_t outbuf = ring + STAGES * STAGE_BYTES;
  // skinny split-K receive slots, after the SwiGLU exchange rows
  const uint32_t pbuf = ring + STAGES * STAGE_BYTES + tc_xch_bytes(BN, EPI, SWAP);
  const int S = p.split;
  const bool clustered = PAIR || S > 1;
  const uint32_t crank = clustered ? cluster_rank() : 0u;
  const int half = PAIR ? static_cast<int>(crank & 1u) : 0;  // which 128 rows of the tile
  const bool leader = (half == 0);
  const uint32_t lead_rank = crank & ~1u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PAIRS; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull_bar[b]), 1);
      mbar_init(smem_u32(&tempty_bar[b]), GROUP * (kEpiThreads / 32));
    }
    mbar_init(smem_u32(&drain_bar), 1);
    mbar_init(smem_u32(&res_bar), 1);
    mbar_init(smem_u32(&recv_bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_p);
    tma_prefetch_desc(&tm_q);
    if (!SWAP && p.out_tma) {
      tma_prefetch_desc(&tm_c);
      if (EPI == EPI_RESIDUAL) tma_prefetch_desc(&tm_r);
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_u32(&tmem_slot), TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(&tmem_slot), TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // the pair signals each other's barriers: both must be initialised first
  if constexpr (PAIR) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  // Skinny split: the CTAs of a cluster push partial rows into each other's
  // shared memory.  A first cluster-barrier phase, arrived at here and waited
  // on just before the first push, makes sure every CTA has started.
  bool push_waited = false;
  if (SWAP && S > 1) cluster_arrive_relaxed();
  pdl_launch_dependents();

  // split mode: this CTA's one tile (for the reduction after the roles)
  int split_prow = 0, split_qcol = 0;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();  // weights: streamed once
      const uint64_t pol_x = l2_policy_evict_last();   // activations: re-read
      // The weight operand does not depend on the previous kernel in the
      // stream, so its loads may start before griddepcontrol.wait.
      const void* tm_w = SWAP ? static_cast<const void*>(&tm_p) : static_cast<const void*>(&tm_q);
      const void* tm_x = SWAP ? static_cast<const void*>(&tm_q) : static_cast<const void*>(&tm_p);
      const uint32_t off_w = SWAP ? 0u : A_BYTES;
      const uint32_t off_x = SWAP ? A_BYTES : 0u;
      // stage st completes on the barrier of its stage pair
      auto full_addr = [&](int st) -> uint32_t {
        const uint32_t a = smem_u32(&full_bar[st >> 1]);
        return PAIR ? mapa_shared(a, lead_rank) : a;
      };
      auto load = [&](uint32_t dst, const void* tm, uint32_t bar, int c0, int c1, uint64_t pol) {
        if constexpr (PAIR) tma_load_2d_pair(dst, tm, bar, c0, c1, pol);
        else tma_load_2d(dst, tm, bar, c0, c1, pol);
      };
      int pend_k[STAGES], pend_row[STAGES];
      uint32_t arm_par[PAIRS];
      // No L2 prefetch of the weight boxes beyond the ring: one SM's TMA unit
      // issues prefetches in order with its loads, so the boxes of a whole K
      // range (28 x 16 KB for gate/up) delay the first token loads by ~3 K
      // cycles, and the loads of a kernel sharing the SM.  Measured on the
      // 22-layer decode step: 1.126 -> 1.044 ms at 32 tokens without it.
      int n_issued = 0;
      bool waited = false;
      int stage = 0;
      uint32_t phase = 0;
      UnitIter it;
      it.init(p, GROUP);
      Unit u;
      bool ok = true;
      while (ok && it.next(u)) {
        int tp, tq;
        tile_coords(u.tile, p, tp, tq);
        const int row_w = SWAP ? tp * kBM : tq * BN + half * QR;
        const int row_x = SWAP ? tq * BN : tp * TILE_P + half * kBM;
        for (int k = u.k0; k < u.k1; ++k) {
          // A whole ring of weight boxes goes out before griddepcontrol.wait,
          // then the activations of those stages, then stage by stage.  (Only
          // the first stage pair before the wait brought the first MMA of an
          // isolated launch ~700 cycles earlier but made the layer step
          // 0.0733 -> 0.0756 ms and decode at 32 tokens 0.964 -> 1.002 ms: the
          // weights streaming during the previous kernel are worth more.)
          if (!waited && n_issued >= STAGES) {
            pdl_wait();
            for (int i = 0; i < n_issued; ++i)
              load(ring + i * STAGE_BYTES + off_x, tm_x, full_addr(i), pend_k[i] * kBK,
                   pend_row[i], pol_x);
            waited = true;
          }
          if (n_issued >= STAGES) {
            // one wait frees a whole pair of stages
            if ((stage & 1) == 0 &&
                !mbar_wait_bounded(smem_u32(&empty_bar[stage >> 1]), phase ^ 1u, &abort_flag,
                                   p.err, DEVERR_TIMEOUT_PRODUCER)) {
              ok = false;
              break;
            }
          }
          const uint32_t sbase = ring + stage * STAGE_BYTES;
          const uint32_t fb = full_addr(stage);
          // the first stage of a pair arms the pair's barrier with the bytes
          // of both stages (of both CTAs of a CTA pair, on the leader's)
          if ((stage & 1) == 0) {
            if (leader) mbar_arrive_expect_tx(smem_u32(&full_bar[stage >> 1]), 2 * GROUP * STAGE_BYTES);
            arm_par[stage >> 1] = phase;
          }
          load(sbase + off_w, tm_w, fb, k * kBK, row_w, pol_w);
          if (waited) {
            load(sbase + off_x, tm_x, fb, k * kBK, row_x, pol_x);
          } else {
            pend_k[stage] = k;
            pend_row[stage] = row_x;
          }
          ++n_issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!waited) {
        pdl_wait();
        const int n = n_issued < STAGES ? n_issued : STAGES;
        for (int i = 0; i < n; ++i)
          load(ring + i * STAGE_BYTES + off_x, tm_x, full_addr(i), pend_k[i] * kBK, pend_row[i],
               pol_x);
      }
      if (!ok) {
        // Unwinding: let copies already in flight land before the CTA exits.
        if (leader) {
          const int n = (n_issued < STAGES ? n_issued : STAGES) / 2;
          for (int i = 0; i < n; ++i) {
            const unsigned long long t0 = global_timer_ns();
            while (!mbar_try_wait(smem_u32(&full_bar[i]), arm_par[i])) {
              if (global_timer_ns() - t0 > 100000000ull) {
                atomicCAS(p.err, 0, DEVERR_TIMEOUT_DRAIN);
                break;
              }
            }
          }
        } else {
          // the peer's copies complete on the leader's barriers: give them
          // time to land
          const unsigned long long t0 = global_timer_ns();
          while (global_timer_ns() - t0 < 2000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      const uint32_t peer = crank ^ 1u;
      auto commit = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          tc_commit_pair(smem_u32(bar));
          tc_commit_pair(mapa_shared(smem_u32(bar), peer));
        } else {
          tc_commit(smem_u32(bar));
        }
      };
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      const uint64_t desc0 = smem_desc_kmajor_sw128(ring);
      UnitIter it;
      it.init(p, GROUP);
      Unit u;
      bool ok = true;
      while (ok && it.next(u)) {
        if (!mbar_wait_bounded(smem_u32(&tempty_bar[acc]), acc_phase ^ 1u, &abort_flag, p.err,
                               DEVERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int k = u.k0; k < u.k1; k += 2) {
          // one wait covers two stages (stage is even here)
          if (!mbar_wait_bounded(smem_u32(&full_bar[stage >> 1]), phase, &abort_flag, p.err,
                                 DEVERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // descriptors differ from the ring's first one only in the start
          // address field (bits 0-13, address >> 4), which never carries
          const uint64_t sd = desc0 + static_cast<uint64_t>((stage * STAGE_BYTES) >> 4);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
              const uint64_t ad = sd + static_cast<uint64_t>((h * STAGE_BYTES + kk * kUmmaK * 2) >> 4);
              const uint64_t bd = ad + static_cast<uint64_t>(A_BYTES >> 4);
              const uint32_t accum = (k + h > u.k0 || kk > 0) ? 1u : 0u;
              if constexpr (PAIR) tc_mma_f16_pair(d, ad, bd, IDESC, accum);
              else tc_mma_f16(d, ad, bd, IDESC, accum);
            }
          }
          // both stages of the pair are free once these MMAs complete
          commit(&empty_bar[stage >> 1]);
          stage += 2;
          if (stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        commit(&tfull_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        // Make sure no MMA is still writing tensor memory before teardown.
        if constexpr (PAIR) tc_commit_pair(smem_u32(&drain_bar));
        else tc_commit(smem_u32(&drain_bar));
        const unsigned long long t0 = global_timer_ns();
        while (!mbar_try_wait(smem_u32(&drain_bar), 0)) {
          if (global_timer_ns() - t0 > 100000000ull) {
            atomicCAS(p.err, 0, DEVERR_TIMEOUT_DRAIN);
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    pdl_wait();
    const int quad = warp & 3;  // tcgen05.ld: warp w reaches lanes 32*(w%4)..+31
    const int lr = quad * 32 + lane;
    const int et = static_cast<int>(threadIdx.x) - 64;  // 0..127
    const uint32_t lead_tempty0 =
        PAIR ? mapa_shared(smem_u32(&tempty_bar[0]), lead_rank) : smem_u32(&tempty_bar[0]);
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t res_phase = 0;
    uint32_t sk_phase = 0;  // recv_bar: stream-K fix-up copies (split == 1 only)
    UnitIter it;
    it.init(p, GROUP);
    Unit u;
    while (it.next(u)) {
      // one thread waits for the accumulator, the others sleep on a named
      // barrier (no polling next to the MMA issuer)
      if (!epi_wait(smem_u32(&tfull_bar[acc]), acc_phase, et, &abort_flag, p.err, &epi_flag)) break;
      tc_fence_after();
      int tp, tq;
      tile_coords(u.tile, p, tp, tq);
      const int prow0 = SWAP ? tp * kBM : tp * TILE_P + half * kBM;
      const int qcol0 = tq * BN;
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      bool ok = true;
      if (S == 1) {
        if constexpr (!SWAP) {
          if (p.sk && u.k0 > 0) {
            // stream-K: this group's range starts inside the tile; its part
            // goes to the group that holds the tile's first k-blocks
            sk_write_partial<BN>(p, &tm_s, taddr, lr, et, outbuf);
          } else {
            int sk_n = 0;
            if (p.sk && u.k1 < p.kb) {
              // stream-K finisher: the contributors are the following groups
              // whose ranges start inside this tile
              const int G = static_cast<int>(gridDim.x) / GROUP;
              const int g = static_cast<int>(blockIdx.x) / GROUP;
              const long long W = static_cast<long long>(it.tiles) * it.kp;
              const long long tile_end = static_cast<long long>(u.tile + 1) * it.kp;
              while (g + 1 + sk_n < G && sk_range_start(W, g + 1 + sk_n, G) < tile_end) ++sk_n;
              const int first = (g + 1) * GROUP + half;
              ok = sk_wait(p.sk_flags, first, sk_n, GROUP, et, &abort_flag, p.err, &epi_flag) &&
                   sk_fixup<BN>(&tm_s, taddr, lr, et, ring, STAGES * STAGE_BYTES, first, sk_n,
                                GROUP, smem_u32(&recv_bar), sk_phase, &abort_flag, p.err,
                                &epi_flag);
            }
            if (ok) {
              if (p.out_tma) {
                ok = emit_tile_tma<DT, BN, EPI>(p, taddr, prow0, qcol0, lr, et, outbuf, &tm_c,
                                                &tm_r, smem_u32(&res_bar), res_phase,
                                                &abort_flag, &epi_flag);
              } else {
                TmemChunks<CW> src{taddr};
                emit_tile<DT, BN, EPI, SWAP, CW>(p, src, prow0, qcol0, lr, xch);
              }
            }
            if (ok && sk_n > 0) {
              // every thread has read the partials: clear the flags for the
              // next call
              named_bar_sync(1, kEpiThreads);
              if (et == 0)
                for (int j = 0; j < sk_n; ++j)
                  p.sk_flags[(g_of_cta<GROUP>() + 1 + j) * GROUP + half] = 0;
            }
          }
        } else {
          TmemChunks<CW> src{taddr};
          emit_tile<DT, BN, EPI, SWAP, CW>(p, src, prow0, qcol0, lr, xch);
        }
      } else {
        split_prow = prow0;
        split_qcol = qcol0;
        if constexpr (SWAP) {
          // Push this thread's partial row to the CTA that owns its feature
          // (local rows go to this CTA's own slots through the same path).
          if (!push_waited) {
            cluster_wait();
            push_waited = true;
          }
          constexpr int F = tc_push_features(EPI);
          constexpr int PITCH = tc_push_pitch(BN, EPI);
          const int f = (EPI == EPI_SWIGLU) ? (lr & 63) : lr;
          const int owner = (f * S) / F;
          const int f0 = (owner * F + S - 1) / S;
          const int rm = (F + S - 1) / S;
          const int col0 = (EPI == EPI_SWIGLU && lr >= 64) ? BN : 0;
          const uint32_t dst = mapa_shared(
              pbuf + static_cast<uint32_t>(((static_cast<int>(crank) * rm + (f - f0)) * PITCH + col0) * 4),
              static_cast<uint32_t>(owner));
          float v[32];
#pragma unroll 1
          for (int c = 0; c < BN; c += CW) {
            if constexpr (CW == 32) tmem_ld_32x32b_x32(taddr + c, v);
            else tmem_ld_32x32b_x16(taddr + c, v);
#pragma unroll
            for (int i = 0; i < CW; i += 4)
              st_cluster_f4(dst + (c + i) * 4, v[i], v[i + 1], v[i + 2], v[i + 3]);
          }
        }
        if constexpr (!SWAP) {
          // wide tiles: stage the column units other CTAs own (this CTA's
          // ring is idle: its MMAs are done)
          fence_proxy_async_smem();
          stage_unowned<DT, BN, EPI>(ring, taddr, lr, S, static_cast<int>(crank) / GROUP);
          fence_proxy_async_smem();
        }
      }
      if (!ok) break;
      if (S == 1) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          const uint32_t te = lead_tempty0 + static_cast<uint32_t>(acc * sizeof(uint64_t));
          if (PAIR && !leader) mbar_arrive_cluster(te);
          else mbar_arrive(te);
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // every TMA store of this CTA has finished before it exits
    if (et == 0) bulk_wait_group<0>();
  }

  if (S > 1) {
    // Every thread of every CTA of the cluster reaches each cluster barrier
    // exactly once, on the normal and on the unwinding path.
    if (threadIdx.x == 64) {
      split_coords[0] = split_prow;
      split_coords[1] = split_qcol;
    }
    const int j = static_cast<int>(crank) / GROUP;  // this CTA's k-split index
    if constexpr (!SWAP) {
      constexpr int U = split_units<BN, EPI>();
      constexpr int UC = unit_cols<EPI>();
      // arm the receive barrier before anyone can send
      if (threadIdx.x == 0)
        mbar_arrive_expect_tx(smem_u32(&recv_bar),
                              static_cast<uint32_t>((S - 1) * owner_units(j, U, S) * 128 * UC * 4));
      // (1) every CTA has staged its blocks, its ring is free to receive,
      // and every receive barrier is armed
      cluster_sync_all();
      if (threadIdx.x == 64 && !abort_flag)
        send_blocks<BN, EPI>(ring, smem_u32(&recv_bar), S, j, half, GROUP);
      if (warp >= 2) {
        const int et = static_cast<int>(threadIdx.x) - 64;
        const bool got = epi_wait(smem_u32(&recv_bar), 0, et, &abort_flag, p.err, &epi_flag);
        const int quad = warp & 3;
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
        if (got && !abort_flag) {
          tc_fence_after();
          reduce_received<DT, BN, EPI>(p, ring, taddr, quad * 32 + lane, S, j, split_coords[0],
                                       split_coords[1]);
        }
      }
      // (2) every copy has landed (each owner waited for its bytes): no CTA
      // leaves while a copy still reads its shared memory
      cluster_sync_all();
    } else {
      // Skinny tiles: each CTA pushed its partial rows before arriving here;
      // after this barrier every CTA reads only its own shared memory, so no
      // CTA's memory is accessed by a peer once it passes it.
      if (!push_waited) cluster_wait();
      cluster_sync_all();
      constexpr int F = tc_push_features(EPI);
      const int f0 = (j * F + S - 1) / S;
      const int f1 = ((j + 1) * F + S - 1) / S;
      if (!abort_flag)
        reduce_pushed<DT, BN, EPI>(p, pbuf, S, split_coords[0], split_coords[1], f0, f1,
                                   (F + S - 1) / S, static_cast<int>(threadIdx.x), kThreads);
    }
  } else if constexpr (PAIR) {
    // neither CTA of the pair may leave while the other can still signal it
    cluster_sync_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side: planning, tensor maps, launch
// ---------------------------------------------------------------------------

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  return fn;
}

struct TmapKey {
  const void* ptr;
  unsigned long long rows, cols;
  int box_cols, box_rows, type;
  bool operator==(const TmapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && box_cols == o.box_cols &&
           box_rows == o.box_rows && type == o.type;
  }
};

struct TmapEntry {
  TmapKey key;
  CUtensorMap map;
  bool used;
};

// Row-major [rows, cols] matrix (leading dimension = cols), boxes of
// box_cols x box_rows with 128-byte swizzle (box_cols * element size is 128
// bytes for every map made here), zero fill outside.  type: 0 f16, 1 bf16,
// 2 f32.  Encoded maps are cached per host thread (encoding costs
// microseconds).
bool make_tmap(CUtensorMap* out, const void* ptr, int type, unsigned long long rows,
               unsigned long long cols, int box_cols, int box_rows) {
  constexpr int kCache = 64;
  thread_local TmapEntry cache[kCache];
  thread_local int victim = 0;
  const TmapKey key{ptr, rows, cols, box_cols, box_rows, type};
  for (int i = 0; i < kCache; ++i) {
    if (cache[i].used && cache[i].key == key) {
      *out = cache[i].map;
      return true;
    }
  }
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  const int esz = (type == 2) ? 4 : 2;
  const CUtensorMapDataType dt = (type == 0)   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                 : (type == 1) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * esz};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(out, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  TmapEntry& e = cache[victim];
  victim = (victim + 1) % kCache;
  e.key = key;
  e.map = *out;
  e.used = true;
  return true;
}

template <int DT, int BN, int EPI, bool SWAP, bool PAIR>
cudaError_t launch_one(const Plan& pl, const CUtensorMap& tp, const CUtensorMap& tq,
                       const CUtensorMap& tc, const CUtensorMap& tr, const CUtensorMap& ts,
                       cudaStream_t stream) {
  constexpr int smem = tc_smem_bytes(BN, EPI, SWAP, PAIR);
  auto kern = tc_linear_kernel<DT, BN, EPI, SWAP, PAIR>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    // every kernel of this library asks for the largest shared-memory
    // carveout, so consecutive kernels can share an SM without reconfiguring it
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  const int cluster = (PAIR ? 2 : 1) * pl.p.split;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int na = 1;
  if (cluster > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, tp, tq, tc, tr, ts, pl.p);
}

// How many clusters of `cluster` CTAs of this tile shape can be resident at
// once (skinny tiles: measured with the SwiGLU epilogue, the largest).
template <int BN, bool SWAP, bool PAIR>
int max_active_clusters(int cluster) {
  constexpr int EPI = SWAP ? EPI_SWIGLU : EPI_NONE;
  constexpr int smem = tc_smem_bytes(BN, EPI, SWAP, PAIR);
  auto kern = tc_linear_kernel<DT_F16, BN, EPI, SWAP, PAIR>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                       cudaSharedmemCarveoutMaxShared);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster * 64);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

struct Maps {
  CUtensorMap p, q, c, r;
  CUtensorMap s;  // stream-K slots: fp32 [grid * 128, bn], 32 x 128 boxes
};

template <int DT, bool SWAP, int BN, bool PAIR>
cudaError_t dispatch_epi(const Plan& pl, int epi, const Maps& m, cudaStream_t s) {
  switch (epi) {
    case EPI_NONE: return launch_one<DT, BN, EPI_NONE, SWAP, PAIR>(pl, m.p, m.q, m.c, m.r, m.s, s);
    case EPI_SWIGLU: return launch_one<DT, BN, EPI_SWIGLU, SWAP, PAIR>(pl, m.p, m.q, m.c, m.r, m.s, s);
    case EPI_RESIDUAL: return launch_one<DT, BN, EPI_RESIDUAL, SWAP, PAIR>(pl, m.p, m.q, m.c, m.r, m.s, s);
    case EPI_F32_OUT: return launch_one<DT, BN, EPI_F32_OUT, SWAP, PAIR>(pl, m.p, m.q, m.c, m.r, m.s, s);
    case EPI_F32_PARTIAL: return launch_one<DT, BN, EPI_F32_PARTIAL, SWAP, PAIR>(pl, m.p, m.q, m.c, m.r, m.s, s);
  }
  return cudaErrorInvalidValue;
}

template <int DT>
cudaError_t dispatch_shape(const Plan& pl, int epi, const Maps& m, cudaStream_t s) {
  if (pl.algo == 1) {
    if (pl.pair) {
      if (pl.bn == 128) return dispatch_epi<DT, false, 128, true>(pl, epi, m, s);
      return dispatch_epi<DT, false, 256, true>(pl, epi, m, s);
    }
    if (pl.bn == 128) return dispatch_epi<DT, false, 128, false>(pl, epi, m, s);
    return dispatch_epi<DT, false, 256, false>(pl, epi, m, s);
  }
  switch (pl.bn) {
    case 16: return dispatch_epi<DT, true, 16, false>(pl, epi, m, s);
    case 32: return dispatch_epi<DT, true, 32, false>(pl, epi, m, s);
    case 64: return dispatch_epi<DT, true, 64, false>(pl, epi, m, s);
  }
  return cudaErrorInvalidValue;
}

// Per-device cache of resident-cluster counts: [shape][cluster size].
struct ClusterCaps {
  int dev = -1;
  int caps[7][9];  // shapes: wide 256, wide 128, skinny 16, 32, 64, pair 256, pair 128
};

int shape_index(int algo, int bn, int pair) {
  if (algo == 1) return pair ? (bn == 256 ? 5 : 6) : (bn == 256 ? 0 : 1);
  return bn == 16 ? 2 : bn == 32 ? 3 : 4;
}

int cluster_cap(int algo, int bn, int pair, int cluster) {
  if (cluster < 1 || cluster > 8) return 0;
  thread_local ClusterCaps cache[8];
  int dev = 0;
  cudaGetDevice(&dev);
  ClusterCaps& c = cache[dev & 7];
  if (c.dev != dev) {
    c.dev = dev;
    for (auto& row : c.caps)
      for (int& v : row) v = -1;
  }
  int& v = c.caps[shape_index(algo, bn, pair)][cluster];
  if (v < 0) {
    if (algo == 1)
      v = pair ? ((bn == 256) ? max_active_clusters<256, false, true>(cluster)
                              : max_active_clusters<128, false, true>(cluster))
               : (bn == 256) ? max_active_clusters<256, false, false>(cluster)
                             : max_active_clusters<128, false, false>(cluster);
    else
      v = (bn == 16) ? max_active_clusters<16, true, false>(cluster)
                     : (bn == 32) ? max_active_clusters<32, true, false>(cluster)
                                  : max_active_clusters<64, true, false>(cluster);
  }
  return v;
}

// Optional tuning override "BN,SPLIT[,PAIR[,SK]]" for wide tiles (ORIN_TC_PLAN).
bool plan_override(int& bn, int& split, int& pair, int& sk) {
  static int o_bn = -1, o_split = -1, o_pair = 0, o_sk = 0;
  static bool read = false;
  if (!read) {
    read = true;
    const char* e = getenv("ORIN_TC_PLAN");
    if (e) {
      const int n = sscanf(e, "%d,%d,%d,%d", &o_bn, &o_split, &o_pair, &o_sk);
      if (n < 2) o_bn = -1;
      if (n < 3) o_pair = 0;
      if (n < 4) o_sk = 0;
    }
    if (o_bn != 128 && o_bn != 256) o_bn = -1;
    if (o_split < 1 || o_split > 8) o_bn = -1;
    if (o_pair && o_split > 4) o_bn = -1;
    if (o_sk && o_split != 1) o_bn = -1;
  }
  if (o_bn < 0) return false;
  bn = o_bn;
  split = o_split;
  pair = o_pair;
  sk = o_sk;
  return true;
}

}  // namespace

size_t sk_workspace_bytes(int grid, int bn) {
  return kSkFlagBytes + static_cast<size_t>(grid) * kBM * bn * sizeof(float);
}

size_t sk_workspace_max_bytes(int sm_count) { return sk_workspace_bytes(sm_count, 256); }

void fill_tiles(Plan& pl, int K, int bn, int split, int pair, int sm_count, int sk_groups = 0) {
  const bool sk = sk_groups > 0;
  TcParams& p = pl.p;
  const int tile_p = pair ? 2 * kBM : kBM;
  const int group = pair ? 2 : 1;
  pl.bn = bn;
  pl.pair = pair;
  p.tiles_p = (p.P + tile_p - 1) / tile_p;
  p.tiles_q = (p.Q + bn - 1) / bn;
  p.kb = (K + kBK - 1) / kBK;
  p.kb += p.kb & 1;  // whole stage pairs; the extra block is zero-filled
  p.group_p = kGroupP;
  p.split = split;
  p.sk = sk ? 1 : 0;
  const int tiles = p.tiles_p * p.tiles_q;
  if (sk) {
    // every co-resident CTA group takes an equal share of tiles x K
    pl.grid = group * sk_groups;
  } else if (split == 1) {
    const int groups = sm_count / group;
    pl.grid = group * (tiles < groups ? tiles : groups);
  } else {
    pl.grid = tiles * split * group;
  }
}

// Choose the tile shape and the split-K factor with a cost model fitted to
// measurements on B200 (microseconds):
//   launch   fixed cost of one launch (set-up, first loads, last epilogue);
//   t_kb     time one CTA needs per 64-deep k-block, growing with the number
//            of CTAs running at once (they share L2 bandwidth);
//   exchange split-K: staging, the cluster barriers and the bulk copies.
// Tiles are dealt in waves of at most `groups` tiles; every wave pays its
// k-blocks at the rate of its own CTA count.
void plan_tc(Plan& pl, int M, int N, int K, int epi, int algo, int sm_count, size_t sk_bytes) {
  const int wrows = (epi == EPI_SWIGLU) ? 2 * N : N;  // rows of W
  TcParams& p = pl.p;
  p = TcParams{};
  p.M = M;
  p.N = N;
  p.K = K;
  pl.algo = algo;
  int kb = (K + kBK - 1) / kBK;
  kb += kb & 1;
  const int G = sm_count;
  if (algo == 2) {
    // skinny: HBM-bound; split K until (almost) every SM streams weights
    const int bn = (M <= 16) ? 16 : (M <= 32) ? 32 : 64;
    p.P = wrows;
    p.Q = M;
    const int tiles = (wrows + kBM - 1) / kBM;
    int split = 1;
    if (tiles < G) {
      split = G / tiles;
      if (split > 8) split = 8;
      if (split > kb / 2) split = kb / 2 > 0 ? kb / 2 : 1;
      // every cluster resident in one wave.  Keeping half of the slots free
      // for the next kernel's CTAs (where two skinny CTAs fit on an SM) cost
      // more than the overlap gained: at 32 tokens q/k/v 8.3 -> 6.6 us, o_proj
      // 8.0 -> 7.0, down 13.3 -> 11.0 without the reservation
      while (split > 1 && cluster_cap(2, bn, 0, split) < tiles) --split;
    }
    fill_tiles(pl, K, bn, split, 0, G);
    return;
  }
  p.P = M;
  p.Q = wrows;
  // a stream-K plan of tile shape (bn, pair) is possible when the workspace
  // holds its slots and every CTA group gets at least one k-block pair
  // The finishers wait on later groups, so every group of a stream-K grid must
  // be resident at once: the grid is the co-resident count of this tile shape
  // (one CTA, or one 2-CTA cluster, per SM pair), at most one group per SM.
  auto sk_groups = [&](int bn, int pair) {
    const int group = pair ? 2 : 1;
    int n = cluster_cap(1, bn, pair, group);
    if (n > G / group) n = G / group;
    return n;
  };
  // Most contributors any tile's finisher adds: groups g whose range starts
  // strictly inside a tile.
  auto sk_max_contributors = [&](long long tiles, int ng) {
    const long long kpp = kb / 2, W = tiles * kpp;
    int most = 0, run = 0;
    long long run_tile = -1;
    for (int g = 1; g < ng; ++g) {
      const long long st = W * g / ng;
      if (st % kpp == 0) continue;
      const long long t = st / kpp;
      run = (t == run_tile) ? run + 1 : 1;
      run_tile = t;
      if (run > most) most = run;
    }
    return most;
  };
  auto sk_possible = [&](int bn, int pair) {
    if (sk_bytes == 0) return false;
    const int group = pair ? 2 : 1;
    const int tile_p = pair ? 2 * kBM : kBM;
    const long long tiles =
        static_cast<long long>((M + tile_p - 1) / tile_p) * ((wrows + bn - 1) / bn);
    const int n = sk_groups(bn, pair);
    const int grid = group * n;
    if (n <= 0 || grid > kSkMaxGrid || sk_bytes < sk_workspace_bytes(grid, bn) ||
        tiles * (kb / 2) < n)
      return false;
    // the finisher stages a 32-column slab (16 KB) of every contributor in its
    // operand ring at once
    const int ring_bytes = tc_stages(bn, pair != 0) * tc_stage_bytes(bn, pair != 0);
    return sk_max_contributors(tiles, n) * 32 * 512 <= ring_bytes;
  };
  int obn = 0, osplit = 0, opair = 0, osk = 0;
  if (plan_override(obn, osplit, opair, osk) && !(epi == EPI_SWIGLU && obn % 128)) {
    if (osk && sk_possible(obn, opair)) {
      fill_tiles(pl, K, obn, 1, opair, G, sk_groups(obn, opair));
      return;
    }
    const int units = (epi == EPI_SWIGLU) ? obn / 64 : obn / 32;
    int sp = osplit > kb / 2 ? kb / 2 : osplit;
    if (sp > units) sp = units;
    const int ring_bytes = tc_stages(obn, opair != 0) * tc_stage_bytes(obn, opair != 0);
    while (sp > 1 && split_smem_bytes(units, epi == EPI_SWIGLU ? 64 : 32, sp) > ring_bytes) --sp;
    fill_tiles(pl, K, obn, sp, opair, G);
    return;
  }
  struct Shape {
    int bn, pair;
    double launch, t0, t_slope;  // t_kb = t0 + t_slope * ctas / sm_count
  };
  const Shape shapes[4] = {{256, 1, 4.0, 0.28, 0.16},
                           {128, 1, 4.0, 0.25, 0.07},
                           {256, 0, 3.5, 0.29, 0.17},
                           {128, 0, 3.5, 0.23, 0.05}};
  auto t_kb = [&](const Shape& sh, long long ctas) {
    return sh.t0 + sh.t_slope * static_cast<double>(ctas) / G;
  };
  double best = 1e30;
  int best_bn = 256, best_split = 1, best_pair = 0;
  int best_sk = 0;  // stream-K groups (0: no stream-K)
  for (const Shape& sh : shapes) {
    if (epi == EPI_SWIGLU && sh.bn % 128) continue;
    const int tile_p = sh.pair ? 2 * kBM : kBM;
    const int group = sh.pair ? 2 : 1;
    const long long tiles =
        static_cast<long long>((M + tile_p - 1) / tile_p) * ((wrows + sh.bn - 1) / sh.bn);
    // persistent, whole K per tile
    const long long groups = G / group;
    double cost = sh.launch;
    for (long long done = 0; done < tiles; done += groups) {
      const long long in_wave = (tiles - done < groups) ? tiles - done : groups;
      cost += kb * t_kb(sh, in_wave * group);
    }
    if (cost < best) {
      best = cost;
      best_bn = sh.bn;
      best_split = 1;
      best_pair = sh.pair;
      best_sk = 0;
    }
    // stream-K: every group takes an equal share of tiles x k-block pairs,
    // all at the full-machine rate; the groups that hold a tile's first
    // k-blocks wait for the other groups' partials of that tile and add them
    // before their last epilogue.  Measured on B200 (K scaled 1024..8192 at
    // M=512): the hand-off (contributor TMA store, flag, finisher TMA load,
    // add) costs ~6-7 us of fixed time over the persistent schedule, so
    // stream-K pays only where it saves more mainloop than that.
    if (sk_possible(sh.bn, sh.pair)) {
      const long long W = tiles * (kb / 2);
      const int ng = sk_groups(sh.bn, sh.pair);
      const long long per = (W + ng - 1) / ng;                   // pairs per group
      const int readers = sk_max_contributors(tiles, ng);
      const double fix = 8.0 + static_cast<double>(readers) * 0.5 * sh.bn / 256.0;
      cost = sh.launch + 2.0 * per * t_kb(sh, ng * group) + fix;
      if (cost < best) {
        best = cost;
        best_bn = sh.bn;
        best_split = 1;
        best_pair = sh.pair;
        best_sk = static_cast<int>(ng);
      }
    }
    // split columns are handed out in units (32 accumulator columns, 64 for
    // SwiGLU pairs): at most one owner per unit
    const int units = (epi == EPI_SWIGLU) ? sh.bn / 64 : sh.bn / 32;
    const int ring_bytes = tc_stages(sh.bn, sh.pair) * tc_stage_bytes(sh.bn, sh.pair);
    for (int s = 2; s * group <= 8 && s <= kb / 2 && s <= units; ++s) {
      if (split_smem_bytes(units, epi == EPI_SWIGLU ? 64 : 32, s) > ring_bytes) continue;
      // split plans run as a single wave of clusters
      const int cap_clusters = cluster_cap(1, sh.bn, sh.pair, s * group);
      if (cap_clusters <= 0 || tiles > cap_clusters) continue;
      const int kbc = 2 * (((kb / 2) + s - 1) / s);
      cost = sh.launch + kbc * t_kb(sh, tiles * s * group) + 2.0 + 2.0 * s;
      if (cost < best) {
        best = cost;
        best_bn = sh.bn;
        best_split = s;
        best_pair = sh.pair;
        best_sk = 0;
      }
    }
  }
  fill_tiles(pl, K, best_bn, best_split, best_pair, G, best_sk);
}

bool encode_tmap_2d(CUtensorMap* out, const void* ptr, int type, unsigned long long rows,
                    unsigned long long cols, int box_cols, int box_rows) {
  return make_tmap(out, ptr, type, rows, cols, box_cols, box_rows);
}

cudaError_t launch_tc(const Plan& pl0, int dtype, int epi, const void* A, const void* W,
                      int* err, cudaStream_t stream, const char** why, void* sk_ws) {
  Plan pl = pl0;
  if (pl.p.sk) {
    if (!sk_ws) {
      if (why) *why = "stream-K plan without a workspace";
      return cudaErrorInvalidValue;
    }
    pl.p.sk_flags = static_cast<int*>(sk_ws);
    pl.p.sk_ws = reinterpret_cast<float*>(static_cast<char*>(sk_ws) + kSkFlagBytes);
  }
  const TcParams& p = pl.p;
  const bool swap = pl.algo == 2;
  const void* pptr = swap ? W : A;
  const void* qptr = swap ? A : W;
  Maps m;
  if (!make_tmap(&m.p, pptr, dtype, static_cast<unsigned long long>(p.P),
                 static_cast<unsigned long long>(p.K), kBK, kBM) ||
      !make_tmap(&m.q, qptr, dtype, static_cast<unsigned long long>(p.Q),
                 static_cast<unsigned long long>(p.K), kBK, tc_qrows(pl.bn, pl.pair != 0))) {
    if (why) *why = "cuTensorMapEncodeTiled failed";
    return cudaErrorInvalidValue;
  }
  m.c = m.p;
  m.r = m.p;
  m.s = m.p;
  if (pl.p.sk &&
      !make_tmap(&m.s, pl.p.sk_ws, 2, static_cast<unsigned long long>(pl.grid) * kBM,
                 static_cast<unsigned long long>(pl.bn), 32, kBM)) {
    if (why) *why = "cuTensorMapEncodeTiled failed (stream-K workspace)";
    return cudaErrorInvalidValue;
  }
  pl.p.out_tma = 0;
  if (!swap && pl.p.split == 1) {
    // wide tiles store through TMA when C (and the residual) rows allow it
    const bool f32 = (epi == EPI_F32_OUT || epi == EPI_F32_PARTIAL);
    const int esz = f32 ? 4 : 2;
    const bool c_ok = (reinterpret_cast<uintptr_t>(p.C) % 16 == 0) && ((p.ldc * esz) % 16 == 0);
    const bool r_ok = (epi != EPI_RESIDUAL) ||
                      ((reinterpret_cast<uintptr_t>(p.R) % 16 == 0) && ((p.ldr * 2) % 16 == 0));
    if (c_ok && r_ok &&
        make_tmap(&m.c, p.C, f32 ? 2 : dtype, static_cast<unsigned long long>(p.M),
                  static_cast<unsigned long long>(p.N), f32 ? 32 : 64, kBM) &&
        (epi != EPI_RESIDUAL ||
         make_tmap(&m.r, p.R, dtype, static_cast<unsigned long long>(p.M),
                   static_cast<unsigned long long>(p.N), 64, kBM)))
      pl.p.out_tma = 1;
  }
  pl.p.err = err;
  if (dtype == DT_F16) return dispatch_shape<DT_F16>(pl, epi, m, stream);
  return dispatch_shape<DT_BF16>(pl, epi, m, stream);
}

}  // namespace orin
