// gemm_tc.cu — the sm_100a linear-layer kernel: C = epilogue(A · W^T).
//
// One persistent kernel template covers both shapes of the hot path:
//   * wide tiles (prefill, M > 64): 128 tokens x 256 weight rows per tile;
//   * skinny tiles (decode, M <= 64): 128 weight rows x {16,32,64} tokens per
//     tile ("swap AB": the weight matrix feeds the 128-lane side of the MMA,
//     so a one-token GEMV still streams weights through the tensor core at
//     full HBM speed, with no CUDA-core fp16->fp32 conversions).
//
// Per CTA (one per SM, 192 threads):
//   warp 0    TMA producer: 2-D tiled loads, 128-byte swizzle, into a
//             STAGES-deep shared-memory ring guarded by mbarriers.  Weight
//             tiles of the first ring pass are issued before the grid waits
//             on the previous kernel (programmatic dependent launch), so a
//             chain of layers keeps HBM busy across kernel boundaries.
//   warp 1    MMA issuer: one thread issues tcgen05.mma.cta_group::1.kind::f16
//             (fp16/bf16 in, fp32 accumulate) into a double-buffered tensor
//             memory accumulator, tcgen05.commit frees ring slots.
//   warps 2-5 epilogue: tcgen05.ld (32 lanes x 32 columns per warp), the
//             fused epilogue (SwiGLU / residual / fp32 widen), global stores.
//
// Scheduling: tiles are rastered in groups of P tiles so concurrently running
// CTAs share operand panels in L2.  Whole waves of tiles are done
// round-robin; the tiles left over (fewer than two waves) are split over all
// CTAs by k-block ranges ("stream-K").  A CTA that holds only part of a tile's
// k-range adds its fp32 partial into a workspace tile (vector atomics, done in
// L2) and bumps the tile's counter; the last arriver reads the sum, applies
// the epilogue, and zeroes the workspace tile and counter again.  No CTA ever
// waits on another CTA.
//
// Every mbarrier wait is bounded (orin_common.cuh): after 2 s the CTA records
// an error code in the device error word and unwinds instead of hanging.
//
// Reference semantics (kernels/matmul.cu:32-43, kernels/gemm_cute.cu:147,
// 176-178): fp32 products and accumulation, one rounding to 16 bits.
#include "orin_common.cuh"
#include "orin_internal.h"

#include <stdio.h>

namespace orin {

constexpr int kBM = 128;       // tile rows = MMA M = tensor-memory lanes
constexpr int kBK = 64;        // K per ring stage: one 128-byte row of 16-bit
constexpr int kUmmaK = 16;     // K per tcgen05.mma kind::f16
constexpr int kThreads = 192;  // 6 warps
constexpr int kEpiThreads = 128;
constexpr int kGroupP = 8;     // P tiles per raster group
constexpr int kMinSplitIters = 4;  // least k-blocks a CTA takes of a split tile

__host__ __device__ constexpr int tc_stage_bytes(int bn) { return kBM * kBK * 2 + bn * kBK * 2; }
__host__ __device__ constexpr int tc_stages(int bn) {
  return (196608 / tc_stage_bytes(bn)) > 12 ? 12 : (196608 / tc_stage_bytes(bn));
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
__host__ __device__ constexpr int tc_smem_bytes(int bn, int epi, bool swap) {
  return tc_stages(bn) * tc_stage_bytes(bn) + tc_xch_bytes(bn, epi, swap) + 1024;
}

// ---------------------------------------------------------------------------
// Work decomposition, computed identically by every role of every CTA.
// ---------------------------------------------------------------------------

struct Seg {
  int tile;
  int k0, k1;     // k-block range [k0, k1)
  int sk;         // -1: this CTA owns the whole tile; else stream-K tile index
  int ncontrib;   // CTAs that contribute to stream-K tile sk
};

struct SegIter {
  int G, c, kb, dp_waves, w, dp_tiles;
  long long pos, end, base, rem;

  __device__ __forceinline__ long long owner(long long i) const {
    const long long big = rem * (base + 1);
    return (i < big) ? i / (base + 1) : rem + (i - big) / base;
  }

  __device__ __forceinline__ void init(const TcParams& p) {
    G = gridDim.x;
    c = blockIdx.x;
    kb = p.kb;
    dp_tiles = p.dp_tiles;
    dp_waves = p.dp_tiles / G;
    w = 0;
    const long long total = static_cast<long long>(p.sk_tiles) * kb;
    const int g = p.sk_ctas;  // CTAs that take part in the split phase
    base = g > 0 ? total / g : 0;
    rem = g > 0 ? total % g : 0;
    if (c < g) {
      pos = c * base + (c < rem ? c : rem);
      end = pos + base + (c < rem ? 1 : 0);
    } else {
      pos = end = 0;
    }
  }

  __device__ __forceinline__ bool next(Seg& s) {
    if (w < dp_waves) {
      s.tile = w * G + c;
      s.k0 = 0;
      s.k1 = kb;
      s.sk = -1;
      s.ncontrib = 1;
      ++w;
      return true;
    }
    if (pos >= end) return false;
    const long long t = pos / kb;
    const int k0 = static_cast<int>(pos - t * kb);
    const long long left = end - pos;
    const int k1 = static_cast<int>((k0 + left < kb) ? (k0 + left) : kb);
    s.tile = dp_tiles + static_cast<int>(t);
    s.k0 = k0;
    s.k1 = k1;
    if (k0 == 0 && k1 == kb) {
      s.sk = -1;
      s.ncontrib = 1;
    } else {
      s.sk = static_cast<int>(t);
      s.ncontrib = static_cast<int>(owner(t * kb + kb - 1) - owner(t * kb) + 1);
    }
    pos += k1 - k0;
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

// Source of accumulator chunks for the epilogue: tensor memory (the CTA owns
// the whole tile) or the stream-K workspace tile (the last arriver), which is
// zeroed as it is read.
template <int CW>
struct TmemChunks {
  uint32_t taddr;  // lane base + accumulator buffer column
  __device__ __forceinline__ void get(int col, float* v) const {
    if constexpr (CW == 32) tmem_ld_32x32b_x32(taddr + col, v);
    else tmem_ld_32x32b_x16(taddr + col, v);
  }
};

template <int CW>
struct WsChunks {
  float* row;  // this thread's row of the workspace tile
  __device__ __forceinline__ void get(int col, float* v) const {
    float4* p = reinterpret_cast<float4*>(row + col);
#pragma unroll
    for (int i = 0; i < CW / 4; ++i) {
      const float4 f = __ldcg(p + i);
      v[4 * i + 0] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
      __stcg(p + i, make_float4(0.f, 0.f, 0.f, 0.f));
    }
  }
};

// Apply the epilogue to one tile row held by this thread (row `lr` of the
// tile) and store it.  Chunks come from `src` CW columns at a time.
template <int DT, int BN, int EPI, bool SWAP, int CW, class Src>
__device__ __forceinline__ void emit_tile(const TcParams& p, const Src& src, int tp, int tq,
                                          int lr, float* xch) {
  using E = Elem<DT>;
  using T = typename E::T;
  const bool vec = p.vec_ok != 0;
  float v[32];
  if constexpr (!SWAP) {
    const int m = tp * kBM + lr;
    const bool mval = m < p.M;
    if constexpr (EPI == EPI_SWIGLU) {
      // Q columns are packed [gate 64 | up 64] groups; output column of the
      // first gate column of group g is (tq*BN + 128g) / 2.
      float u[32];
#pragma unroll 1
      for (int g = 0; g < BN / 128; ++g) {
#pragma unroll 1
        for (int h = 0; h < 64; h += 32) {
          src.get(128 * g + h, v);
          src.get(128 * g + 64 + h, u);
          const int n = (tq * BN + 128 * g) / 2 + h;
          if (mval && n < p.N) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              v[j] = silu_f32(E::round(v[j])) * E::round(u[j]);
            store16_row<DT>(static_cast<T*>(p.C) + m * p.ldc + n, v, 32, p.N - n, vec);
          }
        }
      }
    } else {
#pragma unroll 1
      for (int c = 0; c < BN; c += CW) {
        src.get(c, v);
        const int n = tq * BN + c;
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
    // Skinny: this thread's row is weight row (feature) tp*128 + lr; its
    // columns are tokens tq*BN + c.
    if constexpr (EPI == EPI_SWIGLU) {
      // Packed rows: lanes 0-63 gate, 64-127 up, of output features
      // tp*64 + (lr % 64).
      const int n = tp * 64 + (lr & 63);
#pragma unroll 1
      for (int c = 0; c < BN; c += CW) {
        src.get(c, v);
        if (lr >= 64) {
#pragma unroll
          for (int j = 0; j < CW; ++j) xch[(lr - 64) * 32 + j] = E::round(v[j]);
        }
        named_bar_sync(1, kEpiThreads);
        if (lr < 64 && n < p.N) {
#pragma unroll
          for (int j = 0; j < CW; ++j) {
            const int m = tq * BN + c + j;
            if (m < p.M) {
              const float o = silu_f32(E::round(v[j])) * xch[lr * 32 + j];
              static_cast<T*>(p.C)[m * p.ldc + n] = E::from_f(o);
            }
          }
        }
        named_bar_sync(1, kEpiThreads);
      }
    } else {
      const int n = tp * kBM + lr;
      const bool nval = n < p.N;
#pragma unroll 1
      for (int c = 0; c < BN; c += CW) {
        src.get(c, v);
        if (!nval) continue;
#pragma unroll
        for (int j = 0; j < CW; ++j) {
          const int m = tq * BN + c + j;
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
// The kernel
// ---------------------------------------------------------------------------

template <int DT, int BN, int EPI, bool SWAP>
__global__ void __launch_bounds__(kThreads, 1)
    tc_linear_kernel(const __grid_constant__ CUtensorMap tm_p,
                     const __grid_constant__ CUtensorMap tm_q, const TcParams p) {
  constexpr int STAGES = tc_stages(BN);
  constexpr uint32_t A_BYTES = kBM * kBK * 2;
  constexpr uint32_t STAGE_BYTES = tc_stage_bytes(BN);
  constexpr uint32_t TMEM_COLS = tc_tmem_cols(BN);
  constexpr uint32_t IDESC = instr_desc_f16(DT, kBM, BN);
  constexpr int CW = (BN >= 32) ? 32 : 16;

  extern __shared__ uint8_t dsmem[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  __shared__ int arrival;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t ring = (smem_u32(dsmem) + 1023u) & ~1023u;
  float* xch = reinterpret_cast<float*>(dsmem + (ring - smem_u32(dsmem)) + STAGES * STAGE_BYTES);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull_bar[b]), 1);
      mbar_init(smem_u32(&tempty_bar[b]), kEpiThreads / 32);
    }
    mbar_init(smem_u32(&drain_bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_p);
    tma_prefetch_desc(&tm_q);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();  // weights: streamed once
      const uint64_t pol_x = l2_policy_evict_last();   // activations: re-read
      // Which of the two operands is the weight matrix (independent of the
      // previous kernel in the stream)?
      const void* tm_w = SWAP ? static_cast<const void*>(&tm_p) : static_cast<const void*>(&tm_q);
      const void* tm_x = SWAP ? static_cast<const void*>(&tm_q) : static_cast<const void*>(&tm_p);
      const uint32_t off_w = SWAP ? 0u : A_BYTES;
      const uint32_t off_x = SWAP ? A_BYTES : 0u;
      int pend_k[STAGES], pend_row[STAGES];
      uint32_t arm_par[STAGES];
      int n_issued = 0;
      bool waited = false;
      int stage = 0;
      uint32_t phase = 0;
      SegIter it;
      it.init(p);
      Seg s;
      bool ok = true;
      while (ok && it.next(s)) {
        int tp, tq;
        tile_coords(s.tile, p, tp, tq);
        const int row_w = SWAP ? tp * kBM : tq * BN;
        const int row_x = SWAP ? tq * BN : tp * kBM;
        for (int k = s.k0; k < s.k1; ++k) {
          if (n_issued >= STAGES) {
            if (!waited) {
              pdl_wait();
              for (int i = 0; i < STAGES; ++i)
                tma_load_2d(ring + i * STAGE_BYTES + off_x, tm_x, smem_u32(&full_bar[i]),
                            pend_k[i] * kBK, pend_row[i], pol_x);
              waited = true;
            }
            if (!mbar_wait_bounded(smem_u32(&empty_bar[stage]), phase ^ 1u, &abort_flag, p.err,
                                   DEVERR_TIMEOUT_PRODUCER)) {
              ok = false;
              break;
            }
          }
          const uint32_t sbase = ring + stage * STAGE_BYTES;
          const uint32_t fb = smem_u32(&full_bar[stage]);
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          arm_par[stage] = phase;
          tma_load_2d(sbase + off_w, tm_w, fb, k * kBK, row_w, pol_w);
          if (waited) {
            tma_load_2d(sbase + off_x, tm_x, fb, k * kBK, row_x, pol_x);
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
          tma_load_2d(ring + i * STAGE_BYTES + off_x, tm_x, smem_u32(&full_bar[i]),
                      pend_k[i] * kBK, pend_row[i], pol_x);
      }
      if (!ok) {
        // Unwinding: let copies already in flight land before the CTA exits.
        const int n = n_issued < STAGES ? n_issued : STAGES;
        for (int i = 0; i < n; ++i) {
          const unsigned long long t0 = global_timer_ns();
          while (!mbar_try_wait(smem_u32(&full_bar[i]), arm_par[i])) {
            if (global_timer_ns() - t0 > 100000000ull) {
              atomicCAS(p.err, 0, DEVERR_TIMEOUT_DRAIN);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      SegIter it;
      it.init(p);
      Seg s;
      bool ok = true;
      while (ok && it.next(s)) {
        if (!mbar_wait_bounded(smem_u32(&tempty_bar[acc]), acc_phase ^ 1u, &abort_flag, p.err,
                               DEVERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int k = s.k0; k < s.k1; ++k) {
          if (!mbar_wait_bounded(smem_u32(&full_bar[stage]), phase, &abort_flag, p.err,
                                 DEVERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = ring + stage * STAGE_BYTES;
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            const uint64_t ad = smem_desc_kmajor_sw128(a_addr + kk * kUmmaK * 2);
            const uint64_t bd = smem_desc_kmajor_sw128(b_addr + kk * kUmmaK * 2);
            tc_mma_f16(d, ad, bd, IDESC, (k > s.k0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(smem_u32(&empty_bar[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(smem_u32(&tfull_bar[acc]));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        // Make sure no MMA is still writing tensor memory before teardown.
        tc_commit(smem_u32(&drain_bar));
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
    const int et = threadIdx.x - 64;  // 0..127 within the epilogue group
    int acc = 0;
    uint32_t acc_phase = 0;
    SegIter it;
    it.init(p);
    Seg s;
    while (it.next(s)) {
      const bool failed = !mbar_wait_bounded(smem_u32(&tfull_bar[acc]), acc_phase, &abort_flag,
                                             p.err, DEVERR_TIMEOUT_EPILOGUE);
      // all 128 epilogue threads leave together (the epilogue uses named
      // barriers, which a thread that left early would never reach)
      if (named_bar_or(1, kEpiThreads, failed)) break;
      tc_fence_after();
      int tp, tq;
      tile_coords(s.tile, p, tp, tq);
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (s.sk < 0) {
        TmemChunks<CW> src{taddr};
        emit_tile<DT, BN, EPI, SWAP, CW>(p, src, tp, tq, lr, xch);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&tempty_bar[acc]));
      } else {
        // Partial tile: add into the workspace tile, then count arrivals.
        float* wrow = p.ws + (static_cast<size_t>(s.sk) * kBM + lr) * BN;
        const int prow = tp * kBM + lr;
        const bool rval = prow < p.P;
        float v[32];
#pragma unroll 1
        for (int c = 0; c < BN; c += CW) {
          if constexpr (CW == 32) tmem_ld_32x32b_x32(taddr + c, v);
          else tmem_ld_32x32b_x16(taddr + c, v);
          if (rval) {
#pragma unroll
            for (int i = 0; i < CW / 4; ++i)
              atomicAdd(reinterpret_cast<float4*>(wrow + c) + i,
                        make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&tempty_bar[acc]));
        __threadfence();
        named_bar_sync(1, kEpiThreads);
        if (et == 0) arrival = atomicAdd(p.counters + s.sk, 1);
        named_bar_sync(1, kEpiThreads);
        if (arrival == s.ncontrib - 1) {
          __threadfence();
          WsChunks<CW> src{wrow};
          emit_tile<DT, BN, EPI, SWAP, CW>(p, src, tp, tq, lr, xch);
          if (et == 0) p.counters[s.sk] = 0;
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side: planning, tensor maps, launch
// ---------------------------------------------------------------------------

void plan_tc(Plan& pl, int M, int N, int K, int epi, int algo, int sm_count) {
  const int wrows = (epi == EPI_SWIGLU) ? 2 * N : N;  // rows of W
  TcParams& p = pl.p;
  p = TcParams{};
  p.M = M;
  p.N = N;
  p.K = K;
  pl.algo = algo;
  if (algo == 2) {
    pl.bn = (M <= 16) ? 16 : (M <= 32) ? 32 : 64;
    p.P = wrows;
    p.Q = M;
  } else {
    pl.bn = 256;
    p.P = M;
    p.Q = wrows;
  }
  p.tiles_p = (p.P + kBM - 1) / kBM;
  p.tiles_q = (p.Q + pl.bn - 1) / pl.bn;
  p.kb = (K + kBK - 1) / kBK;
  p.group_p = kGroupP;
  const int tiles = p.tiles_p * p.tiles_q;
  const int G = sm_count;
  // Whole waves: one tile per CTA, full K.  The tiles left over (fewer than
  // a wave) are split by k-blocks so every CTA gets a share, but no CTA gets
  // less than kMinSplitIters k-blocks (fewer partial sums to combine).
  p.dp_tiles = (tiles / G) * G;
  p.sk_tiles = tiles - p.dp_tiles;
  const long long sk_iters = static_cast<long long>(p.sk_tiles) * p.kb;
  long long sk_ctas = sk_iters / kMinSplitIters;
  if (sk_ctas < p.sk_tiles) sk_ctas = p.sk_tiles;
  if (sk_ctas > G) sk_ctas = G;
  p.sk_ctas = p.sk_tiles > 0 ? static_cast<int>(sk_ctas) : 0;
  pl.grid = p.dp_tiles > 0 ? G : p.sk_ctas;
  const size_t part = static_cast<size_t>(p.sk_tiles) * kBM * pl.bn * sizeof(float);
  pl.ws_bytes = (p.sk_tiles > 0) ? part + static_cast<size_t>(p.sk_tiles) * sizeof(int) : 0;
}

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
  int box_rows, dt;
  bool operator==(const TmapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && box_rows == o.box_rows &&
           dt == o.dt;
  }
};

struct TmapEntry {
  TmapKey key;
  CUtensorMap map;
  bool used;
};

// Row-major [rows, cols] 16-bit matrix (leading dimension = cols), boxes of
// 64 columns x box_rows rows, 128-byte swizzle, zero fill outside.  Encoded
// maps are cached per host thread (encoding costs microseconds).
bool make_tmap(CUtensorMap* out, const void* ptr, int dt, unsigned long long rows,
               unsigned long long cols, int box_rows) {
  constexpr int kCache = 64;
  thread_local TmapEntry cache[kCache];
  thread_local int victim = 0;
  const TmapKey key{ptr, rows, cols, box_rows, dt};
  for (int i = 0; i < kCache; ++i) {
    if (cache[i].used && cache[i].key == key) {
      *out = cache[i].map;
      return true;
    }
  }
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(out, dt == DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                   2, const_cast<void*>(ptr), dims, strides, box, estr,
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

template <int DT, int BN, int EPI, bool SWAP>
cudaError_t launch_one(const Plan& pl, const CUtensorMap& tp, const CUtensorMap& tq,
                       cudaStream_t stream) {
  constexpr int smem = tc_smem_bytes(BN, EPI, SWAP);
  auto kern = tc_linear_kernel<DT, BN, EPI, SWAP>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tp, tq, pl.p);
}

template <int DT, bool SWAP, int BN>
cudaError_t dispatch_epi(const Plan& pl, int epi, const CUtensorMap& a, const CUtensorMap& b,
                         cudaStream_t s) {
  switch (epi) {
    case EPI_NONE: return launch_one<DT, BN, EPI_NONE, SWAP>(pl, a, b, s);
    case EPI_SWIGLU: return launch_one<DT, BN, EPI_SWIGLU, SWAP>(pl, a, b, s);
    case EPI_RESIDUAL: return launch_one<DT, BN, EPI_RESIDUAL, SWAP>(pl, a, b, s);
    case EPI_F32_OUT: return launch_one<DT, BN, EPI_F32_OUT, SWAP>(pl, a, b, s);
    case EPI_F32_PARTIAL: return launch_one<DT, BN, EPI_F32_PARTIAL, SWAP>(pl, a, b, s);
  }
  return cudaErrorInvalidValue;
}

template <int DT>
cudaError_t dispatch_shape(const Plan& pl, int epi, const CUtensorMap& a, const CUtensorMap& b,
                           cudaStream_t s) {
  if (pl.algo == 1) return dispatch_epi<DT, false, 256>(pl, epi, a, b, s);
  switch (pl.bn) {
    case 16: return dispatch_epi<DT, true, 16>(pl, epi, a, b, s);
    case 32: return dispatch_epi<DT, true, 32>(pl, epi, a, b, s);
    case 64: return dispatch_epi<DT, true, 64>(pl, epi, a, b, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_tc(const Plan& pl0, int dtype, int epi, const void* A, const void* W,
                      void* ws, int* err, cudaStream_t stream, const char** why) {
  Plan pl = pl0;
  const TcParams& p = pl.p;
  const bool swap = pl.algo == 2;
  const void* pptr = swap ? W : A;
  const void* qptr = swap ? A : W;
  CUtensorMap tmp, tmq;
  if (!make_tmap(&tmp, pptr, dtype, static_cast<unsigned long long>(p.P),
                 static_cast<unsigned long long>(p.K), kBM) ||
      !make_tmap(&tmq, qptr, dtype, static_cast<unsigned long long>(p.Q),
                 static_cast<unsigned long long>(p.K), pl.bn)) {
    if (why) *why = "cuTensorMapEncodeTiled failed";
    return cudaErrorInvalidValue;
  }
  pl.p.err = err;
  if (p.sk_tiles > 0) {
    pl.p.ws = static_cast<float*>(ws);
    pl.p.counters = reinterpret_cast<int*>(static_cast<char*>(ws) +
                                           static_cast<size_t>(p.sk_tiles) * kBM * pl.bn * sizeof(float));
  }
  if (dtype == DT_F16) return dispatch_shape<DT_F16>(pl, epi, tmp, tmq, stream);
  return dispatch_shape<DT_BF16>(pl, epi, tmp, tmq, stream);
}

}  // namespace orin
