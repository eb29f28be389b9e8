// attention_tc.cu — prefill attention on the 5th-generation tensor cores.
//
// The same attention as attention.cu (the reference's sink + sliding-window
// GQA attention, kernels/attention.cu:27-138, over the ring pools of
// src/kv_cache.cu:21-41): query token qi of a call of seq_len new tokens and
// cache_len positions sits at ap = cache_len - seq_len + qi and attends to the
// positions p <= ap with p < n_sink or p >= ap + 1 - W, each read through its
// pool slot (after the call's own K/V were scattered), with fp32 scores
// scale * q.k, an fp32 softmax and one 16-bit rounding of sum_p softmax_p v_p.
//
// Kernel (calls of many tokens; decode keeps the split-key mma.sync kernel):
// one CTA per 128 query rows of one KV head — a row is a (token, query head)
// pair, the heads of one GQA group stacked so they share every K/V tile —
// and 10 warps:
//   warp 0     TMA producer: K and V tiles of 128 pool slots (2-D boxes of
//              64 columns x 128 slots, 128-byte swizzle, no multicast) into
//              two-stage K and V rings; a K stage is free once S has read it,
//              a V stage once P V has;
//   warp 1     MMA issuer: S = Q K^T (M = 128 rows, N = 128 keys, K = head_dim)
//              into one of two tensor-memory buffers, then O += P V
//              (N = head_dim, K = 128 keys) into a tensor-memory accumulator,
//              V read as an MN-major operand straight from its TMA tile; S of
//              tile j + 1 is issued before P V of tile j;
//   warps 2-9  softmax, two threads per row (one per 64-key half): the row's
//              maximum from tensor memory, masks as two slot ranges per row,
//              P = 2^(c s - c m) rounded to 16 bits into one of two 128-byte-
//              swizzled P tiles in shared memory (the A operand of P V), O
//              rescaled in tensor memory only when a row maximum grows by
//              more than 2^8; at the end O / l, rounded and stored.
// CTAs start with the row blocks that have the most key tiles.
//
// Head dim 64 has a second form, attn_tc_pp_kernel: two 128-row query tiles
// per CTA sharing every K/V tile, four softmax warps per tile at one thread
// per row, the tensor core working on one tile while the other is in softmax.
// It halves the grid, so the launcher takes it only where every CTA has the
// same key tiles and halving the CTAs halves the waves.
//
// Keys are taken in slot order, 128 slots per tile (softmax does not depend on
// the order of its terms): slot s holds, for a query at ap, the logical
// position the reference reads there — s itself for a sink slot (attended if
// s <= ap), and for a window slot the one position p in [ap + 1 - W, ap] with
// n_sink + (p - n_sink) % W == s (attended if p >= n_sink).  While no query of
// the CTA has wrapped the ring (ap < n_sink + W), slots equal positions and the
// tiles past the last query's position are skipped (the causal half).
// Every wait is bounded (2 s, device error code).
#include <type_traits>

#include "orin_common.cuh"
#include "orin_internal.h"

namespace orin {

namespace {

constexpr int kAtThreads = 320;  // producer, MMA, 8 softmax warps
constexpr int kAtRows = 128;   // query rows per CTA (MMA M)
constexpr int kAtKeys = 128;   // key slots per tile (MMA N of S, K of P V)
constexpr int kAtStages = 2;   // K/V ring
constexpr uint32_t kAtom = kAtRows * 128;  // one 64-column x 128-row 16-bit box: 16 KB
constexpr uint32_t kPBytes = 2 * kAtom;     // one P tile: 128 rows x 128 keys, 16-bit
// O is rescaled only when a row's maximum grows by more than 2^kLazy in the
// exponent; until then P is taken against the older, smaller maximum (at
// most 2^kLazy, exact in 16 bits relative to its size) and O / l is
// unchanged because l is summed against the same maximum.
constexpr float kLazy = 8.f;

struct AttnTcParams {
  void* out;        // [seq_len, num_heads, head_dim] 16-bit
  const void* q;    // [seq_len, num_heads, head_dim] 16-bit
  int seq_len, cache_len, num_heads, num_kv_heads, n_sink, window;
  float scale;
  int group;  // G = num_heads / num_kv_heads
  int hpb;    // group heads per row block (min(G, 128))
  int tpb;    // tokens per row block (128 / hpb)
  int hsb;    // row blocks per (token block, group) when G > 128
  int row_blocks;  // per KV head
  int* err;
};

// Shared memory (after 1024-byte alignment): Q (head_dim / 64 boxes), the K
// ring, the V ring (head_dim / 64 boxes per stage), two P tiles (two 64-key
// boxes each).
template <int HD>
constexpr uint32_t at_q_bytes() { return (HD / 64) * kAtom; }
template <int HD>
constexpr uint32_t at_stage_bytes() { return 2 * (HD / 64) * kAtom; }
template <int HD>
constexpr uint32_t at_smem_bytes() {
  return 1024 + at_q_bytes<HD>() + kAtStages * at_stage_bytes<HD>() + 2 * kPBytes;
}

// Byte offset of 16-byte chunk j of row r in a 128-byte-swizzled box.
__device__ __forceinline__ uint32_t at_sw128(int r, int j) {
  return static_cast<uint32_t>(r * 128 + ((j ^ (r & 7)) << 4));
}

// Shared-memory descriptor of an MN-major operand in 128-byte-swizzle boxes:
// 64 contiguous MN elements per 128-byte row, rows along K; 8-row atoms 1024 B
// apart along K (stride byte offset), 64-element MN blocks `lbo` bytes apart
// (leading byte offset).
__device__ __forceinline__ uint64_t smem_desc_mnmajor_sw128(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Lane 0 of a softmax warp waits (bounded) on `bar` for the warp; false, in
// every lane, on timeout.  The softmax warps never wait for one another.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int lane,
                                          volatile int* abort_flag, int* err) {
  int ok = 1;
  if (lane == 0)
    ok = mbar_wait_bounded(bar, parity, abort_flag, err, DEVERR_TIMEOUT_EPILOGUE) ? 1 : 0;
  __syncwarp();
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Two 64-column loads (32 lanes x 32 bits) and one wait, in one statement.
__device__ __forceinline__ void tmem_ld_32x32b_x64x2(uint32_t taddr0, uint32_t taddr1, float* v0,
                                                     float* v1) {
  uint32_t r[128];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
      "%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
      "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
      "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63"
      "}, [%128];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
      "%64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, "
      "%80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, "
      "%96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, "
      "%112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127"
      "}, [%129];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
        "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
        "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]),
        "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]),
        "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]),
        "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]),
        "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]),
        "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]),
        "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]),
        "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]),
        "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]),
        "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]),
        "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]),
        "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]),
        "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]),
        "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]),
        "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]),
        "=r"(r[126]), "=r"(r[127])
      : "r"(taddr0), "r"(taddr1)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    v0[i] = __uint_as_float(r[i]);
    v1[i] = __uint_as_float(r[64 + i]);
  }
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The row's attended slots as two ranges [0, a_hi) and [b_lo, b_hi): the
// sinks, and the window positions [max(n_sink, ap + 1 - W), ap], whose slots
// are one run of ring residues (split in two where it wraps).
__device__ __forceinline__ void row_ranges(int ap, bool row_ok, int n_sink, int window,
                                           int& a_hi, int& b_lo, int& b_hi) {
  const int slots = n_sink + window;
  a_hi = b_lo = b_hi = 0;
  if (!row_ok) return;
  if (ap < n_sink) {
    a_hi = ap + 1;
    return;
  }
  const int w_lo = max(n_sink, ap + 1 - window);
  if (ap - w_lo + 1 >= window) {
    a_hi = slots;
    return;
  }
  const int r_lo = (w_lo - n_sink) % window, r_hi = (ap - n_sink) % window;
  if (r_lo == 0) {
    a_hi = n_sink + r_hi + 1;
  } else if (r_lo <= r_hi) {
    a_hi = n_sink;
    b_lo = n_sink + r_lo;
    b_hi = n_sink + r_hi + 1;
  } else {
    a_hi = n_sink + r_hi + 1;
    b_lo = n_sink + r_lo;
    b_hi = slots;
  }
}

// bits [lo, hi) of 64
__device__ __forceinline__ uint64_t range_bits64(int lo, int hi) {
  lo = max(lo, 0);
  hi = min(hi, 64);
  if (hi <= lo) return 0ull;
  const uint64_t top = hi == 64 ? ~0ull : ((1ull << hi) - 1ull);
  return top & ~((1ull << lo) - 1ull);
}

// -inf for the 64 keys [k0, k0 + 64) of v outside the ranges; skipped when
// every lane of the warp attends to all of them
__device__ __forceinline__ void mask64(float* v, int k0, int a_hi, int b_lo, int b_hi) {
  const uint64_t bits = range_bits64(0, a_hi - k0) | range_bits64(b_lo - k0, b_hi - k0);
  if (!__all_sync(0xffffffffu, bits == ~0ull)) {
    const uint32_t lo = static_cast<uint32_t>(bits), hi = static_cast<uint32_t>(bits >> 32);
#pragma unroll
    for (int i = 0; i < 64; ++i)
      if (!(((i < 32 ? lo : hi) >> (i & 31)) & 1u)) v[i] = -INFINITY;
  }
}

template <int DT, int HD>
__global__ void __launch_bounds__(kAtThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const AttnTcParams p) {
  using E = Elem<DT>;
  constexpr int NB = HD / 64;  // 64-column boxes per row of Q, K, V
  constexpr uint32_t IDESC_S = instr_desc_f16(DT, kAtRows, kAtKeys);
  constexpr uint32_t IDESC_O = instr_desc_f16(DT, kAtRows, HD) | (1u << 16);  // B MN-major
  constexpr uint32_t TMEM_COLS = 512;  // S x 2 (256 columns) + O (head_dim)
  constexpr uint32_t O_COL = 2 * kAtKeys;
  constexpr uint32_t TILE_BYTES = NB * kAtom;  // one K or one V tile

  extern __shared__ uint8_t at_dsmem[];
  __shared__ __align__(8) uint64_t k_full[kAtStages];
  __shared__ __align__(8) uint64_t k_empty[kAtStages];
  __shared__ __align__(8) uint64_t v_full[kAtStages];
  __shared__ __align__(8) uint64_t v_empty[kAtStages];
  __shared__ __align__(8) uint64_t s_full[2];   // S of tile j in buffer j % 2
  __shared__ __align__(8) uint64_t p_full[2];   // P of tile j in buffer j % 2
  __shared__ __align__(8) uint64_t pv_done[2];  // P V of tile j (and all before)
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  __shared__ float l_half[2][kAtRows];  // the two halves of each row's sum

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t base_s = (smem_u32(at_dsmem) + 1023u) & ~1023u;
  const uint32_t q_s = base_s;
  const uint32_t k_ring = q_s + TILE_BYTES;
  const uint32_t v_ring = k_ring + kAtStages * TILE_BYTES;
  const uint32_t p_s = v_ring + kAtStages * TILE_BYTES;

  // CTAs in launch order take the row blocks with the most key tiles first
  // (the last tokens), so the short causal blocks fill the last wave
  const int kvh = static_cast<int>(blockIdx.x % p.num_kv_heads);
  const int rb = p.row_blocks - 1 - static_cast<int>(blockIdx.x / p.num_kv_heads);
  const int tb = rb / p.hsb, hs = rb % p.hsb;
  const int t_lo = tb * p.tpb;
  const int base = p.cache_len - p.seq_len;
  int t_hi = t_lo + p.tpb - 1;
  if (t_hi > p.seq_len - 1) t_hi = p.seq_len - 1;
  const int slots = p.n_sink + p.window;
  const int ap_max = base + t_hi;
  // tiles of 128 slots to visit: all of them once a query may have wrapped
  // the ring, else the slots up to the last query's position
  const int n_tiles = (ap_max < slots) ? ap_max / kAtKeys + 1 : (slots + kAtKeys - 1) / kAtKeys;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kAtStages; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&k_empty[s]), 1);
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 1);
    }
    mbar_init(smem_u32(&s_full[0]), 1);
    mbar_init(smem_u32(&s_full[1]), 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&p_full[b]), 8);  // one arrival per softmax warp
      mbar_init(smem_u32(&pv_done[b]), 1);
    }
    mbar_init(smem_u32(&drain_bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  // q and the pools come from the previous kernels
  pdl_wait();
  // Q rows into shared memory (K-major, 128-byte swizzle), every thread
  const uint16_t* qg = static_cast<const uint16_t*>(p.q);
  for (int c = threadIdx.x; c < kAtRows * (HD / 8); c += kAtThreads) {
    const int r = c / (HD / 8), j = c % (HD / 8);  // row, 16-byte chunk of the row
    const int tr = r / p.hpb, hr = hs * p.hpb + r % p.hpb;
    const int tok = t_lo + tr;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (tr < p.tpb && tok < p.seq_len && hr < p.group)
      v = *reinterpret_cast<const uint4*>(
          qg + (static_cast<size_t>(tok) * p.num_heads + kvh * p.group + hr) * HD + 8 * j);
    const uint32_t a = q_s + (j / 8) * kAtom + at_sw128(r, j % 8);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // K tile j into stage j % 2 once S of tile j - 2 is done with it, V tile j
    // once P V of tile j - 2 is
    if (lane == 0) {
      int n_k = 0, n_v = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % kAtStages;
        const uint32_t par = ((j / kAtStages) - 1) & 1u;
        if (j >= kAtStages && !mbar_wait_bounded(smem_u32(&k_empty[st]), par, &abort_flag, p.err,
                                                 DEVERR_TIMEOUT_PRODUCER))
          break;
        mbar_arrive_expect_tx(smem_u32(&k_full[st]), TILE_BYTES);
#pragma unroll
        for (int c = 0; c < NB; ++c)
          tma_load_2d_plain(k_ring + st * TILE_BYTES + c * kAtom, &tm_k, smem_u32(&k_full[st]),
                            kvh * HD + 64 * c, j * kAtKeys);
        ++n_k;
        if (j >= kAtStages && !mbar_wait_bounded(smem_u32(&v_empty[st]), par, &abort_flag, p.err,
                                                 DEVERR_TIMEOUT_PRODUCER))
          break;
        mbar_arrive_expect_tx(smem_u32(&v_full[st]), TILE_BYTES);
#pragma unroll
        for (int c = 0; c < NB; ++c)
          tma_load_2d_plain(v_ring + st * TILE_BYTES + c * kAtom, &tm_v, smem_u32(&v_full[st]),
                            kvh * HD + 64 * c, j * kAtKeys);
        ++n_v;
      }
      if (abort_flag) {
        // let the copies in flight land before the CTA exits
        auto drain = [&](uint64_t* full, int n) {
          for (int j = n > kAtStages ? n - kAtStages : 0; j < n; ++j) {
            const unsigned long long t0 = global_timer_ns();
            while (!mbar_try_wait(smem_u32(&full[j % kAtStages]), (j / kAtStages) & 1u))
              if (global_timer_ns() - t0 > 100000000ull) break;
          }
        };
        drain(k_full, n_k);
        drain(v_full, n_v);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint64_t qd0 = smem_desc_kmajor_sw128(q_s);
      const uint64_t pd0 = smem_desc_kmajor_sw128(p_s);
      const uint64_t pd1 = smem_desc_kmajor_sw128(p_s + kPBytes);
      auto issue_s = [&](int j) -> bool {
        const int st = j % kAtStages;
        if (!mbar_wait_bounded(smem_u32(&k_full[st]), (j / kAtStages) & 1u, &abort_flag, p.err,
                               DEVERR_TIMEOUT_MMA))
          return false;
        tc_fence_after();
        const uint64_t kd0 = smem_desc_kmajor_sw128(k_ring + st * TILE_BYTES);
        const uint32_t d = tmem_base + static_cast<uint32_t>((j & 1) * kAtKeys);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t off = static_cast<uint64_t>(((kk / 4) * kAtom + (kk % 4) * 32) >> 4);
          tc_mma_f16(d, qd0 + off, kd0 + off, IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&s_full[j & 1]));
        tc_commit(smem_u32(&k_empty[st]));
        return true;
      };
      bool ok = n_tiles > 0 ? issue_s(0) : true;
      for (int j = 0; ok && j < n_tiles; ++j) {
        // S of the next tile goes ahead of this tile's softmax
        if (j + 1 < n_tiles && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        // P of tile j is in shared memory and O rescaled
        const int st = j % kAtStages;
        if (!mbar_wait_bounded(smem_u32(&p_full[j & 1]), (j >> 1) & 1u, &abort_flag, p.err,
                               DEVERR_TIMEOUT_MMA) ||
            !mbar_wait_bounded(smem_u32(&v_full[st]), (j / kAtStages) & 1u, &abort_flag, p.err,
                               DEVERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // V: MN-major, head_dim in 64-element blocks one box (16 KB) apart
        const uint64_t vd0 = smem_desc_mnmajor_sw128(v_ring + st * TILE_BYTES, kAtom);
#pragma unroll
        for (int kk = 0; kk < kAtKeys / 16; ++kk) {
          const uint64_t aoff = static_cast<uint64_t>(((kk / 4) * kAtom + (kk % 4) * 32) >> 4);
          const uint64_t boff = static_cast<uint64_t>((kk * 16 * 128) >> 4);  // 16 keys
          tc_mma_f16(tmem_base + O_COL, ((j & 1) ? pd1 : pd0) + aoff, vd0 + boff, IDESC_O,
                     (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(smem_u32(&pv_done[j & 1]));
        tc_commit(smem_u32(&v_empty[st]));
      }
      if (!ok) {
        tc_commit(smem_u32(&drain_bar));
        const unsigned long long t0 = global_timer_ns();
        while (!mbar_try_wait(smem_u32(&drain_bar), 0))
          if (global_timer_ns() - t0 > 100000000ull) break;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    // Two threads per row, in warps w and w + 4 (the same tensor-memory lane
    // quarter): half h takes keys [64 h, 64 h + 64) of each tile for P and
    // columns [h HD / 2, (h + 1) HD / 2) of O.  Both read the whole row of S
    // for its maximum (max is exact in any order, so the two agree bit for
    // bit and take the same rescaling decisions); the halves of the row sum
    // meet once, at the end.
    constexpr int KH = kAtKeys / 2;  // keys per half
    constexpr int OH = HD / 2;       // O columns per half
    const int quad = warp & 3;
    const int h = (warp - 2) >> 2;
    const int r = quad * 32 + lane;  // this thread's row (= tensor-memory lane)
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const int tr = r / p.hpb, hr = hs * p.hpb + r % p.hpb;
    const int tok = t_lo + tr;
    const bool row_ok = tr < p.tpb && tok < p.seq_len && hr < p.group;
    const int ap = base + tok;
    int a_hi, b_lo, b_hi;
    row_ranges(ap, row_ok, p.n_sink, p.window, a_hi, b_lo, b_hi);
    // a warp with no valid row only keeps the P hand-off in step
    const bool dead = __all_sync(0xffffffffu, !row_ok);
    // masks the keys [k0, k0 + N) of v outside the row's ranges (a bit per
    // key); the warp skips it when every lane attends to all of them
    auto mask = [&](float* v, int k0, auto n_tag) {
      constexpr int N = decltype(n_tag)::value;
      const uint64_t bits = range_bits64(0, a_hi - k0) | range_bits64(b_lo - k0, b_hi - k0);
      const uint64_t all = N == 64 ? ~0ull : ((1ull << N) - 1ull);
      if (!__all_sync(0xffffffffu, (bits & all) == all)) {
        const uint32_t lo = static_cast<uint32_t>(bits), hi = static_cast<uint32_t>(bits >> 32);
#pragma unroll
        for (int i = 0; i < N; ++i)
          if (!(((i < 32 ? lo : hi) >> (i & 31)) & 1u)) v[i] = -INFINITY;
      }
    };
    // exp(scale * (s - m)) = 2^(s * c - m * c), c = scale * log2(e)
    const float c = p.scale * 1.4426950408889634f;
    // m: the maximum P is taken against (raw score units); l: this half's sum
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int b = j & 1;
      if (!warp_wait(smem_u32(&s_full[b]), (j >> 1) & 1u, lane, &abort_flag, p.err)) {
        ok = false;
        break;
      }
      if (dead) {
        // S of tile j exists, so P V of tile j - 2 was issued: this arrival
        // cannot land in an earlier phase of p_full[b]
        if (lane == 0) mbar_arrive(smem_u32(&p_full[b]));
        continue;
      }
      tc_fence_after();
      const uint32_t s_t = lane_base + static_cast<uint32_t>(b * kAtKeys);
      const int s0 = j * kAtKeys;
      // this half of the row, and the other half for the maximum only
      float sv[KH], so[KH];
      tmem_ld_32x32b_x64x2(s_t + h * KH, s_t + (1 - h) * KH, sv, so);
      mask(sv, s0 + h * KH, std::integral_constant<int, KH>());
      mask(so, s0 + (1 - h) * KH, std::integral_constant<int, KH>());
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = fmaxf(sv[i], so[i]);
#pragma unroll
      for (int i = 8; i < KH; ++i) mx[i & 7] = fmaxf(mx[i & 7], fmaxf(sv[i], so[i]));
      const float m_tile =
          fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      // the warp moves its rows' maxima (and rescales O) only when one of them
      // grows by more than 2^kLazy; a row with nothing attended yet keeps
      // m = -inf and adds nothing
      const bool grow = (m_tile - m_run) * c > kLazy;  // false for -inf - -inf
      float alpha = 1.f;
      const bool rescale = __any_sync(0xffffffffu, grow);
      if (rescale) {
        const float m_new = fmaxf(m_run, m_tile);
        alpha = (m_new == -INFINITY) ? 1.f : ex2_approx((m_run - m_new) * c);
        m_run = m_new;
      }
      if (j > 0 && rescale) {
        // O holds P V of every earlier tile: wait for the last one
        if (!warp_wait(smem_u32(&pv_done[b ^ 1]), ((j - 1) >> 1) & 1u, lane, &abort_flag,
                       p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < OH; cc += 32) {
          float v[32];
          tmem_ld_32x32b_x32(lane_base + O_COL + h * OH + cc, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tmem_st_32x32b_x32(lane_base + O_COL + h * OH + cc, v);
        }
      } else if (j >= 2) {
        // P buffer b was last read by P V of tile j - 2
        if (!warp_wait(smem_u32(&pv_done[b]), ((j >> 1) - 1) & 1u, lane, &abort_flag, p.err)) {
          ok = false;
          break;
        }
      }
      const float mc = (m_run == -INFINITY) ? 0.f : m_run * c;
      float sum[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sum[i] = 0.f;
#pragma unroll
      for (int i = 0; i < KH; ++i) {
        sv[i] = ex2_approx(fmaf(sv[i], c, -mc));  // masked: 2^-inf = 0
        sum[i & 7] += sv[i];
      }
      // P rounded to 16 bits: this half is box h of P tile b, row r
      const uint32_t pb = p_s + static_cast<uint32_t>(b) * kPBytes + static_cast<uint32_t>(h) * kAtom;
#pragma unroll
      for (int ch = 0; ch < KH / 8; ++ch) {
        const uint32_t addr = pb + at_sw128(r, ch);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr),
                     "r"(E::pack2(sv[8 * ch + 0], sv[8 * ch + 1])),
                     "r"(E::pack2(sv[8 * ch + 2], sv[8 * ch + 3])),
                     "r"(E::pack2(sv[8 * ch + 4], sv[8 * ch + 5])),
                     "r"(E::pack2(sv[8 * ch + 6], sv[8 * ch + 7]))
                     : "memory");
      }
      l_run = l_run * alpha + ((sum[0] + sum[1]) + (sum[2] + sum[3])) +
              ((sum[4] + sum[5]) + (sum[6] + sum[7]));
      fence_proxy_async_smem();  // P, written by threads, is read by the tensor core
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&p_full[b]));
    }
    if (ok && n_tiles > 0)
      ok = warp_wait(smem_u32(&pv_done[(n_tiles - 1) & 1]), ((n_tiles - 1) >> 1) & 1u, lane,
                     &abort_flag, p.err);
    // the two halves of the row sum; both warps of the pair get here (every
    // wait above is bounded) and agree on whether to write
    l_half[h][r] = l_run;
    if (named_bar_and(1 + quad, 64, ok) && n_tiles > 0) {
      tc_fence_after();
      const float l = l_half[0][r] + l_half[1][r];
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint16_t* dst = static_cast<uint16_t*>(p.out) +
                      (static_cast<size_t>(tok) * p.num_heads + kvh * p.group + hr) * HD + h * OH;
#pragma unroll 1
      for (int cc = 0; cc < OH; cc += 32) {
        float v[32];
        tmem_ld_32x32b_x32(lane_base + O_COL + h * OH + cc, v);
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 u;
            u.x = E::pack2(v[i + 0] * inv, v[i + 1] * inv);
            u.y = E::pack2(v[i + 2] * inv, v[i + 3] * inv);
            u.z = E::pack2(v[i + 4] * inv, v[i + 5] * inv);
            u.w = E::pack2(v[i + 6] * inv, v[i + 7] * inv);
            *reinterpret_cast<uint4*>(dst + cc + i) = u;
          }
        }
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
// Head dim 64: two 128-row query tiles per CTA in ping-pong.  Tiles A and B
// (row blocks 2c and 2c + 1 of one KV head) share every K/V tile; warps 2-5
// run tile A's softmax and warps 6-9 tile B's, one thread per row, so the
// tensor core computes S or P V of one tile while the other is in softmax:
//   S_A(j), S_B(j); then per tile t: [P_t(j) ready] P V_t(j), S_t(j + 1).
// Tensor memory: S_A, S_B (128 columns each), O_A, O_B (64 each).  Shared
// memory: Q_A, Q_B, two-stage K and V rings, P_A, P_B (one per tile: a tile's
// softmax waits for its P V of tile j - 1 before writing P of tile j).
// ---------------------------------------------------------------------------

constexpr int kPpThreads = 320;

template <int DT>
__global__ void __launch_bounds__(kPpThreads, 1)
    attn_tc_pp_kernel(const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v, const AttnTcParams p) {
  using E = Elem<DT>;
  constexpr int HD = 64;
  constexpr uint32_t IDESC_S = instr_desc_f16(DT, kAtRows, kAtKeys);
  constexpr uint32_t IDESC_O = instr_desc_f16(DT, kAtRows, HD) | (1u << 16);  // B MN-major
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t O_COL = 2 * kAtKeys;  // O_t at O_COL + t * HD
  constexpr uint32_t TILE = kAtom;          // one 64-column x 128-row box

  extern __shared__ uint8_t pp_dsmem[];
  __shared__ __align__(8) uint64_t k_full[kAtStages];
  __shared__ __align__(8) uint64_t k_empty[kAtStages];
  __shared__ __align__(8) uint64_t v_full[kAtStages];
  __shared__ __align__(8) uint64_t v_empty[kAtStages];
  __shared__ __align__(8) uint64_t s_full[2];   // per query tile
  __shared__ __align__(8) uint64_t p_full[2];   // per query tile, one arrival per warp
  __shared__ __align__(8) uint64_t pv_done[2];  // per query tile
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t base_s = (smem_u32(pp_dsmem) + 1023u) & ~1023u;
  const uint32_t q_s = base_s;                     // Q_A, Q_B
  const uint32_t k_ring = q_s + 2 * TILE;
  const uint32_t v_ring = k_ring + kAtStages * TILE;
  const uint32_t p_s = v_ring + kAtStages * TILE;  // P_A, P_B (two boxes each)

  // CTAs in launch order take the row-block pairs with the most key tiles first
  const int kvh = static_cast<int>(blockIdx.x % p.num_kv_heads);
  const int pairs = (p.row_blocks + 1) / 2;
  const int pair = pairs - 1 - static_cast<int>(blockIdx.x / p.num_kv_heads);
  const int base = p.cache_len - p.seq_len;
  const int slots = p.n_sink + p.window;
  // tile t is row block 2 * pair + t: tokens from tile_lo(t), head slice tile_hs(t)
  auto tile_lo = [&](int t) { return ((2 * pair + t) / p.hsb) * p.tpb; };
  auto tile_hs = [&](int t) { return (2 * pair + t) % p.hsb; };
  auto tile_ok = [&](int t) { return 2 * pair + t < p.row_blocks; };
  int ap_max = 0;
  for (int t = 0; t < 2; ++t) {
    if (tile_ok(t)) {
      const int t_hi = min(tile_lo(t) + p.tpb - 1, p.seq_len - 1);
      ap_max = max(ap_max, base + t_hi);
    }
  }
  const int n_tiles = (ap_max < slots) ? ap_max / kAtKeys + 1 : (slots + kAtKeys - 1) / kAtKeys;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kAtStages; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&k_empty[s]), 1);
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&s_full[t]), 1);
      mbar_init(smem_u32(&p_full[t]), 4);
      mbar_init(smem_u32(&pv_done[t]), 1);
    }
    mbar_init(smem_u32(&drain_bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  pdl_wait();
  // both tiles' Q rows into shared memory (K-major, 128-byte swizzle)
  const uint16_t* qg = static_cast<const uint16_t*>(p.q);
  for (int c = threadIdx.x; c < 2 * kAtRows * (HD / 8); c += kPpThreads) {
    const int t = c / (kAtRows * (HD / 8));
    const int cc = c % (kAtRows * (HD / 8));
    const int r = cc / (HD / 8), j = cc % (HD / 8);
    const int tr = r / p.hpb, hr = tile_hs(t) * p.hpb + r % p.hpb;
    const int tok = tile_lo(t) + tr;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (tile_ok(t) && tr < p.tpb && tok < p.seq_len && hr < p.group)
      v = *reinterpret_cast<const uint4*>(
          qg + (static_cast<size_t>(tok) * p.num_heads + kvh * p.group + hr) * HD + 8 * j);
    const uint32_t a = q_s + t * TILE + at_sw128(r, j);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int n_k = 0, n_v = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % kAtStages;
        const uint32_t par = ((j / kAtStages) - 1) & 1u;
        if (j >= kAtStages && !mbar_wait_bounded(smem_u32(&k_empty[st]), par, &abort_flag, p.err,
                                                 DEVERR_TIMEOUT_PRODUCER))
          break;
        mbar_arrive_expect_tx(smem_u32(&k_full[st]), TILE);
        tma_load_2d_plain(k_ring + st * TILE, &tm_k, smem_u32(&k_full[st]), kvh * HD,
                          j * kAtKeys);
        ++n_k;
        if (j >= kAtStages && !mbar_wait_bounded(smem_u32(&v_empty[st]), par, &abort_flag, p.err,
                                                 DEVERR_TIMEOUT_PRODUCER))
          break;
        mbar_arrive_expect_tx(smem_u32(&v_full[st]), TILE);
        tma_load_2d_plain(v_ring + st * TILE, &tm_v, smem_u32(&v_full[st]), kvh * HD,
                          j * kAtKeys);
        ++n_v;
      }
      if (abort_flag) {
        auto drain = [&](uint64_t* full, int n) {
          for (int j = n > kAtStages ? n - kAtStages : 0; j < n; ++j) {
            const unsigned long long t0 = global_timer_ns();
            while (!mbar_try_wait(smem_u32(&full[j % kAtStages]), (j / kAtStages) & 1u))
              if (global_timer_ns() - t0 > 100000000ull) break;
          }
        };
        drain(k_full, n_k);
        drain(v_full, n_v);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      auto issue_s = [&](int t, int j) -> bool {
        const int st = j % kAtStages;
        if (t == 0 && !mbar_wait_bounded(smem_u32(&k_full[st]), (j / kAtStages) & 1u, &abort_flag,
                                         p.err, DEVERR_TIMEOUT_MMA))
          return false;
        tc_fence_after();
        const uint64_t qd = smem_desc_kmajor_sw128(q_s + t * TILE);
        const uint64_t kd = smem_desc_kmajor_sw128(k_ring + st * TILE);
        const uint32_t d = tmem_base + static_cast<uint32_t>(t * kAtKeys);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t off = static_cast<uint64_t>((kk * 32) >> 4);
          tc_mma_f16(d, qd + off, kd + off, IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&s_full[t]));
        if (t == 1) tc_commit(smem_u32(&k_empty[st]));  // both tiles' S read K(j)
        return true;
      };
      auto issue_pv = [&](int t, int j) -> bool {
        const int st = j % kAtStages;
        if (!mbar_wait_bounded(smem_u32(&p_full[t]), j & 1u, &abort_flag, p.err,
                               DEVERR_TIMEOUT_MMA) ||
            (t == 0 && !mbar_wait_bounded(smem_u32(&v_full[st]), (j / kAtStages) & 1u,
                                          &abort_flag, p.err, DEVERR_TIMEOUT_MMA)))
          return false;
        tc_fence_after();
        const uint64_t pd = smem_desc_kmajor_sw128(p_s + t * 2 * TILE);
        const uint64_t vd = smem_desc_mnmajor_sw128(v_ring + st * TILE, TILE);
#pragma unroll
        for (int kk = 0; kk < kAtKeys / 16; ++kk) {
          const uint64_t aoff = static_cast<uint64_t>(((kk / 4) * TILE + (kk % 4) * 32) >> 4);
          const uint64_t boff = static_cast<uint64_t>((kk * 16 * 128) >> 4);  // 16 keys
          tc_mma_f16(tmem_base + O_COL + t * HD, pd + aoff, vd + boff, IDESC_O,
                     (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(smem_u32(&pv_done[t]));
        if (t == 1) tc_commit(smem_u32(&v_empty[st]));  // both tiles' P V read V(j)
        return true;
      };
      bool ok = n_tiles == 0 || (issue_s(0, 0) && issue_s(1, 0));
      for (int j = 0; ok && j < n_tiles; ++j) {
        // per tile: P V of tile j once its P is ready, then its S of tile j + 1
        // (its S buffer was read before P was written)
        for (int t = 0; ok && t < 2; ++t) {
          if (!issue_pv(t, j) || (j + 1 < n_tiles && !issue_s(t, j + 1))) ok = false;
        }
      }
      if (!ok) {
        tc_commit(smem_u32(&drain_bar));
        const unsigned long long t0 = global_timer_ns();
        while (!mbar_try_wait(smem_u32(&drain_bar), 0))
          if (global_timer_ns() - t0 > 100000000ull) break;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int t = (warp - 2) >> 2;  // query tile
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // this thread's row (= tensor-memory lane)
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t s_t = lane_base + static_cast<uint32_t>(t * kAtKeys);
    const uint32_t o_t = lane_base + O_COL + static_cast<uint32_t>(t * HD);
    const int tr = r / p.hpb, hr = tile_hs(t) * p.hpb + r % p.hpb;
    const int tok = tile_lo(t) + tr;
    const bool row_ok = tile_ok(t) && tr < p.tpb && tok < p.seq_len && hr < p.group;
    const int ap = base + tok;
    int a_hi, b_lo, b_hi;
    row_ranges(ap, row_ok, p.n_sink, p.window, a_hi, b_lo, b_hi);
    const bool dead = __all_sync(0xffffffffu, !row_ok);
    const float c = p.scale * 1.4426950408889634f;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    const uint32_t pb = p_s + static_cast<uint32_t>(t * 2) * TILE;
    for (int j = 0; j < n_tiles; ++j) {
      if (!warp_wait(smem_u32(&s_full[t]), j & 1u, lane, &abort_flag, p.err)) {
        ok = false;
        break;
      }
      if (dead) {
        if (lane == 0) mbar_arrive(smem_u32(&p_full[t]));
        continue;
      }
      tc_fence_after();
      // one row is 128 scores, more than the 168 registers a thread has at
      // 320 threads leave room for: the first half is read for the maximum
      // and read again for its exponentials (S stays until P is published)
      const int s0 = j * kAtKeys;
      float sv[64];
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        tmem_ld_32x32b_x32x2(s_t + half * 64, s_t + half * 64 + 32, sv, sv + 32);
        mask64(sv, s0 + half * 64, a_hi, b_lo, b_hi);
#pragma unroll
        for (int i = 0; i < 64; ++i) mx[i & 7] = fmaxf(mx[i & 7], sv[i]);
      }
      const float m_tile = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                 fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      const bool grow = (m_tile - m_run) * c > kLazy;
      float alpha = 1.f;
      const bool rescale = __any_sync(0xffffffffu, grow);
      if (rescale) {
        const float m_new = fmaxf(m_run, m_tile);
        alpha = (m_new == -INFINITY) ? 1.f : ex2_approx((m_run - m_new) * c);
        m_run = m_new;
      }
      // P V of tile j - 1 has finished: P's buffer is free and O is final
      if (j > 0) {
        if (!warp_wait(smem_u32(&pv_done[t]), (j - 1) & 1u, lane, &abort_flag, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (rescale) {
#pragma unroll 1
          for (int cc = 0; cc < HD; cc += 32) {
            float v[32];
            tmem_ld_32x32b_x32(o_t + cc, v);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= alpha;
            tmem_st_32x32b_x32(o_t + cc, v);
          }
        }
      }
      const float mc = (m_run == -INFINITY) ? 0.f : m_run * c;
      float sum[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sum[i] = 0.f;
      // the second half is still in sv; then the first half again
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int half = 1 - pass;
        if (pass == 1) {
          tmem_ld_32x32b_x32x2(s_t, s_t + 32, sv, sv + 32);
          mask64(sv, s0, a_hi, b_lo, b_hi);
        }
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          sv[i] = ex2_approx(fmaf(sv[i], c, -mc));
          sum[i & 7] += sv[i];
        }
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint32_t addr = pb + static_cast<uint32_t>(half) * TILE + at_sw128(r, ch);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr),
                       "r"(E::pack2(sv[8 * ch + 0], sv[8 * ch + 1])),
                       "r"(E::pack2(sv[8 * ch + 2], sv[8 * ch + 3])),
                       "r"(E::pack2(sv[8 * ch + 4], sv[8 * ch + 5])),
                       "r"(E::pack2(sv[8 * ch + 6], sv[8 * ch + 7]))
                       : "memory");
        }
      }
      l_run = l_run * alpha + ((sum[0] + sum[1]) + (sum[2] + sum[3])) +
              ((sum[4] + sum[5]) + (sum[6] + sum[7]));
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&p_full[t]));
    }
    if (ok && n_tiles > 0 &&
        warp_wait(smem_u32(&pv_done[t]), (n_tiles - 1) & 1u, lane, &abort_flag, p.err)) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      uint16_t* dst = static_cast<uint16_t*>(p.out) +
                      (static_cast<size_t>(tok) * p.num_heads + kvh * p.group + hr) * HD;
#pragma unroll 1
      for (int cc = 0; cc < HD; cc += 32) {
        float v[32];
        tmem_ld_32x32b_x32(o_t + cc, v);
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 u;
            u.x = E::pack2(v[i + 0] * inv, v[i + 1] * inv);
            u.y = E::pack2(v[i + 2] * inv, v[i + 3] * inv);
            u.z = E::pack2(v[i + 4] * inv, v[i + 5] * inv);
            u.w = E::pack2(v[i + 6] * inv, v[i + 7] * inv);
            *reinterpret_cast<uint4*>(dst + cc + i) = u;
          }
        }
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

// 1024 alignment slack + Q_A, Q_B + K and V rings + P_A, P_B
constexpr uint32_t kPpSmem = 1024 + (2 + 2 * kAtStages + 4) * kAtom;

template <int DT>
cudaError_t launch_pp(const AttnTcParams& p, const void* k_pool, const void* v_pool,
                      cudaStream_t s) {
  CUtensorMap tk, tv;
  const long long slots = static_cast<long long>(p.n_sink) + p.window;
  const unsigned long long rows =
      static_cast<unsigned long long>(p.cache_len < slots ? p.cache_len : slots);
  const unsigned long long cols = static_cast<unsigned long long>(p.num_kv_heads) * 64;
  if (!encode_tmap_2d(&tk, k_pool, DT, rows, cols, 64, kAtKeys) ||
      !encode_tmap_2d(&tv, v_pool, DT, rows, cols, 64, kAtKeys))
    return cudaErrorInvalidValue;
  auto kern = attn_tc_pp_kernel<DT>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kPpSmem);
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  const int pairs = (p.row_blocks + 1) / 2;
  return launch_pdl_smem(kern, dim3(pairs * p.num_kv_heads), dim3(kPpThreads), kPpSmem, s, tk,
                         tv, p);
}

template <int DT, int HD>
cudaError_t launch_at(const AttnTcParams& p, int row_blocks, const void* k_pool,
                      const void* v_pool, cudaStream_t s) {
  CUtensorMap tk, tv;
  // only slots that hold a written position: the rest read as zeros (a slot
  // no call has written yet may hold any bits, and 0 * NaN would reach O)
  const long long slots = static_cast<long long>(p.n_sink) + p.window;
  const unsigned long long rows =
      static_cast<unsigned long long>(p.cache_len < slots ? p.cache_len : slots);
  const unsigned long long cols = static_cast<unsigned long long>(p.num_kv_heads) * HD;
  if (!encode_tmap_2d(&tk, k_pool, DT, rows, cols, 64, kAtKeys) ||
      !encode_tmap_2d(&tv, v_pool, DT, rows, cols, 64, kAtKeys))
    return cudaErrorInvalidValue;
  auto kern = attn_tc_kernel<DT, HD>;
  constexpr int smem = static_cast<int>(at_smem_bytes<HD>());
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  return launch_pdl_smem(kern, dim3(row_blocks * p.num_kv_heads), dim3(kAtThreads), smem, s, tk,
                         tv, p);
}

}  // namespace

bool attention_tc_supported(int seq_len, int num_heads, int num_kv_heads, int head_dim,
                            int n_sink, int window) {
  if (head_dim != 64 && head_dim != 128) return false;
  if (num_kv_heads < 1 || num_heads % num_kv_heads != 0) return false;
  const int group = num_heads / num_kv_heads;
  // calls with a full block of rows; a group either divides 128 or is a
  // multiple of it
  if (static_cast<long long>(seq_len) * group < kAtRows) return false;
  if (group <= kAtRows ? (kAtRows % group) != 0 : (group % kAtRows) != 0) return false;
  if (num_kv_heads > 65535 || window < 1 || n_sink < 0) return false;
  return true;
}

namespace {

// Whether two query tiles per CTA beat one.  Both kernels hold one CTA per
// SM.  A paired step (two tiles' softmax on the same eight warps, the tensor
// core working on one tile while the other is in softmax) measured 1.74x a
// single tile's step on B200, so pairing pays only where every CTA has the
// same key tiles (every row attends the whole ring: no causal tail for the
// one-tile grid's heaviest-first order to pack) and halving the CTAs halves
// the waves (1020 x 2048 tokens, 32/4 heads of 64: 256 CTAs in two waves
// 37.1 us, 128 paired CTAs in one 32.2 us; the causal 1028 x 1028 chunk
// 22.5 us against 29.0 paired).
bool pairs_pay(const AttnTcParams& p) {
  const long long first_ap = static_cast<long long>(p.cache_len) - p.seq_len;
  if (first_ap < static_cast<long long>(p.n_sink) + p.window - 1) return false;
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int n_sm = (dev >= 0 && dev < 64) ? sms[dev] : 0;
  if (n_sm == 0) {
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    if (n_sm <= 0) return false;
    if (dev >= 0 && dev < 64) sms[dev] = n_sm;
  }
  const long long one = static_cast<long long>(p.row_blocks) * p.num_kv_heads;
  const long long two = static_cast<long long>((p.row_blocks + 1) / 2) * p.num_kv_heads;
  const long long waves_one = (one + n_sm - 1) / n_sm, waves_two = (two + n_sm - 1) / n_sm;
  return waves_one >= 2 * waves_two;
}

}  // namespace

cudaError_t launch_attention_tc(void* out, const void* q, const void* k_pool, const void* v_pool,
                                int seq_len, int cache_len, int num_heads, int num_kv_heads,
                                int head_dim, float scale, int n_sink, int window, int dtype,
                                int* err, cudaStream_t s, int pairing) {
  AttnTcParams p;
  p.out = out;
  p.q = q;
  p.seq_len = seq_len;
  p.cache_len = cache_len;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.n_sink = n_sink;
  p.window = window;
  p.scale = scale;
  p.group = num_heads / num_kv_heads;
  p.hpb = p.group < kAtRows ? p.group : kAtRows;
  p.tpb = kAtRows / p.hpb;
  p.hsb = (p.group + p.hpb - 1) / p.hpb;
  p.err = err;
  const long long rb = static_cast<long long>((seq_len + p.tpb - 1) / p.tpb) * p.hsb;
  if (rb * num_kv_heads > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  const int row_blocks = static_cast<int>(rb);
  p.row_blocks = row_blocks;
  if (head_dim == 64 && (pairing == 2 || (pairing == 0 && pairs_pay(p)))) {
    return dtype == DT_F16 ? launch_pp<DT_F16>(p, k_pool, v_pool, s)
                           : launch_pp<DT_BF16>(p, k_pool, v_pool, s);
  }
  if (head_dim == 64)
    return dtype == DT_F16 ? launch_at<DT_F16, 64>(p, row_blocks, k_pool, v_pool, s)
                           : launch_at<DT_BF16, 64>(p, row_blocks, k_pool, v_pool, s);
  return dtype == DT_F16 ? launch_at<DT_F16, 128>(p, row_blocks, k_pool, v_pool, s)
                         : launch_at<DT_BF16, 128>(p, row_blocks, k_pool, v_pool, s);
}

}  // namespace orin
