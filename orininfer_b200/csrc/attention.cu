// attention.cu — sink + sliding-window GQA attention over the ring KV pool,
// and the scatter of a call's new K/V rows into that pool.
//
// Pool layout (the reference's, src/kv_cache.cu:21-41): per layer one K and
// one V pool of n_sink + W slots, slot-major [slot][num_kv_heads][head_dim].
// Logical position p lives in slot p (p < n_sink) or n_sink + (p - n_sink) % W.
//
// Attention (kernels/attention.cu:27-138): query token qi of a call with
// seq_len new tokens and cache_len positions in total sits at
// ap = cache_len - seq_len + qi and attends to every position p with
//   p <= ap  and  (p < n_sink  or  p >= ap + 1 - W),
// read through its slot after the call's own tokens were scattered (so a
// chunk that wraps the ring reads its own later tokens in the wrapped slots,
// as the reference does):
//   out[qi, h] = round16( sum_p softmax_p(scale * q[qi, h] . k[p, h / G]) v[p, h / G] )
// with G = num_heads / num_kv_heads, fp32 scores, fp32 softmax and fp32 sums.
//
// Kernel: one CTA (4 warps) per (row block, kv head, key split).  A row is one
// (token, query head) pair; the heads of one GQA group share the K/V tiles, so
// a row block stacks tokens x group heads (16 rows per warp, the m16n8k16 tile).
// Keys stream through shared memory in 64-key tiles (cp.async, two stages,
// rows padded by 16 bytes so the fragment loads are bank-conflict free) in the
// order of their logical positions: the sink range, then the window range.
// The split partials of a decode row block (16 rows) are merged by the last
// of its split CTAs to arrive (an arrival counter in the workspace's first
// 4 KB, which every call leaves zero), in split order; those of a prefill row
// block (64 rows, too many for one CTA's loads in flight) by a combine launch
// over every SM.
// S = Q K^T and O += P V run on mma.sync m16n8k16 with an online softmax in
// registers.  Prefill blocks put 4 warps on 64 rows; decode blocks put the 4
// warps on one 16-row group and split each key tile between them, and split
// the key range across CTAs; partials (running max, sum, unnormalised O)
// merge in shared memory and, across CTAs, as above.  Every CTA lets the next
// kernel launch at once, and a single-token call's splits whose first tile
// ends before the new token issue their K/V loads before the dependency wait.
#include <cstdlib>
#include <cstring>

#include "orin_common.cuh"
#include "orin_internal.h"

namespace orin {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kKeyTile = 64;

struct AttnParams {
  void* out;           // [seq_len, num_heads, head_dim] 16-bit
  const void* q;       // [seq_len, num_heads, head_dim] 16-bit
  const void* k_pool;  // [n_sink + W, num_kv_heads, head_dim] 16-bit
  const void* v_pool;
  float* ws;           // split partials (splits > 1): O [splits][rows][HD], then (m, l) pairs
  int* counters;       // splits > 1: one arrival counter per (grid x, grid y), zero between calls
  int merge_here;      // splits > 1: the last split CTA merges (else attn_combine_kernel)
  int own_slots_only;  // the kernel before this one wrote only the call's own positions' slots
  int seq_len, cache_len, num_heads, num_kv_heads, n_sink, window;
  float scale;
  int group;   // G = num_heads / num_kv_heads
  int hpb;     // group heads per row block
  int tpb;     // tokens per row block
  int hsb;     // row blocks per (token block, group) when G > rows per block
  int splits;  // key splits (grid z)
  int batch;   // sequences (grid y = batch * num_kv_heads); rows [batch][seq_len][heads]
  long long pool_stride;  // elements from one sequence's pools to the next
};

// Pool slot of logical position p (src/kv_cache.cu:29-31).
__device__ __forceinline__ int ring_slot(int p, int n_sink, int window) {
  return p < n_sink ? p : n_sink + (p - n_sink) % window;
}

__device__ __forceinline__ void cp_async_16(void* smem, const void* gmem, bool full) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int n = full ? 16 : 0;  // 0 bytes read: the 16 bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t lds32(const uint16_t* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

// Four 8x8 16-bit matrices, transposed: lane l gives the row address of
// matrix l / 8, row l % 8; register i receives matrix i's elements
// (2 * (lane % 4) + {0, 1}, lane / 4).
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const uint16_t* p) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}

// D += A B, m16n8k16, fp32 accumulate.  Fragments (lane = 4 g + q):
//   A: a0 = (g, 2q..2q+1), a1 = (g+8, 2q..), a2 = (g, 2q+8..), a3 = (g+8, 2q+8..)
//   B: b0 = (k 2q..2q+1, n g), b1 = (k 2q+8..2q+9, n g)
//   D: d0, d1 = (g, 2q..2q+1), d2, d3 = (g+8, 2q..2q+1)
template <int DT>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (DT == DT_F16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Key ranges of one row block: tokens [t_lo, t_hi] attend to the sink range
// [0, sink_cnt) and the window range [win_lo, win_lo + win_cnt).
struct KeyRanges {
  int sink_cnt, win_lo, win_cnt, tiles_sink, tiles;
};

__device__ __host__ __forceinline__ KeyRanges key_ranges(int ap_lo, int ap_hi, int n_sink,
                                                        int window) {
  KeyRanges r;
  r.sink_cnt = ap_hi + 1 < n_sink ? ap_hi + 1 : n_sink;
  int lo = ap_lo + 1 - window;
  if (lo < n_sink) lo = n_sink;
  r.win_lo = lo;
  r.win_cnt = ap_hi >= lo ? ap_hi - lo + 1 : 0;
  r.tiles_sink = (r.sink_cnt + kKeyTile - 1) / kKeyTile;
  r.tiles = r.tiles_sink + (r.win_cnt + kKeyTile - 1) / kKeyTile;
  return r;
}

template <int HD>
constexpr int attn_pitch() { return HD + 8; }  // 16-bit elements per staged key row
template <int HD>
constexpr int attn_stage_elems() { return kKeyTile * attn_pitch<HD>(); }
template <int HD>
constexpr int attn_smem_bytes() {
  return 4 * attn_stage_elems<HD>() * 2;  // 2 stages x (K, V)
}

// RW = warps stacked on rows (4: 64 rows, prefill), the other 4 / RW warps
// split each key tile.
// out[orow][d, d + 4) = round16(o / l) over the key splits' partials, in
// split order with a running maximum (flash-decoding style): o = sum_s f_s O_s,
// l = sum_s f_s l_s, f_s = exp(m_s - max m).  The partials are read through L2
// (written by other CTAs), 16 splits' loads in flight before their updates.
template <int DT, int HD>
__device__ __forceinline__ void merge_splits(void* out, const float* ws, int rows_total,
                                             int splits, int orow, int d) {
  using E = Elem<DT>;
  const float* mlb = ws + static_cast<size_t>(splits) * rows_total * HD;
  float m = -INFINITY, l = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
  constexpr int kB = 16;
  for (int sp = 0; sp < splits; sp += kB) {
    float2 mlv[kB];
    float4 ov[kB];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      if (sp + u < splits) {
        const size_t pr = static_cast<size_t>(sp + u) * rows_total + orow;
        mlv[u] = __ldcg(reinterpret_cast<const float2*>(mlb + pr * 2));
        ov[u] = __ldcg(reinterpret_cast<const float4*>(ws + pr * HD + d));
      } else {
        mlv[u] = make_float2(-INFINITY, 0.f);
        ov[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      if (mlv[u].x == -INFINITY) continue;  // a split with no attended key adds nothing
      const float m_new = fmaxf(m, mlv[u].x);
      const float a = m == -INFINITY ? 0.f : __expf(m - m_new);
      const float f = __expf(mlv[u].x - m_new);
      l = l * a + f * mlv[u].y;
      o[0] = o[0] * a + f * ov[u].x;
      o[1] = o[1] * a + f * ov[u].y;
      o[2] = o[2] * a + f * ov[u].z;
      o[3] = o[3] * a + f * ov[u].w;
      m = m_new;
    }
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + static_cast<size_t>(orow) * HD + d) =
      make_uint2(E::pack2(o[0] * inv, o[1] * inv), E::pack2(o[2] * inv, o[3] * inv));
}

template <int DT, int HD, int RW>
__global__ void __launch_bounds__(kAttnThreads)
    attn_kernel(const AttnParams p) {
  using E = Elem<DT>;
  constexpr int KW = 4 / RW;          // warps sharing a row group
  constexpr int KC = kKeyTile / KW;   // keys per warp per tile
  constexpr int NB = KC / 8;          // S n-blocks per warp
  constexpr int KS = HD / 16;         // k-steps of Q K^T
  constexpr int ON = HD / 8;          // O n-blocks
  constexpr int PITCH = attn_pitch<HD>();
  constexpr int R = 16 * RW;          // rows per block
  constexpr int OP = HD + 4;          // fp32 pitch of the merge area
  static_assert(KC % 16 == 0, "a warp's key slice must cover whole k-steps");
  static_assert(KW * R * OP * 4 <= attn_smem_bytes<HD>(), "merge area must fit the stages");

  extern __shared__ __align__(16) uint16_t attn_smem[];
  __shared__ float s_m[KW * R];
  __shared__ float s_l[KW * R];

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q4 = lane & 3;
  const int rw = warp % RW, kw = warp / RW;

  const int kvh = blockIdx.y % p.num_kv_heads;
  const int bseq = blockIdx.y / p.num_kv_heads;  // sequence of this CTA
  const int tb = blockIdx.x / p.hsb, hs = blockIdx.x % p.hsb;
  const int t_lo = tb * p.tpb;
  int t_hi = t_lo + p.tpb - 1;
  if (t_hi > p.seq_len - 1) t_hi = p.seq_len - 1;
  const int base = p.cache_len - p.seq_len;
  const KeyRanges kr = key_ranges(base + t_lo, base + t_hi, p.n_sink, p.window);
  const int per = (kr.tiles + p.splits - 1) / p.splits;
  const int tile0 = blockIdx.z * per;
  int tile1 = tile0 + per;
  if (tile1 > kr.tiles) tile1 = kr.tiles;

  // The two rows of this lane: warp rows g and g + 8 of row group rw.
  int tok[2], head[2], ap[2];
  bool rv[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = rw * 16 + g + 8 * i;
    const int tr = r / p.hpb, hr = hs * p.hpb + r % p.hpb;
    tok[i] = t_lo + tr;
    head[i] = kvh * p.group + hr;
    rv[i] = tr < p.tpb && tok[i] < p.seq_len && hr < p.group;
    ap[i] = base + tok[i];
  }

  const uint16_t* kpool = static_cast<const uint16_t*>(p.k_pool) + bseq * p.pool_stride;
  const uint16_t* vpool = static_cast<const uint16_t*>(p.v_pool) + bseq * p.pool_stride;
  // this sequence's first q / out row
  const size_t row_base = static_cast<size_t>(bseq) * p.seq_len * p.num_heads;
  // stage s: K at 2 s, V at 2 s + 1 (in units of one staged tile)
  auto sK = [&](int stage) { return attn_smem + (2 * stage) * attn_stage_elems<HD>(); };
  auto sV = [&](int stage) { return attn_smem + (2 * stage + 1) * attn_stage_elems<HD>(); };

  auto tile_start = [&](int t, int& end) {
    if (t < kr.tiles_sink) {
      end = kr.sink_cnt;
      return t * kKeyTile;
    }
    end = kr.win_lo + kr.win_cnt;
    return kr.win_lo + (t - kr.tiles_sink) * kKeyTile;
  };
  auto load_tile = [&](int t, int stage) {
    int end;
    const int start = tile_start(t, end);
    constexpr int CPR = HD / 8;  // 16-byte chunks per key row
    for (int c = tid; c < kKeyTile * CPR; c += kAttnThreads) {
      const int row = c / CPR, col = (c % CPR) * 8;
      const int pos = start + row;
      const bool ok = pos < end;
      size_t off = 0;
      if (ok)
        off = (static_cast<size_t>(ring_slot(pos, p.n_sink, p.window)) * p.num_kv_heads + kvh) *
                  HD + col;
      cp_async_16(sK(stage) + row * PITCH + col, kpool + off, ok);
      cp_async_16(sV(stage) + row * PITCH + col, vpool + off, ok);
    }
  };

  // The next kernel (o_proj's weight stream) may be scheduled at once: it
  // waits for this grid's end before reading the output, and streams its
  // weights meanwhile.
  pdl_launch_dependents();
  // q and the new token's K/V row come from the previous kernels.  When the
  // caller states that the kernel before this call wrote no pool slot but
  // those of the call's own positions (own_slots_only: the decoder's RoPE +
  // append), a single-token call's one new position, base, is the last of
  // the window range and every other attended position sits in a slot
  // nothing in flight writes: a first tile that ends before base is loaded
  // before griddepcontrol.wait, overlapping the previous kernel's tail.
  bool early = false;
  if (p.own_slots_only && p.seq_len == 1 && tile0 < tile1) {
    int end;
    const int start = tile_start(tile0, end);
    early = min(start + kKeyTile, end) - 1 < base;
  }
  if (early) load_tile(tile0, 0);
  pdl_wait();
  if (!early && tile0 < tile1) load_tile(tile0, 0);
  cp_async_commit();

  // Q fragments of the two rows, straight from global memory.
  uint32_t qa[KS][4];
  {
    const uint16_t* qb = static_cast<const uint16_t*>(p.q) + row_base * HD;
    const uint16_t* q0 =
        rv[0] ? qb + (static_cast<size_t>(tok[0]) * p.num_heads + head[0]) * HD : nullptr;
    const uint16_t* q1 =
        rv[1] ? qb + (static_cast<size_t>(tok[1]) * p.num_heads + head[1]) * HD : nullptr;
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      const int c = 16 * s + 2 * q4;
      qa[s][0] = q0 ? *reinterpret_cast<const uint32_t*>(q0 + c) : 0u;
      qa[s][1] = q1 ? *reinterpret_cast<const uint32_t*>(q1 + c) : 0u;
      qa[s][2] = q0 ? *reinterpret_cast<const uint32_t*>(q0 + c + 8) : 0u;
      qa[s][3] = q1 ? *reinterpret_cast<const uint32_t*>(q1 + c + 8) : 0u;
    }
  }

  float o[ON][4];
#pragma unroll
  for (int j = 0; j < ON; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};

  for (int t = tile0; t < tile1; ++t) {
    const int stage = (t - tile0) & 1;
    if (t + 1 < tile1) load_tile(t + 1, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    int end;
    const int start = tile_start(t, end);
    const uint16_t* k_s = sK(stage) + (kw * KC) * PITCH;
    const uint16_t* v_s = sV(stage) + (kw * KC) * PITCH;

    // S = Q K^T over this warp's KC keys
    float s[NB][4];
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
      const uint16_t* kr_row = k_s + (8 * j + g) * PITCH + 2 * q4;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks)
        mma16816<DT>(s[j], qa[ks], lds32(kr_row + 16 * ks), lds32(kr_row + 16 * ks + 8));
    }

    // mask, scale and the online softmax of the two rows
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < NB; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = e >> 1;
        const int pos = start + kw * KC + 8 * j + 2 * q4 + (e & 1);
        const bool ok = rv[i] && pos < end && pos <= ap[i] &&
                        (pos < p.n_sink || pos >= ap[i] + 1 - p.window);
        s[j][e] = ok ? s[j][e] * p.scale : -INFINITY;
        mx[i] = fmaxf(mx[i], s[j][e]);
      }
    float alpha[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
      const float m_new = fmaxf(m_run[i], mx[i]);
      // a row with nothing valid yet keeps m = -inf and adds nothing
      alpha[i] = m_new == -INFINITY ? 1.f : __expf(m_run[i] - m_new);
      mx[i] = m_new == -INFINITY ? 0.f : m_new;
      m_run[i] = m_new;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < NB; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = e >> 1;
        const float v = __expf(s[j][e] - mx[i]);  // exp(-inf) = 0 for masked keys
        s[j][e] = v;
        rs[i] += v;
      }
#pragma unroll
    for (int i = 0; i < 2; ++i) l_run[i] = l_run[i] * alpha[i] + rs[i];
#pragma unroll
    for (int j = 0; j < ON; ++j) {
      o[j][0] *= alpha[0];
      o[j][1] *= alpha[0];
      o[j][2] *= alpha[1];
      o[j][3] *= alpha[1];
    }

    // O += P V: the S accumulators of n-blocks 2u, 2u+1 are the A fragment of
    // k-step u; V's B fragments come transposed from shared memory.
#pragma unroll
    for (int u = 0; u < KC / 16; ++u) {
      uint32_t pa[4];
      pa[0] = E::pack2(s[2 * u][0], s[2 * u][1]);
      pa[1] = E::pack2(s[2 * u][2], s[2 * u][3]);
      pa[2] = E::pack2(s[2 * u + 1][0], s[2 * u + 1][1]);
      pa[3] = E::pack2(s[2 * u + 1][2], s[2 * u + 1][3]);
      const int mi = lane >> 3;
      const uint16_t* vrow = v_s + (16 * u + (mi & 1) * 8 + (lane & 7)) * PITCH + (mi >> 1) * 8;
#pragma unroll
      for (int jp = 0; jp < ON / 2; ++jp) {
        uint32_t b[4];
        ldmatrix_x4_trans(b, vrow + 16 * jp);
        mma16816<DT>(o[2 * jp], pa, b[0], b[1]);
        mma16816<DT>(o[2 * jp + 1], pa, b[2], b[3]);
      }
    }
    __syncthreads();  // this stage is refilled by the next iteration's load
  }
  cp_async_wait<0>();
  __syncthreads();

  // Partials of every warp into shared memory (the stages are free now).
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    l_run[i] += __shfl_xor_sync(0xffffffffu, l_run[i], 1);
    l_run[i] += __shfl_xor_sync(0xffffffffu, l_run[i], 2);
  }
  float* s_o = reinterpret_cast<float*>(attn_smem);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int r = kw * R + rw * 16 + g + 8 * i;
#pragma unroll
    for (int j = 0; j < ON; ++j)
      *reinterpret_cast<float2*>(s_o + r * OP + 8 * j + 2 * q4) =
          make_float2(o[j][2 * i], o[j][2 * i + 1]);
    if (q4 == 0) {
      s_m[r] = m_run[i];
      s_l[r] = l_run[i];
    }
  }
  __syncthreads();

  // Merge the KW partials of each row; write the row (one split) or this
  // split's partial.
  const int rows_total = p.batch * p.seq_len * p.num_heads;
  for (int idx = tid; idx < R * (HD / 2); idx += kAttnThreads) {
    const int r = idx / (HD / 2), d = (idx % (HD / 2)) * 2;
    const int tr = r / p.hpb, hr = hs * p.hpb + r % p.hpb;
    const int tk = t_lo + tr;
    if (!(tr < p.tpb && tk < p.seq_len && hr < p.group)) continue;
    const int orow = static_cast<int>(row_base) + tk * p.num_heads + kvh * p.group + hr;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < KW; ++w) m = fmaxf(m, s_m[w * R + r]);
    float l = 0.f, ox = 0.f, oy = 0.f;
#pragma unroll
    for (int w = 0; w < KW; ++w) {
      const float mw = s_m[w * R + r];
      const float f = mw == -INFINITY ? 0.f : __expf(mw - m);
      l += f * s_l[w * R + r];
      const float2 v = *reinterpret_cast<const float2*>(s_o + (w * R + r) * OP + d);
      ox += f * v.x;
      oy += f * v.y;
    }
    if (p.splits == 1) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      *reinterpret_cast<uint32_t*>(static_cast<uint16_t*>(p.out) +
                                   static_cast<size_t>(orow) * HD + d) =
          E::pack2(ox * inv, oy * inv);
    } else {
      const size_t prow = static_cast<size_t>(blockIdx.z) * rows_total + orow;
      *reinterpret_cast<float2*>(p.ws + prow * HD + d) = make_float2(ox, oy);
      if (d == 0) {
        float* ml = p.ws + static_cast<size_t>(p.splits) * rows_total * HD + prow * 2;
        ml[0] = m;
        ml[1] = l;
      }
    }
  }
  if (p.splits == 1 || !p.merge_here) return;
  // The last split CTA of this row block to arrive merges the splits.  Its
  // partials are fenced before the arrival; the other splits' are read
  // through L2 after it (threadfence, atomic, threadfence).
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    int* cnt = p.counters + blockIdx.y * gridDim.x + blockIdx.x;
    const int last = atomicAdd(cnt, 1) == p.splits - 1;
    if (last) *cnt = 0;  // every split has arrived: zero for the next call
    s_last = last;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = tid; idx < R * (HD / 4); idx += kAttnThreads) {
    const int r = idx / (HD / 4), d = (idx % (HD / 4)) * 4;
    const int tr = r / p.hpb, hr = hs * p.hpb + r % p.hpb;
    const int tk = t_lo + tr;
    if (!(tr < p.tpb && tk < p.seq_len && hr < p.group)) continue;
    const int orow = static_cast<int>(row_base) + tk * p.num_heads + kvh * p.group + hr;
    merge_splits<DT, HD>(p.out, p.ws, rows_total, p.splits, orow, d);
  }
}

// The split partials of prefill row blocks merged, one thread per 4 output
// dims of a row.
template <int DT, int HD>
__global__ void __launch_bounds__(128)
    attn_combine_kernel(void* out, const float* ws, int rows_total, int splits) {
  pdl_wait();
  pdl_launch_dependents();
  const long long idx = static_cast<long long>(blockIdx.x) * 128 + threadIdx.x;
  if (idx >= static_cast<long long>(rows_total) * (HD / 4)) return;
  merge_splits<DT, HD>(out, ws, rows_total, splits, static_cast<int>(idx / (HD / 4)),
                       static_cast<int>(idx % (HD / 4)) * 4);
}

// The call's new K/V rows into their pool slots (src/kv_cache.cu:21-41).  When
// more than W window positions land in one call, two tokens share a slot; the
// later token is the one kept (what a sequential append leaves), so the
// earlier one is skipped.  One CTA per token, 16-byte copies when the rows
// allow them.
__global__ void __launch_bounds__(128)
    kv_scatter_kernel(uint16_t* k_pool, uint16_t* v_pool, const uint16_t* k_src,
                      const uint16_t* v_src, int seq_len, int start_pos, int n_sink, int window,
                      int kv_dim, int vec) {
  pdl_wait();
  const int t = blockIdx.x;
  const int pos = start_pos + t;
  if (pos >= n_sink && t + window < seq_len) return;  // a later token owns the slot
  const size_t dst = static_cast<size_t>(ring_slot(pos, n_sink, window)) * kv_dim;
  const size_t src = static_cast<size_t>(t) * kv_dim;
  if (vec) {
    for (int c = threadIdx.x; c < kv_dim / 8; c += blockDim.x) {
      reinterpret_cast<uint4*>(k_pool + dst)[c] = reinterpret_cast<const uint4*>(k_src + src)[c];
      reinterpret_cast<uint4*>(v_pool + dst)[c] = reinterpret_cast<const uint4*>(v_src + src)[c];
    }
  } else {
    for (int c = threadIdx.x; c < kv_dim; c += blockDim.x) {
      k_pool[dst + c] = k_src[src + c];
      v_pool[dst + c] = v_src[src + c];
    }
  }
  pdl_launch_dependents();
}

template <int DT, int HD, int RW>
cudaError_t launch_attn_kernel(const AttnParams& p, int row_blocks, cudaStream_t s) {
  auto kern = attn_kernel<DT, HD, RW>;
  constexpr int smem = attn_smem_bytes<HD>();
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  return launch_pdl_smem(kern, dim3(row_blocks, p.num_kv_heads * p.batch, p.splits),
                         dim3(kAttnThreads), smem, s, p);
}

template <int DT, int HD>
cudaError_t attn_dispatch(const AttnParams& p, int rw, int row_blocks, cudaStream_t s) {
  cudaError_t e = rw == 1 ? launch_attn_kernel<DT, HD, 1>(p, row_blocks, s)
                          : launch_attn_kernel<DT, HD, 4>(p, row_blocks, s);
  if (e != cudaSuccess || p.splits == 1 || p.merge_here) return e;
  const int rows_total = p.batch * p.seq_len * p.num_heads;
  const long long items = static_cast<long long>(rows_total) * (HD / 4);
  return launch_pdl_smem(attn_combine_kernel<DT, HD>, dim3(static_cast<unsigned>((items + 127) / 128)),
                         dim3(128), 0, s, p.out, static_cast<const float*>(p.ws), rows_total,
                         p.splits);
}

}  // namespace

namespace {

// ORIN_ATTN_SPLITS: tuning override, the most key splits a decode row block
// takes (read once per process; 0 or unset: the planner's choice).
int attention_split_cap() {
  static const int v = [] {
    const char* e = std::getenv("ORIN_ATTN_SPLITS");
    const int n = e ? std::atoi(e) : 0;
    return n > 0 ? n : 0;
  }();
  return v;
}

}  // namespace

AttnPlan plan_attention(int seq_len, int cache_len, int num_heads, int num_kv_heads,
                        int head_dim, int n_sink, int window, size_t workspace_bytes) {
  AttnPlan pl = {};
  const int group = num_heads / num_kv_heads;
  pl.rw = static_cast<long long>(seq_len) * group <= 32 ? 1 : 4;
  const int rows = 16 * pl.rw;
  pl.hpb = group < rows ? group : rows;
  pl.tpb = rows / pl.hpb;
  pl.hsb = (group + pl.hpb - 1) / pl.hpb;
  const long long token_blocks = (seq_len + pl.tpb - 1) / pl.tpb;
  pl.row_blocks = token_blocks * pl.hsb;
  // Split the keys across CTAs only when the row blocks leave SMs idle
  // (aiming at two CTAs per SM of a B200's 148).
  constexpr int kSMs = 148;
  const long long ctas = pl.row_blocks * num_kv_heads;
  int splits = 1;
  if (ctas < kSMs) {
    // key tiles of the row block with the most keys (the last one)
    const int last_lo = static_cast<int>((token_blocks - 1) * pl.tpb);
    const int base = cache_len - seq_len;
    const KeyRanges kr = key_ranges(base + last_lo, cache_len - 1, n_sink, window);
    long long want = (2 * kSMs + ctas - 1) / ctas;
    if (want > kr.tiles) want = kr.tiles;
    if (want > 256) want = 256;
    if (pl.rw == 1 && attention_split_cap() > 0 && want > attention_split_cap())
      want = attention_split_cap();
    splits = want < 1 ? 1 : static_cast<int>(want);
    const size_t per_split =
        static_cast<size_t>(seq_len) * num_heads * (head_dim + 2) * sizeof(float);
    while (splits > 1 &&
           (workspace_bytes < kAttnCounterBytes ||
            static_cast<size_t>(splits) * per_split > workspace_bytes - kAttnCounterBytes))
      --splits;
    // one arrival counter per CTA row of the grid
    if (ctas > kAttnCounterBytes / static_cast<long long>(sizeof(int))) splits = 1;
  }
  pl.splits = splits;
  pl.workspace_bytes = splits > 1 ? kAttnCounterBytes + static_cast<size_t>(splits) * seq_len *
                                                            num_heads * (head_dim + 2) *
                                                            sizeof(float)
                                  : 0;
  return pl;
}

namespace {

// ORIN_ATTN_KERNEL: 0 automatic, 1 "mma" (the mma.sync kernel), 2 "tc" (the
// tensor-core kernel wherever it applies), 3 "tc1" / 4 "tc2" (the tensor-core
// kernel with one / two query tiles per CTA; two needs head dim 64).
int attention_kernel_override() {
  static const int v = [] {
    const char* e = std::getenv("ORIN_ATTN_KERNEL");
    if (!e) return 0;
    if (std::strcmp(e, "mma") == 0) return 1;
    if (std::strcmp(e, "tc") == 0) return 2;
    if (std::strcmp(e, "tc1") == 0) return 3;
    if (std::strcmp(e, "tc2") == 0) return 4;
    return 0;
  }();
  return v;
}

}  // namespace

cudaError_t launch_attention(void* out, const void* q, const void* k_pool, const void* v_pool,
                             int seq_len, int cache_len, int num_heads, int num_kv_heads,
                             int head_dim, float scale, int n_sink, int window, int dtype,
                             void* workspace, size_t workspace_bytes, cudaStream_t s, int batch,
                             long long pool_stride, int* err, int flags) {
  if (seq_len <= 0 || batch <= 0) return cudaSuccess;
  if (batch == 1 && attention_tc_supported(seq_len, num_heads, num_kv_heads, head_dim, n_sink,
                                           window)) {
    // the tensor-core kernel has no key split, so it wants some row blocks:
    // measured on B200 with 1028 cached keys and more, it is ahead from 32
    // CTAs of 128 rows (128 tokens x 32/4 heads: 18.0 us against 21.6 for
    // the split-key kernel) and level at 16 (17.6 against 17.0)
    const int ov = attention_kernel_override();
    const int group = num_heads / num_kv_heads;
    const long long rows = static_cast<long long>(seq_len) * group;
    const long long ctas = (rows + 127) / 128 * num_kv_heads;
    if (ov >= 2 || (ov == 0 && ctas >= 32))
      return launch_attention_tc(out, q, k_pool, v_pool, seq_len, cache_len, num_heads,
                                 num_kv_heads, head_dim, scale, n_sink, window, dtype, err, s,
                                 ov >= 3 ? ov - 2 : 0);
  }
  // each sequence plans alone, on its share of the partials' part of the
  // workspace (the arrival counters at its start serve the whole call)
  const size_t share = (workspace && workspace_bytes > kAttnCounterBytes)
                           ? (workspace_bytes - kAttnCounterBytes) / batch + kAttnCounterBytes
                           : 0;
  AttnPlan pl = plan_attention(seq_len, cache_len, num_heads, num_kv_heads, head_dim, n_sink,
                               window, share);
  if (pl.row_blocks * num_kv_heads * batch > kAttnCounterBytes / static_cast<long long>(sizeof(int)))
    pl.splits = 1;
  if (pl.row_blocks > 0x7fffffffLL || static_cast<long long>(num_kv_heads) * batch > 65535 ||
      static_cast<long long>(batch) * seq_len * num_heads > 0x7fffffffLL)
    return cudaErrorInvalidConfiguration;
  AttnParams p;
  p.out = out;
  p.q = q;
  p.k_pool = k_pool;
  p.v_pool = v_pool;
  p.counters = static_cast<int*>(workspace);
  p.ws = workspace ? reinterpret_cast<float*>(static_cast<char*>(workspace) + kAttnCounterBytes)
                   : nullptr;
  p.seq_len = seq_len;
  p.cache_len = cache_len;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.n_sink = n_sink;
  p.window = window;
  p.scale = scale;
  p.group = num_heads / num_kv_heads;
  p.hpb = pl.hpb;
  p.tpb = pl.tpb;
  p.hsb = pl.hsb;
  p.splits = pl.splits;
  // decode row blocks merge in the kernel; prefill row blocks in a combine
  // launch (64 rows x 10 splits on one CTA: 32.3 us against 17.0 for the
  // 64 x 2048-token call of 32/4 heads of 64)
  p.merge_here = pl.rw == 1 ? 1 : 0;
  p.own_slots_only = (flags & kAttnOwnSlotsOnly) ? 1 : 0;
  p.batch = batch;
  p.pool_stride = pool_stride;
  const int rb = static_cast<int>(pl.row_blocks);
  if (dtype == DT_F16)
    return head_dim == 64 ? attn_dispatch<DT_F16, 64>(p, pl.rw, rb, s)
                          : attn_dispatch<DT_F16, 128>(p, pl.rw, rb, s);
  return head_dim == 64 ? attn_dispatch<DT_BF16, 64>(p, pl.rw, rb, s)
                        : attn_dispatch<DT_BF16, 128>(p, pl.rw, rb, s);
}

cudaError_t launch_kv_scatter(void* k_pool, void* v_pool, const void* k_src, const void* v_src,
                              int seq_len, int start_pos, int n_sink, int window, int kv_dim,
                              cudaStream_t s) {
  if (seq_len <= 0) return cudaSuccess;
  const bool vec = kv_dim % 8 == 0 &&
                   ((reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool) |
                     reinterpret_cast<uintptr_t>(k_src) | reinterpret_cast<uintptr_t>(v_src)) &
                    15) == 0;
  return launch_pdl_smem(kv_scatter_kernel, dim3(seq_len), dim3(128), 0, s,
                         static_cast<uint16_t*>(k_pool), static_cast<uint16_t*>(v_pool),
                         static_cast<const uint16_t*>(k_src), static_cast<const uint16_t*>(v_src),
                         seq_len, start_pos, n_sink, window, kv_dim, vec ? 1 : 0);
}

}  // namespace orin
