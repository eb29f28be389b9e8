// norm_rope.cu — the elementwise steps around the projections:
//   * the embedding row gather (kernels/embedding.cu:4-21);
//   * RMSNorm over rows (kernels/rmsnorm.cu:7-34): out = round16(x * r * w),
//     r = rsqrtf(sum(x^2) / dim + eps), fp32;
//   * rotary embedding, rotate-half pairs (i, i + head_dim/2) of every head
//     (kernels/rope.cu:7-37): angle = pos * powf(theta, -2 i / head_dim),
//     x0' = x0 cos - x1 sin, x1' = x0 sin + x1 cos, each rounded to 16 bits;
//   * the fused step this library runs after its single q/k/v projection
//     (token rows [q | k | v]): the optional per-head q/k RMSNorm of Qwen3
//     (src/model.cu:64-67), the rotation, q into its own buffer
//     [seq, heads, head_dim] and k/v into their ring slots
//     (src/kv_cache.cu:21-41) — five reference launches in one, with the same
//     rounding points.
#include "orin_common.cuh"
#include "orin_internal.h"

namespace orin {

namespace {

constexpr int kNormThreads = 256;

template <int DT>
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_kernel(typename Elem<DT>::T* out, const typename Elem<DT>::T* x,
                   const typename Elem<DT>::T* w, int dim, float eps, int vec) {
  using E = Elem<DT>;
  using T = typename E::T;
  // The next kernel may be scheduled at once (it waits for this grid's end
  // before reading the output) and start streaming its weights; the norm
  // weight does not depend on the previous kernel either, so each thread's
  // first two vectors of it come in before the wait.
  pdl_launch_dependents();
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
  uint4 w_early[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
  if (vec) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int c = threadIdx.x + k * kNormThreads;
      if (c < dim / 8) w_early[k] = w4[c];
    }
  }
  pdl_wait();
  const size_t row = blockIdx.x;
  const T* xr = x + row * dim;
  T* orow = out + row * dim;
  __shared__ float red[kNormThreads / 32];
  float ss = 0.f;
  if (vec) {
    for (int c = threadIdx.x; c < dim / 8; c += kNormThreads) {
      const uint4 u = reinterpret_cast<const uint4*>(xr)[c];
      const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = E::unpack2(wd[i]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
  } else {
    for (int i = threadIdx.x; i < dim; i += kNormThreads) {
      const float v = E::to_f(xr[i]);
      ss += v * v;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float r = rsqrtf(tot / static_cast<float>(dim) + eps);
  if (vec) {
    for (int c = threadIdx.x, k = 0; c < dim / 8; c += kNormThreads, ++k) {
      const uint4 u = reinterpret_cast<const uint4*>(xr)[c];
      const uint4 g = k == 0 ? w_early[0] : k == 1 ? w_early[1] : w4[c];
      const uint32_t xd[4] = {u.x, u.y, u.z, u.w};
      const uint32_t wd[4] = {g.x, g.y, g.z, g.w};
      uint32_t od[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = E::unpack2(xd[i]);
        const float2 b = E::unpack2(wd[i]);
        od[i] = E::pack2(a.x * r * b.x, a.y * r * b.y);
      }
      reinterpret_cast<uint4*>(orow)[c] = make_uint4(od[0], od[1], od[2], od[3]);
    }
  } else {
    for (int i = threadIdx.x; i < dim; i += kNormThreads)
      orow[i] = E::from_f(E::to_f(xr[i]) * r * E::to_f(w[i]));
  }
}

// out[t] = table[ids[t]] (one CTA per token, 16-byte copies when rows allow);
// an id outside [0, vocab) gives a zero row.
__global__ void __launch_bounds__(256)
    embedding_kernel(uint16_t* out, const uint16_t* table, const int32_t* ids, int hidden,
                     int vocab, int vec) {
  pdl_launch_dependents();  // the next kernel waits for this grid's end anyway
  pdl_wait();
  const int t = blockIdx.x;
  const int id = ids[t];
  const bool ok = id >= 0 && id < vocab;
  uint16_t* dst = out + static_cast<size_t>(t) * hidden;
  const uint16_t* src = table + static_cast<size_t>(ok ? id : 0) * hidden;
  if (vec) {
    for (int c = threadIdx.x; c < hidden / 8; c += blockDim.x)
      reinterpret_cast<uint4*>(dst)[c] =
          ok ? reinterpret_cast<const uint4*>(src)[c] : make_uint4(0, 0, 0, 0);
  } else {
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) dst[c] = ok ? src[c] : 0;
  }
  pdl_launch_dependents();
}

// One thread per (token, head, pair) of q and then k, in place.
template <int DT>
__global__ void __launch_bounds__(256)
    rope_kernel(typename Elem<DT>::T* q, typename Elem<DT>::T* k, int seq_len, int num_heads,
                int num_kv_heads, int head_dim, int start_pos, float theta) {
  using E = Elem<DT>;
  pdl_wait();
  const int half = head_dim >> 1;
  const long long nq = static_cast<long long>(seq_len) * num_heads * half;
  const long long nk = static_cast<long long>(seq_len) * num_kv_heads * half;
  long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= nq + nk) return;
  typename Elem<DT>::T* base = q;
  int heads = num_heads;
  if (t >= nq) {
    t -= nq;
    base = k;
    heads = num_kv_heads;
  }
  const int i = static_cast<int>(t % half);
  const long long hs = t / half;  // token * heads + head
  const int tok = static_cast<int>(hs / heads);
  float c, s;
  rope_angle(start_pos + tok, i, head_dim, theta, c, s);
  typename Elem<DT>::T* v = base + hs * head_dim;
  const float x0 = E::to_f(v[i]), x1 = E::to_f(v[i + half]);
  v[i] = E::from_f(x0 * c - x1 * s);
  v[i + half] = E::from_f(x0 * s + x1 * c);
}

// One warp per (token, head slot): slots [0, H) are q heads, [H, H + KV) k
// heads, [H + KV, H + 2 KV) v heads of the token's row [q | k | v].  Lane l
// holds pairs l, l + 32, ... (head_dim / 64 of them).
template <int DT, int HD>
__global__ void __launch_bounds__(256)
    qkv_rope_append_kernel(typename Elem<DT>::T* q_out, const typename Elem<DT>::T* qkv,
                           const typename Elem<DT>::T* q_norm, const typename Elem<DT>::T* k_norm,
                           typename Elem<DT>::T* k_pool, typename Elem<DT>::T* v_pool,
                           int seq_len, int start_pos, int num_heads, int num_kv_heads, float eps,
                           float theta, int n_sink, int window, int batch,
                           long long pool_stride) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int HALF = HD / 2;
  constexpr int PL = HALF / 32;  // pairs per lane
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int slots = num_heads + 2 * num_kv_heads;
  if (wid >= static_cast<long long>(batch) * seq_len * slots) return;
  // row tg of the call = token tok of sequence b (sequences one after another)
  const long long tg = wid / slots;
  const int b = static_cast<int>(tg / seq_len);
  const int tok = static_cast<int>(tg - static_cast<long long>(b) * seq_len);
  const int slot = static_cast<int>(wid % slots);
  const int pos = start_pos + tok;
  k_pool += b * pool_stride;
  v_pool += b * pool_stride;
  // a later token of this call that lands in the same ring slot owns it
  const bool pool_owner = !(pos >= n_sink && tok + window < seq_len);
  const T* src = qkv + static_cast<size_t>(tg) * slots * HD + static_cast<size_t>(slot) * HD;
  const size_t kv_dim = static_cast<size_t>(num_kv_heads) * HD;
  const size_t ring = static_cast<size_t>(pos < n_sink ? pos : n_sink + (pos - n_sink) % window);

  if (slot >= num_heads + num_kv_heads) {  // v: straight into the pool
    if (!pool_owner) return;
    const int h = slot - num_heads - num_kv_heads;
    T* dst = v_pool + ring * kv_dim + static_cast<size_t>(h) * HD;
#pragma unroll
    for (int j = 0; j < PL; ++j) {
      dst[lane + 32 * j] = src[lane + 32 * j];
      dst[lane + 32 * j + HALF] = src[lane + 32 * j + HALF];
    }
    return;
  }
  const bool is_q = slot < num_heads;
  float x0[PL], x1[PL];
#pragma unroll
  for (int j = 0; j < PL; ++j) {
    x0[j] = E::to_f(src[lane + 32 * j]);
    x1[j] = E::to_f(src[lane + 32 * j + HALF]);
  }
  const T* nw = is_q ? q_norm : k_norm;
  if (nw) {  // per-head RMSNorm, rounded to 16 bits as its own kernel would
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PL; ++j) ss += x0[j] * x0[j] + x1[j] * x1[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / static_cast<float>(HD) + eps);
#pragma unroll
    for (int j = 0; j < PL; ++j) {
      x0[j] = E::round(x0[j] * r * E::to_f(nw[lane + 32 * j]));
      x1[j] = E::round(x1[j] * r * E::to_f(nw[lane + 32 * j + HALF]));
    }
  }
  T* dst;
  if (is_q) {
    dst = q_out + (static_cast<size_t>(tg) * num_heads + slot) * HD;
  } else {
    if (!pool_owner) return;
    dst = k_pool + ring * kv_dim + static_cast<size_t>(slot - num_heads) * HD;
  }
#pragma unroll
  for (int j = 0; j < PL; ++j) {
    const int i = lane + 32 * j;
    float c, s;
    rope_angle(pos, i, HD, theta, c, s);
    dst[i] = E::from_f(x0[j] * c - x1[j] * s);
    dst[i + HALF] = E::from_f(x0[j] * s + x1[j] * c);
  }
}

template <int DT>
cudaError_t rmsnorm_t(void* out, const void* x, const void* w, int rows, int dim, float eps,
                      cudaStream_t s) {
  using T = typename Elem<DT>::T;
  const bool vec = dim % 8 == 0 &&
                   ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(x) |
                     reinterpret_cast<uintptr_t>(w)) &
                    15) == 0;
  return launch_pdl_smem(rmsnorm_kernel<DT>, dim3(rows), dim3(kNormThreads), 0, s,
                         static_cast<T*>(out), static_cast<const T*>(x),
                         static_cast<const T*>(w), dim, eps, vec ? 1 : 0);
}

template <int DT>
cudaError_t rope_t(void* q, void* k, int seq_len, int num_heads, int num_kv_heads, int head_dim,
                   int start_pos, float theta, cudaStream_t s) {
  using T = typename Elem<DT>::T;
  const long long n =
      static_cast<long long>(seq_len) * (num_heads + num_kv_heads) * (head_dim / 2);
  const long long blocks = (n + 255) / 256;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  return launch_pdl_smem(rope_kernel<DT>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s,
                           static_cast<T*>(q), static_cast<T*>(k), seq_len, num_heads,
                           num_kv_heads, head_dim, start_pos, theta);
}

template <int DT, int HD>
cudaError_t qkv_rope_append_t(void* q_out, const void* qkv, const void* q_norm,
                              const void* k_norm, void* k_pool, void* v_pool, int seq_len,
                              int start_pos, int num_heads, int num_kv_heads, float eps,
                              float theta, int n_sink, int window, int batch,
                              long long pool_stride, cudaStream_t s) {
  using T = typename Elem<DT>::T;
  const long long warps =
      static_cast<long long>(batch) * seq_len * (num_heads + 2 * num_kv_heads);
  const long long blocks = (warps + 7) / 8;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  return launch_pdl_smem(qkv_rope_append_kernel<DT, HD>, dim3(static_cast<unsigned>(blocks)),
                         dim3(256), 0, s, static_cast<T*>(q_out), static_cast<const T*>(qkv),
                         static_cast<const T*>(q_norm), static_cast<const T*>(k_norm),
                         static_cast<T*>(k_pool), static_cast<T*>(v_pool), seq_len, start_pos,
                         num_heads, num_kv_heads, eps, theta, n_sink, window, batch, pool_stride);
}

}  // namespace

cudaError_t launch_embedding(void* out, const void* table, const int* ids, int seq_len,
                             int hidden, int vocab, cudaStream_t s) {
  if (seq_len <= 0) return cudaSuccess;
  const bool vec = hidden % 8 == 0 &&
                   ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(table)) &
                    15) == 0;
  return launch_pdl_smem(embedding_kernel, dim3(seq_len), dim3(256), 0, s,
                           static_cast<uint16_t*>(out), static_cast<const uint16_t*>(table),
                           reinterpret_cast<const int32_t*>(ids), hidden, vocab, vec ? 1 : 0);
}

cudaError_t launch_rmsnorm(void* out, const void* x, const void* w, int rows, int dim, float eps,
                           int dtype, cudaStream_t s) {
  if (rows <= 0) return cudaSuccess;
  return dtype == DT_F16 ? rmsnorm_t<DT_F16>(out, x, w, rows, dim, eps, s)
                         : rmsnorm_t<DT_BF16>(out, x, w, rows, dim, eps, s);
}

cudaError_t launch_rope(void* q, void* k, int seq_len, int num_heads, int num_kv_heads,
                        int head_dim, int start_pos, float theta, int dtype, cudaStream_t s) {
  if (seq_len <= 0) return cudaSuccess;
  return dtype == DT_F16
             ? rope_t<DT_F16>(q, k, seq_len, num_heads, num_kv_heads, head_dim, start_pos, theta, s)
             : rope_t<DT_BF16>(q, k, seq_len, num_heads, num_kv_heads, head_dim, start_pos, theta,
                               s);
}

cudaError_t launch_qkv_rope_append(void* q_out, const void* qkv, const void* q_norm,
                                   const void* k_norm, void* k_pool, void* v_pool, int seq_len,
                                   int start_pos, int num_heads, int num_kv_heads, int head_dim,
                                   float eps, float theta, int n_sink, int window, int dtype,
                                   cudaStream_t s, int batch, long long pool_stride) {
  if (seq_len <= 0 || batch <= 0) return cudaSuccess;
#define ORIN_QKV_ROPE(DTV, HDV)                                                               \
  qkv_rope_append_t<DTV, HDV>(q_out, qkv, q_norm, k_norm, k_pool, v_pool, seq_len, start_pos, \
                              num_heads, num_kv_heads, eps, theta, n_sink, window, batch,      \
                              pool_stride, s)
  if (dtype == DT_F16) return head_dim == 64 ? ORIN_QKV_ROPE(DT_F16, 64) : ORIN_QKV_ROPE(DT_F16, 128);
  return head_dim == 64 ? ORIN_QKV_ROPE(DT_BF16, 64) : ORIN_QKV_ROPE(DT_BF16, 128);
#undef ORIN_QKV_ROPE
}

}  // namespace orin
