// model_step.cpp — the reference's per-token call sequence (Model::forward,
// src/model.cu:20-131: embedding, per layer RMSNorm, q/k/v matmuls, the
// per-head q/k RMSNorm, RoPE, the K/V append, attention, o_proj + add, RMSNorm,
// gate/up matmuls, SwiGLU, down + add, then the final RMSNorm, LM head and
// bf16 -> fp32 logits) written
// against include/orin_kernels.h, the C++ drop-in signatures liborin_b200.so
// exports, plus orin_kv_append for the append KVCache::append_kv does.
//
// Usage: model_step <out.bin>   (writes the fp32 logits of one decode token
// after a 16-token prompt; seeded random bf16 weights, 2 layers, TinyLlama
// widths).  Exit status 0 on success.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <random>
#include <vector>

#include "orin_b200.h"
#include "orin_kernels.h"

namespace {

constexpr int H = 2048, NH = 32, NKV = 4, HD = 64, IM = 5632, V = 32000, LAYERS = 2;
constexpr int QD = NH * HD, KVD = NKV * HD, N_SINK = 4, WINDOW = 60;
constexpr float EPS = 1e-5f, THETA = 10000.f;

#define CHECK(x)                                                              \
  do {                                                                        \
    cudaError_t e_ = (x);                                                     \
    if (e_ != cudaSuccess) {                                                  \
      std::fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));          \
      return 1;                                                               \
    }                                                                         \
  } while (0)

__nv_bfloat16* upload(std::mt19937& g, size_t n, float scale, bool ones = false) {
  std::normal_distribution<float> d(0.f, 1.f);
  std::vector<__nv_bfloat16> h(n);
  for (auto& v : h) v = __float2bfloat16(ones ? 1.f : d(g) * scale);
  __nv_bfloat16* p = nullptr;
  if (cudaMalloc(&p, n * sizeof(__nv_bfloat16)) != cudaSuccess) return nullptr;
  cudaMemcpy(p, h.data(), n * sizeof(__nv_bfloat16), cudaMemcpyHostToDevice);
  return p;
}

struct Layer {
  __nv_bfloat16 *in_norm, *q, *k, *v, *q_norm, *k_norm, *o, *post_norm, *gate, *up, *down,
      *k_pool, *v_pool;
};

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: %s <out.bin>\n", argv[0]);
    return 2;
  }
  std::mt19937 g(1234);
  std::vector<Layer> L(LAYERS);
  for (auto& l : L) {
    l.in_norm = upload(g, H, 0.f, true);
    l.q = upload(g, size_t(QD) * H, 0.02f);
    l.k = upload(g, size_t(KVD) * H, 0.02f);
    l.v = upload(g, size_t(KVD) * H, 0.02f);
    l.q_norm = upload(g, HD, 0.f, true);
    l.k_norm = upload(g, HD, 0.f, true);
    l.o = upload(g, size_t(H) * QD, 0.02f);
    l.post_norm = upload(g, H, 0.f, true);
    l.gate = upload(g, size_t(IM) * H, 0.02f);
    l.up = upload(g, size_t(IM) * H, 0.02f);
    l.down = upload(g, size_t(H) * IM, 0.02f);
    CHECK(cudaMalloc(&l.k_pool, size_t(N_SINK + WINDOW) * KVD * 2));
    CHECK(cudaMalloc(&l.v_pool, size_t(N_SINK + WINDOW) * KVD * 2));
    CHECK(cudaMemset(l.k_pool, 0, size_t(N_SINK + WINDOW) * KVD * 2));
    CHECK(cudaMemset(l.v_pool, 0, size_t(N_SINK + WINDOW) * KVD * 2));
  }
  __nv_bfloat16* embed = upload(g, size_t(V) * H, 0.02f);
  __nv_bfloat16* final_norm = upload(g, H, 0.f, true);
  __nv_bfloat16* lm_head = upload(g, size_t(V) * H, 0.02f);
  const int max_seq = 16;
  __nv_bfloat16 *x, *buf_b, *scratch;
  float* logits;
  int32_t* ids;
  CHECK(cudaMalloc(&x, size_t(max_seq) * H * 2));
  CHECK(cudaMalloc(&buf_b, size_t(max_seq) * H * 2));
  CHECK(cudaMalloc(&scratch, size_t(max_seq) * 2 * IM * 2 + size_t(V) * 2));
  CHECK(cudaMalloc(&logits, size_t(V) * 4));
  CHECK(cudaMalloc(&ids, max_seq * 4));

  int start = 0;
  std::vector<int32_t> prompt(max_seq);
  for (int i = 0; i < max_seq; ++i) prompt[i] = int32_t((i * 7919) % V);
  for (int step = 0; step < 2; ++step) {
    const int seq = step == 0 ? max_seq : 1;
    CHECK(cudaMemcpy(ids, prompt.data(), seq * 4, cudaMemcpyHostToDevice));
    kernels::embedding(x, embed, ids, seq, H);
    for (auto& l : L) {
      __nv_bfloat16* q = scratch;
      __nv_bfloat16* k = scratch + size_t(seq) * QD;
      __nv_bfloat16* v = scratch + size_t(seq) * (QD + KVD);
      kernels::rmsnorm(buf_b, x, l.in_norm, seq, H, EPS);
      kernels::matmul(q, buf_b, l.q, seq, QD, H);
      kernels::matmul(k, buf_b, l.k, seq, KVD, H);
      kernels::matmul(v, buf_b, l.v, seq, KVD, H);
      kernels::rmsnorm(q, q, l.q_norm, seq * NH, HD, EPS);
      kernels::rmsnorm(k, k, l.k_norm, seq * NKV, HD, EPS);
      kernels::rope(q, k, seq, NH, NKV, HD, start, THETA);
      if (orin_kv_append(l.k_pool, l.v_pool, k, v, seq, start, N_SINK, WINDOW, KVD, ORIN_BF16,
                         nullptr) != ORIN_OK)
        return 1;
      kernels::attention(buf_b, q, l.k_pool, l.v_pool, seq, start + seq, NH, NKV, HD,
                         1.0f / std::sqrt(float(HD)), N_SINK, WINDOW);
      kernels::matmul(scratch, buf_b, l.o, seq, H, QD);
      kernels::add(x, scratch, seq * H);
      kernels::rmsnorm(buf_b, x, l.post_norm, seq, H, EPS);
      __nv_bfloat16* gate = scratch;
      __nv_bfloat16* up = scratch + size_t(seq) * IM;
      kernels::matmul(gate, buf_b, l.gate, seq, IM, H);
      kernels::matmul(up, buf_b, l.up, seq, IM, H);
      kernels::fused_silu_mul(gate, gate, up, seq, IM);
      kernels::matmul(buf_b, gate, l.down, seq, H, IM);
      kernels::add(x, buf_b, seq * H);
    }
    kernels::rmsnorm(buf_b, x, final_norm, seq, H, EPS);
    kernels::matmul(scratch, buf_b + size_t(seq - 1) * H, lm_head, 1, V, H);
    kernels::bf16_to_fp32(logits, scratch, V);
    start += seq;
    CHECK(cudaDeviceSynchronize());
    if (orin_device_check(nullptr) != ORIN_OK) return 1;
    // greedy next token, as the reference's sampler picks it
    std::vector<float> h(V);
    CHECK(cudaMemcpy(h.data(), logits, size_t(V) * 4, cudaMemcpyDeviceToHost));
    int best = 0;
    for (int i = 1; i < V; ++i)
      if (h[i] > h[best]) best = i;
    prompt[0] = best;
  }
  std::vector<float> h(V);
  CHECK(cudaMemcpy(h.data(), logits, size_t(V) * 4, cudaMemcpyDeviceToHost));
  FILE* f = std::fopen(argv[1], "wb");
  if (!f) return 1;
  std::fwrite(h.data(), 4, V, f);
  std::fclose(f);
  return 0;
}
