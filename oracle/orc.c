/*
 * orc.c — CPU oracle for the linear-layer hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the test-suite, the
 * smoke check and the bench's CPU-baseline leg compare the CUDA kernels
 * against; no product code path links or calls it.
 *
 * It restates, in plain C, the arithmetic of the reference's GEMM path:
 *   kernels/matmul.cu:25-44   gemv_kernel: C[n] = bf16(sum_k f32(A[k])*f32(B[n,k]))
 *   kernels/matmul.cu:59-68   cublasGemmEx, 16-bit in/out, CUBLAS_COMPUTE_32F
 *   kernels/gemm_cute.cu:147,176-178  fp32 accumulator, one rounding to 16 bits
 *   kernels/fused_swiglu.cu:11-15     out = bf16(g/(1+expf(-g)) * u), fp32 math
 *   kernels/softmax.cu:81             x = bf16(f32(x) + f32(y))
 *   kernels/softmax.cu:89             out = f32(in)
 *   src/model.cu:98-110,125-130       where the model rounds between those steps
 * for both 16-bit types (fp16 and bf16; the reference itself is bf16-only).
 *
 * Parity pin: tests/golden/ holds outputs of the reference's own kernels
 * (compiled from its sources by oracle/Makefile and run on a B200) for seeded
 * inputs; tests/test_oracle.py checks this file against them.
 *
 * Accumulation is fp32, like the reference; the summation order is a fixed
 * 8-lane strided order (lane j sums k = j mod 8, then a pairwise tree), which
 * mirrors the reference GEMV's thread-strided partial sums + tree reduction.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { ORC_F16 = 0, ORC_BF16 = 1 };
enum { ORC_EPI_NONE = 0, ORC_EPI_SWIGLU = 1, ORC_EPI_RESIDUAL = 2, ORC_EPI_F32_OUT = 3,
       ORC_EPI_F32_PARTIAL = 4 };

/* ---------------------------------------------------------------- 16-bit <-> f32 */

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Round to nearest even (what __float2bfloat16 does); NaN stays NaN. */
static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

static inline float f16_to_f32(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

/* IEEE binary16 round-to-nearest-even (what __float2half_rn does). */
static inline uint16_t f32_to_f16(float f) {
    _Float16 v = (_Float16)f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

static inline float to_f(uint16_t h, int dt) { return dt == ORC_F16 ? f16_to_f32(h) : bf16_to_f32(h); }
static inline uint16_t from_f(float f, int dt) { return dt == ORC_F16 ? f32_to_f16(f) : f32_to_bf16(f); }
static inline float round16(float f, int dt) { return to_f(from_f(f, dt), dt); }

void orc_widen(const uint16_t* in, float* out, long long n, int dt) {
    for (long long i = 0; i < n; ++i) out[i] = to_f(in[i], dt);
}

void orc_round(const float* in, uint16_t* out, long long n, int dt) {
    for (long long i = 0; i < n; ++i) out[i] = from_f(in[i], dt);
}

/* ---------------------------------------------------------------- fp32 GEMM */

typedef float v8 __attribute__((vector_size(32)));

static inline float hsum8(v8 v) {
    /* pairwise tree over the 8 lanes: ((0+4)+(2+6)) + ((1+5)+(3+7)) */
    float a0 = v[0] + v[4], a1 = v[1] + v[5], a2 = v[2] + v[6], a3 = v[3] + v[7];
    return (a0 + a2) + (a1 + a3);
}

static inline v8 load8(const float* p) {
    v8 v;
    memcpy(&v, p, sizeof(v));
    return v;
}

/* C[m][n] = sum_k A[m][k] * W[n][k] for a 4 x 2 block, fp32. */
__attribute__((target_clones("avx512f", "avx2", "default")))
static void micro_4x2(const float* A, const float* W, float* C, int M, int N, int K,
                      int m0, int n0) {
    const int mr = (M - m0) < 4 ? (M - m0) : 4;
    const int nr = (N - n0) < 2 ? (N - n0) : 2;
    const float* a[4];
    const float* w[2];
    for (int i = 0; i < 4; ++i) a[i] = A + (size_t)(m0 + (i < mr ? i : 0)) * K;
    for (int j = 0; j < 2; ++j) w[j] = W + (size_t)(n0 + (j < nr ? j : 0)) * K;
    v8 acc[4][2];
    for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 2; ++j) acc[i][j] = (v8){0, 0, 0, 0, 0, 0, 0, 0};
    int k = 0;
    for (; k + 8 <= K; k += 8) {
        const v8 w0 = load8(w[0] + k), w1 = load8(w[1] + k);
        for (int i = 0; i < 4; ++i) {
            const v8 av = load8(a[i] + k);
            acc[i][0] += av * w0;
            acc[i][1] += av * w1;
        }
    }
    for (int i = 0; i < mr; ++i)
        for (int j = 0; j < nr; ++j) {
            v8 t = acc[i][j];
            /* K tail continues the same lane assignment (k mod 8) */
            for (int kk = k; kk < K; ++kk) t[kk - k] += a[i][kk] * w[j][kk];
            C[(size_t)(m0 + i) * N + n0 + j] = hsum8(t);
        }
}

/* Multithreaded fp32 GEMM, C[M,N] = A[M,K] . W[N,K]^T.  threads <= 0: all. */
void orc_gemm_f32(const float* A, const float* W, float* C, int M, int N, int K, int threads) {
    const int nb = (N + 7) / 8;  /* 8 weight rows per task: they stay in L1/L2 */
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
#endif
    for (int b = 0; b < nb; ++b) {
        const int n_lo = b * 8;
        const int n_hi = (n_lo + 8 < N) ? n_lo + 8 : N;
        for (int m0 = 0; m0 < M; m0 += 4)
            for (int n0 = n_lo; n0 < n_hi; n0 += 2) micro_4x2(A, W, C, M, N, K, m0, n0);
    }
}

/* ---------------------------------------------------------------- linear layer */

static inline float silu(float g) { return g / (1.0f + expf(-g)); }

/*
 * C = epilogue(A . W^T) with the reference's rounding points.
 *   NONE      C16 = round16(acc)
 *   SWIGLU    W is [2N,K] packed in 64-row gate/up groups; C16[M,N] =
 *             round16(silu(round16(g)) * round16(u))
 *   RESIDUAL  C16 = round16(R + round16(acc))
 *   F32_OUT   C32 = round16(acc) widened
 *   F32_PARTIAL C32 = acc
 */
int orc_linear(void* C, const uint16_t* A, const uint16_t* W, int M, int N, int K, int dt, int epi,
               const uint16_t* R, int threads) {
    const int wrows = (epi == ORC_EPI_SWIGLU) ? 2 * N : N;
    float* a = (float*)malloc(sizeof(float) * (size_t)M * K);
    float* w = (float*)malloc(sizeof(float) * (size_t)wrows * K);
    float* acc = (float*)malloc(sizeof(float) * (size_t)M * wrows);
    if (!a || !w || !acc) {
        free(a); free(w); free(acc);
        return -1;
    }
    orc_widen(A, a, (long long)M * K, dt);
    orc_widen(W, w, (long long)wrows * K, dt);
    orc_gemm_f32(a, w, acc, M, wrows, K, threads);
    for (int m = 0; m < M; ++m) {
        for (int n = 0; n < N; ++n) {
            const size_t o = (size_t)m * N + n;
            if (epi == ORC_EPI_SWIGLU) {
                const int gr = (n / 64) * 128 + (n % 64);
                const float g = round16(acc[(size_t)m * wrows + gr], dt);
                const float u = round16(acc[(size_t)m * wrows + gr + 64], dt);
                ((uint16_t*)C)[o] = from_f(silu(g) * u, dt);
            } else {
                const float v = acc[(size_t)m * wrows + n];
                switch (epi) {
                    case ORC_EPI_NONE: ((uint16_t*)C)[o] = from_f(v, dt); break;
                    case ORC_EPI_RESIDUAL:
                        ((uint16_t*)C)[o] = from_f(to_f(R[o], dt) + round16(v, dt), dt);
                        break;
                    case ORC_EPI_F32_OUT: ((float*)C)[o] = round16(v, dt); break;
                    default: ((float*)C)[o] = v; break;
                }
            }
        }
    }
    free(a); free(w); free(acc);
    return 0;
}

/*
 * The reference's decode GEMV in its exact summation order
 * (kernels/matmul.cu:25-44, launched at :49-51 with T = min(K, 256) threads):
 * thread t accumulates k = t, t+T, ... with fused multiply-adds, then
 * for (s = T/2; s > 0; s >>= 1) sdata[t] += sdata[t+s] for t < s.
 * When T is not a power of two that tree never adds some partial sums
 * (e.g. T = 200 loses sdata[24] at s = 12); this restatement keeps that
 * behaviour so it can be compared bit-for-bit with the reference's output.
 * The product kernels compute the full sum instead.
 */
void orc_gemv_reference_order(uint16_t* C, const uint16_t* A, const uint16_t* B, int N, int K,
                              int dt) {
    const int T = K < 256 ? K : 256;
    float* sd = (float*)malloc(sizeof(float) * (size_t)T);
    if (!sd) return;
    for (int n = 0; n < N; ++n) {
        const uint16_t* b = B + (size_t)n * K;
        for (int t = 0; t < T; ++t) {
            float sum = 0.0f;
            for (int k = t; k < K; k += T) sum = fmaf(to_f(A[k], dt), to_f(b[k], dt), sum);
            sd[t] = sum;
        }
        for (int st = T / 2; st > 0; st >>= 1)
            for (int t = 0; t < st; ++t) sd[t] += sd[t + st];
        C[n] = from_f(sd[0], dt);
    }
    free(sd);
}

/* kernels/fused_swiglu.cu:11-15 */
void orc_silu_mul(uint16_t* out, const uint16_t* g, const uint16_t* u, long long n, int dt) {
    for (long long i = 0; i < n; ++i) out[i] = from_f(silu(to_f(g[i], dt)) * to_f(u[i], dt), dt);
}

/* kernels/softmax.cu:78-83 */
void orc_add(uint16_t* x, const uint16_t* y, long long n, int dt) {
    for (long long i = 0; i < n; ++i) x[i] = from_f(to_f(x[i], dt) + to_f(y[i], dt), dt);
}

/* Packed gate/up layout the fused SwiGLU reads (64-row groups). */
void orc_pack_gate_up(uint16_t* wp, const uint16_t* wg, const uint16_t* wu, int IM, int K) {
    for (long long r = 0; r < 2LL * IM; ++r) {
        const long long g = r / 128, h = r % 128;
        const uint16_t* src = (h < 64 ? wg : wu) + (g * 64 + (h % 64)) * (long long)K;
        memcpy(wp + r * K, src, sizeof(uint16_t) * (size_t)K);
    }
}

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
