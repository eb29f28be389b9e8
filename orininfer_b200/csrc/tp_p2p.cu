// tp_p2p.cu — the row-parallel reduction over NVLink peer memory.
//
// Replaces NCCL's fp32 all-reduce after the o_proj / down_proj partial GEMMs
// when the communicator has a peer-memory region (orin_tp_enable_p2p).  Every
// rank's region holds its fp32 partial [M, N] (written by its GEMM), a 16-bit
// result buffer and a flag block; peers map each other's regions (CUDA IPC),
// so this kernel reads and writes them with plain loads and stores.
//
// One kernel, the same grid of G blocks on every rank.  Rank r owns an even
// share of the rows; block b handles chunk b of every rank's share, so block
// b only ever synchronises with block b of each peer (no grid-wide step):
//   1. "ready": signal every peer's block b (flag store after a fence),
//      wait (bounded) for theirs — all partials are complete;
//   2. sum chunk b of this rank's rows over ranks 0..W-1 in that order (every
//      element is summed once, by its owner, in the same order for any rank
//      count), apply residual and rounding, write C and this rank's result;
//   3. "done": signal every peer's block b, wait for theirs — their chunk b
//      results are complete;
//   4. copy chunk b of every peer's rows from its result buffer into C.
// A block leaves only after every peer's block b finished reading this rank's
// partial (their step 3 follows their step 2), so the next GEMM may overwrite
// it; it rewrites its result chunk only after every peer's block b started the
// next call (step 1), i.e. finished copying.  Flags carry per-block epochs in
// device memory, advanced by the block itself, so captured graphs replay
// correctly.  Every wait gives up after 2 s, records a device error code and
// returns (orin_device_check reports it; the communicator is then unusable).
// Plain peer loads and stores only: no multimem, no TMA.
#include "orin_common.cuh"
#include "orin_internal.h"

namespace orin {
namespace {

constexpr int kP2PThreads = 256;
constexpr unsigned long long kPeerWaitNs = 2000000000ull;

// Flag store into a peer's memory after this block's writes.  The fence is
// GPU-scope on purpose: a peer reads this rank's buffers over NVLink from
// this GPU's L2 (peer memory is not cached on the reading side, and the
// reading loads are volatile), so completing the writes at GPU scope before
// the flag leaves is what makes them visible to the peer.  A system-scope
// release also drains to host-coherent level and measured 2-3 us per signal
// (the whole reduction: 29 us instead of 12 us at M=512, TP2).
__device__ __forceinline__ void signal_store(int* p, int v) {
  asm volatile("fence.acq_rel.gpu;\n\tst.relaxed.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v)
               : "memory");
}

__device__ __forceinline__ int ld_relaxed_sys(const int* p) {
  int v;
  asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// After a flag poll: later loads (of peer buffers) are ordered after it.
__device__ __forceinline__ void fence_acquire_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

// Another GPU's memory (or ours, written by another GPU): no L1 copy.
__device__ __forceinline__ float4 ld_peer_f4(const float* p) {
  float4 v;
  asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ld_peer_u4(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Threads p < world (p != rank) each wait for peer p's flag of this block to
// reach e (relaxed polls, then a fence); the block proceeds together.
__device__ bool wait_block_peers(const P2PView& v, int base, int e, volatile int* abort_flag) {
  const int p = threadIdx.x;
  if (p < v.world && p != v.rank) {
    const int* f = v.local_flags + base + blockIdx.x * kP2PMaxRanks + p;
    const unsigned long long t0 = global_timer_ns();
    while (ld_relaxed_sys(f) < e) {
      if (global_timer_ns() - t0 > kPeerWaitNs) {
        atomicCAS(v.err, 0, DEVERR_TIMEOUT_PEER);
        *abort_flag = 1;
        break;
      }
    }
    fence_acquire_gpu();
  }
  __syncthreads();
  return *abort_flag == 0;
}

// Thread p (p != rank) tells peer p's block of the same index: "e".  The block
// barrier before it orders every thread's writes before the fence.
__device__ void signal_block_peers(const P2PView& v, int base, int e) {
  const int p = threadIdx.x;
  if (p < v.world && p != v.rank)
    signal_store(v.flags[p] + base + blockIdx.x * kP2PMaxRanks + v.rank, e);
}

// Chunk b of rank q's rows, in elements (multiples of 8).
__device__ __forceinline__ void chunk_of(const P2PView& v, int q, long long& lo, long long& hi) {
  const long long s0 = v.row0[q] * v.N;
  const long long s1 = v.row0[q + 1] * v.N;
  const long long per = (((s1 - s0) / 8 + gridDim.x - 1) / gridDim.x) * 8;
  lo = s0 + per * blockIdx.x;
  hi = lo + per < s1 ? lo + per : s1;
  if (lo > s1) lo = s1;
}

template <int DT>
__global__ void __launch_bounds__(kP2PThreads) p2p_allreduce_kernel(const P2PView v) {
  using E = Elem<DT>;
  using T = typename E::T;
  __shared__ int abort_flag;
  // launched early (programmatic dependent launch): the partial GEMM is
  // complete after this
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) abort_flag = 0;
  __syncthreads();
  const int e = v.epoch[blockIdx.x] + 1;
  const bool peers = v.world > 1;
  if (peers) {
    __syncthreads();  // every thread has read the epoch before thread 0 can move it
    signal_block_peers(v, kP2PArrive, e);
    if (!wait_block_peers(v, kP2PArrive, e, &abort_flag)) return;
  }
  T* C = static_cast<T*>(v.C);
  T* Res = static_cast<T*>(v.result_local);
  const T* R = static_cast<const T*>(v.R);
  long long lo, hi;
  chunk_of(v, v.rank, lo, hi);
  for (long long i = lo + 8 * threadIdx.x; i < hi; i += 8 * kP2PThreads) {
    // every rank's loads are issued before the first add (peer loads take
    // 1-2 us; issued one rank at a time they would serialise), then summed in
    // rank order
    float4 a[kP2PMaxRanks], b[kP2PMaxRanks];
#pragma unroll
    for (int p = 0; p < kP2PMaxRanks; ++p) {
      if (p < v.world) {
        a[p] = ld_peer_f4(v.partial[p] + i);
        b[p] = ld_peer_f4(v.partial[p] + i + 4);
      }
    }
    float s[8] = {a[0].x, a[0].y, a[0].z, a[0].w, b[0].x, b[0].y, b[0].z, b[0].w};
#pragma unroll
    for (int p = 1; p < kP2PMaxRanks; ++p) {
      if (p < v.world) {
        s[0] += a[p].x; s[1] += a[p].y; s[2] += a[p].z; s[3] += a[p].w;
        s[4] += b[p].x; s[5] += b[p].y; s[6] += b[p].z; s[7] += b[p].w;
      }
    }
    float o[8];
    if (R) {
      const uint4 r = *reinterpret_cast<const uint4*>(R + i);
      const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = E::unpack2(rw[j]);
        o[2 * j] = f.x + E::round(s[2 * j]);
        o[2 * j + 1] = f.y + E::round(s[2 * j + 1]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = s[j];
    }
    const uint4 packed = make_uint4(E::pack2(o[0], o[1]), E::pack2(o[2], o[3]),
                                    E::pack2(o[4], o[5]), E::pack2(o[6], o[7]));
    *reinterpret_cast<uint4*>(C + i) = packed;
    if (peers) *reinterpret_cast<uint4*>(Res + i) = packed;
  }
  if (peers) {
    __syncthreads();
    signal_block_peers(v, kP2PDone, e);
    if (!wait_block_peers(v, kP2PDone, e, &abort_flag)) return;
    for (int q = 0; q < v.world; ++q) {
      if (q == v.rank) continue;
      chunk_of(v, q, lo, hi);
      const T* src = static_cast<const T*>(v.result[q]);
      // four chunks in flight per thread before their stores
      constexpr int kU = 4;
      for (long long i0 = lo + 8 * threadIdx.x; i0 < hi; i0 += 8LL * kP2PThreads * kU) {
        uint4 t[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const long long i = i0 + 8LL * kP2PThreads * u;
          if (i < hi) t[u] = ld_peer_u4(src + i);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const long long i = i0 + 8LL * kP2PThreads * u;
          if (i < hi) *reinterpret_cast<uint4*>(C + i) = t[u];
        }
      }
    }
  }
  if (threadIdx.x == 0) v.epoch[blockIdx.x] = e;
}

}  // namespace

// Up to kP2PMaxBlocks blocks (256 threads x 98 registers: two per SM when
// alone, one beside a GEMM CTA), so the grid need not be resident at once.
// Progress needs less: block b waits only for block b of each peer, and the
// blocks of a grid are dispatched in index order, so the lowest unfinished
// index is resident on every rank and completes, which frees its slots for
// the next.  (A grid capped at one block per SM was measured 11 % slower on
// the Llama-3 layer at TP2: too few loads in flight.)  Every wait still gives
// up after 2 s.
int p2p_blocks(long long most_rows, int N) {
  long long b = (most_rows * N / 8 + kP2PThreads - 1) / kP2PThreads;
  if (b > kP2PMaxBlocks) b = kP2PMaxBlocks;
  if (b < 1) b = 1;
  return static_cast<int>(b);
}

cudaError_t launch_p2p_reduce(const P2PView& v, int dtype, cudaStream_t s) {
  long long most = 0;
  for (int p = 0; p < v.world; ++p) {
    const long long rows = v.row0[p + 1] - v.row0[p];
    most = rows > most ? rows : most;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p2p_blocks(most, v.N));
  cfg.blockDim = dim3(kP2PThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return (dtype == DT_F16) ? cudaLaunchKernelEx(&cfg, p2p_allreduce_kernel<DT_F16>, v)
                           : cudaLaunchKernelEx(&cfg, p2p_allreduce_kernel<DT_BF16>, v);
}

}  // namespace orin
