// Tensor-parallel exchange of the RowParallel output over NVLink peer memory,
// fused with the split-K reduction before it and the residual add + RMSNorm
// after it.
//
// At TP > 1 each rank holds a partial o_proj / down_proj output.  The
// reference all-reduces it in bf16 (RowParallelLinear.forward,
// parallel_layers.py:190-195), then the block adds the residual and applies
// the next RMSNorm (model/model.py:259-265).  For decode-sized batches this
// kernel does all of it in one launch:
//   1. sum this rank's split-K fp32 partials (split order) and round to bf16:
//      the rank's own F.linear output;
//   2. push it into the exchange buffers of the other ranks (CUDA IPC
//      mappings, NVLink) as flagged words: every 8-byte word carries two bf16
//      values and the call's sequence number, written with one 8-byte store,
//      so a reader knows a word has arrived by its flag alone -- no fences
//      and no separate arrival flags on the critical path;
//   3. sum the ranks' bf16 outputs in fp32 in rank order, round to bf16 (the
//      all-reduced tensor), add the residual in bf16 and apply the RMSNorm
//      with the same thread layout and rounding as the norm kernels.
// one-shot: every rank pushes its whole output to every rank.
// two-shot: rank p owns the 8-column vectors [p*nv/t, (p+1)*nv/t); phase 1
//   pushes each slice to its owner, the owner sums it and pushes the reduced
//   slice to every rank (phase 2): 2(t-1)/t of the output crosses NVLink per
//   rank instead of (t-1), for one more one-way latency.
// Both modes sum in the same order, so they give identical bits; at two
// ranks both equal NCCL's bf16 sum.
//
// Sequence numbers: CTA j of every launch handles rows j, j + kArSlots, ...
// and keeps its call count in seen[j] (this rank's buffer); words of call c
// carry c (never 0, the buffer starts zeroed), so nothing is ever reset and
// CUDA-graph replays stay in step.  The receive areas are double-buffered by
// the parity of c: a rank starts writing call c + 2 only after it received
// every peer's words of call c + 1, which each peer writes only after its
// call c kernel (and so its reads of the parity-c buffer) completed, so two
// buffers suffice.  Every wait gives up after the peer wait limit, reports
// ERR_PEER_TIMEOUT, poisons this rank's buffer and lets the kernel finish
// (the output is then invalid).  A timed-out call leaves the ranks out of
// step for good (later calls would each wait out the limit), so every later
// call on a poisoned buffer skips its waits and the host, which reads the
// error word after each step, raises.  The limit is long (20 s) because a
// rank's host can stall for seconds (a large pickle, a garbage collection)
// while its peers are already waiting on the GPU.
#include <cstring>

#include "common.cuh"
#include "host.h"
#include "norm_row.cuh"

namespace aacc {

constexpr int kArMaxWorld = 8;
constexpr int kArSlots = 128;
constexpr int64_t kArHeaderBytes = 16384;  // seen[kArSlots] | poison word at 8192, padded
constexpr int64_t kDefaultPeerWaitMs = 20000;
static int64_t g_peer_wait_ms = kDefaultPeerWaitMs;  // host-side setting, passed to every launch

struct ArPeers {
  char* buf[kArMaxWorld];
};

__device__ __forceinline__ uint32_t* ar_seen(char* b) { return reinterpret_cast<uint32_t*>(b); }
__device__ __forceinline__ uint32_t* ar_poison(char* b) { return reinterpret_cast<uint32_t*>(b + 8192); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// 8 bf16 values (uint4) as four flagged words, stored as two 16-byte
// vectors of 8-byte elements (each element is single-copy atomic).
__device__ __forceinline__ void st_flagged(uint64_t* dst, uint4 v, uint32_t seq) {
  const uint64_t f = (uint64_t)seq << 32;
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(f | v.x), "l"(f | v.y) : "memory");
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst + 2), "l"(f | v.z), "l"(f | v.w) : "memory");
}

// Wait until the four flagged words at src carry `seq` and return their data.
__device__ __forceinline__ uint4 ld_flagged(const uint64_t* src, uint32_t seq, unsigned* err, bool& ok,
                                            uint32_t* poison, uint64_t wait_ns) {
  uint64_t a, b, c, d;
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(src) : "memory");
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(c), "=l"(d) : "l"(src + 2) : "memory");
    if ((uint32_t)(a >> 32) == seq && (uint32_t)(b >> 32) == seq && (uint32_t)(c >> 32) == seq &&
        (uint32_t)(d >> 32) == seq)
      break;
    if (!ok) break;  // an earlier wait of this thread already timed out
    if ((i & 15) == 0) {
      if (*reinterpret_cast<volatile uint32_t*>(poison)) {  // another thread of this rank gave up already
        ok = false;
        break;
      }
      const uint64_t now = global_ns();
      if (i == 0) {
        t0 = now;
      } else if (now - t0 > wait_ns || i > (1u << 28)) {
        report(err, ERR_PEER_TIMEOUT);
        atomicExch(poison, 1u);
        ok = false;
        break;
      }
    }
  }
  return make_uint4((uint32_t)a, (uint32_t)b, (uint32_t)c, (uint32_t)d);
}

__device__ __forceinline__ uint4 pack8(const float (&a)[8]) {
  uint4 u;
  u.x = pack_bf16(a[0], a[1]);
  u.y = pack_bf16(a[2], a[3]);
  u.z = pack_bf16(a[4], a[5]);
  u.w = pack_bf16(a[6], a[7]);
  return u;
}
__device__ __forceinline__ void add8(float (&a)[8], uint4 u) {
  float2 f;
  f = unpack_bf16(u.x); a[0] += f.x; a[1] += f.y;
  f = unpack_bf16(u.y); a[2] += f.x; a[3] += f.y;
  f = unpack_bf16(u.z); a[4] += f.x; a[5] += f.y;
  f = unpack_bf16(u.w); a[6] += f.x; a[7] += f.y;
}

template <int V, bool kTwoShot>
__global__ void __launch_bounds__(kNormMaxThreads)
    tp_allreduce_norm_kernel(const void* __restrict__ src, int splits, const __grid_constant__ ArPeers peers,
                             int world, int rank, int64_t max_rows, bf16* __restrict__ residual,
                             const bf16* __restrict__ w, bf16* __restrict__ y, int64_t M, int hidden, float eps,
                             unsigned* err, uint64_t wait_ns) {
  griddep_wait();
  griddep_launch();
  const int j = blockIdx.x, tid = threadIdx.x, nt = blockDim.x;
  char* own = peers.buf[rank];
  const uint32_t s0 = *reinterpret_cast<volatile uint32_t*>(ar_seen(own) + j);
  const uint32_t seq = s0 + 1;
  const int64_t par = s0 & 1;
  const int nv = hidden / 8;
  const int slice = nv / world;             // two-shot: vectors owned by each rank
  const int64_t row_words = hidden / 2;     // flagged words per row
  // word (not byte) offsets into a buffer
  auto recv1 = [&](char* b, int from, int64_t m, int c) {
    return reinterpret_cast<uint64_t*>(b + kArHeaderBytes) + ((par * world + from) * max_rows + m) * row_words + c * 4;
  };
  auto recv2 = [&](char* b, int64_t m, int c) {
    return reinterpret_cast<uint64_t*>(b + kArHeaderBytes) + (2 * world * max_rows + par * max_rows + m) * row_words +
           c * 4;
  };
  // A poisoned buffer (an earlier call timed out) skips every wait.
  bool ok = *reinterpret_cast<volatile uint32_t*>(ar_poison(own)) == 0;
  uint32_t* poison = ar_poison(own);
  // The first row's residual is local and already final: load it now so its
  // latency hides under the exchange.
  uint4 res0[V];
  if (j < M) {
#pragma unroll
    for (int v = 0; v < V; ++v) res0[v] = *reinterpret_cast<const uint4*>(residual + (int64_t)j * hidden + (v * nt + tid) * 8);
  }

  // 1. this rank's bf16 GEMM output, pushed to the owners (two-shot) or to everyone.
  for (int64_t m = j; m < M; m += kArSlots) {
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = v * nt + tid;
      uint4 pk;
      if (splits > 0) {
        float a[8];
        sum_partials8(static_cast<const float*>(src) + m * hidden + c * 8, splits, M * hidden, a);
        pk = pack8(a);
      } else {
        pk = *reinterpret_cast<const uint4*>(static_cast<const bf16*>(src) + m * hidden + c * 8);
      }
      if (kTwoShot) {
        st_flagged(recv1(peers.buf[c / slice], rank, m, c), pk, seq);
      } else {
        for (int p = 0; p < world; ++p) st_flagged(recv1(peers.buf[(rank + p) % world], rank, m, c), pk, seq);
      }
    }
  }

  // 2. (two-shot) reduce the owned slice and push it to every rank.
  if (kTwoShot) {
    for (int64_t m = j; m < M; m += kArSlots) {
      for (int c = rank * slice + tid; c < (rank + 1) * slice; c += nt) {
        float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int from = 0; from < world; ++from) add8(a, ld_flagged(recv1(own, from, m, c), seq, err, ok, poison, wait_ns));
        const uint4 pk = pack8(a);
        for (int p = 0; p < world; ++p) st_flagged(recv2(peers.buf[(rank + p) % world], m, c), pk, seq);
      }
    }
  }

  // 3. all-reduced bf16 delta -> residual add -> RMSNorm.
  for (int64_t m = j; m < M; m += kArSlots) {
    float h[V * 8];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = v * nt + tid;
      float d[8];
      if (kTwoShot) {
        const uint4 u = ld_flagged(recv2(own, m, c), seq, err, ok, poison, wait_ns);
        float2 f;
        f = unpack_bf16(u.x); d[0] = f.x; d[1] = f.y;
        f = unpack_bf16(u.y); d[2] = f.x; d[3] = f.y;
        f = unpack_bf16(u.z); d[4] = f.x; d[5] = f.y;
        f = unpack_bf16(u.w); d[6] = f.x; d[7] = f.y;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) d[i] = 0.f;
        for (int from = 0; from < world; ++from) add8(d, ld_flagged(recv1(own, from, m, c), seq, err, ok, poison, wait_ns));
#pragma unroll
        for (int i = 0; i < 8; ++i) d[i] = rbf(d[i]);
      }
      bf16* rp = residual + m * hidden + c * 8;
      const uint4 r = m == j ? res0[v] : *reinterpret_cast<const uint4*>(rp);
      const uint32_t* ru = reinterpret_cast<const uint32_t*>(&r);
      uint4 o;
      uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 rf = unpack_bf16(ru[q]);
        h[v * 8 + 2 * q] = rbf(rf.x + d[2 * q]);
        h[v * 8 + 2 * q + 1] = rbf(rf.y + d[2 * q + 1]);
        ou[q] = pack_bf16(h[v * 8 + 2 * q], h[v * 8 + 2 * q + 1]);
      }
      *reinterpret_cast<uint4*>(rp) = o;
    }
    norm_row<V>(h, w, y + m * hidden, eps, hidden);
    __syncthreads();  // norm_row's reduction scratch is reused by the next row
  }
  __syncthreads();
  if (tid == 0) ar_seen(own)[j] = seq;
}

}  // namespace aacc

using namespace aacc;

extern "C" {

int aacc_tp_set_peer_wait_ms(int64_t ms) {
  if (ms < 1 || ms > 600000) return set_error(AACC_ERR_INVALID, "tp_set_peer_wait_ms: %lld ms outside [1, 600000]",
                                              (long long)ms);
  g_peer_wait_ms = ms;
  return AACC_OK;
}

int64_t aacc_tp_exchange_bytes(int world, int64_t max_rows, int64_t hidden) {
  if (world < 1 || max_rows < 1 || hidden < 1) return 0;
  return kArHeaderBytes + (2 * world + 2) * max_rows * hidden * 4;  // 4 bytes per bf16 as flagged words
}

int aacc_peer_buffer_alloc(int64_t bytes, void** ptr, void* ipc_handle) {
  if (bytes <= 0 || !ptr || !ipc_handle) return set_error(AACC_ERR_INVALID, "peer_buffer_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return set_error(AACC_ERR_CUDA, "peer_buffer_alloc: cudaMalloc(%lld): %s", (long long)bytes,
                                         cudaGetErrorString(e));
  e = cudaMemset(p, 0, (size_t)bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_error(AACC_ERR_CUDA, "peer_buffer_alloc: %s", cudaGetErrorString(e));
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return AACC_OK;
}

int aacc_peer_buffer_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return set_error(AACC_ERR_INVALID, "peer_buffer_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(AACC_ERR_CUDA, "peer_buffer_open: %s", cudaGetErrorString(e));
  *ptr = p;
  return AACC_OK;
}

int aacc_peer_buffer_close(void* peer_ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
  return e == cudaSuccess ? AACC_OK : set_error(AACC_ERR_CUDA, "peer_buffer_close: %s", cudaGetErrorString(e));
}

int aacc_peer_buffer_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? AACC_OK : set_error(AACC_ERR_CUDA, "peer_buffer_free: %s", cudaGetErrorString(e));
}

int aacc_tp_allreduce_add_rmsnorm(const void* src, int splits, void* const* buffers, int world, int rank,
                                  int two_shot, int64_t max_rows, void* residual, const void* w, void* y, int64_t M,
                                  int64_t hidden, float eps, cudaStream_t stream) {
  int threads, V;
  int st = norm_shape(M, hidden, "tp_allreduce_add_rmsnorm", &threads, &V);
  if (st) return st;
  if (world < 2 || world > kArMaxWorld || rank < 0 || rank >= world || !buffers)
    return set_error(AACC_ERR_INVALID, "tp_allreduce_add_rmsnorm: world %d / rank %d (2..%d ranks)", world, rank,
                     kArMaxWorld);
  if (M > max_rows) return set_error(AACC_ERR_INVALID, "tp_allreduce_add_rmsnorm: %lld rows > exchange capacity %lld",
                                     (long long)M, (long long)max_rows);
  if (splits < 0 || splits > 64) return set_error(AACC_ERR_INVALID, "tp_allreduce_add_rmsnorm: splits %d", splits);
  if (M == 0) return AACC_OK;  // every rank sees the same M: all skip together
  if (two_shot && (hidden / 8) % world)
    return set_error(AACC_ERR_INVALID, "tp_allreduce_add_rmsnorm: two-shot needs hidden/8 divisible by %d", world);
  if (!aligned16(src) || !aligned16(residual) || !aligned16(w) || !aligned16(y))
    return set_error(AACC_ERR_INVALID, "tp_allreduce_add_rmsnorm: operands must be 16-byte aligned");
  ArPeers peers{};
  for (int p = 0; p < world; ++p) {
    if (!buffers[p] || !aligned16(buffers[p]))
      return set_error(AACC_ERR_INVALID, "tp_allreduce_add_rmsnorm: exchange buffer %d missing or unaligned", p);
    peers.buf[p] = static_cast<char*>(buffers[p]);
  }
  unsigned* err = device_error_ptr();
  const uint64_t wait_ns = (uint64_t)g_peer_wait_ms * 1000000ull;
  cudaError_t le;
#define AACC_AR_LAUNCH(VV)                                                                                        \
  le = two_shot ? launch_k(tp_allreduce_norm_kernel<VV, true>, dim3(kArSlots), dim3(threads), 0, stream, src,    \
                           splits, peers, world, rank, max_rows, (bf16*)residual, (const bf16*)w, (bf16*)y, M,  \
                           (int)hidden, eps, err, wait_ns)                                                                \
                : launch_k(tp_allreduce_norm_kernel<VV, false>, dim3(kArSlots), dim3(threads), 0, stream, src,   \
                           splits, peers, world, rank, max_rows, (bf16*)residual, (const bf16*)w, (bf16*)y, M,  \
                           (int)hidden, eps, err, wait_ns)
  switch (V) {
    case 1: AACC_AR_LAUNCH(1); break;
    case 2: AACC_AR_LAUNCH(2); break;
    case 3: AACC_AR_LAUNCH(3); break;
    case 4: AACC_AR_LAUNCH(4); break;
    case 5: AACC_AR_LAUNCH(5); break;
    case 6: AACC_AR_LAUNCH(6); break;
    case 7: AACC_AR_LAUNCH(7); break;
    default: AACC_AR_LAUNCH(8); break;
  }
#undef AACC_AR_LAUNCH
  return check_launch("tp_allreduce_add_rmsnorm", le);
}

}  // extern "C"
