// Cluster split-K tcgen05 GEMM for decode-sized batches (M <= 256 rows) with
// the epilogue fused in.
//
//   out = x @ w^T,  x: [M][K] activations (K-major), w: [N][K] weights.
//
// A decode projection streams 4-50 MB of weights against a few hundred
// activation rows, so a grid of one CTA per 128-column output tile leaves
// most SMs idle.  Here the K dimension of every output tile is split over the
// S CTAs of one thread-block cluster (grid (N/128, M tiles, S), cluster
// (1, 1, S)):
//
//   1. each CTA runs the TMA -> tcgen05.mma -> TMEM pipeline of gemm_tc.cu
//      over its slice of K (the same slab order and MMA sequence);
//   2. it stages its fp32 partial tile in its own shared memory (the ring is
//      free by then; 16-byte chunks XOR-swizzled by row, conflict-free);
//   3. cluster barrier; CTA j then owns rows [j*R/S, (j+1)*R/S) of the tile
//      and sums the S partials of those rows straight from the peers' shared
//      memory (distributed shared memory, addresses from mapa), in split
//      order -- the same fp32 additions, in the same order, as gemm_splitk +
//      the split-K epilogue kernels, so the result is bit-identical to that
//      path at equal splits;
//   4. it runs the epilogue on its rows: q/k RMSNorm + RoPE + KV-cache store
//      (QKV), SiLU-mul (interleaved gate/up), or a bf16 store (o / down, whose
//      residual add + RMSNorm needs whole rows and follows in add_rmsnorm or
//      the TP exchange);
//   5. a second cluster barrier keeps every CTA's staging alive until its
//      peers have read it.
//
// No fp32 partials go through HBM and no epilogue kernel is launched.  Both
// cluster barriers are reached on every path (a wait that runs out only
// skips the stores).  No load uses cluster multicast: every CTA fetches its
// own tiles.
#include <mutex>

#include "common.cuh"
#include "host.h"
#include "qkv_epilogue.cuh"
#include "tcgen05.cuh"

namespace aacc {

enum ClusterEpiKind { CEPI_STORE = 0, CEPI_SILU = 1, CEPI_QKV = 2 };

struct ClusterEpi {
  bf16* out;    // STORE: [M][N]; SILU: [M][N / 2]
  int64_t ldo;  // row stride of out, elements
  QkvEpi qkv;   // QKV
};

// 16 warps: three run the mainloop (TMA, MMA, TMEM allocation); all of them
// drain TMEM and run the reduction + epilogue, which is latency-bound.
constexpr int kClusterThreads = 512;
constexpr int kMaxClusterSplits = 16;

template <int MT>
struct ClusterCfg {
  static constexpr int A_BYTES = MT * 128 * 128;  // MT*128 rows x 64 bf16
  static constexpr int B_BYTES = 128 * 128;       // 128 weight rows x 64 bf16
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = MT == 1 ? 6 : 4;  // 192 KB ring
  static constexpr int RING = STAGES * STAGE_BYTES;
  static constexpr int STAGING = MT * 128 * 512;  // fp32 partial tile, rows x 128 columns
  static_assert(STAGING <= RING, "the partial tile reuses the ring");
  static constexpr int TMEM_COLS = MT * 128;
  static constexpr size_t SMEM = size_t(RING) + 1024 + 256;
};

// Generic address of the same shared-memory location in cluster CTA `rank`;
// plain loads through it read that CTA's shared memory, and the compiler can
// issue several of them back to back.
template <typename T>
__device__ __forceinline__ const T* cluster_peer(const T* local, uint32_t rank) {
  uint64_t r;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(reinterpret_cast<uint64_t>(local)), "r"(rank));
  return reinterpret_cast<const T*>(r);
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Byte offset of 16-byte chunk `chunk` (0..31) of staged row `row`.
__device__ __forceinline__ uint32_t stg_off(int row, int chunk) {
  return (uint32_t)(row * 512 + ((chunk ^ (row & 31)) << 4));
}

template <int MT, int EPI>
__global__ void __launch_bounds__(kClusterThreads, 1)
    gemm_cluster_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb, int64_t M,
                        int64_t N, int K, int S, ClusterEpi p, unsigned* err) {
  using C = ClusterCfg<MT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_ring = base;
  uint8_t* b_ring = base + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + C::RING);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accum = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_launch();
  const int split = (int)cluster_rank();  // cluster (1, 1, S) over grid z: rank == blockIdx.z % S
  const int64_t m0 = (int64_t)blockIdx.y * (128 * MT);
  const int64_t n0 = (int64_t)blockIdx.x * 128;
  const int nk_all = K / 64;
  const int kb0 = (int)((int64_t)split * nk_all / S);
  const int nk = (int)((int64_t)(split + 1) * nk_all / S) - kb0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  volatile int* abort = abort_flag;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer: weights (no dependency) first, then activations ----------------
    tma_prefetch_desc(&tma);
    tma_prefetch_desc(&tmb);
    const uint64_t pol_a = policy_evict_last(), pol_b = policy_evict_first();
    const int pre = nk < C::STAGES ? nk : C::STAGES;
    for (int kb = 0; kb < pre; ++kb) {
      mbar_arrive_expect_tx(&full[kb], C::STAGE_BYTES);
      tma_load_2d_hint(b_ring + kb * C::B_BYTES, &tmb, &full[kb], (kb0 + kb) * 64, (int)n0, pol_b);
    }
    griddep_wait();
    for (int kb = 0; kb < pre; ++kb)
      tma_load_2d_hint(a_ring + kb * C::A_BYTES, &tma, &full[kb], (kb0 + kb) * 64, (int)m0, pol_a);
    int issued = pre;
    for (int kb = pre; kb < nk; ++kb) {
      const int st = kb % C::STAGES;
      if (!mbar_wait(&empty[st], ((kb / C::STAGES) - 1) & 1, err, abort)) break;
      mbar_arrive_expect_tx(&full[st], C::STAGE_BYTES);
      tma_load_2d_hint(a_ring + st * C::A_BYTES, &tma, &full[st], (kb0 + kb) * 64, (int)m0, pol_a);
      tma_load_2d_hint(b_ring + st * C::B_BYTES, &tmb, &full[st], (kb0 + kb) * 64, (int)n0, pol_b);
      ++issued;
    }
    // every issued copy has landed before the ring is reused for staging
    for (int st = 0; st < C::STAGES && st < issued; ++st) {
      const int last = st + ((issued - 1 - st) / C::STAGES) * C::STAGES;
      mbar_wait(&full[st], (last / C::STAGES) & 1, err, nullptr);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = umma_idesc_bf16<128>();
    for (int kb = 0; kb < nk; ++kb) {
      const int st = kb % C::STAGES;
      if (!mbar_wait(&full[st], (kb / C::STAGES) & 1, err, abort)) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(a_ring + st * C::A_BYTES);
      const uint32_t b_addr = smem_u32(b_ring + st * C::B_BYTES);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          umma_bf16(tmem + mt * 128, umma_desc_sw128(a_addr + mt * 128 * 128 + kk * 32),
                    umma_desc_sw128(b_addr + kk * 32), idesc, (kb | kk) != 0);
        }
      }
      umma_commit(&empty[st]);
    }
    umma_commit(accum);  // fires once every MMA issued above has completed
  }

  // ---------------- stage this split's fp32 partial tile ----------------
  __syncwarp();
  griddep_wait();  // outputs may alias buffers the previous kernel still read
  const bool have = mbar_wait(accum, 0, err, nullptr);
  tc_fence_after();
  __syncthreads();  // the producer's final waits are done: the ring is free
  // Warp w drains TMEM lanes 32*(w%4).. (its lane quarter): with MT = 2,
  // warps 4-7 / 12-15 take the second 128-row tile; the warps that share a
  // quarter and a tile split the 128 columns.
  const int quarter = warp & 3;
  const int mt_row = MT == 2 ? (warp >> 2) & 1 : 0;
  const int cparts = MT == 2 ? 2 : 4, cpart = MT == 2 ? warp >> 3 : warp >> 2;
  const int srow = mt_row * 128 + quarter * 32 + lane;  // row of the tile this thread drains
  const int c_lo = cpart * (128 / cparts), c_hi = c_lo + 128 / cparts;
  const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16) + mt_row * 128;
  uint8_t* stg = base;
#pragma unroll 1
  for (int c = c_lo; c < c_hi; c += 16) {
    float v[16];
    tmem_ld16(trow + c, v);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4*>(stg + stg_off(srow, c / 4 + j)) =
          make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
  cluster_sync_all();  // every split's partial tile is staged and visible to the cluster

  // ---------------- sum the S partials of this CTA's rows (split order), epilogue ----------------
  // Two rows per warp per iteration; for each, all S partial loads are issued
  // before the first addition, so the remote reads overlap.
  const bool ok = have && !*abort;
  const int R = MT * 128;
  const int r_lo = split * R / S, r_hi = (split + 1) * R / S;
  constexpr int kWarps = kClusterThreads / 32;
  if constexpr (EPI == CEPI_SILU) {
    // lane l: output columns 2l, 2l+1 = gate columns 2l, 2l+1 and up columns 64+2l, 64+2l+1
#pragma unroll 1
    for (int r0 = r_lo + warp; r0 < r_hi; r0 += 2 * kWarps) {
      float2 g[2], u[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = min(r0 + h * kWarps, r_hi - 1);
        const float2* pg = reinterpret_cast<const float2*>(stg + stg_off(r, lane >> 1) + (lane & 1) * 8);
        const float2* pu = reinterpret_cast<const float2*>(stg + stg_off(r, 16 + (lane >> 1)) + (lane & 1) * 8);
        float2 vg[kMaxClusterSplits], vu[kMaxClusterSplits];
#pragma unroll
        for (int q = 0; q < kMaxClusterSplits; ++q)
          if (q < S) {
            vg[q] = *cluster_peer(pg, q);
            vu[q] = *cluster_peer(pu, q);
          }
        g[h] = vg[0];
        u[h] = vu[0];
#pragma unroll
        for (int q = 1; q < kMaxClusterSplits; ++q)
          if (q < S) {
            g[h].x += vg[q].x;
            g[h].y += vg[q].y;
            u[h].x += vu[q].x;
            u[h].y += vu[q].y;
          }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = r0 + h * kWarps;
        const int64_t m = m0 + r;
        if (ok && r < r_hi && m < M)
          *reinterpret_cast<uint32_t*>(p.out + m * p.ldo + n0 / 2 + 2 * lane) =
              pack_bf16(silu_mul(g[h].x, u[h].x), silu_mul(g[h].y, u[h].y));
      }
    }
  } else {
    // lane l: columns 4l..4l+3 of the tile
#pragma unroll 1
    for (int r0 = r_lo + warp; r0 < r_hi; r0 += 2 * kWarps) {
      float4 acc[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = min(r0 + h * kWarps, r_hi - 1);
        const float4* pa = reinterpret_cast<const float4*>(stg + stg_off(r, lane));
        float4 v[kMaxClusterSplits];
#pragma unroll
        for (int q = 0; q < kMaxClusterSplits; ++q)
          if (q < S) v[q] = *cluster_peer(pa, q);
        acc[h] = v[0];
#pragma unroll
        for (int q = 1; q < kMaxClusterSplits; ++q)
          if (q < S) {
            acc[h].x += v[q].x;
            acc[h].y += v[q].y;
            acc[h].z += v[q].z;
            acc[h].w += v[q].w;
          }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = r0 + h * kWarps;
        const int64_t m = m0 + r;
        if (!ok || r >= r_hi || m >= M) continue;  // warp-uniform
        if constexpr (EPI == CEPI_QKV) {
          const float a4[4] = {acc[h].x, acc[h].y, acc[h].z, acc[h].w};
          qkv_head_epilogue(a4, lane, m, (int)(n0 / 128), p.qkv);
        } else {
          uint2 o;
          o.x = pack_bf16(acc[h].x, acc[h].y);
          o.y = pack_bf16(acc[h].z, acc[h].w);
          *reinterpret_cast<uint2*>(p.out + m * p.ldo + n0 + 4 * lane) = o;
        }
      }
    }
  }
  cluster_sync_all();  // the peers have finished reading this CTA's staging

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS)
                 : "memory");
  }
}

// ---- host: plan and launch ---------------------------------------------------

struct ClusterPlan {
  int mt;       // 1: 128-row tiles, 2: one 256-row tile
  int m_tiles;  // tiles over M
  int splits;   // CTAs per cluster = K slices per output tile
};

template <int MT>
static const void* cluster_kernel_ptr(int epi) {
  switch (epi) {
    case CEPI_SILU: return reinterpret_cast<const void*>(gemm_cluster_kernel<MT, CEPI_SILU>);
    case CEPI_QKV: return reinterpret_cast<const void*>(gemm_cluster_kernel<MT, CEPI_QKV>);
    default: return reinterpret_cast<const void*>(gemm_cluster_kernel<MT, CEPI_STORE>);
  }
}

static int prepare_kernel(const void* fn, size_t smem) {
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  return e == cudaSuccess ? AACC_OK : set_error(AACC_ERR_CUDA, "gemm_cluster: %s", cudaGetErrorString(e));
}

// CTAs with clusters of s that can be resident at once on the current device
// (cached per device; queried on first use, which the engine makes before it
// captures any graph, since every shape runs eagerly first).
static int resident_ctas(int mt, int s) {
  static std::mutex mu;
  static int cache[64][3][kMaxClusterSplits + 1];
  int dev = 0;
  if (mt < 1 || mt > 2 || s < 1 || s > kMaxClusterSplits) return 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lk(mu);
  int& c = cache[dev][mt][s];
  if (c == 0) {
    const size_t smem = mt == 2 ? ClusterCfg<2>::SMEM : ClusterCfg<1>::SMEM;
    const void* fn = mt == 2 ? cluster_kernel_ptr<2>(CEPI_STORE) : cluster_kernel_ptr<1>(CEPI_STORE);
    if (prepare_kernel(fn, smem)) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, (unsigned)s);
    cfg.blockDim = dim3(kClusterThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = (unsigned)s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    c = n > 0 ? n * s : -1;
  }
  return c > 0 ? c : 0;
}

// Tile shape and split count for an M x N x K decode GEMM: among the shapes
// whose CTAs all fit on the GPU at once, the one that moves the fewest bytes
// through the busiest SM (K slabs x slab bytes, plus half the partial bytes it
// reads back from its peers); `want_splits` > 0 forces the split count.
static ClusterPlan plan_cluster(int64_t M, int64_t N, int64_t K, int want_splits) {
  const int nk = (int)(K / 64);
  const int n_tiles = (int)(N / 128);
  ClusterPlan best{M > 128 ? 2 : 1, 1, 1};
  if (want_splits > 0) {
    best.splits = want_splits;
    return best;
  }
  double best_cost = 1e30;
  for (int mt = 1; mt <= 2; ++mt) {
    if (mt == 2 && M <= 128) continue;
    const int m_tiles = (int)((M + 128 * mt - 1) / (128 * mt));
    for (int s = 1; s <= kMaxClusterSplits && s <= nk; ++s) {
      const int ctas = n_tiles * m_tiles * s;
      if (ctas > resident_ctas(mt, s)) continue;
      const double slab_kb = mt * 16.0 + 16.0;
      const double cost = ((nk + s - 1) / s) * slab_kb + (s > 1 ? 0.5 * mt * 64.0 * (s - 1) / s : 0.0);
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best = ClusterPlan{mt, m_tiles, s};
      }
    }
  }
  return best;
}

template <int MT, int EPI>
static int launch_cluster_gemm(const void* x, const void* w, int64_t M, int64_t N, int64_t K, const ClusterPlan& pl,
                               const ClusterEpi& p, cudaStream_t stream) {
  using C = ClusterCfg<MT>;
  CUtensorMap ta, tb;
  int st = make_tmap_2d(&ta, x, K, M, K * 2, 64, 128 * MT, true);
  if (st) return st;
  st = make_tmap_2d(&tb, w, K, N, K * 2, 64, 128, true);
  if (st) return st;
  static std::mutex mu;
  static unsigned long long ready = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!(ready & (1ull << (dev & 63)))) {
      st = prepare_kernel(reinterpret_cast<const void*>(gemm_cluster_kernel<MT, EPI>), C::SMEM);
      if (st) return st;
      ready |= 1ull << (dev & 63);
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(N / 128), (unsigned)pl.m_tiles, (unsigned)pl.splits);
  cfg.blockDim = dim3(kClusterThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = (unsigned)pl.splits;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return check_launch("gemm_cluster_kernel",
                      cudaLaunchKernelEx(&cfg, gemm_cluster_kernel<MT, EPI>, ta, tb, M, N, (int)K, pl.splits, p,
                                         device_error_ptr()));
}

template <int EPI>
static int cluster_gemm(const void* x, const void* w, int64_t M, int64_t N, int64_t K, int splits,
                        const ClusterEpi& p, cudaStream_t stream, const char* what) {
  if (M < 0 || M > 256 || N <= 0 || N % 128 || K <= 0 || K % 64)
    return set_error(AACC_ERR_INVALID, "%s: need 0 <= M <= 256, N %% 128 == 0, K %% 64 == 0 (M %lld N %lld K %lld)",
                     what, (long long)M, (long long)N, (long long)K);
  if (N / 128 >= 65536) return set_error(AACC_ERR_UNSUPPORTED, "%s: N too large", what);
  if (splits < 0 || splits > kMaxClusterSplits || splits > K / 64)
    return set_error(AACC_ERR_INVALID, "%s: splits %d outside [0, min(%d, K/64)]", what, splits, kMaxClusterSplits);
  if (!aligned16(x) || !aligned16(w)) return set_error(AACC_ERR_INVALID, "%s: operands must be 16-byte aligned", what);
  if (M == 0) return AACC_OK;
  const ClusterPlan pl = plan_cluster(M, N, K, splits);
  return pl.mt == 2 ? launch_cluster_gemm<2, EPI>(x, w, M, N, K, pl, p, stream)
                    : launch_cluster_gemm<1, EPI>(x, w, M, N, K, pl, p, stream);
}

}  // namespace aacc

using namespace aacc;

extern "C" {

int aacc_gemm_cluster_plan(int64_t M, int64_t N, int64_t K, int* mt, int* m_tiles, int* splits) {
  if (M <= 0 || M > 256 || N <= 0 || N % 128 || K <= 0 || K % 64 || !mt || !m_tiles || !splits)
    return set_error(AACC_ERR_INVALID, "gemm_cluster_plan: bad sizes");
  const ClusterPlan pl = plan_cluster(M, N, K, 0);
  *mt = pl.mt;
  *m_tiles = pl.m_tiles;
  *splits = pl.splits;
  return AACC_OK;
}

int64_t aacc_gemm_cluster_capacity(int tile_rows_128, int splits) { return resident_ctas(tile_rows_128, splits); }

int aacc_gemm_cluster(const void* x, const void* w, void* out, int64_t M, int64_t N, int64_t K, int splits,
                      cudaStream_t stream) {
  if (!aligned16(out)) return set_error(AACC_ERR_INVALID, "gemm_cluster: output must be 16-byte aligned");
  ClusterEpi p{};
  p.out = (bf16*)out;
  p.ldo = N;
  return cluster_gemm<CEPI_STORE>(x, w, M, N, K, splits, p, stream, "gemm_cluster");
}

int aacc_gemm_silu_mul_cluster(const void* x, const void* w_gate_up, void* out, int64_t M, int64_t I, int64_t K,
                               int splits, cudaStream_t stream) {
  if (I <= 0 || I % 64) return set_error(AACC_ERR_INVALID, "gemm_silu_mul_cluster: I must be a multiple of 64");
  if (!aligned16(out)) return set_error(AACC_ERR_INVALID, "gemm_silu_mul_cluster: output must be 16-byte aligned");
  ClusterEpi p{};
  p.out = (bf16*)out;
  p.ldo = I;
  return cluster_gemm<CEPI_SILU>(x, w_gate_up, M, 2 * I, K, splits, p, stream, "gemm_silu_mul_cluster");
}

int aacc_qkv_norm_rope_store_cluster(const void* x, const void* w_qkv, const void* q_norm_w, const void* k_norm_w,
                                     float eps, const int64_t* positions, const void* rope_cos_sin, int64_t max_pos,
                                     const int64_t* slot_mapping, void* q_out, void* k_cache, void* v_cache,
                                     int64_t num_blocks, int num_q_heads, int num_kv_heads, int block_size, int64_t M,
                                     int64_t K, int splits, cudaStream_t stream) {
  if (num_q_heads <= 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks <= 0 || max_pos <= 0)
    return set_error(AACC_ERR_INVALID, "qkv_norm_rope_store_cluster: bad sizes");
  if (!aligned16(q_out) || !aligned16(k_cache) || !aligned16(v_cache))
    return set_error(AACC_ERR_INVALID, "qkv_norm_rope_store_cluster: pointers must be 16-byte aligned");
  ClusterEpi p{};
  p.qkv = QkvEpi{(const bf16*)q_norm_w, (const bf16*)k_norm_w, eps, positions, (const bf16*)rope_cos_sin, max_pos,
                 slot_mapping, (bf16*)q_out, (bf16*)k_cache, (bf16*)v_cache, num_blocks * block_size, num_q_heads,
                 num_kv_heads, block_size, device_error_ptr()};
  const int64_t N = (int64_t)(num_q_heads + 2 * num_kv_heads) * 128;
  return cluster_gemm<CEPI_QKV>(x, w_qkv, M, N, K, splits, p, stream, "qkv_norm_rope_store_cluster");
}

}  // extern "C"
