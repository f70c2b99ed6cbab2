// Split-K GEMMs for decode batches of at most 64 rows, weights as the MMA's
// 128-row operand:
//
//   D[n][b] = sum_k w[n][k] * x[b][k]   (tcgen05.mma M = 128 weight rows,
//                                        N = NB batch rows, K = 16)
//
// At a handful of rows the cost of a projection is streaming its weights, and
// the general kernel (activations as the 128-row operand) spends most of its
// 192 KB of shared memory on padding rows of x: one CTA fits on an SM, so the
// next projection cannot start fetching its weights until the SM is free.
// Here a ring stage is a 128 x 64 weight slab (16 KB) plus an NB x 64 slab of
// x (2-8 KB): four stages take ~74-98 KB, two or three CTAs share an SM, and
// each CTA issues its whole weight slice before griddepcontrol.wait -- so a
// projection's weight stream overlaps the kernel before it (programmatic
// dependent launch) and only x, the MMAs and the epilogue follow the wait.
//
// Grid: (N / 128 weight tiles) x splits; CTA (tile, s) covers K slabs
// [s * kb, (s + 1) * kb).  Warp 0 (one lane) is the TMA producer, warp 1 (one
// lane) issues the MMAs, warp 2 owns TMEM; then all four warps drain TMEM
// (thread t = weight row n_base + t, one fp32 column per batch row) and write
// the fp32 partials part[s][b][n] -- the layout of the general split-K GEMM,
// so the split-K epilogues and the tensor-parallel exchange take either.
//
// SK_QKV / SK_SILU also finish their tile in the same launch: every CTA
// publishes its partials, bumps the tile's counter, and the last of the tile's
// `splits` CTAs sums the partials in split order and runs the epilogue of
// splitk_qkv_kernel / splitk_silu_kernel on them (a 128-column tile is one
// attention head, or 64 gate + 64 up rows): the same arithmetic, so the same
// bits for the same partials.  The last CTA resets its counter to zero for
// the next launch.
#include "common.cuh"
#include "host.h"
#include "qkv_epilogue.cuh"
#include "tcgen05.cuh"

namespace aacc {

enum SkinnyEpi { SK_PARTIAL = 0, SK_QKV = 1, SK_SILU = 2 };

constexpr int kSkThreads = 128;
constexpr int kSkStages = 4;
constexpr int kSkWBytes = 128 * 128;  // 128 weight rows x 64 bf16

template <int NB>
struct SkinnyCfg {
  static constexpr int X_BYTES = NB * 128;  // NB rows x 64 bf16
  static constexpr int TMEM_COLS = NB < 32 ? 32 : NB;
  static constexpr size_t SMEM = size_t(kSkStages) * (kSkWBytes + X_BYTES) + 1024 + 256;
};

struct SkinnyParams {
  float* part;       // [splits][M][N]
  int kb_per_split;  // 64-wide K slabs per CTA
  int* counters;     // SK_QKV / SK_SILU: one zeroed int per 128-row tile
  QkvEpi qkv;        // SK_QKV
  bf16* act;         // SK_SILU: [M][N / 2]
  unsigned* err;
};

template <int NB, int EPI>
__global__ void __launch_bounds__(kSkThreads)
    skinny_gemm_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx, int64_t M,
                       int64_t N, SkinnyParams p) {
  using C = SkinnyCfg<NB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* w_ring = base;
  uint8_t* x_ring = base + kSkStages * kSkWBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(x_ring + kSkStages * C::X_BYTES);
  uint64_t* empty = full + kSkStages;
  uint64_t* accum = empty + kSkStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_launch();
  const int tile = blockIdx.x;
  const int64_t n_base = (int64_t)tile * 128;
  const int split = blockIdx.y, splits = gridDim.y;
  const int kb0 = split * p.kb_per_split, nk = p.kb_per_split;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSkStages; ++i) {
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
    // ---------------- TMA producer ----------------
    tma_prefetch_desc(&tmw);
    tma_prefetch_desc(&tmx);
    const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
    // Weights first, before waiting on the kernel that writes x.
    const int pre = nk < kSkStages ? nk : kSkStages;
    for (int kb = 0; kb < pre; ++kb) {
      mbar_arrive_expect_tx(&full[kb], kSkWBytes + C::X_BYTES);
      tma_load_2d_hint(w_ring + kb * kSkWBytes, &tmw, &full[kb], (kb0 + kb) * 64, (int)n_base, pol_w);
    }
    griddep_wait();
    for (int kb = 0; kb < pre; ++kb)
      tma_load_2d_hint(x_ring + kb * C::X_BYTES, &tmx, &full[kb], (kb0 + kb) * 64, 0, pol_x);
    int issued = pre;
    for (int kb = pre; kb < nk; ++kb) {
      const int st = kb % kSkStages;
      if (!mbar_wait(&empty[st], ((kb / kSkStages) - 1) & 1, p.err, abort)) break;
      mbar_arrive_expect_tx(&full[st], kSkWBytes + C::X_BYTES);
      tma_load_2d_hint(w_ring + st * kSkWBytes, &tmw, &full[st], (kb0 + kb) * 64, (int)n_base, pol_w);
      tma_load_2d_hint(x_ring + st * C::X_BYTES, &tmx, &full[st], (kb0 + kb) * 64, 0, pol_x);
      ++issued;
    }
    for (int st = 0; st < kSkStages && st < issued; ++st) {  // no copy in flight at exit
      const int last = st + ((issued - 1 - st) / kSkStages) * kSkStages;
      mbar_wait(&full[st], (last / kSkStages) & 1, p.err, nullptr);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = umma_idesc_m128(NB, false);
    for (int kb = 0; kb < nk; ++kb) {
      const int st = kb % kSkStages;
      if (!mbar_wait(&full[st], (kb / kSkStages) & 1, p.err, abort)) break;
      tc_fence_after();
      const uint32_t wa = smem_u32(w_ring + st * kSkWBytes), xa = smem_u32(x_ring + st * C::X_BYTES);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16(tmem, umma_desc_sw128(wa + kk * 32), umma_desc_sw128(xa + kk * 32), idesc, (kb | kk) != 0);
      umma_commit(&empty[st]);
    }
    umma_commit(accum);
  }

  // ---------------- partials: thread t = weight row n_base + t ----------------
  __syncwarp();
  griddep_wait();  // the partial buffer may still be read by the previous kernel
  const bool have = mbar_wait(accum, 0, p.err, nullptr);
  tc_fence_after();
  const bool ok = have && !*abort;
  const int64_t n = n_base + threadIdx.x;
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  float* dst = p.part + (int64_t)split * M * N + n;
#pragma unroll
  for (int g = 0; g < NB / 16; ++g) {
    float v[16];
    tmem_ld16(trow + 16 * g, v);
    if (ok && n < N) {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (16 * g + j < M) dst[(int64_t)(16 * g + j) * N] = v[j];
    }
  }

  if constexpr (EPI != SK_PARTIAL) {
    // ---------------- the tile's last CTA: split sum + epilogue ----------------
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      int last = 0;
      if (ok) {
        last = atomicAdd(&p.counters[tile], 1) == splits - 1;
        if (last) p.counters[tile] = 0;
        __threadfence();
      }
      *last_flag = last;
    }
    __syncthreads();
    if (*last_flag) {
      __threadfence();  // the other CTAs' partials (read through L2 below)
      const int64_t stride = M * N;
      if constexpr (EPI == SK_QKV) {
        // warp w: rows w, w + 4, ... (four per pass, their split sums loaded
        // together); lane l: head columns 4l..4l+3
        for (int64_t m0 = warp; m0 < M; m0 += 16) {
          float4 s4[4];
#pragma unroll
          for (int r = 0; r < 4; ++r)
            if (m0 + 4 * r < M) s4[r] = __ldcg(reinterpret_cast<const float4*>(p.part + (m0 + 4 * r) * N + n_base +
                                                                                 4 * lane));
#pragma unroll 4
          for (int s = 1; s < splits; ++s) {
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              if (m0 + 4 * r >= M) continue;
              const float4 b = __ldcg(reinterpret_cast<const float4*>(p.part + (int64_t)s * stride +
                                                                      (m0 + 4 * r) * N + n_base + 4 * lane));
              s4[r].x += b.x;
              s4[r].y += b.y;
              s4[r].z += b.z;
              s4[r].w += b.w;
            }
          }
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            if (m0 + 4 * r >= M) continue;  // warp-uniform
            const float acc[4] = {s4[r].x, s4[r].y, s4[r].z, s4[r].w};
            qkv_head_epilogue(acc, lane, m0 + 4 * r, tile, p.qkv);
          }
        }
      } else {
        // gate rows n_base..+63, up rows n_base+64..+127: output columns
        // tile*64 + c; thread t: column t % 64, rows t / 64, + 2, ... (eight
        // per pass, their split sums loaded together)
        const int c = threadIdx.x & 63;
        const int64_t I = N / 2;
        for (int64_t m0 = threadIdx.x >> 6; m0 < M; m0 += 16) {
          float g[8], u[8];
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            if (m0 + 2 * r >= M) continue;
            const float* src = p.part + (m0 + 2 * r) * N + n_base + c;
            g[r] = __ldcg(src);
            u[r] = __ldcg(src + 64);
          }
#pragma unroll 2
          for (int s = 1; s < splits; ++s) {
#pragma unroll
            for (int r = 0; r < 8; ++r) {
              if (m0 + 2 * r >= M) continue;
              const float* src = p.part + (int64_t)s * stride + (m0 + 2 * r) * N + n_base + c;
              g[r] += __ldcg(src);
              u[r] += __ldcg(src + 64);
            }
          }
#pragma unroll
          for (int r = 0; r < 8; ++r)
            if (m0 + 2 * r < M) p.act[(m0 + 2 * r) * I + (int64_t)tile * 64 + c] = tobf(silu_mul(g[r], u[r]));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS)
                 : "memory");
  }
}

template <int NB, int EPI>
static int launch_skinny(const void* x, const void* w, int64_t M, int64_t N, int64_t K, int splits,
                         const SkinnyParams& p, cudaStream_t stream) {
  using C = SkinnyCfg<NB>;
  CUtensorMap tw, tx;
  int st = make_tmap_2d(&tw, w, K, N, K * 2, 64, 128, true);
  if (st) return st;
  st = make_tmap_2d(&tx, x, K, M, K * 2, 64, NB, true);
  if (st) return st;
  set_smem_once<skinny_gemm_kernel<NB, EPI>>((int)C::SMEM);
  dim3 grid((unsigned)(N / 128), (unsigned)splits);
  return check_launch("skinny_gemm_kernel", launch_k(skinny_gemm_kernel<NB, EPI>, grid, dim3(kSkThreads), C::SMEM,
                                                     stream, tw, tx, M, N, p));
}

template <int EPI>
static int skinny_dispatch(const void* x, const void* w, int64_t M, int64_t N, int64_t K, int splits, SkinnyParams p,
                           cudaStream_t stream) {
  p.kb_per_split = (int)(K / 64) / splits;
  p.err = device_error_ptr();
  if (M <= 16) return launch_skinny<16, EPI>(x, w, M, N, K, splits, p, stream);
  if (M <= 32) return launch_skinny<32, EPI>(x, w, M, N, K, splits, p, stream);
  return launch_skinny<64, EPI>(x, w, M, N, K, splits, p, stream);
}

static int skinny_check(const void* x, const void* w, const float* part, int64_t M, int64_t N, int64_t K, int splits,
                        const char* what) {
  if (M < 0 || M > 64 || N <= 0 || N % 128 || K <= 0 || K % 64 || splits < 1 || (K / 64) % splits)
    return set_error(AACC_ERR_INVALID, "%s: need M <= 64, N %% 128 == 0, K %% 64 == 0, splits | K/64 "
                     "(M %lld N %lld K %lld splits %d)", what, (long long)M, (long long)N, (long long)K, splits);
  if (N / 128 > 65535 || splits > 65535 || N >= (int64_t(1) << 31))
    return set_error(AACC_ERR_UNSUPPORTED, "%s: dimension too large", what);
  if (!aligned16(x) || !aligned16(w) || !aligned16(part))
    return set_error(AACC_ERR_INVALID, "%s: operands must be 16-byte aligned", what);
  return AACC_OK;
}

}  // namespace aacc

using namespace aacc;

extern "C" {

int aacc_gemm_skinny_splitk(const void* x, const void* w, float* partial, int64_t M, int64_t N, int64_t K,
                            int splits, cudaStream_t stream) {
  int st = skinny_check(x, w, partial, M, N, K, splits, "gemm_skinny_splitk");
  if (st || M == 0) return st;
  SkinnyParams p{};
  p.part = partial;
  return skinny_dispatch<SK_PARTIAL>(x, w, M, N, K, splits, p, stream);
}

int aacc_skinny_qkv_norm_rope_store(const void* x, const void* w_qkv, float* partial, int splits, int* counters,
                                    const void* q_norm_w, const void* k_norm_w, float eps, const int64_t* positions,
                                    const void* rope_cos_sin, int64_t max_pos, const int64_t* slot_mapping,
                                    void* q_out, void* k_cache, void* v_cache, int64_t num_blocks, int num_q_heads,
                                    int num_kv_heads, int block_size, int64_t M, int64_t K, cudaStream_t stream) {
  const int64_t N = (int64_t)(num_q_heads + 2 * num_kv_heads) * 128;
  int st = skinny_check(x, w_qkv, partial, M, N, K, splits, "skinny_qkv_norm_rope_store");
  if (st || M == 0) return st;
  if (num_q_heads <= 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks <= 0 || max_pos <= 0 || !counters)
    return set_error(AACC_ERR_INVALID, "skinny_qkv_norm_rope_store: bad sizes");
  if (!aligned16(q_out) || !aligned16(k_cache) || !aligned16(v_cache))
    return set_error(AACC_ERR_INVALID, "skinny_qkv_norm_rope_store: pointers must be 16-byte aligned");
  SkinnyParams p{};
  p.part = partial;
  p.counters = counters;
  p.qkv = QkvEpi{(const bf16*)q_norm_w, (const bf16*)k_norm_w, eps, positions, (const bf16*)rope_cos_sin, max_pos,
                 slot_mapping, (bf16*)q_out, (bf16*)k_cache, (bf16*)v_cache, num_blocks * block_size, num_q_heads,
                 num_kv_heads, block_size, device_error_ptr()};
  return skinny_dispatch<SK_QKV>(x, w_qkv, M, N, K, splits, p, stream);
}

int aacc_skinny_silu_mul(const void* x, const void* w_gate_up, float* partial, int splits, int* counters, void* out,
                         int64_t M, int64_t I, int64_t K, cudaStream_t stream) {
  int st = skinny_check(x, w_gate_up, partial, M, 2 * I, K, splits, "skinny_silu_mul");
  if (st || M == 0) return st;
  if (!counters) return set_error(AACC_ERR_INVALID, "skinny_silu_mul: counters required");
  SkinnyParams p{};
  p.part = partial;
  p.counters = counters;
  p.act = (bf16*)out;
  return skinny_dispatch<SK_SILU>(x, w_gate_up, M, 2 * I, K, splits, p, stream);
}

}  // extern "C"
