// tcgen05 / TMEM GEMMs with fused epilogues for the Qwen3 projections.
//
//   out = x @ w^T,  x: [M][K] activations (A, K-major), w: [N][K] weights
//   (B, K-major, the nn.Linear layout).
//
// One CTA computes an (MT*128) x BN output tile.  Warp 0 (one elected lane)
// streams 64-wide K slabs of A and B into a STAGES-deep ring with TMA
// (128-byte swizzle); warp 1 (one lane) issues tcgen05.mma (M=128, N=BN,
// K=16, bf16 in / fp32 accumulate) into TMEM, releasing ring slots with
// tcgen05.commit; warp 2 owns the TMEM allocation.  After the last slab all
// eight warps drain TMEM with tcgen05.ld (warp w reads TMEM lanes
// 32*(w%4)..+31, i.e. one output row per thread) and run the epilogue:
//
//   EPI_STORE   bf16(acc)
//   EPI_SILU    bf16(silu(bf16(gate))) * bf16(up) on interleaved gate/up rows
//   EPI_QKV     per-head RMSNorm (q_norm / k_norm) + RoPE for Q/K heads, then
//               Q to q_out and K/V rows straight into the paged KV cache
//   EPI_ARGMAX  per-row (max, first index) of bf16(acc) over each 128-column
//               group (lm_head + greedy sampling without materialised logits);
//               rows with a temperature > 0 take the max of
//               bf16(acc / T) + Gumbel noise instead (temperature sampling)
//
// Decode batches (M <= 256) are weight-bandwidth bound: every weight byte is
// read once (MT=2 keeps both 128-row halves of the batch in one CTA);
// prefill tiles (MT=2, BN=256) are tensor-pipe bound.
#include "common.cuh"
#include "host.h"
#include "sample.cuh"
#include "tcgen05.cuh"

namespace aacc {

enum Epi { EPI_STORE = 0, EPI_SILU = 1, EPI_QKV = 2, EPI_ARGMAX = 3, EPI_PARTIAL = 4 };

struct EpiParams {
  bf16* out;
  int64_t ldo;
  const bf16* bias;  // EPI_STORE: optional per-column bias [N], added in fp32 before the bf16 rounding
  // EPI_PARTIAL (split-K): fp32 partial sums part[split][M][N]
  float* part;
  int64_t part_rows;  // M
  int kb_per_split;   // 64-wide K slabs per split (grid.z splits); 0 = all
  // EPI_QKV
  const bf16* qn_w;
  const bf16* kn_w;
  float eps;
  const int64_t* positions;
  const bf16* rope;  // [max_pos][128] = cos[64] | sin[64]
  int64_t max_pos;
  const int64_t* slot_mapping;
  bf16* k_cache;
  bf16* v_cache;
  int64_t num_slots;
  int Hq, Hkv, bs;
  // EPI_ARGMAX
  float* part_val;
  int32_t* part_idx;
  int64_t n_groups;
  const float* temperature;  // per row, NULL = all greedy
  const int64_t* seeds;      // per row
  const int64_t* counters;   // per row (position of the sampled token's input)
  int64_t vocab_offset;      // global id of column 0 (vocab-parallel shard)
  unsigned* err;
};

constexpr int kGemmThreads = 256;

template <int BN, int MT>
struct GemmCfg {
  static constexpr int A_BYTES = MT * 128 * 128;  // MT*128 rows x 64 bf16
  static constexpr int B_BYTES = BN * 128;        // BN rows x 64 bf16
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES > 8 ? 8 : (200 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = MT * BN;  // 128, 256 or 512
  static constexpr size_t SMEM = size_t(STAGES) * STAGE_BYTES + 1024 + 256;
};

// ---- epilogues: one thread = one output row, 128 columns ------------------
// `tcol` is the TMEM address of column 0 of this 128-column group for this
// warp's lane quarter; `n0` the global column of that column 0.
template <int EPI>
__device__ __forceinline__ void epilogue_group(uint32_t tcol, int64_t m, bool row_ok, int64_t n0, int64_t N,
                                               const EpiParams& p) {
  if constexpr (EPI == EPI_STORE) {
#pragma unroll 1
    for (int c = 0; c < 128; c += 16) {
      float v[16];
      tmem_ld16(tcol + c, v);
      if (p.bias) {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (n0 + c + i < N) v[i] += bf(p.bias[n0 + c + i]);
      }
      if (row_ok) {
        if (n0 + c + 16 <= N) {
          store16_bf16(p.out + m * p.ldo + n0 + c, v);
        } else {
          for (int i = 0; i < 16; ++i)
            if (n0 + c + i < N) p.out[m * p.ldo + n0 + c + i] = tobf(v[i]);
        }
      }
    }
  } else if constexpr (EPI == EPI_PARTIAL) {
    // fp32 partial of this K split; summed (in split order) by the consumer.
    float* dst = p.part + ((int64_t)blockIdx.z * p.part_rows + m) * N + n0;
#pragma unroll 1
    for (int c = 0; c < 128; c += 16) {
      float v[16];
      tmem_ld16(tcol + c, v);
      if (row_ok) {
        if (n0 + c + 16 <= N) {
          float4* d4 = reinterpret_cast<float4*>(dst + c);
          d4[0] = make_float4(v[0], v[1], v[2], v[3]);
          d4[1] = make_float4(v[4], v[5], v[6], v[7]);
          d4[2] = make_float4(v[8], v[9], v[10], v[11]);
          d4[3] = make_float4(v[12], v[13], v[14], v[15]);
        } else {
          for (int i = 0; i < 16; ++i)
            if (n0 + c + i < N) dst[c + i] = v[i];
        }
      }
    }
  } else if constexpr (EPI == EPI_SILU) {
    const int64_t ob = n0 / 2;  // output column of gate column n0
#pragma unroll 1
    for (int c = 0; c < 64; c += 16) {
      float gv[16], uv[16];
      tmem_ld16(tcol + c, gv);
      tmem_ld16(tcol + 64 + c, uv);
      if (row_ok && n0 + 128 <= N) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float gg = rbf(gv[i]);
          const float act = rbf(gg / (1.0f + expf(-gg)));
          gv[i] = act * rbf(uv[i]);
        }
        store16_bf16(p.out + m * p.ldo + ob + c, gv);
      }
    }
  } else if constexpr (EPI == EPI_QKV) {
    const int hh = (int)(n0 / 128);
    const bool is_q = hh < p.Hq, is_k = !is_q && hh < p.Hq + p.Hkv;
    bf16* dst = nullptr;
    if (row_ok) {
      if (is_q) {
        dst = p.out + m * p.ldo + (int64_t)hh * 128;
      } else {
        const int64_t slot = p.slot_mapping[m];
        if (slot >= p.num_slots) report(p.err, ERR_SLOT_OOB);
        if (slot >= 0 && slot < p.num_slots) {
          const int kvh = is_k ? hh - p.Hq : hh - p.Hq - p.Hkv;
          const int64_t off = ((slot / p.bs) * p.Hkv + kvh) * p.bs + slot % p.bs;
          dst = (is_k ? p.k_cache : p.v_cache) + off * 128;
        }
      }
    }
    if (!is_q && !is_k) {  // V head: plain store
#pragma unroll 1
      for (int c = 0; c < 128; c += 16) {
        float v[16];
        tmem_ld16(tcol + c, v);
        if (dst) store16_bf16(dst + c, v);
      }
      return;
    }
    // Pass 1: sum of squares of the bf16-rounded projection.
    float ss = 0.f;
#pragma unroll 1
    for (int c = 0; c < 128; c += 16) {
      float v[16];
      tmem_ld16(tcol + c, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float x = rbf(v[i]);
        ss += x * x;
      }
    }
    const float r = rsqrtf(ss / 128.f + p.eps);
    const bf16* nw = is_q ? p.qn_w : p.kn_w;
    int64_t pos = row_ok ? p.positions[m] : 0;
    if (pos < 0 || pos >= p.max_pos) {
      if (row_ok) report(p.err, ERR_POS_OOB);
      pos = 0;
    }
    const bf16* cs = p.rope + pos * 128;
    // Pass 2: normalise, weight, rotate (pairs i and i+64), store.
#pragma unroll 1
    for (int c = 0; c < 64; c += 16) {
      float x1[16], x2[16], w1[16], w2[16], cv[16], sv[16];
      tmem_ld16(tcol + c, x1);
      tmem_ld16(tcol + 64 + c, x2);
      load16_bf16(nw + c, w1);
      load16_bf16(nw + 64 + c, w2);
      load16_bf16(cs + c, cv);
      load16_bf16(cs + 64 + c, sv);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float y1 = rbf(w1[i] * rbf(rbf(x1[i]) * r));
        const float y2 = rbf(w2[i] * rbf(rbf(x2[i]) * r));
        x1[i] = rbf(y1 * cv[i]) + rbf(-y2 * sv[i]);
        x2[i] = rbf(y2 * cv[i]) + rbf(y1 * sv[i]);
      }
      if (dst) {
        store16_bf16(dst + c, x1);
        store16_bf16(dst + 64 + c, x2);
      }
    }
  } else {  // EPI_ARGMAX
    float best = -INFINITY;
    int32_t bi = 0x7fffffff;
    float temp = 0.f;
    uint64_t key = 0;
    if (row_ok && p.temperature) {
      temp = p.temperature[m];
      if (temp > 0.f) key = sample_key(p.seeds[m], p.counters[m]);
    }
#pragma unroll 1
    for (int c = 0; c < 128; c += 16) {
      float v[16];
      tmem_ld16(tcol + c, v);
      if (row_ok) {
        if (temp > 0.f) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int64_t n = n0 + c + i;
            const float x = rbf(rbf(v[i]) / temp) + gumbel_noise(key, (uint32_t)(p.vocab_offset + n));
            if (n < N && x > best) {
              best = x;
              bi = (int32_t)n;
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int64_t n = n0 + c + i;
            const float x = rbf(v[i]);
            if (n < N && x > best) {
              best = x;
              bi = (int32_t)n;
            }
          }
        }
        if (p.out) {
          if (n0 + c + 16 <= N) {
            store16_bf16(p.out + m * p.ldo + n0 + c, v);
          } else {
            for (int i = 0; i < 16; ++i)
              if (n0 + c + i < N) p.out[m * p.ldo + n0 + c + i] = tobf(v[i]);
          }
        }
      }
    }
    if (row_ok) {
      const int64_t gidx = n0 / 128;
      p.part_val[m * p.n_groups + gidx] = best;
      p.part_idx[m * p.n_groups + gidx] = bi;
    }
  }
}

template <int BN, int MT, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb, int64_t M,
                   int64_t N, int K, EpiParams p) {
  using C = GemmCfg<BN, MT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_ring = base;
  uint8_t* b_ring = base + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accum = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_launch();
  const int64_t m0 = (int64_t)blockIdx.y * (128 * MT);
  const int64_t n_base = (int64_t)blockIdx.x * BN;
  // K slabs of this split: [kb0, kb0 + nk).
  const int nk_all = K / 64;
  const int kb0 = p.kb_per_split > 0 ? (int)blockIdx.z * p.kb_per_split : 0;
  const int nk = p.kb_per_split > 0 ? min(p.kb_per_split, nk_all - kb0) : nk_all;

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
    // ---------------- TMA producer ----------------
    tma_prefetch_desc(&tma);
    tma_prefetch_desc(&tmb);
    const uint64_t pol_a = policy_evict_last(), pol_b = policy_evict_first();
    // The weights (B) do not depend on the previous kernel: start streaming
    // the first ring's worth of them before waiting for it, then load the
    // activations (A), which the previous kernel wrote.
    const int pre = nk < C::STAGES ? nk : C::STAGES;
    for (int kb = 0; kb < pre; ++kb) {
      mbar_arrive_expect_tx(&full[kb], C::STAGE_BYTES);
      tma_load_2d_hint(b_ring + kb * C::B_BYTES, &tmb, &full[kb], (kb0 + kb) * 64, (int)n_base, pol_b);
    }
    griddep_wait();
    for (int kb = 0; kb < pre; ++kb)
      tma_load_2d_hint(a_ring + kb * C::A_BYTES, &tma, &full[kb], (kb0 + kb) * 64, (int)m0, pol_a);
    int issued = pre;
    for (int kb = pre; kb < nk; ++kb) {
      const int st = kb % C::STAGES;
      if (!mbar_wait(&empty[st], ((kb / C::STAGES) - 1) & 1, p.err, abort)) break;
      mbar_arrive_expect_tx(&full[st], C::STAGE_BYTES);
      tma_load_2d_hint(a_ring + st * C::A_BYTES, &tma, &full[st], (kb0 + kb) * 64, (int)m0, pol_a);
      tma_load_2d_hint(b_ring + st * C::B_BYTES, &tmb, &full[st], (kb0 + kb) * 64, (int)n_base, pol_b);
      ++issued;
    }
    for (int st = 0; st < C::STAGES && st < issued; ++st) {
      const int last = st + ((issued - 1 - st) / C::STAGES) * C::STAGES;
      mbar_wait(&full[st], (last / C::STAGES) & 1, p.err, nullptr);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc = umma_idesc_bf16<BN>();
    for (int kb = 0; kb < nk; ++kb) {
      const int st = kb % C::STAGES;
      if (!mbar_wait(&full[st], (kb / C::STAGES) & 1, p.err, abort)) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(a_ring + st * C::A_BYTES);
      const uint32_t b_addr = smem_u32(b_ring + st * C::B_BYTES);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          umma_bf16(tmem + mt * BN, umma_desc_sw128(a_addr + mt * 128 * 128 + kk * 32),
                    umma_desc_sw128(b_addr + kk * 32), idesc, (kb | kk) != 0);
        }
      }
      umma_commit(&empty[st]);
    }
    umma_commit(accum);  // fires once every MMA issued above has completed
  }

  // ---------------- epilogue: all eight warps ----------------
  __syncwarp();
  griddep_wait();  // outputs may alias buffers the previous kernel still read
  const bool have = mbar_wait(accum, 0, p.err, nullptr);
  tc_fence_after();
  const int quarter = warp & 3, wset = warp >> 2;
  const int mt = (MT == 2) ? wset : 0;
  const int64_t m = m0 + mt * 128 + quarter * 32 + lane;
  const bool row_ok = have && !*abort && m < M;
  const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16) + mt * BN;
#pragma unroll 1
  for (int g = 0; g < BN / 128; ++g) {
    if (MT == 1 && (g & 1) != wset) continue;
    // A 128-column group entirely past N (the tail tile of a BN=256 grid)
    // has nothing to store and no partial slot; skip it (warp-uniform).
    if (n_base + g * 128 >= N) continue;
    epilogue_group<EPI>(trow + g * 128, m, row_ok, n_base + g * 128, N, p);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS) : "memory");
  }
}

// Merge per-group argmax partials: highest value wins, first index on ties.
__global__ void argmax_merge_groups_kernel(const float* __restrict__ pv, const int32_t* __restrict__ pi,
                                           int64_t n_groups, int64_t vocab_offset, int64_t* __restrict__ tokens,
                                           float* __restrict__ best_val) {
  griddep_wait();
  griddep_launch();
  const int64_t m = blockIdx.x;
  float best = -INFINITY;
  int32_t bi = 0x7fffffff;
  for (int64_t gi = threadIdx.x; gi < n_groups; gi += blockDim.x) {
    const float v = pv[m * n_groups + gi];
    const int32_t i = pi[m * n_groups + gi];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, best, o);
    const int32_t i = __shfl_xor_sync(0xffffffffu, bi, o);
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  __shared__ float sv[32];
  __shared__ int32_t si[32];
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k)
      if (sv[k] > best || (sv[k] == best && si[k] < bi)) {
        best = sv[k];
        bi = si[k];
      }
    tokens[m] = (bi == 0x7fffffff ? 0 : bi) + vocab_offset;
    if (best_val) best_val[m] = best;
  }
}

// ---- host launch --------------------------------------------------------------
template <int BN, int MT, int EPI>
static int launch_gemm(const void* x, const void* w, int64_t M, int64_t N, int64_t K, const EpiParams& p,
                       cudaStream_t stream, int splits = 1) {
  using C = GemmCfg<BN, MT>;
  CUtensorMap ta, tb;
  int st = make_tmap_2d(&ta, x, K, M, K * 2, 64, 128 * MT, true);
  if (st) return st;
  st = make_tmap_2d(&tb, w, K, N, K * 2, 64, BN, true);
  if (st) return st;
  auto kern = gemm_tc_kernel<BN, MT, EPI>;
  set_smem_once<gemm_tc_kernel<BN, MT, EPI>>((int)C::SMEM);
  dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + 128 * MT - 1) / (128 * MT)), (unsigned)splits);
  return check_launch("gemm_tc_kernel",
                      launch_k(kern, grid, dim3(kGemmThreads), C::SMEM, stream, ta, tb, M, N, (int)K, p));
}

// Tile shapes: decode batches (M <= 256) use 128x128 tiles, one CTA per
// 128-row half of the batch, so twice the CTAs stream the weights (the second
// read of a weight tile hits L2) and twice the SMs share the tensor work --
// at M = 256 a weight byte feeds 256 FMAs, so the decode GEMMs need every
// SM's tensor pipe as much as its bandwidth.  Prefill uses 256x256 tiles.
//
// The lm_head (EPI_ARGMAX, N = vocab: thousands of tiles) is the exception:
// there every SM is busy anyway and the per-SM shared-memory fill (TMA
// throughput) is the limit, so 256x256 tiles, which re-read the activations
// half as often and the weights once, are faster from M = 129 up.
template <int EPI>
static int gemm_dispatch(const void* x, const void* w, int64_t M, int64_t N, int64_t K, const EpiParams& p,
                         cudaStream_t stream, int splits = 1) {
  if (M <= 128 || (M <= 256 && EPI != EPI_ARGMAX)) return launch_gemm<128, 1, EPI>(x, w, M, N, K, p, stream, splits);
  return launch_gemm<256, 2, EPI>(x, w, M, N, K, p, stream, splits);
}

static int gemm_check(const void* x, const void* w, int64_t M, int64_t N, int64_t K, const char* what) {
  if (M < 0 || N <= 0 || K <= 0 || K % 64)
    return set_error(AACC_ERR_INVALID, "%s: need K %% 64 == 0 (M %lld N %lld K %lld)", what, (long long)M,
                     (long long)N, (long long)K);
  if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31))
    return set_error(AACC_ERR_UNSUPPORTED, "%s: dimension too large", what);
  if (!aligned16(x) || !aligned16(w)) return set_error(AACC_ERR_INVALID, "%s: operands must be 16-byte aligned", what);
  return AACC_OK;
}

}  // namespace aacc

using namespace aacc;

extern "C" {

int aacc_gemm(const void* x, const void* w, void* out, int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  int st = gemm_check(x, w, M, N, K, "gemm");
  if (st || M == 0) return st;
  if (!aligned16(out) || (N % 8)) return set_error(AACC_ERR_INVALID, "gemm: output must be 16-byte aligned rows");
  EpiParams p{};
  p.out = (bf16*)out;
  p.ldo = N;
  p.err = device_error_ptr();
  return gemm_dispatch<EPI_STORE>(x, w, M, N, K, p, stream);
}

int aacc_gemm_bias(const void* x, const void* w, const void* bias, void* out, int64_t M, int64_t N, int64_t K,
                   cudaStream_t stream) {
  int st = gemm_check(x, w, M, N, K, "gemm_bias");
  if (st || M == 0) return st;
  if (!aligned16(out) || (N % 8)) return set_error(AACC_ERR_INVALID, "gemm_bias: output must be 16-byte aligned rows");
  EpiParams p{};
  p.out = (bf16*)out;
  p.ldo = N;
  p.bias = (const bf16*)bias;
  p.err = device_error_ptr();
  return gemm_dispatch<EPI_STORE>(x, w, M, N, K, p, stream);
}

int aacc_gemm_splitk(const void* x, const void* w, float* partial, int64_t M, int64_t N, int64_t K, int splits,
                     cudaStream_t stream) {
  int st = gemm_check(x, w, M, N, K, "gemm_splitk");
  if (st || M == 0) return st;
  const int nk = (int)(K / 64);
  if (splits < 1 || nk % splits)
    return set_error(AACC_ERR_INVALID, "gemm_splitk: splits %d must divide K/64 = %d", splits, nk);
  if (!aligned16(partial) || (N % 4)) return set_error(AACC_ERR_INVALID, "gemm_splitk: partial rows must be 16-byte aligned");
  EpiParams p{};
  p.part = partial;
  p.part_rows = M;
  p.kb_per_split = nk / splits;
  p.err = device_error_ptr();
  return gemm_dispatch<EPI_PARTIAL>(x, w, M, N, K, p, stream, splits);
}

int aacc_gemm_silu_mul(const void* x, const void* w_gate_up, void* out, int64_t M, int64_t I, int64_t K,
                       cudaStream_t stream) {
  int st = gemm_check(x, w_gate_up, M, 2 * I, K, "gemm_silu_mul");
  if (st || M == 0) return st;
  if (I % 64) return set_error(AACC_ERR_INVALID, "gemm_silu_mul: intermediate size must be a multiple of 64");
  if (!aligned16(out)) return set_error(AACC_ERR_INVALID, "gemm_silu_mul: output must be 16-byte aligned");
  EpiParams p{};
  p.out = (bf16*)out;
  p.ldo = I;
  p.err = device_error_ptr();
  return gemm_dispatch<EPI_SILU>(x, w_gate_up, M, 2 * I, K, p, stream);
}

int aacc_qkv_norm_rope_store(const void* x, const void* w_qkv, const void* q_norm_w, const void* k_norm_w, float eps,
                             const int64_t* positions, const void* rope_cos_sin, int64_t max_pos,
                             const int64_t* slot_mapping, void* q_out, void* k_cache, void* v_cache,
                             int64_t num_blocks, int num_q_heads, int num_kv_heads, int block_size, int64_t M,
                             int64_t K, cudaStream_t stream) {
  const int64_t N = (int64_t)(num_q_heads + 2 * num_kv_heads) * 128;
  int st = gemm_check(x, w_qkv, M, N, K, "qkv_norm_rope_store");
  if (st || M == 0) return st;
  if (num_q_heads <= 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks <= 0 || max_pos <= 0)
    return set_error(AACC_ERR_INVALID, "qkv_norm_rope_store: bad sizes");
  if (!aligned16(q_out) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(rope_cos_sin) ||
      !aligned16(q_norm_w) || !aligned16(k_norm_w))
    return set_error(AACC_ERR_INVALID, "qkv_norm_rope_store: pointers must be 16-byte aligned");
  EpiParams p{};
  p.out = (bf16*)q_out;
  p.ldo = (int64_t)num_q_heads * 128;
  p.qn_w = (const bf16*)q_norm_w;
  p.kn_w = (const bf16*)k_norm_w;
  p.eps = eps;
  p.positions = positions;
  p.rope = (const bf16*)rope_cos_sin;
  p.max_pos = max_pos;
  p.slot_mapping = slot_mapping;
  p.k_cache = (bf16*)k_cache;
  p.v_cache = (bf16*)v_cache;
  p.num_slots = num_blocks * block_size;
  p.Hq = num_q_heads;
  p.Hkv = num_kv_heads;
  p.bs = block_size;
  p.err = device_error_ptr();
  return gemm_dispatch<EPI_QKV>(x, w_qkv, M, N, K, p, stream);
}

int64_t aacc_lm_head_workspace_bytes(int64_t M, int64_t vocab) {
  return M * ((vocab + 127) / 128) * (int64_t)(sizeof(float) + sizeof(int32_t));
}

int aacc_lm_head_argmax(const void* x, const void* w, int64_t M, int64_t vocab, int64_t K, int64_t vocab_offset,
                        int64_t* tokens, float* best_val, void* logits, void* workspace, int64_t workspace_bytes,
                        cudaStream_t stream) {
  return aacc_lm_head_sample(x, w, M, vocab, K, vocab_offset, nullptr, nullptr, nullptr, tokens, best_val, logits,
                             workspace, workspace_bytes, stream);
}

int aacc_lm_head_sample(const void* x, const void* w, int64_t M, int64_t vocab, int64_t K, int64_t vocab_offset,
                        const float* temperature, const int64_t* seeds, const int64_t* counters, int64_t* tokens,
                        float* best_val, void* logits, void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  int st = gemm_check(x, w, M, vocab, K, "lm_head_argmax");
  if (temperature && (!seeds || !counters))
    return set_error(AACC_ERR_INVALID, "lm_head_sample: temperatures need seeds and counters");
  if (st || M == 0) return st;
  const int64_t groups = (vocab + 127) / 128;
  if (!workspace || workspace_bytes < aacc_lm_head_workspace_bytes(M, vocab))
    return set_error(AACC_ERR_INVALID, "lm_head_argmax: workspace too small");
  if (logits && (!aligned16(logits) || vocab % 8))
    return set_error(AACC_ERR_INVALID, "lm_head_argmax: logits rows must be 16-byte aligned");
  EpiParams p{};
  p.out = (bf16*)logits;
  p.ldo = vocab;
  p.part_val = (float*)workspace;
  p.part_idx = (int32_t*)((float*)workspace + M * groups);
  p.n_groups = groups;
  p.temperature = temperature;
  p.seeds = seeds;
  p.counters = counters;
  p.vocab_offset = vocab_offset;
  p.err = device_error_ptr();
  st = gemm_dispatch<EPI_ARGMAX>(x, w, M, vocab, K, p, stream);
  if (st) return st;
  return check_launch("argmax_merge_groups",
                      launch_k(argmax_merge_groups_kernel, dim3((unsigned)M), dim3(256), 0, stream,
                               (const float*)p.part_val, (const int32_t*)p.part_idx, groups, vocab_offset, tokens,
                               best_val));
}

}  // extern "C"
