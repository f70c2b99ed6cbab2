// Causal (chunked) prefill attention over the paged KV cache on mma.sync
// (the legacy tensor-core path): aacc_prefill_attention_mma.  The engine's
// path is the tcgen05 kernel in prefill_attn_tc.cu; this one serves block
// sizes that are not multiples of 128 and A/B timing.
//
// One CTA per (64-query tile, query head, sequence).  The chunk's K/V (and
// every earlier chunk of the same sequence) are already in the paged pool, so
// the kernel only reads the cache: a producer warp streams 64-token K/V tiles
// with TMA (128-byte swizzle) through an mbarrier ring, and four consumer
// warps (16 query rows each) run S = Q K^T and O += P V on mma.sync
// m16n8k16 with an fp32 online softmax and a causal mask
// key_pos <= query_pos (query i of the chunk sits at ctx_start + i).
#include "common.cuh"
#include "host.h"

namespace aacc {

constexpr int kPD = 128;
constexpr int kPTile = 64;
constexpr int kPConsumers = 4;
constexpr int kPThreads = (kPConsumers + 1) * 32;
constexpr int kPStages = 3;
constexpr int kPHalf = kPTile * 64 * 2;

struct PrefillSmem {
  bf16 tiles[kPStages][4][kPTile * 64];
  uint64_t full[kPStages];
  uint64_t empty[kPStages];
  int abort;
};

__global__ void __launch_bounds__(kPThreads, 2)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                        const bf16* __restrict__ q, bf16* __restrict__ out, const int32_t* __restrict__ bt,
                        int64_t max_blocks, const int64_t* __restrict__ seq_rows, const int32_t* __restrict__ cu_q,
                        const int32_t* __restrict__ ctx_start, int Hq, int Hkv, int bs, int64_t num_blocks,
                        int n_qtiles, float scale_log2, unsigned* err) {
  extern __shared__ uint8_t smem_raw[];
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  griddep_wait();
  griddep_launch();
  const int qt = n_qtiles - 1 - (int)blockIdx.x;  // heaviest tiles first
  const int hq = blockIdx.y;
  const int64_t s = blockIdx.z;
  const int64_t q0 = cu_q[s];
  const int q_len = cu_q[s + 1] - (int)q0;
  if (qt * kPTile >= q_len) return;
  const int G = Hq / Hkv;
  const int kvh = hq / G;
  const int64_t row = seq_rows[s];
  const int64_t c0 = ctx_start[s];
  const int rows_here = min(kPTile, q_len - qt * kPTile);
  const int64_t p_last = c0 + qt * kPTile + rows_here - 1;  // position of the last query of the tile
  int ntiles = (int)(p_last / kPTile) + 1;
  if ((int64_t)ntiles * kPTile > max_blocks * bs) {
    if (threadIdx.x == 0) report(err, ERR_CTX_OOB);
    ntiles = (int)(max_blocks * bs / kPTile);
  }

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kPConsumers);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  volatile int* abort = &sm.abort;

  if (warp == kPConsumers) {
    if (lane == 0) {
      const int32_t* btrow = bt + row * max_blocks;
      int issued = 0;
      for (int i = 0; i < ntiles; ++i) {
        const int st = i % kPStages;
        if (i >= kPStages && !mbar_wait(&sm.empty[st], ((i / kPStages) - 1) & 1, err, abort)) break;
        const int64_t t0 = (int64_t)i * kPTile;
        int64_t blk = btrow[t0 / bs];
        if (blk < 0 || blk >= num_blocks) {
          report(err, ERR_BLOCK_OOB);
          blk = 0;
        }
        const int r = (int)((blk * Hkv + kvh) * bs + t0 % bs);
        mbar_arrive_expect_tx(&sm.full[st], 4 * kPHalf);
        tma_load_2d(sm.tiles[st][0], &tmk, &sm.full[st], 0, r);
        tma_load_2d(sm.tiles[st][1], &tmk, &sm.full[st], 64, r);
        tma_load_2d(sm.tiles[st][2], &tmv, &sm.full[st], 0, r);
        tma_load_2d(sm.tiles[st][3], &tmv, &sm.full[st], 64, r);
        ++issued;
      }
      for (int st = 0; st < kPStages && st < issued; ++st) {
        const int last = st + ((issued - 1 - st) / kPStages) * kPStages;
        mbar_wait(&sm.full[st], (last / kPStages) & 1, err, nullptr);
      }
    }
    return;
  }

  const int g = lane >> 2, c = lane & 3;
  const int r_lo = qt * kPTile + 16 * warp + g;  // query row within the sequence chunk
  const int r_hi = r_lo + 8;
  const int64_t pos_lo = c0 + r_lo, pos_hi = c0 + r_hi;
  uint32_t qa[8][4];
  {
    const int64_t ld = (int64_t)Hq * kPD;
    const bf16* ql = q + (q0 + min(r_lo, q_len - 1)) * ld + (int64_t)hq * kPD;
    const bf16* qh = q + (q0 + min(r_hi, q_len - 1)) * ld + (int64_t)hq * kPD;
    const bool vl = r_lo < q_len, vh = r_hi < q_len;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      qa[kk][0] = vl ? *reinterpret_cast<const uint32_t*>(ql + 16 * kk + 2 * c) : 0u;
      qa[kk][1] = vh ? *reinterpret_cast<const uint32_t*>(qh + 16 * kk + 2 * c) : 0u;
      qa[kk][2] = vl ? *reinterpret_cast<const uint32_t*>(ql + 16 * kk + 2 * c + 8) : 0u;
      qa[kk][3] = vh ? *reinterpret_cast<const uint32_t*>(qh + 16 * kk + 2 * c + 8) : 0u;
    }
  }
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  const int mi = lane >> 3, r8 = lane & 7;

  for (int i = 0; i < ntiles; ++i) {
    const int st = i % kPStages;
    if (!mbar_wait(&sm.full[st], (i / kPStages) & 1, err, abort)) break;
    const uint32_t kb = smem_u32(sm.tiles[st][0]);
    const uint32_t vb = smem_u32(sm.tiles[st][2]);
    float sc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int chunk = 2 * kk + (mi & 1);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = 16 * j + (mi >> 1) * 8 + r8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kb + (chunk >> 3) * kPHalf + swz128(key, chunk & 7), b0, b1, b2, b3);
        mma_bf16_16816(sc[2 * j], qa[kk], b0, b1);
        mma_bf16_16816(sc[2 * j + 1], qa[kk], b2, b3);
      }
    }
    const int64_t kbase = (int64_t)i * kPTile + 2 * c;
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int64_t k0 = kbase + 8 * n, k1 = k0 + 1;
      sc[n][0] = (k0 <= pos_lo) ? sc[n][0] * scale_log2 : -INFINITY;
      sc[n][1] = (k1 <= pos_lo) ? sc[n][1] * scale_log2 : -INFINITY;
      sc[n][2] = (k0 <= pos_hi) ? sc[n][2] * scale_log2 : -INFINITY;
      sc[n][3] = (k1 <= pos_hi) ? sc[n][3] * scale_log2 : -INFINITY;
      mx_lo = fmaxf(mx_lo, fmaxf(sc[n][0], sc[n][1]));
      mx_hi = fmaxf(mx_hi, fmaxf(sc[n][2], sc[n][3]));
    }
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
    const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
    const float mu_lo = (mn_lo == -INFINITY) ? 0.f : mn_lo, mu_hi = (mn_hi == -INFINITY) ? 0.f : mn_hi;
    const float a_lo = exp2f(m_lo - mu_lo), a_hi = exp2f(m_hi - mu_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    float s_lo = 0.f, s_hi = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      sc[n][0] = exp2f(sc[n][0] - mu_lo);
      sc[n][1] = exp2f(sc[n][1] - mu_lo);
      sc[n][2] = exp2f(sc[n][2] - mu_hi);
      sc[n][3] = exp2f(sc[n][3] - mu_hi);
      s_lo += sc[n][0] + sc[n][1];
      s_hi += sc[n][2] + sc[n][3];
    }
    l_lo = l_lo * a_lo + s_lo;
    l_hi = l_hi * a_hi + s_hi;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= a_lo;
      o[j][1] *= a_lo;
      o[j][2] *= a_hi;
      o[j][3] *= a_hi;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // 16-key k-steps of the PV product
      uint32_t pa[4];
      pa[0] = pack_bf16(sc[2 * j][0], sc[2 * j][1]);
      pa[1] = pack_bf16(sc[2 * j][2], sc[2 * j][3]);
      pa[2] = pack_bf16(sc[2 * j + 1][0], sc[2 * j + 1][1]);
      pa[3] = pack_bf16(sc[2 * j + 1][2], sc[2 * j + 1][3]);
      const int key = 16 * j + (mi & 1) * 8 + r8;
#pragma unroll
      for (int jp = 0; jp < 8; ++jp) {
        const int chunk = 2 * jp + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vb + (chunk >> 3) * kPHalf + swz128(key, chunk & 7), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * jp], pa, b0, b1);
        mma_bf16_16816(o[2 * jp + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[st]);
  }
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  const float il = l_lo > 0.f ? 1.f / l_lo : 0.f, ih = l_hi > 0.f ? 1.f / l_hi : 0.f;
  const int64_t ld = (int64_t)Hq * kPD;
  if (r_lo < q_len) {
    bf16* dst = out + (q0 + r_lo) * ld + (int64_t)hq * kPD;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      *reinterpret_cast<uint32_t*>(dst + 8 * j + 2 * c) = pack_bf16(o[j][0] * il, o[j][1] * il);
  }
  if (r_hi < q_len) {
    bf16* dst = out + (q0 + r_hi) * ld + (int64_t)hq * kPD;
#pragma unroll
    for (int j = 0; j < 16; ++j)
      *reinterpret_cast<uint32_t*>(dst + 8 * j + 2 * c) = pack_bf16(o[j][2] * ih, o[j][3] * ih);
  }
}

}  // namespace aacc

using namespace aacc;

extern "C" {

int aacc_prefill_attention_mma(const void* q, void* out, const void* k_cache, const void* v_cache, int64_t num_blocks,
                           const int32_t* block_tables, int64_t max_blocks, const int64_t* seq_rows, const int32_t* cu_q,
                           const int32_t* ctx_start, int64_t num_seqs, int64_t max_q_len, int num_q_heads,
                           int num_kv_heads, int block_size, float scale, cudaStream_t stream) {
  if (num_seqs < 0 || max_q_len < 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || block_size <= 0 ||
      block_size % kPTile || num_blocks <= 0 || max_blocks <= 0)
    return set_error(AACC_ERR_INVALID, "prefill_attention: bad sizes");
  if (num_seqs == 0 || max_q_len == 0) return AACC_OK;
  if (num_seqs > 65535) return set_error(AACC_ERR_UNSUPPORTED, "prefill_attention: too many sequences per call");
  const int64_t rows = num_blocks * num_kv_heads * block_size;
  if (rows >= (int64_t(1) << 31)) return set_error(AACC_ERR_UNSUPPORTED, "prefill_attention: pool too large");
  CUtensorMap tmk, tmv;
  int st = make_tmap_2d(&tmk, k_cache, kPD, rows, kPD * 2, 64, kPTile, true);
  if (st) return st;
  st = make_tmap_2d(&tmv, v_cache, kPD, rows, kPD * 2, 64, kPTile, true);
  if (st) return st;
  const int n_qtiles = (int)((max_q_len + kPTile - 1) / kPTile);
  const size_t smem = sizeof(PrefillSmem) + 1024;
  set_smem_once<prefill_attn_kernel>((int)smem);
  dim3 grid(n_qtiles, num_q_heads, (unsigned)num_seqs);
  return check_launch("prefill_attn_kernel",
                      launch_k(prefill_attn_kernel, grid, dim3(kPThreads), smem, stream, tmk, tmv, (const bf16*)q,
                               (bf16*)out, block_tables, max_blocks, seq_rows, cu_q, ctx_start, num_q_heads,
                               num_kv_heads, block_size, num_blocks, n_qtiles, scale * kLog2e, device_error_ptr()));
}

}  // extern "C"
