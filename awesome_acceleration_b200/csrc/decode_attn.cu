// Paged-KV decode attention (one query token per sequence, GQA).
//
// Work decomposition: one CTA per (context split, kv head, sequence).  A
// dedicated producer warp streams 64-token K and V tiles of the split from
// the paged pool into a STAGES-deep shared-memory ring with TMA tensor copies
// (128-byte swizzle, completion on mbarriers).  Four consumer warps each own
// 16 tokens of every tile and compute S = Q K^T and O += P V with
// mma.sync m16n8k16 (the G query heads that share the kv head are the rows of
// the A operand), keeping an online softmax in fp32.  The four partial
// (max, sum, O) triples are merged in shared memory; a split either writes
// the final bf16 output (single split) or an fp32 partial, and the last
// split CTA of a (sequence, kv head) to finish, found with an atomic counter
// in the workspace, merges the partials in split order and resets the
// counter (no separate combine launch).
//
// The kernel is HBM-bound: each K/V byte of the context is read once per
// kv head.  Algorithmic bytes per call = sum(ctx) * Hkv * 128 * 2 * 2.
#include <mutex>

#include "common.cuh"
#include "host.h"

namespace aacc {

constexpr int kD = 128;
constexpr int kTile = 64;
constexpr int kConsumerWarps = 4;
constexpr int kDecodeThreads = (kConsumerWarps + 1) * 32;
constexpr int kDecodeStages = 3;
constexpr int kHalfTileBytes = kTile * 64 * 2;  // 64 rows x 64 dims bf16 = 8 KB

struct DecodeSmem {
  // [stage][K half0, K half1, V half0, V half1], each 8 KB, 1024-aligned.
  bf16 tiles[kDecodeStages][4][kTile * 64];
  uint64_t full[kDecodeStages];
  uint64_t empty[kDecodeStages];
  float red_m[kConsumerWarps][8];
  float red_l[kConsumerWarps][8];
  int abort;
};

template <int G>
__global__ void __launch_bounds__(kDecodeThreads, 2)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                        const bf16* __restrict__ q, bf16* __restrict__ out, float* __restrict__ ws_o,
                        float* __restrict__ ws_ml, const int32_t* __restrict__ bt, int64_t max_blocks,
                        const int64_t* __restrict__ rows, const int32_t* __restrict__ seqlens, int ctx_add,
                        int Hkv, int bs, int64_t num_blocks, int64_t max_ctx, int split_tokens, int max_splits,
                        float scale_log2, int* __restrict__ cnt, unsigned* err) {
  extern __shared__ uint8_t smem_raw[];
  DecodeSmem& sm = *reinterpret_cast<DecodeSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  griddep_wait();  // q, the new K/V rows and seqlens come from the previous kernels
  griddep_launch();

  const int s = blockIdx.x, h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int Hq = Hkv * G;
  const int64_t row = rows[b];
  int64_t ctx = row < 0 ? 0 : (int64_t)seqlens[row] + ctx_add;  // negative rows are padding
  if (ctx > max_ctx) {  // max_ctx <= max_blocks * bs and <= max_splits * split_tokens
    if (threadIdx.x == 0 && s == 0) report(err, ERR_CTX_OOB);
    ctx = max_ctx;
  }
  if (ctx <= 0) {
    // Nothing to attend to: define the output as zeros.
    if (s == 0)
      for (int i = threadIdx.x; i < G * kD; i += blockDim.x)
        out[(b * Hq + (int64_t)h * G) * kD + i] = tobf(0.f);
    return;
  }
  const int n_splits = (int)((ctx + split_tokens - 1) / split_tokens);
  if (s >= n_splits) return;
  const int64_t t_begin = (int64_t)s * split_tokens;
  const int64_t t_end = min(t_begin + split_tokens, ctx);
  const int ntiles = (int)((t_end - t_begin + kTile - 1) / kTile);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kDecodeStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kConsumerWarps);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  volatile int* abort = &sm.abort;

  if (warp == kConsumerWarps) {
    // ---------------- producer warp ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      const int32_t* btrow = bt + row * max_blocks;
      // K/V tiles are read exactly once: evict_first keeps them from
      // displacing the projection weights held in L2 across the attention.
      const uint64_t pol = policy_evict_first();
      int issued = 0;
      for (int i = 0; i < ntiles; ++i) {
        const int st = i % kDecodeStages;
        if (i >= kDecodeStages && !mbar_wait(&sm.empty[st], ((i / kDecodeStages) - 1) & 1, err, abort)) break;
        const int64_t t0 = t_begin + (int64_t)i * kTile;
        int64_t blk = btrow[t0 / bs];
        if (blk < 0 || blk >= num_blocks) {
          report(err, ERR_BLOCK_OOB);
          blk = 0;  // keep the pipeline moving on a valid address; the result is flagged
        }
        const int r = (int)((blk * Hkv + h) * bs + t0 % bs);
        mbar_arrive_expect_tx(&sm.full[st], 4 * kHalfTileBytes);
        tma_load_2d_hint(sm.tiles[st][0], &tmk, &sm.full[st], 0, r, pol);
        tma_load_2d_hint(sm.tiles[st][1], &tmk, &sm.full[st], 64, r, pol);
        tma_load_2d_hint(sm.tiles[st][2], &tmv, &sm.full[st], 0, r, pol);
        tma_load_2d_hint(sm.tiles[st][3], &tmv, &sm.full[st], 64, r, pol);
        ++issued;
      }
      // Drain: every copy this CTA issued has landed before the CTA may exit.
      for (int st = 0; st < kDecodeStages && st < issued; ++st) {
        const int last = st + ((issued - 1 - st) / kDecodeStages) * kDecodeStages;
        mbar_wait(&sm.full[st], (last / kDecodeStages) & 1, err, nullptr);
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int g = lane >> 2, c = lane & 3;
  // Q as the A operand: rows = the G query heads of this kv head (rows >= G are zero).
  uint32_t qa[8][4];
  {
    const bf16* qrow = q + (b * Hq + (int64_t)h * G + (g < G ? g : 0)) * kD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t lo = 0, hi = 0;
      if (g < G) {
        lo = *reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 2 * c);
        hi = *reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 2 * c + 8);
      }
      qa[kk][0] = lo;
      qa[kk][1] = 0;
      qa[kk][2] = hi;
      qa[kk][3] = 0;
    }
  }
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;

  const int mi = lane >> 3, r8 = lane & 7;
  const int ktok = 16 * warp + (mi >> 1) * 8 + r8;  // K ldmatrix row (token within tile)
  const int vtok = 16 * warp + (mi & 1) * 8 + r8;   // V ldmatrix row
  bool ok = true;
  for (int i = 0; i < ntiles; ++i) {
    const int st = i % kDecodeStages;
    if (!mbar_wait(&sm.full[st], (i / kDecodeStages) & 1, err, abort)) {
      ok = false;
      break;
    }
    const uint32_t kb = smem_u32(sm.tiles[st][0]);
    const uint32_t vb = smem_u32(sm.tiles[st][2]);
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int chunk = 2 * kk + (mi & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kb + (chunk >> 3) * kHalfTileBytes + swz128(ktok, chunk & 7), b0, b1, b2, b3);
      mma_bf16_16816(sc[0], qa[kk], b0, b1);
      mma_bf16_16816(sc[1], qa[kk], b2, b3);
    }
    const int64_t tbase = t_begin + (int64_t)i * kTile + 16 * warp + 2 * c;
    float x[4];
    x[0] = (tbase + 0 < t_end) ? sc[0][0] * scale_log2 : -INFINITY;
    x[1] = (tbase + 1 < t_end) ? sc[0][1] * scale_log2 : -INFINITY;
    x[2] = (tbase + 8 < t_end) ? sc[1][0] * scale_log2 : -INFINITY;
    x[3] = (tbase + 9 < t_end) ? sc[1][1] * scale_log2 : -INFINITY;
    float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = exp2f(m_run - m_use);
    float p[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) p[j] = exp2f(x[j] - m_use);
    l_run = l_run * alpha + (p[0] + p[1] + p[2] + p[3]);
    m_run = m_new;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= alpha;
      o[j][1] *= alpha;
    }
    uint32_t pa[4];
    pa[0] = pack_bf16(p[0], p[1]);
    pa[1] = 0;
    pa[2] = pack_bf16(p[2], p[3]);
    pa[3] = 0;
#pragma unroll
    for (int jp = 0; jp < 8; ++jp) {
      const int chunk = 2 * jp + (mi >> 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vb + (chunk >> 3) * kHalfTileBytes + swz128(vtok, chunk & 7), b0, b1, b2, b3);
      mma_bf16_16816(o[2 * jp], pa, b0, b1);
      mma_bf16_16816(o[2 * jp + 1], pa, b2, b3);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[st]);
  }
  // Quad-reduce the row sum (all four lanes of a quad hold the same running max).
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);

  // Merge the four consumer warps through shared memory (reusing the tile ring).
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32));
  float* red_o = reinterpret_cast<float*>(&sm.tiles[0][0][0]);  // [warp][G][128]
  if (g < G) {
    if (c == 0) {
      sm.red_m[warp][g] = ok ? m_run : -INFINITY;
      sm.red_l[warp][g] = ok ? l_run : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      red_o[(warp * G + g) * kD + 8 * j + 2 * c] = o[j][0];
      red_o[(warp * G + g) * kD + 8 * j + 2 * c + 1] = o[j][1];
    }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32));
  const int d = threadIdx.x;  // 0..127
#pragma unroll
  for (int gg = 0; gg < G; ++gg) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm.red_m[w][gg]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float f = exp2f(sm.red_m[w][gg] - Mu);
      L += f * sm.red_l[w][gg];
      O += f * red_o[(w * G + gg) * kD + d];
    }
    const int64_t qh = b * Hq + (int64_t)h * G + gg;
    if (n_splits == 1) {
      out[qh * kD + d] = tobf(L > 0.f ? O / L : 0.f);
    } else {
      ws_o[(qh * max_splits + s) * kD + d] = O;
      if (d == 0) {
        ws_ml[(qh * max_splits + s) * 2 + 0] = M;
        ws_ml[(qh * max_splits + s) * 2 + 1] = L;
      }
    }
  }
  if (n_splits == 1 || cnt == nullptr) return;
  // The last split CTA of this (sequence, kv head) to finish merges all
  // splits (threadfence-reduction pattern) and resets the counter to zero.
  __threadfence();
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32));
  __shared__ int s_last;
  if (d == 0) {
    const int prev = atomicAdd(&cnt[b * Hkv + h], 1);
    s_last = (prev == n_splits - 1);
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32));
  if (!s_last) return;
  __threadfence();
#pragma unroll
  for (int gg = 0; gg < G; ++gg) {
    const int64_t qh = b * Hq + (int64_t)h * G + gg;
    const volatile float* ml = ws_ml + qh * max_splits * 2;
    const volatile float* po = ws_o + qh * max_splits * kD;
    float M = -INFINITY;
    for (int t = 0; t < n_splits; ++t) M = fmaxf(M, ml[2 * t]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float L = 0.f, O = 0.f;
    for (int t = 0; t < n_splits; ++t) {
      const float f = exp2f(ml[2 * t] - Mu);
      L += f * ml[2 * t + 1];
      O += f * po[t * kD + d];
    }
    out[qh * kD + d] = tobf(L > 0.f ? O / L : 0.f);
  }
  if (d == 0) cnt[b * Hkv + h] = 0;
}

// Context tokens one CTA streams: as few splits as keep ~8 CTAs per SM in
// flight, at most 2048 tokens.  Every extra split costs a CTA's set-up and a
// partial (O, max, sum) written and merged; the cap bounds the imbalance
// between rows of very different lengths.  Measured on the B200 (same-box
// A/B): cfg2 engine step, attention only, ctx 1536: 7.70 ms at 512-token
// splits, 6.76 ms at 2048; cfg3 (ctx U[512,4096]): 6.02 / 6.40 / 6.45 /
// 6.36 TB/s at 512 / 1024 / 2048 / unsplit.
static int default_split(int64_t batch, int Hkv, int64_t max_ctx) {
  const int64_t target = 148 * 8;  // CTAs to keep every SM busy (two resident, several waves)
  int64_t want = (target + batch * Hkv - 1) / (batch * Hkv);
  int64_t split = (max_ctx + want - 1) / want;
  split = ((split + kTile - 1) / kTile) * kTile;
  if (split < kTile) split = kTile;
  if (split > 2048) split = 2048;
  return (int)split;
}

static size_t decode_smem_bytes() { return sizeof(DecodeSmem) + 1024; }

// Argument checks shared by both decode-attention entry points; they run
// before either one touches the device or the stream.
static int decode_check(const char* what, int64_t batch, int64_t num_blocks, int64_t max_blocks, int num_q_heads,
                        int num_kv_heads, int block_size, int64_t max_context, int split_tokens) {
  if (batch < 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads || block_size <= 0 ||
      block_size % kTile || num_blocks <= 0 || max_blocks <= 0 || max_context <= 0)
    return set_error(AACC_ERR_INVALID, "%s: bad sizes", what);
  const int G = num_q_heads / num_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8)
    return set_error(AACC_ERR_UNSUPPORTED, "%s: q/kv head ratio %d not in {1,2,4,8}", what, G);
  if (num_blocks * num_kv_heads * block_size >= (int64_t(1) << 31))
    return set_error(AACC_ERR_UNSUPPORTED, "%s: pool too large", what);
  if (split_tokens > 0 && split_tokens % kTile)
    return set_error(AACC_ERR_INVALID, "%s: split_tokens must be a multiple of %d", what, kTile);
  return AACC_OK;
}

}  // namespace aacc

using namespace aacc;

extern "C" {

int64_t aacc_paged_decode_workspace_bytes(int64_t batch, int num_q_heads, int64_t max_context, int split_tokens) {
  if (split_tokens <= 0) split_tokens = default_split(batch, 1, max_context);  // upper bound on splits
  int64_t max_splits = (max_context + split_tokens - 1) / split_tokens;
  if (max_splits < 1) max_splits = 1;
  // partial O | partial (max, sum) | one merge counter per (row, kv head) (<= q heads)
  return batch * num_q_heads * max_splits * (kD + 2) * (int64_t)sizeof(float) +
         batch * num_q_heads * (int64_t)sizeof(int);
}

int aacc_paged_decode_attention(const void* q, void* out, const void* k_cache, const void* v_cache, int64_t num_blocks,
                                const int32_t* block_tables, int64_t max_blocks, const int64_t* slot_indices,
                                const int32_t* seqlens, int ctx_add, int64_t batch, int num_q_heads,
                                int num_kv_heads, int block_size, float scale, int split_tokens,
                                int64_t max_context, void* workspace, int64_t workspace_bytes,
                                cudaStream_t stream) {
  int st = decode_check("paged_decode_attention", batch, num_blocks, max_blocks, num_q_heads, num_kv_heads,
                        block_size, max_context, split_tokens);
  if (st || batch == 0) return st;
  const int G = num_q_heads / num_kv_heads;
  if (max_context > max_blocks * block_size) max_context = max_blocks * block_size;
  const int64_t rows = num_blocks * num_kv_heads * block_size;
  if (split_tokens <= 0) split_tokens = default_split(batch, num_kv_heads, max_context);
  const int max_splits = (int)((max_context + split_tokens - 1) / split_tokens);
  if (max_splits > 1) {
    const int64_t need = batch * num_q_heads * (int64_t)max_splits * (kD + 2) * (int64_t)sizeof(float) +
                         batch * num_kv_heads * (int64_t)sizeof(int);
    if (!workspace || workspace_bytes < need)
      return set_error(AACC_ERR_INVALID, "paged_decode_attention: workspace %lld < %lld bytes",
                       (long long)workspace_bytes, (long long)need);
  }
  CUtensorMap tmk, tmv;
  st = make_tmap_2d(&tmk, k_cache, kD, rows, kD * 2, 64, kTile, true);
  if (st) return st;
  st = make_tmap_2d(&tmv, v_cache, kD, rows, kD * 2, 64, kTile, true);
  if (st) return st;
  float* ws_o = static_cast<float*>(workspace);
  float* ws_ml = ws_o ? ws_o + batch * num_q_heads * (int64_t)max_splits * kD : nullptr;
  int* cnt = ws_ml ? reinterpret_cast<int*>(ws_ml + batch * num_q_heads * (int64_t)max_splits * 2) : nullptr;
  const float scale_log2 = scale * kLog2e;
  unsigned* err = device_error_ptr();
  dim3 grid(max_splits, num_kv_heads, (unsigned)batch);
  const size_t smem = decode_smem_bytes();
  cudaError_t le;
#define AACC_LAUNCH_DECODE(GG)                                                                                     \
  {                                                                                                                \
    set_smem_once<paged_decode_kernel<GG>>((int)smem);                                                             \
    le = launch_k(paged_decode_kernel<GG>, grid, dim3(kDecodeThreads), smem, stream, tmk, tmv, (const bf16*)q,     \
                  (bf16*)out, ws_o, ws_ml, block_tables, max_blocks, slot_indices, seqlens, ctx_add, num_kv_heads, \
                  block_size, num_blocks, max_context, split_tokens, max_splits, scale_log2, cnt, err);            \
  }
  switch (G) {
    case 1: AACC_LAUNCH_DECODE(1) break;
    case 2: AACC_LAUNCH_DECODE(2) break;
    case 4: AACC_LAUNCH_DECODE(4) break;
    default: AACC_LAUNCH_DECODE(8) break;
  }
#undef AACC_LAUNCH_DECODE
  return check_launch("paged_decode_kernel", le);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot allocate device memory at all: a plugin run by a host
// runtime that owns every device allocation and forbids its plugins to call
// cudaMalloc, or a service that must keep a fixed device-memory footprint
// after start-up.  For them aacc_paged_decode_attention_noalloc takes no
// workspace: its split partials and merge counters live in the file-scope
// array below, of fixed size kNoAllocScratchBytes, which every GPU that loads
// this library holds until the process exits.  The first call on a device
// (with that device current) looks up the array's device address with
// cudaGetSymbolAddress, so make that first call before any stream capture.
// Every call on a device shares the one array and leaves its last contents
// behind; the merge counters, the only part that must start at zero, are
// cleared on the caller's stream before each launch.  Calls that overlap on
// the GPU (different streams, concurrently) race on the array.
// ---------------------------------------------------------------------------
namespace aacc {

constexpr int64_t kNoAllocScratchBytes = int64_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64];

static int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64)
    return set_error(AACC_ERR_CUDA, "paged_decode_attention_noalloc: no current device (%s)",
                     cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(AACC_ERR_CUDA, "paged_decode_attention_noalloc: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return AACC_OK;
}

}  // namespace aacc

extern "C" {

int64_t aacc_paged_decode_noalloc_capacity_bytes(void) { return kNoAllocScratchBytes; }

int aacc_paged_decode_attention_noalloc(const void* q, void* out, const void* k_cache, const void* v_cache,
                                        int64_t num_blocks, const int32_t* block_tables, int64_t max_blocks,
                                        const int64_t* slot_indices, const int32_t* seqlens, int ctx_add,
                                        int64_t batch, int num_q_heads, int num_kv_heads, int block_size,
                                        float scale, int split_tokens, int64_t max_context, cudaStream_t stream) {
  // Every argument check comes before the scratch lookup and the counter
  // clear, so a rejected call leaves nothing on the caller's stream.
  int st = decode_check("paged_decode_attention_noalloc", batch, num_blocks, max_blocks, num_q_heads, num_kv_heads,
                        block_size, max_context, split_tokens);
  if (st || batch == 0) return st;
  // The same split plan as aacc_paged_decode_attention, to size the scratch.
  int64_t ctx = max_context > max_blocks * block_size ? max_blocks * block_size : max_context;
  const int split = split_tokens > 0 ? split_tokens : default_split(batch, num_kv_heads, ctx);
  const int64_t max_splits = (ctx + split - 1) / split;
  const int64_t partial_bytes = batch * num_q_heads * max_splits * (kD + 2) * (int64_t)sizeof(float);
  const int64_t counter_bytes = batch * num_kv_heads * (int64_t)sizeof(int);
  if (max_splits > 1 && partial_bytes + counter_bytes > kNoAllocScratchBytes)
    return set_error(AACC_ERR_INVALID,
                     "paged_decode_attention_noalloc: %lld rows x %d q heads x %lld splits need %lld bytes of "
                     "scratch; the static scratch holds %lld bytes (use aacc_paged_decode_attention with a "
                     "workspace, or fewer rows / a larger split_tokens)",
                     (long long)batch, num_q_heads, (long long)max_splits,
                     (long long)(partial_bytes + counter_bytes), (long long)kNoAllocScratchBytes);
  void* scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st) return st;
  if (max_splits > 1) {
    cudaError_t e = cudaMemsetAsync(static_cast<char*>(scratch) + partial_bytes, 0, counter_bytes, stream);
    if (e != cudaSuccess)
      return set_error(AACC_ERR_CUDA, "paged_decode_attention_noalloc: clearing counters: %s", cudaGetErrorString(e));
  }
  return aacc_paged_decode_attention(q, out, k_cache, v_cache, num_blocks, block_tables, max_blocks, slot_indices,
                                     seqlens, ctx_add, batch, num_q_heads, num_kv_heads, block_size, scale, split,
                                     ctx, scratch, kNoAllocScratchBytes, stream);
}

}  // extern "C"
