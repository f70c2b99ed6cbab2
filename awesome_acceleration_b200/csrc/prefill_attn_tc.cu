// Causal (chunked) prefill attention over the paged KV cache on tcgen05 /
// TMEM: the B200 form of flash_attn_varlen_func (llm.py:178-184) for a chunk
// whose K/V are already stored in the paged pool.
//
// A work item is a pair of query tiles of one (sequence, kv head); one
// persistent CTA per SM walks its items (see FlashItems).  A tile's 128 MMA
// rows are 128 / G query positions times the G query heads that share the kv
// head (row r = position p * G + head g, P = 128 / G), so every K/V byte is
// read once per kv head, not once per query head; the two tiles (A: positions
// [qs, qs + P), B: the next P) share every K/V tile.  Each Q tile arrives by
// TMA as two 3-D boxes (64 dims x G heads x P tokens) next to the first K
// tile.  Per 128-key tile:
//
//   producer warp   TMA: K and V tiles (two 64-column halves each, 128-byte
//                   swizzle) from the paged pool into a ring of three 32 KB
//                   slots, K one tile ahead of V (K0 K1 V0 K2 V1 K3 V2 ...);
//                   a slot is free once both tiles' MMA issuers released it;
//   MMA warps       one issuing thread per tile: S_t(i+1) = Q_t K_{i+1}^T
//                   into tile t's TMEM score columns as soon as tile t's
//                   softmax group has read S_t(i) into registers (so it runs
//                   under that group's exponentials), and O_t += P_t(i) V_i
//                   into its TMEM accumulator once the group has written P
//                   (V read as an MN-major operand, in place);
//   softmax groups  4 warps per tile, one thread per row: S from TMEM, causal
//                   mask key_pos <= query_pos (query p of the chunk sits at
//                   ctx_start + tile start + p) on the tiles that cross the
//                   diagonal, fp32 online softmax in base 2 (SFU exponential),
//                   P rounded to bf16 into the tile's own P buffer (as
//                   FlashAttention-2 rounds P before the PV product), so
//                   neither group waits for the other's P.V; at the
//                   end O / l out.  The reference maximum of a row moves only
//                   when the row's running maximum exceeds it by more than
//                   2^8 (in exp2 units, as FlashAttention-4 does): P stays
//                   <= 256, O / l is the same quotient, and the O rescale in
//                   TMEM (a read-modify-write on the critical path) is rare.
//
// TMEM: S_A | S_B | O_A | O_B (128 columns each).
//
// Every wait is bounded; a wait that runs out reports ERR_WAIT_TIMEOUT and
// the CTA stops issuing work, drains its own copies and frees TMEM.
#include <algorithm>

#include "common.cuh"
#include "host.h"
#include "tcgen05.cuh"

namespace aacc {

constexpr int kFD = 128;            // head dim
constexpr int kFKeys = 128;         // keys per K/V tile
constexpr int kFSlots = 3;          // K/V ring: 32 KB slots holding K0 K1 V0 K2 V1 ...
constexpr int kFGroupWarps = 4;     // one softmax group: a thread per MMA row of one query tile
constexpr int kFSoftmaxWarps = 2 * kFGroupWarps;
constexpr int kFThreads = (kFSoftmaxWarps + 3) * 32;  // + producer, + one MMA issuer per tile
constexpr int kFHalf = 128 * 128;   // bytes of one 64-column half of a 128-row bf16 tile
constexpr float kFRescaleLog2 = 8.f;  // move a row's reference maximum when exp2 would exceed 2^8

struct FlashSmem {
  uint8_t kv[kFSlots][2][kFHalf];   // a K or V tile: 128 keys x 128 dims as two 64-dim halves
  uint8_t q[2][2][kFHalf];          // two query tiles: 128 rows x 128 dims as two 64-dim halves
  uint8_t p[2][2][kFHalf];          // per tile, P: 128 rows x 128 keys as two 64-key halves
  uint64_t full[kFSlots];
  uint64_t empty[kFSlots];
  uint64_t q_full;                  // the item's Q tiles landed
  uint64_t q_free;                  // the item's last S done: Q buffers may be refilled
  uint64_t s_full[2];               // per tile: S ready
  uint64_t s_free[2];               // per tile: S read into registers (its TMEM may be overwritten)
  uint64_t p_full[2];               // per tile: P written, O corrected
  uint64_t pv_done[2];              // per tile: O += P V done
  uint64_t o_free[2];               // per tile: the item's O read out of TMEM
  uint32_t tmem_slot;
  int abort;
};

// 2^x with the SFU's approximate exponential (PTX ex2.approx.ftz.f32); 2^-inf = 0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One work item: a pair of query tiles of one (sequence, kv head).  Items run
// pair-major, heaviest (latest positions, most key tiles) first: item j has
// pair n_pairs - 1 - j / (Hkv * n_seqs).  Returns false for a pair past the
// end of its sequence's chunk.
struct FlashItem {
  int64_t q0, c0, row;
  int kvh, qs0, q_len, rows_a, rows_b, nt_a, nt_b, nkv;
  bool have_b, clamped;
};

template <int P>
__device__ __forceinline__ bool flash_item(int j, int n_pairs, int Hkv, int n_seqs, const int32_t* __restrict__ cu_q,
                                           const int32_t* __restrict__ ctx_start,
                                           const int64_t* __restrict__ seq_rows, int64_t kv_cap, FlashItem& it) {
  const int per_pair = Hkv * n_seqs;
  const int pair = n_pairs - 1 - j / per_pair, rem = j % per_pair;
  const int s = rem / Hkv;
  it.kvh = rem % Hkv;
  it.q0 = cu_q[s];
  it.q_len = cu_q[s + 1] - (int)it.q0;
  it.qs0 = pair * 2 * P;  // tile A: positions [qs0, qs0 + P); tile B: the next P
  if (it.qs0 >= it.q_len) return false;
  it.c0 = ctx_start[s];
  it.row = seq_rows[s];
  it.rows_a = min(P, it.q_len - it.qs0);
  it.rows_b = it.qs0 + P < it.q_len ? min(P, it.q_len - it.qs0 - P) : 0;
  it.nt_a = (int)((it.c0 + it.qs0 + it.rows_a - 1) / kFKeys) + 1;
  it.nt_b = it.rows_b ? (int)((it.c0 + it.qs0 + P + it.rows_b - 1) / kFKeys) + 1 : 0;
  it.clamped = it.nt_a > kv_cap || it.nt_b > kv_cap;
  it.nt_a = min(it.nt_a, (int)kv_cap);
  it.nt_b = min(it.nt_b, (int)kv_cap);
  it.have_b = it.nt_b > 0;
  it.nkv = max(it.nt_a, it.nt_b);
  return true;
}

// The items of this CTA in snake order: round r takes item r * gridDim.x + k
// with k = blockIdx.x on even rounds and gridDim.x - 1 - blockIdx.x on odd
// ones, which evens out the heaviest-first sequence across CTAs.
template <int P>
struct FlashItems {
  int r = 0;
  __device__ __forceinline__ bool next(FlashItem& it, int n_items, int n_pairs, int Hkv, int n_seqs,
                                       const int32_t* cu_q, const int32_t* ctx_start, const int64_t* seq_rows,
                                       int64_t kv_cap) {
    const int G = gridDim.x, k = blockIdx.x;
    while (r * G < n_items) {
      const int j = r * G + ((r & 1) ? G - 1 - k : k);
      ++r;
      if (j < n_items && flash_item<P>(j, n_pairs, Hkv, n_seqs, cu_q, ctx_start, seq_rows, kv_cap, it)) return true;
    }
    return false;
  }
};

// Persistent: one CTA per SM walks its items (FlashItems);
// barriers and TMEM are set up once, and every barrier's phase runs on across
// items, so an item's loads and first S start while the previous item's
// softmax groups finish and store O.
template <int G>
__global__ void __launch_bounds__(kFThreads, 1)
    flash_prefill_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                         const __grid_constant__ CUtensorMap tmq, bf16* __restrict__ out, const int32_t* __restrict__ bt,
                         int64_t max_blocks, const int64_t* __restrict__ seq_rows, const int32_t* __restrict__ cu_q,
                         const int32_t* __restrict__ ctx_start, int Hq, int Hkv, int bs, int64_t num_blocks,
                         int n_pairs, int n_seqs, float scale_log2, unsigned* err) {
  constexpr int P = 128 / G;  // query positions per tile
  extern __shared__ uint8_t smem_raw[];
  FlashSmem& sm = *reinterpret_cast<FlashSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  griddep_wait();
  griddep_launch();
  const int n_items = n_pairs * Hkv * n_seqs;
  const int64_t kv_cap = max_blocks * bs / kFKeys;  // key tiles the block table can hold
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kFSlots; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 2);  // one arrival per tile's MMA issuer
    }
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_free, 2);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.s_free[t], kFGroupWarps * 32);
      mbar_init(&sm.p_full[t], kFGroupWarps * 32);
      mbar_init(&sm.pv_done[t], 1);
      mbar_init(&sm.o_free[t], kFGroupWarps * 32);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == kFSoftmaxWarps + 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_slot)),
                 "r"(512u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_slot;  // S_A | S_B | O_A | O_B, 128 columns each
  volatile int* abort = &sm.abort;

  if (warp == kFSoftmaxWarps) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      int U = 0, nq = 0;  // K/V units issued, items whose Q was loaded (running over items)
      bool ok = true;
      FlashItems<P> items;
      FlashItem it;
      while (ok && items.next(it, n_items, n_pairs, Hkv, n_seqs, cu_q, ctx_start, seq_rows, kv_cap)) {
        if (it.clamped) report(err, ERR_CTX_OOB);
        // Q tiles (K-major, 128-byte swizzle; row = position * G + head), once
        // the previous item's last S has read the buffers.  Rows past the
        // chunk hold other tokens (or zeros past the last) and are never stored.
        if (nq > 0 && !(ok = mbar_wait(&sm.q_free, (nq - 1) & 1, err, abort))) break;
        mbar_arrive_expect_tx(&sm.q_full, (it.have_b ? 4 : 2) * kFHalf);
        for (int t = 0; t < (it.have_b ? 2 : 1); ++t)
          for (int h = 0; h < 2; ++h)
            tma_load_3d(sm.q[t][h], &tmq, &sm.q_full, 64 * h, it.kvh * G, (int)(it.q0 + it.qs0 + t * P));
        ++nq;
        const int32_t* btrow = bt + it.row * max_blocks;
        // unit u of the item: K_0, then K_{j+1}, V_j for j = 0 .. nkv-2, then V_{nkv-1}
        for (int u = 0; u < 2 * it.nkv; ++u) {
          const int sl = U % kFSlots;
          if (U >= kFSlots && !(ok = mbar_wait(&sm.empty[sl], ((U / kFSlots) - 1) & 1, err, abort))) break;
          const int w = u - 1;
          const bool is_v = u > 0 && (w >= 2 * (it.nkv - 1) || (w & 1));
          const int tile = u == 0 ? 0 : (w >= 2 * (it.nkv - 1) ? it.nkv - 1 : (w >> 1) + (is_v ? 0 : 1));
          const int64_t t0 = (int64_t)tile * kFKeys;
          int64_t blk = btrow[t0 / bs];
          if (blk < 0 || blk >= num_blocks) {
            report(err, ERR_BLOCK_OOB);
            blk = 0;
          }
          const int r = (int)((blk * Hkv + it.kvh) * bs + t0 % bs);
          const CUtensorMap* tm = is_v ? &tmv : &tmk;
          mbar_arrive_expect_tx(&sm.full[sl], 2 * kFHalf);
          tma_load_2d(sm.kv[sl][0], tm, &sm.full[sl], 0, r);
          tma_load_2d(sm.kv[sl][1], tm, &sm.full[sl], 64, r);
          ++U;
        }
      }
      // No copy in flight at exit (normally the MMA thread has waited for all).
      if (nq > 0) mbar_wait(&sm.q_full, (nq - 1) & 1, err, nullptr);
      for (int sl = 0; sl < kFSlots && sl < U; ++sl) {
        const int last = sl + ((U - 1 - sl) / kFSlots) * kFSlots;
        mbar_wait(&sm.full[sl], (last / kFSlots) & 1, err, nullptr);
      }
    }
  } else if (warp > kFSoftmaxWarps) {
    // ---------------- MMA issuers: warp 9 for tile A, warp 10 for tile B ----------------
    // Each walks its item's K/V units in ring order -- K_0 K_1 V_0 K_2 V_1 ...
    // V_{nkv-1}, which is also its issue order S(0) S(1) PV(0) S(2) PV(1) ... --
    // issuing S_t(j) for K_j (once its group has read the previous scores)
    // and PV_t(j) for V_j (once its group has written P(j); the item's first
    // PV also once the group has read the previous item's O), and releasing
    // every unit on the ring's two-arrival empty barrier, with a plain
    // arrival for units its tile does not use.  The two tiles never wait for
    // each other.
    const int t = warp - kFSoftmaxWarps - 1;
    if (lane == 0) {
      constexpr uint32_t id_s = umma_idesc_m128(kFKeys, false);  // S = Q K^T: both K-major (over dims)
      constexpr uint32_t id_pv = umma_idesc_m128(kFD, true);     // O += P V: V is N(dims)-major
      auto wait_bar = [&](uint64_t* bar, int phase) -> bool {
        if (!mbar_wait(bar, phase & 1, err, abort)) return false;
        tc_fence_after();
        return true;
      };
      const uint32_t qb = smem_u32(sm.q[t][0]), pb = smem_u32(sm.p[t][0]);
      const uint32_t tS = tmem + 128 * t, tO = tmem + 256 + 128 * t;
      // running counts over items: units, items, waits on s_free / p_full / o_free, items with this tile
      int V = 0, nq = 0, nsf = 0, npf = 0, nof = 0, seen = 0;
      bool ok = true;
      FlashItems<P> items;
      FlashItem it;
      while (ok && items.next(it, n_items, n_pairs, Hkv, n_seqs, cu_q, ctx_start, seq_rows, kv_cap)) {
        const int nkv = it.nkv, nt = t ? it.nt_b : it.nt_a;  // nt_b = 0 when the item has no tile B
        if (!(ok = wait_bar(&sm.q_full, nq++))) break;
        if (nt == 0) mbar_arrive(&sm.q_free);  // this tile reads no Q in this item
        for (int u = 0; ok && u < 2 * nkv; ++u) {
          const int w = u - 1;
          const bool is_v = u > 0 && (w >= 2 * (nkv - 1) || (w & 1));
          const int j = u == 0 ? 0 : (w >= 2 * (nkv - 1) ? nkv - 1 : (w >> 1) + (is_v ? 0 : 1));
          const int uu = V++;
          if (!(ok = wait_bar(&sm.full[uu % kFSlots], uu / kFSlots))) break;
          if (j >= nt) {
            mbar_arrive(&sm.empty[uu % kFSlots]);  // a key tile past this tile's diagonal
            continue;
          }
          const uint32_t kv = smem_u32(sm.kv[uu % kFSlots][0]);
          if (!is_v) {
            if ((j > 0 || seen) && !(ok = wait_bar(&sm.s_free[t], nsf++))) break;  // S_t read
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {  // 16 dims per step
              const uint32_t off = (uint32_t)((kk >> 2) * kFHalf + (kk & 3) * 32);
              umma_bf16(tS, umma_desc_sw128(qb + off), umma_desc_sw128(kv + off), id_s, kk != 0);
            }
            umma_commit(&sm.s_full[t]);
            if (j == nt - 1) umma_commit(&sm.q_free);  // this tile's last S of the item
          } else {
            if (j == 0 && seen && !(ok = wait_bar(&sm.o_free[t], nof++))) break;  // previous O read
            if (!(ok = wait_bar(&sm.p_full[t], npf++))) break;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {  // 16 keys per step
              const uint64_t a = umma_desc_sw128(pb + (uint32_t)((kk >> 2) * kFHalf + (kk & 3) * 32));
              const uint64_t b = umma_desc_sw128_mn(kv + (uint32_t)(kk * 16 * 128), kFHalf);
              umma_bf16(tO, a, b, id_pv, (j | kk) != 0);
            }
            umma_commit(&sm.pv_done[t]);
          }
          umma_commit(&sm.empty[uu % kFSlots]);
        }
        if (nt > 0) ++seen;
      }
    }
  } else {
    // ---------------- softmax groups: group t = tile t, thread = row = TMEM lane ----------------
    // Rows past the end of the chunk are never stored and each MMA row is
    // independent, so they need no masking: only tiles that cross the causal
    // diagonal are masked.  The running maximum is kept on raw scores (the
    // scale is positive), so each exponent is one FFMA + EX2.
    const int t = warp / kFGroupWarps, r = threadIdx.x % 128, p = r / G, g = r % G;
    const uint32_t lane_off = (uint32_t)((warp % kFGroupWarps) * 32) << 16;
    const uint32_t tS = tmem + 128 * t, tO = tmem + 256 + 128 * t;
    int nsf = 0, npd = 0;  // waits on s_full / pv_done (running over items)
    bool ok = true;
    FlashItems<P> items;
    FlashItem it;
    while (ok && items.next(it, n_items, n_pairs, Hkv, n_seqs, cu_q, ctx_start, seq_rows, kv_cap)) {
      if (t == 1 && !it.have_b) continue;
      const int qs = it.qs0 + t * P, ntiles = t ? it.nt_b : it.nt_a;
      const bool row_valid = p < (t ? it.rows_b : it.rows_a);
      const int pos = (int)(it.c0 + qs + p), pos_min = (int)(it.c0 + qs);
      bf16* const dst = out + ((it.q0 + qs + p) * Hq + (int64_t)it.kvh * G + g) * kFD;
      float m = -INFINITY, l = 0.f;
      for (int i = 0; i < ntiles; ++i) {
        if (!mbar_wait(&sm.s_full[t], (nsf++) & 1, err, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[kFKeys];
        uint32_t srow = tS + lane_off;
        asm volatile("" : "+r"(srow));
#pragma unroll
        for (int c = 0; c < kFKeys / 32; ++c) tmem_ld32_async(srow + 32 * c, sv + 32 * c);
        tmem_wait_ld();
        tmem_pin(sv);
        tc_fence_before();
        mbar_arrive(&sm.s_free[t]);  // the MMA may now overwrite S_t with the next scores
        const int k0 = i * kFKeys;
        if (k0 + kFKeys - 1 > pos_min) {  // tile crosses the diagonal (warp-uniform)
#pragma unroll
          for (int jj = 0; jj < kFKeys; ++jj)
            if (k0 + jj > pos) sv[jj] = -INFINITY;
        }
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int jj = 0; jj < kFKeys; jj += 4) {
#pragma unroll
          for (int u = 0; u < 4; ++u) mx[u] = fmaxf(mx[u], sv[jj + u]);
        }
        // m: the row's reference maximum (raw score); it moves to the tile's
        // maximum only when that exceeds it by more than 8 / scale_log2.
        const float m_tile = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        const float m_new = (m_tile - m) * scale_log2 > kFRescaleLog2 ? m_tile : m;  // m = -inf: moves
        const float msc = (m_new == -INFINITY ? 0.f : m_new) * scale_log2;
        const float alpha = m_new == m ? 1.f : fast_exp2(fmaf(m, scale_log2, -msc));  // m = -inf: 0
        float rs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int jj = 0; jj < kFKeys; jj += 4) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            sv[jj + u] = fast_exp2(fmaf(sv[jj + u], scale_log2, -msc));
            rs[u] += sv[jj + u];
          }
        }
        l = l * alpha + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
        m = m_new;
        // This tile's previous P.V must be done: it reads this tile's P
        // buffer and updates O, which a rescale reads below.
        if (i > 0) {
          if (!mbar_wait(&sm.pv_done[t], (npd++) & 1, err, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (i > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {  // tcgen05.ld/st are warp-wide
#pragma unroll 1
          for (int c = 0; c < kFD / 16; ++c) {
            float ov[16];
            tmem_ld16(tO + lane_off + 16 * c, ov);
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) ov[jj] *= alpha;
            tmem_st16(tO + lane_off + 16 * c, ov);
          }
          tmem_wait_st();
        }
        {
          // row base in the tile's P buffer, recomputed per step (kept out of
          // registers across the loop); 16-byte chunk c of the row lands at
          // chunk (c ^ row) % 8 of its 64-key half (128-byte swizzle)
          uint32_t prow = smem_u32(sm.p[t][0]) + (uint32_t)r * 128u;
          asm volatile("" : "+r"(prow));
          const uint32_t r7 = (uint32_t)(r & 7);
#pragma unroll
          for (int c = 0; c < 16; ++c) {  // 8 keys per 16-byte chunk
            const uint32_t addr = prow + (uint32_t)(c >> 3) * kFHalf + ((((uint32_t)c & 7u) ^ r7) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr),
                         "r"(pack_bf16(sv[8 * c + 0], sv[8 * c + 1])), "r"(pack_bf16(sv[8 * c + 2], sv[8 * c + 3])),
                         "r"(pack_bf16(sv[8 * c + 4], sv[8 * c + 5])), "r"(pack_bf16(sv[8 * c + 6], sv[8 * c + 7]))
                         : "memory");
          }
        }
        fence_proxy_async();
        tc_fence_before();
        mbar_arrive(&sm.p_full[t]);
      }
      if (!ok) break;
      // ---------------- item epilogue: O / l, then O's TMEM is free ----------------
      if (!mbar_wait(&sm.pv_done[t], (npd++) & 1, err, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float il = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {  // 64 columns per TMEM round trip
        float ov[64];
        tmem_ld32_async(tO + lane_off + 64 * h, ov);
        tmem_ld32_async(tO + lane_off + 64 * h + 32, ov + 32);
        tmem_wait_ld();
        tmem_pin(ov);
        if (h == 1) {  // O is in registers: the next item's first P.V may overwrite it
          tc_fence_before();
          mbar_arrive(&sm.o_free[t]);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float o16[16];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) o16[jj] = ov[16 * c + jj] * il;
          if (row_valid) store16_bf16(dst + 64 * h + 16 * c, o16);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kFSoftmaxWarps + 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
  }
}

}  // namespace aacc

using namespace aacc;

extern "C" int aacc_prefill_attention_mma(const void* q, void* out, const void* k_cache, const void* v_cache,
                                          int64_t num_blocks, const int32_t* block_tables, int64_t max_blocks,
                                          const int64_t* seq_rows, const int32_t* cu_q, const int32_t* ctx_start,
                                          int64_t num_seqs, int64_t max_q_len, int num_q_heads, int num_kv_heads,
                                          int block_size, float scale, cudaStream_t stream);

namespace aacc {
static bool prefill_use_mma() {
  static const bool on = [] {
    const char* v = getenv("AACC_PREFILL_ATTN");
    return v && v[0] == 'm';
  }();
  return on;
}
}  // namespace aacc

extern "C" {

int aacc_prefill_attention(const void* q, void* out, int64_t num_tokens, const void* k_cache, const void* v_cache,
                           int64_t num_blocks, const int32_t* block_tables, int64_t max_blocks, const int64_t* seq_rows,
                           const int32_t* cu_q, const int32_t* ctx_start, int64_t num_seqs, int64_t max_q_len,
                           int num_q_heads, int num_kv_heads, int block_size, float scale, cudaStream_t stream) {
  if (num_seqs < 0 || max_q_len < 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || block_size <= 0 ||
      block_size % 64 || num_blocks <= 0 || max_blocks <= 0 || num_tokens < 0 || max_q_len > num_tokens)
    return set_error(AACC_ERR_INVALID, "prefill_attention: bad sizes");
  const int G = num_q_heads / num_kv_heads;
  // The tensor-core kernel takes 128-key tiles (block sizes that are multiples
  // of 128) and 1, 2, 4 or 8 query heads per kv head; the mma.sync kernel
  // covers 64-token blocks and other ratios.
  if (block_size % kFKeys || (G != 1 && G != 2 && G != 4 && G != 8) || prefill_use_mma())
    return aacc_prefill_attention_mma(q, out, k_cache, v_cache, num_blocks, block_tables, max_blocks, seq_rows, cu_q,
                                      ctx_start, num_seqs, max_q_len, num_q_heads, num_kv_heads, block_size, scale,
                                      stream);
  if (num_seqs == 0 || max_q_len == 0) return AACC_OK;
  if (num_seqs > 65535 || num_tokens >= (int64_t(1) << 31))
    return set_error(AACC_ERR_UNSUPPORTED, "prefill_attention: too many sequences or tokens per call");
  const int64_t rows = num_blocks * num_kv_heads * block_size;
  if (rows >= (int64_t(1) << 31)) return set_error(AACC_ERR_UNSUPPORTED, "prefill_attention: pool too large");
  if (!aligned16(q) || !aligned16(out)) return set_error(AACC_ERR_INVALID, "prefill_attention: q/out must be 16-byte aligned");
  const int P = 128 / G;
  CUtensorMap tmk, tmv, tmq;
  int st = make_tmap_2d(&tmk, k_cache, kFD, rows, kFD * 2, 64, kFKeys, true);
  if (st) return st;
  st = make_tmap_2d(&tmv, v_cache, kFD, rows, kFD * 2, 64, kFKeys, true);
  if (st) return st;
  // q as [token][head][dim]: boxes of 64 dims x G heads x P tokens
  st = make_tmap_3d(&tmq, q, kFD, num_q_heads, num_tokens, kFD * 2, (uint64_t)num_q_heads * kFD * 2, 64, G, P, true);
  if (st) return st;
  const int n_pairs = (int)((max_q_len + 2 * P - 1) / (2 * P));
  const int64_t n_items = (int64_t)n_pairs * num_kv_heads * num_seqs;
  if (n_items >= (int64_t(1) << 31)) return set_error(AACC_ERR_UNSUPPORTED, "prefill_attention: too many work items");
  const size_t smem = sizeof(FlashSmem) + 1024;
  dim3 grid((unsigned)std::min<int64_t>(n_items, sm_count()));
  cudaError_t le;
#define AACC_LAUNCH_FLASH(GG)                                                                                      \
  {                                                                                                                \
    set_smem_once<flash_prefill_kernel<GG>>((int)smem);                                                            \
    le = launch_k(flash_prefill_kernel<GG>, grid, dim3(kFThreads), smem, stream, tmk, tmv, tmq,                    \
                  (bf16*)out, block_tables, max_blocks, seq_rows, cu_q, ctx_start, num_q_heads, num_kv_heads,       \
                  block_size, num_blocks, n_pairs, (int)num_seqs, scale * kLog2e, device_error_ptr());             \
  }
  switch (G) {
    case 1: AACC_LAUNCH_FLASH(1) break;
    case 2: AACC_LAUNCH_FLASH(2) break;
    case 4: AACC_LAUNCH_FLASH(4) break;
    default: AACC_LAUNCH_FLASH(8) break;
  }
#undef AACC_LAUNCH_FLASH
  return check_launch("flash_prefill_kernel", le);
}

}  // extern "C"
