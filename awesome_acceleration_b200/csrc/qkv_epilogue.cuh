// Warp-cooperative epilogue of the fused QKV projection for one (token, head):
// per-head q/k RMSNorm (model/model.py:219-222, rounding as RMSNorm.forward,
// :47-52), RoPE on Q and K (:80-92, bf16 table, pairs (i, i+64)), then Q to
// q_out and K/V straight into the paged KV cache.  Lane l holds the fp32
// projection sums of head columns 4l..4l+3.  Shared by the split-K epilogue
// kernel and the cluster split-K GEMM, so both round at the same points.
#pragma once
#include "common.cuh"

namespace aacc {

struct QkvEpi {
  const bf16* qn_w;
  const bf16* kn_w;
  float eps;
  const int64_t* positions;
  const bf16* rope;  // [max_pos][128] = cos[64] | sin[64]
  int64_t max_pos;
  const int64_t* slot_mapping;
  bf16* q_out;  // [M][Hq][128]
  bf16* k_cache;
  bf16* v_cache;
  int64_t num_slots;
  int Hq, Hkv, bs;
  unsigned* err;
};

__device__ __forceinline__ void qkv_head_epilogue(const float (&acc)[4], int lane, int64_t m, int hh,
                                                  const QkvEpi& a) {
  const int c = 4 * lane;  // column within the head
  float x[4] = {rbf(acc[0]), rbf(acc[1]), rbf(acc[2]), rbf(acc[3])};
  const bool is_q = hh < a.Hq, is_k = !is_q && hh < a.Hq + a.Hkv;
  bf16* dst = nullptr;
  if (is_q) {
    dst = a.q_out + (m * a.Hq + hh) * 128;
  } else {
    const int64_t slot = a.slot_mapping[m];
    if (slot >= a.num_slots && lane == 0) report(a.err, ERR_SLOT_OOB);
    if (slot >= 0 && slot < a.num_slots) {
      const int kvh = is_k ? hh - a.Hq : hh - a.Hq - a.Hkv;
      dst = (is_k ? a.k_cache : a.v_cache) + (((slot / a.bs) * a.Hkv + kvh) * a.bs + slot % a.bs) * 128;
    }
  }
  if (is_q || is_k) {
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / 128.f + a.eps);
    const bf16* nw = (is_q ? a.qn_w : a.kn_w) + c;
    float y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) y[i] = rbf(bf(nw[i]) * rbf(x[i] * r));
    int64_t pos = a.positions[m];
    if (pos < 0 || pos >= a.max_pos) {
      if (lane == 0) report(a.err, ERR_POS_OOB);
      pos = 0;
    }
    const int ci = c & 63;  // frequency index (the table's cos/sin repeat every 64 columns)
    const bf16* cs = a.rope + pos * 128;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float partner = __shfl_xor_sync(0xffffffffu, y[i], 16);  // column c+i +/- 64
      const float cv = bf(cs[ci + i]), sv = bf(cs[64 + ci + i]);
      x[i] = (c < 64) ? rbf(y[i] * cv) + rbf(-partner * sv) : rbf(y[i] * cv) + rbf(partner * sv);
    }
  }
  if (dst) {
    uint2 o;
    o.x = pack_bf16(x[0], x[1]);
    o.y = pack_bf16(x[2], x[3]);
    *reinterpret_cast<uint2*>(dst + c) = o;
  }
}

// bf16(silu(bf16(g))) * bf16(u) (model/model.py:189-190, MLP.forward's eager bf16 ops).
__device__ __forceinline__ float silu_mul(float g, float u) {
  const float gg = rbf(g);
  return rbf(gg / (1.0f + expf(-gg))) * rbf(u);
}

}  // namespace aacc
