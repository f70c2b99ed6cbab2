// Epilogues of split-K decode GEMMs: sum the fp32 partials (split order),
// then apply the same epilogue math as the fused GEMM epilogues, rounding at
// the reference's points.
//
//   splitk_qkv_kernel:  per (token, head) warp, lane l owns columns 4l..4l+3:
//                       q/k RMSNorm over the head (warp reduction), RoPE
//                       pairs (i, i+64) across lanes l and l^16, stores Q to
//                       q_out and K/V rows into the paged cache.
//   splitk_silu_kernel: bf16(silu(bf16(gate))) * bf16(up) over gate/up rows
//                       interleaved in groups of 64.
#include "common.cuh"
#include "host.h"
#include "qkv_epilogue.cuh"

namespace aacc {

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

__global__ void __launch_bounds__(128)
    splitk_qkv_kernel(const float* __restrict__ part, int S, int64_t M, QkvEpi a) {
  griddep_wait();
  griddep_launch();
  const int heads = a.Hq + 2 * a.Hkv;
  const int64_t item = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (item >= M * heads) return;
  const int lane = threadIdx.x & 31;
  const int64_t m = item / heads;
  const int hh = (int)(item % heads);
  const int64_t N = (int64_t)heads * 128;
  const float* src = part + m * N + (int64_t)hh * 128 + 4 * lane;
  float4 s4 = ld4(src);
#pragma unroll 8  // several splits' loads in flight; additions stay in split order
  for (int s = 1; s < S; ++s) {
    const float4 b = ld4(src + (int64_t)s * M * N);
    s4.x += b.x;
    s4.y += b.y;
    s4.z += b.z;
    s4.w += b.w;
  }
  const float acc[4] = {s4.x, s4.y, s4.z, s4.w};
  qkv_head_epilogue(acc, lane, m, hh, a);
}

__global__ void splitk_silu_kernel(const float* __restrict__ part, int S, int64_t M, int64_t I,
                                   bf16* __restrict__ out) {
  // one thread = 8 consecutive output columns of one row
  griddep_wait();
  griddep_launch();
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t per_row = I / 8;
  if (t >= M * per_row) return;
  const int64_t m = t / per_row;
  const int64_t j = (t % per_row) * 8;
  const int64_t N = 2 * I;
  const int64_t gcol = (j / 64) * 128 + (j % 64);
  const float* g0 = part + m * N + gcol;
  float g[8], u[8];
  {
    float4 a = ld4(g0), b = ld4(g0 + 4), c = ld4(g0 + 64), d = ld4(g0 + 68);
    g[0] = a.x; g[1] = a.y; g[2] = a.z; g[3] = a.w; g[4] = b.x; g[5] = b.y; g[6] = b.z; g[7] = b.w;
    u[0] = c.x; u[1] = c.y; u[2] = c.z; u[3] = c.w; u[4] = d.x; u[5] = d.y; u[6] = d.z; u[7] = d.w;
  }
#pragma unroll 8
  for (int s = 1; s < S; ++s) {
    const float* gs = g0 + (int64_t)s * M * N;
    float4 a = ld4(gs), b = ld4(gs + 4), c = ld4(gs + 64), d = ld4(gs + 68);
    g[0] += a.x; g[1] += a.y; g[2] += a.z; g[3] += a.w; g[4] += b.x; g[5] += b.y; g[6] += b.z; g[7] += b.w;
    u[0] += c.x; u[1] += c.y; u[2] += c.z; u[3] += c.w; u[4] += d.x; u[5] += d.y; u[6] += d.z; u[7] += d.w;
  }
  float r[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) r[i] = silu_mul(g[i], u[i]);
  uint4 o;
  o.x = pack_bf16(r[0], r[1]);
  o.y = pack_bf16(r[2], r[3]);
  o.z = pack_bf16(r[4], r[5]);
  o.w = pack_bf16(r[6], r[7]);
  *reinterpret_cast<uint4*>(out + m * I + j) = o;
}

}  // namespace aacc

using namespace aacc;

extern "C" {

int aacc_splitk_qkv_norm_rope_store(const float* partial, int splits, const void* q_norm_w, const void* k_norm_w,
                                    float eps, const int64_t* positions, const void* rope_cos_sin, int64_t max_pos,
                                    const int64_t* slot_mapping, void* q_out, void* k_cache, void* v_cache,
                                    int64_t num_blocks, int num_q_heads, int num_kv_heads, int block_size, int64_t M,
                                    cudaStream_t stream) {
  if (M < 0 || splits < 1 || num_q_heads <= 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks <= 0 ||
      max_pos <= 0)
    return set_error(AACC_ERR_INVALID, "splitk_qkv_norm_rope_store: bad sizes");
  if (M == 0) return AACC_OK;
  if (!aligned16(partial) || !aligned16(q_out) || !aligned16(k_cache) || !aligned16(v_cache))
    return set_error(AACC_ERR_INVALID, "splitk_qkv_norm_rope_store: pointers must be 16-byte aligned");
  const int64_t items = M * (num_q_heads + 2 * num_kv_heads);
  QkvEpi a{(const bf16*)q_norm_w, (const bf16*)k_norm_w, eps, positions, (const bf16*)rope_cos_sin, max_pos,
           slot_mapping, (bf16*)q_out, (bf16*)k_cache, (bf16*)v_cache, num_blocks * block_size, num_q_heads,
           num_kv_heads, block_size, device_error_ptr()};
  return check_launch("splitk_qkv_norm_rope_store",
                      launch_k(splitk_qkv_kernel, dim3((unsigned)((items + 3) / 4)), dim3(128), 0, stream, partial,
                               splits, M, a));
}

int aacc_splitk_silu_mul(const float* partial, int splits, void* out, int64_t M, int64_t I, cudaStream_t stream) {
  if (M < 0 || I <= 0 || I % 64 || splits < 1 || !aligned16(partial) || !aligned16(out))
    return set_error(AACC_ERR_INVALID, "splitk_silu_mul: I must be a multiple of 64, pointers 16-byte aligned");
  if (M == 0) return AACC_OK;
  const int64_t n = M * I / 8;
  return check_launch("splitk_silu_mul", launch_k(splitk_silu_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256),
                                                  0, stream, partial, splits, M, I, (bf16*)out));
}

}  // extern "C"
