// Row-wise RMSNorm building blocks shared by the norm kernels and the
// tensor-parallel exchange kernel, so that every path rounds identically:
// fp32 sum of squares (per-thread in column order, then warp butterfly, then
// warps in order), x * rsqrt(mean + eps) rounded to bf16, then the bf16
// weight multiply rounded to bf16 (model/model.py:47-52).
//
// Thread layout: min(128, hidden/8) threads per row; thread t owns the
// 8-column vectors v * threads + t for v < V = hidden / (8 * threads).
#pragma once

#include "common.cuh"

namespace aacc {

constexpr int kNormMaxThreads = 128;

template <int V>
__device__ __forceinline__ void norm_row(float (&x)[V * 8], const bf16* __restrict__ w, bf16* __restrict__ y,
                                         float eps, int hidden) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < V * 8; ++i) ss += x[i] * x[i];
  __shared__ float red[kNormMaxThreads / 32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)hidden + eps);
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int col = (v * blockDim.x + threadIdx.x) * 8;
    uint4 wv = *reinterpret_cast<const uint4*>(w + col);
    const uint32_t* wu = reinterpret_cast<const uint32_t*>(&wv);
    uint4 ov;
    uint32_t* ou = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 wf = unpack_bf16(wu[j]);
      float a = rbf(x[v * 8 + 2 * j] * r), b2 = rbf(x[v * 8 + 2 * j + 1] * r);
      ou[j] = pack_bf16(wf.x * a, wf.y * b2);
    }
    *reinterpret_cast<uint4*>(y + col) = ov;
  }
}

template <int V>
__device__ __forceinline__ void load_row(float (&x)[V * 8], const bf16* __restrict__ src) {
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int col = (v * blockDim.x + threadIdx.x) * 8;
    uint4 u = *reinterpret_cast<const uint4*>(src + col);
    const uint32_t* p = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = unpack_bf16(p[j]);
      x[v * 8 + 2 * j] = f.x;
      x[v * 8 + 2 * j + 1] = f.y;
    }
  }
}

// Sum the split-K partials of 8 consecutive columns (split order, fp32).
// The loop is unrolled so that several splits' loads are in flight at once;
// the additions keep split order.
__device__ __forceinline__ void sum_partials8(const float* __restrict__ part, int S, int64_t split_stride, float (&d)[8]) {
  float4 a = reinterpret_cast<const float4*>(part)[0], b = reinterpret_cast<const float4*>(part)[1];
  d[0] = a.x; d[1] = a.y; d[2] = a.z; d[3] = a.w; d[4] = b.x; d[5] = b.y; d[6] = b.z; d[7] = b.w;
#pragma unroll 8
  for (int s = 1; s < S; ++s) {
    a = reinterpret_cast<const float4*>(part + s * split_stride)[0];
    b = reinterpret_cast<const float4*>(part + s * split_stride)[1];
    d[0] += a.x; d[1] += a.y; d[2] += a.z; d[3] += a.w; d[4] += b.x; d[5] += b.y; d[6] += b.z; d[7] += b.w;
  }
}

inline int norm_shape(int64_t rows, int64_t hidden, const char* what, int* threads, int* V) {
  if (rows < 0 || hidden < 256 || hidden % 256 || (hidden > 1024 && hidden % 1024) || hidden > 8192)
    return set_error(AACC_ERR_UNSUPPORTED, "%s: hidden %lld must be 256..1024 in steps of 256 or a multiple of 1024 "
                     "up to 8192", what, (long long)hidden);
  if (rows > 0x7fffffff) return set_error(AACC_ERR_INVALID, "%s: too many rows", what);
  *threads = hidden >= 1024 ? 128 : (int)(hidden / 8);
  *V = (int)(hidden / (8 * *threads));
  return AACC_OK;
}

}  // namespace aacc
