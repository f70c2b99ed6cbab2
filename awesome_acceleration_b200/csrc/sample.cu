// Greedy and temperature sampling over materialised logits, and the
// vocab-parallel argmax merge.
#include "common.cuh"
#include "host.h"
#include "sample.cuh"

namespace aacc {

__device__ __forceinline__ void better(float& bv, int64_t& bi, float v, int64_t i) {
  if (v > bv || (v == bv && i < bi)) {
    bv = v;
    bi = i;
  }
}

__device__ __forceinline__ void block_argmax(float& bv, int64_t& bi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t i = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, v, i);
  }
  __shared__ float sv[32];
  __shared__ int64_t si[32];
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k) better(bv, bi, sv[k], si[k]);
}

// torch.argmax semantics on bf16 rows: highest value, first index on ties.
__global__ void argmax_rows_kernel(const bf16* __restrict__ logits, int64_t vocab, int64_t* __restrict__ tokens) {
  griddep_wait();
  griddep_launch();
  const int64_t m = blockIdx.x;
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  const bf16* row = logits + m * vocab;
  for (int64_t n = threadIdx.x; n < vocab; n += blockDim.x) better(bv, bi, bf(row[n]), n);
  block_argmax(bv, bi);
  if (threadIdx.x == 0) tokens[m] = bi == INT64_MAX ? 0 : bi;
}

// Temperature sampling over materialised bf16 logits: the same Gumbel-max
// draw (and noise) as the lm_head epilogue; rows with T <= 0 stay greedy.
__global__ void sample_rows_kernel(const bf16* __restrict__ logits, int64_t vocab, const float* __restrict__ temp,
                                   const int64_t* __restrict__ seeds, const int64_t* __restrict__ counters,
                                   int64_t* __restrict__ tokens) {
  griddep_wait();
  griddep_launch();
  const int64_t m = blockIdx.x;
  const float t = temp[m];
  const uint64_t key = sample_key(seeds[m], counters[m]);
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  const bf16* row = logits + m * vocab;
  for (int64_t n = threadIdx.x; n < vocab; n += blockDim.x) {
    const float x = bf(row[n]);
    better(bv, bi, t > 0.f ? rbf(x / t) + gumbel_noise(key, (uint32_t)n) : x, n);
  }
  block_argmax(bv, bi);
  if (threadIdx.x == 0) tokens[m] = bi == INT64_MAX ? 0 : bi;
}

// Shard s's candidate of row m is (cv[s * sv + m], ci[s * si + m]).
__global__ void argmax_merge_kernel(const float* __restrict__ cv, const int64_t* __restrict__ ci, int shards,
                                    int64_t sv, int64_t si, int64_t* __restrict__ tokens) {
  griddep_wait();
  griddep_launch();
  const int64_t m = blockIdx.x;
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  for (int s = threadIdx.x; s < shards; s += blockDim.x) better(bv, bi, cv[s * sv + m], ci[s * si + m]);
  block_argmax(bv, bi);
  if (threadIdx.x == 0) tokens[m] = bi == INT64_MAX ? 0 : bi;
}

}  // namespace aacc

using namespace aacc;

extern "C" {

int aacc_argmax_rows(const void* logits, int64_t M, int64_t vocab, int64_t* tokens, cudaStream_t stream) {
  if (M < 0 || vocab <= 0) return set_error(AACC_ERR_INVALID, "argmax_rows: bad sizes");
  if (M == 0) return AACC_OK;
  return check_launch("argmax_rows", launch_k(argmax_rows_kernel, dim3((unsigned)M), dim3(512), 0, stream,
                                              (const bf16*)logits, vocab, tokens));
}

int aacc_sample_rows(const void* logits, int64_t M, int64_t vocab, const float* temperature, const int64_t* seeds,
                     const int64_t* counters, int64_t* tokens, cudaStream_t stream) {
  if (M < 0 || vocab <= 0 || (M > 0 && (!temperature || !seeds || !counters)))
    return set_error(AACC_ERR_INVALID, "sample_rows: bad sizes or missing temperature/seeds/counters");
  if (M == 0) return AACC_OK;
  return check_launch("sample_rows", launch_k(sample_rows_kernel, dim3((unsigned)M), dim3(512), 0, stream,
                                              (const bf16*)logits, vocab, temperature, seeds, counters, tokens));
}

int aacc_argmax_merge(const float* cand_val, const int64_t* cand_idx, int64_t M, int shards, int64_t* tokens,
                      cudaStream_t stream) {
  return aacc_argmax_merge_strided(cand_val, cand_idx, M, shards, M, M, tokens, stream);
}

int aacc_argmax_merge_strided(const float* cand_val, const int64_t* cand_idx, int64_t M, int shards,
                              int64_t val_shard_stride, int64_t idx_shard_stride, int64_t* tokens,
                              cudaStream_t stream) {
  if (M < 0 || shards <= 0 || val_shard_stride < M || idx_shard_stride < M)
    return set_error(AACC_ERR_INVALID, "argmax_merge: bad sizes or shard strides");
  if (M == 0) return AACC_OK;
  return check_launch("argmax_merge", launch_k(argmax_merge_kernel, dim3((unsigned)M), dim3(32), 0, stream, cand_val,
                                               cand_idx, shards, val_shard_stride, idx_shard_stride, tokens));
}

}  // extern "C"
