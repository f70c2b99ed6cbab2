// Paged KV-cache store and the per-step slot bookkeeping kernels.
#include "common.cuh"
#include "host.h"

namespace aacc {

// One warp per (token, kv head): lanes 0-15 move the 256-byte K row, lanes
// 16-31 the V row, 16 bytes each.
__global__ void kv_store_kernel(const bf16* __restrict__ k, const bf16* __restrict__ v, int64_t T,
                                int64_t ks, int64_t vs, const int64_t* __restrict__ slot_mapping,
                                bf16* __restrict__ kc, bf16* __restrict__ vc, int64_t num_slots, int Hkv,
                                int bs, unsigned* err) {
  griddep_wait();
  griddep_launch();
  int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (warp >= T * Hkv) return;
  int64_t t = warp / Hkv;
  int h = (int)(warp % Hkv);
  int64_t slot = slot_mapping[t];
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (lane == 0) report(err, ERR_SLOT_OOB);
    return;
  }
  int64_t blk = slot / bs, off = slot % bs;
  int64_t dst = ((blk * Hkv + h) * bs + off) * 128;
  int c = lane & 15;
  if (lane < 16) {
    const uint4* src = reinterpret_cast<const uint4*>(k + t * ks + (int64_t)h * 128) + c;
    reinterpret_cast<uint4*>(kc + dst)[c] = *src;
  } else {
    const uint4* src = reinterpret_cast<const uint4*>(v + t * vs + (int64_t)h * 128) + c;
    reinterpret_cast<uint4*>(vc + dst)[c] = *src;
  }
}

__global__ void decode_slot_mapping_kernel(const int64_t* __restrict__ rows, const int32_t* __restrict__ seqlens,
                                           const int32_t* __restrict__ bt, int64_t max_blocks, int bs,
                                           int64_t num_blocks, int64_t* __restrict__ out, int64_t B,
                                           unsigned* err) {
  griddep_wait();
  griddep_launch();
  int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int64_t row = rows[b];
  if (row < 0) {  // padding row of a bucketed batch: no cache slot
    out[b] = -1;
    return;
  }
  int64_t n = seqlens[row];
  int64_t j = n / bs;
  if (j >= max_blocks) {
    report(err, ERR_CTX_OOB);
    out[b] = -1;
    return;
  }
  int64_t blk = bt[row * max_blocks + j];
  if (blk < 0 || blk >= num_blocks) {
    report(err, ERR_BLOCK_OOB);
    out[b] = -1;
    return;
  }
  out[b] = blk * bs + n % bs;
}

__global__ void advance_seqlens_kernel(const int64_t* __restrict__ rows, int32_t* __restrict__ seqlens,
                                       int64_t* __restrict__ positions, int64_t B) {
  griddep_wait();
  griddep_launch();
  int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B && rows[b] >= 0) {  // negative rows are padding
    atomicAdd(&seqlens[rows[b]], 1);
    if (positions) positions[b] += 1;
  }
}

// dst[i] = src[idx[i]] for rows of `row_bytes` bytes (16-byte multiple).
__global__ void gather_rows_kernel(const uint4* __restrict__ src, const int64_t* __restrict__ idx, int64_t n_src,
                                   int64_t vec_per_row, uint4* __restrict__ dst, unsigned* err) {
  griddep_wait();
  griddep_launch();
  const int64_t i = blockIdx.x;
  int64_t r = idx[i];
  if (r < 0 || r >= n_src) {
    if (threadIdx.x == 0) report(err, ERR_SLOT_OOB);
    r = 0;
  }
  for (int64_t v = threadIdx.x; v < vec_per_row; v += blockDim.x) dst[i * vec_per_row + v] = src[r * vec_per_row + v];
}

}  // namespace aacc

using namespace aacc;

extern "C" {

int aacc_kv_store(const void* k, const void* v, int64_t num_tokens, int64_t k_row_stride, int64_t v_row_stride,
                  const int64_t* slot_mapping, void* k_cache, void* v_cache, int64_t num_blocks, int num_kv_heads,
                  int block_size, cudaStream_t stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || block_size <= 0 || num_blocks <= 0)
    return set_error(AACC_ERR_INVALID, "kv_store: bad sizes");
  if (num_tokens == 0) return AACC_OK;
  if (!aligned16(k) || !aligned16(v) || !aligned16(k_cache) || !aligned16(v_cache) || (k_row_stride % 8) ||
      (v_row_stride % 8))
    return set_error(AACC_ERR_INVALID, "kv_store: pointers/strides must be 16-byte aligned");
  int64_t warps = num_tokens * num_kv_heads;
  int threads = 256;
  int64_t blocks = (warps + 7) / 8;
  return check_launch("kv_store", launch_k(kv_store_kernel, dim3((unsigned)blocks), dim3(threads), 0, stream,
                                           (const bf16*)k, (const bf16*)v, num_tokens, k_row_stride, v_row_stride,
                                           slot_mapping, (bf16*)k_cache, (bf16*)v_cache, num_blocks * block_size,
                                           num_kv_heads, block_size, device_error_ptr()));
}

int aacc_decode_slot_mapping(const int64_t* slot_indices, const int32_t* seqlens, const int32_t* block_tables,
                             int64_t max_blocks, int block_size, int64_t num_blocks, int64_t* slot_mapping_out,
                             int64_t batch, cudaStream_t stream) {
  if (batch < 0 || max_blocks <= 0 || block_size <= 0) return set_error(AACC_ERR_INVALID, "slot_mapping: bad sizes");
  if (batch == 0) return AACC_OK;
  return check_launch("decode_slot_mapping",
                      launch_k(decode_slot_mapping_kernel, dim3((unsigned)((batch + 127) / 128)), dim3(128), 0,
                               stream, slot_indices, seqlens, block_tables, max_blocks, block_size, num_blocks,
                               slot_mapping_out, batch, device_error_ptr()));
}

int aacc_gather_rows(const void* src, int64_t n_src, int64_t row_bytes, const int64_t* idx, int64_t n, void* dst,
                     cudaStream_t stream) {
  if (n < 0 || n_src <= 0 || row_bytes <= 0 || row_bytes % 16 || !aligned16(src) || !aligned16(dst))
    return set_error(AACC_ERR_INVALID, "gather_rows: rows must be 16-byte multiples and aligned");
  if (n == 0) return AACC_OK;
  return check_launch("gather_rows", launch_k(gather_rows_kernel, dim3((unsigned)n), dim3(128), 0, stream,
                                              (const uint4*)src, idx, n_src, row_bytes / 16, (uint4*)dst,
                                              device_error_ptr()));
}

int aacc_advance_seqlens(const int64_t* slot_indices, int32_t* seqlens, int64_t* positions, int64_t batch,
                         cudaStream_t stream) {
  if (batch < 0) return set_error(AACC_ERR_INVALID, "advance_seqlens: bad batch");
  if (batch == 0) return AACC_OK;
  return check_launch("advance_seqlens", launch_k(advance_seqlens_kernel, dim3((unsigned)((batch + 127) / 128)),
                                                  dim3(128), 0, stream, slot_indices, seqlens, positions, batch));
}

}  // extern "C"
