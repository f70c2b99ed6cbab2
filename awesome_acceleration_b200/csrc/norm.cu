// RMSNorm family: plain, fused residual-add + RMSNorm, and fused embedding
// gather + RMSNorm.  One CTA per row with min(128, hidden/8) threads; each
// thread keeps V x 8 values in registers (16-byte vector loads), V =
// hidden / (8 * threads).
//
// Rounding follows the eager reference (model/model.py:47-52): fp32 sum of
// squares, x * rsqrt(mean + eps) rounded to bf16, then the bf16 weight
// multiply rounded to bf16.  The residual add rounds to bf16 first
// (model/model.py:259, :265).
#include "common.cuh"
#include "host.h"
#include "norm_row.cuh"

namespace aacc {

// x[r][c] <- bf16(x[r][c] + bias[c]), 8 columns per thread (the eager bf16
// `output + self.bias` after the RowParallel all-reduce).
__global__ void bias_add_kernel(bf16* __restrict__ x, const bf16* __restrict__ bias, int64_t n8, int64_t cols8) {
  griddep_wait();
  griddep_launch();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  uint4 xv = reinterpret_cast<uint4*>(x)[i];
  const uint4 bv = reinterpret_cast<const uint4*>(bias)[i % cols8];
  uint32_t* xs = reinterpret_cast<uint32_t*>(&xv);
  const uint32_t* bs = reinterpret_cast<const uint32_t*>(&bv);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 a = unpack_bf16(xs[j]), b = unpack_bf16(bs[j]);
    xs[j] = pack_bf16(a.x + b.x, a.y + b.y);
  }
  reinterpret_cast<uint4*>(x)[i] = xv;
}

template <int V>
__global__ void __launch_bounds__(kNormMaxThreads) rmsnorm_kernel(const bf16* __restrict__ x,
                                                                  const bf16* __restrict__ w, bf16* __restrict__ y,
                                                                  int hidden, float eps) {
  griddep_wait();
  griddep_launch();
  const int64_t row = blockIdx.x;
  float v[V * 8];
  load_row<V>(v, x + row * hidden);
  norm_row<V>(v, w, y + row * hidden, eps, hidden);
}

template <int V>
__global__ void __launch_bounds__(kNormMaxThreads)
    add_rmsnorm_kernel(const bf16* __restrict__ delta, bf16* __restrict__ residual, const bf16* __restrict__ w,
                       bf16* __restrict__ y, int hidden, float eps) {
  griddep_wait();
  griddep_launch();
  const int64_t row = blockIdx.x;
  float a[V * 8], d[V * 8];
  load_row<V>(a, residual + row * hidden);
  load_row<V>(d, delta + row * hidden);
#pragma unroll
  for (int vv = 0; vv < V; ++vv) {
    const int col = (vv * blockDim.x + threadIdx.x) * 8;
    uint4 ov;
    uint32_t* ou = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = vv * 8 + 2 * j;
      a[i] = rbf(a[i] + d[i]);
      a[i + 1] = rbf(a[i + 1] + d[i + 1]);
      ou[j] = pack_bf16(a[i], a[i + 1]);
    }
    *reinterpret_cast<uint4*>(residual + row * hidden + col) = ov;
  }
  norm_row<V>(a, w, y + row * hidden, eps, hidden);
}

template <int V>
__global__ void __launch_bounds__(kNormMaxThreads)
    splitk_add_rmsnorm_kernel(const float* __restrict__ part, int S, int64_t rows, bf16* __restrict__ residual,
                              const bf16* __restrict__ w, bf16* __restrict__ y, int hidden, float eps) {
  griddep_wait();
  griddep_launch();
  const int64_t row = blockIdx.x;
  const int64_t stride = rows * hidden;
  float a[V * 8];
  load_row<V>(a, residual + row * hidden);
#pragma unroll
  for (int vv = 0; vv < V; ++vv) {
    const int col = (vv * blockDim.x + threadIdx.x) * 8;
    float d[8];
    sum_partials8(part + row * hidden + col, S, stride, d);
    uint4 ov;
    uint32_t* ou = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = vv * 8 + 2 * j;
      a[i] = rbf(a[i] + rbf(d[2 * j]));
      a[i + 1] = rbf(a[i + 1] + rbf(d[2 * j + 1]));
      ou[j] = pack_bf16(a[i], a[i + 1]);
    }
    *reinterpret_cast<uint4*>(residual + row * hidden + col) = ov;
  }
  norm_row<V>(a, w, y + row * hidden, eps, hidden);
}

__global__ void splitk_reduce_kernel(const float* __restrict__ part, int S, int64_t n8, int64_t stride,
                                     bf16* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float d[8];
  sum_partials8(part + i * 8, S, stride, d);
  uint4 ov;
  ov.x = pack_bf16(d[0], d[1]);
  ov.y = pack_bf16(d[2], d[3]);
  ov.z = pack_bf16(d[4], d[5]);
  ov.w = pack_bf16(d[6], d[7]);
  reinterpret_cast<uint4*>(out)[i] = ov;
}

template <int V>
__global__ void __launch_bounds__(kNormMaxThreads)
    embed_rmsnorm_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ table, int64_t vocab,
                         bf16* __restrict__ residual, const bf16* __restrict__ w, bf16* __restrict__ y, int hidden,
                         float eps, unsigned* err) {
  griddep_wait();
  griddep_launch();
  const int64_t row = blockIdx.x;
  int64_t id = ids[row];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) report(err, ERR_TOKEN_OOB);
    id = 0;
  }
  float a[V * 8];
  load_row<V>(a, table + id * hidden);
#pragma unroll
  for (int vv = 0; vv < V; ++vv) {
    const int col = (vv * blockDim.x + threadIdx.x) * 8;
    *reinterpret_cast<uint4*>(residual + row * hidden + col) =
        *reinterpret_cast<const uint4*>(table + id * hidden + col);
  }
  norm_row<V>(a, w, y + row * hidden, eps, hidden);
}

// threads = min(128, hidden/8) (a multiple of 32); V = hidden / (8 * threads).
}  // namespace aacc

using namespace aacc;

#define AACC_NORM_LAUNCH(KV, ...) le = launch_k(KV, dim3((unsigned)rows), dim3(threads), 0, stream, __VA_ARGS__)
#define AACC_NORM_DISPATCH(KERNEL, ...)                         \
  cudaError_t le;                                               \
  switch (V) {                                                  \
    case 1: AACC_NORM_LAUNCH(KERNEL<1>, __VA_ARGS__); break;    \
    case 2: AACC_NORM_LAUNCH(KERNEL<2>, __VA_ARGS__); break;    \
    case 3: AACC_NORM_LAUNCH(KERNEL<3>, __VA_ARGS__); break;    \
    case 4: AACC_NORM_LAUNCH(KERNEL<4>, __VA_ARGS__); break;    \
    case 5: AACC_NORM_LAUNCH(KERNEL<5>, __VA_ARGS__); break;    \
    case 6: AACC_NORM_LAUNCH(KERNEL<6>, __VA_ARGS__); break;    \
    case 7: AACC_NORM_LAUNCH(KERNEL<7>, __VA_ARGS__); break;    \
    default: AACC_NORM_LAUNCH(KERNEL<8>, __VA_ARGS__); break;   \
  }

extern "C" {

int aacc_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t hidden, float eps, cudaStream_t stream) {
  int threads, V;
  int st = norm_shape(rows, hidden, "rmsnorm", &threads, &V);
  if (st || rows == 0) return st;
  AACC_NORM_DISPATCH(rmsnorm_kernel, (const bf16*)x, (const bf16*)w, (bf16*)y, (int)hidden, eps)
  return check_launch("rmsnorm", le);
}

int aacc_add_rmsnorm(const void* delta, void* residual, const void* w, void* y, int64_t rows, int64_t hidden, float eps,
                     cudaStream_t stream) {
  int threads, V;
  int st = norm_shape(rows, hidden, "add_rmsnorm", &threads, &V);
  if (st || rows == 0) return st;
  AACC_NORM_DISPATCH(add_rmsnorm_kernel, (const bf16*)delta, (bf16*)residual, (const bf16*)w, (bf16*)y, (int)hidden,
                     eps)
  return check_launch("add_rmsnorm", le);
}

int aacc_splitk_add_rmsnorm(const float* partial, int splits, void* residual, const void* w, void* y, int64_t rows,
                            int64_t hidden, float eps, cudaStream_t stream) {
  int threads, V;
  int st = norm_shape(rows, hidden, "splitk_add_rmsnorm", &threads, &V);
  if (st || rows == 0) return st;
  if (splits < 1 || !aligned16(partial)) return set_error(AACC_ERR_INVALID, "splitk_add_rmsnorm: bad partials");
  AACC_NORM_DISPATCH(splitk_add_rmsnorm_kernel, partial, splits, rows, (bf16*)residual, (const bf16*)w, (bf16*)y,
                     (int)hidden, eps)
  return check_launch("splitk_add_rmsnorm", le);
}

int aacc_splitk_reduce(const float* partial, int splits, void* out, int64_t rows, int64_t cols, cudaStream_t stream) {
  if (rows < 0 || cols <= 0 || cols % 8 || splits < 1 || !aligned16(partial) || !aligned16(out))
    return set_error(AACC_ERR_INVALID, "splitk_reduce: cols must be a multiple of 8, pointers 16-byte aligned");
  if (rows == 0) return AACC_OK;
  const int64_t n8 = rows * cols / 8;
  return check_launch("splitk_reduce", launch_k(splitk_reduce_kernel, dim3((unsigned)((n8 + 255) / 256)), dim3(256),
                                                0, stream, partial, splits, n8, rows * cols, (bf16*)out));
}

int aacc_bias_add(void* x, const void* bias, int64_t rows, int64_t cols, cudaStream_t stream) {
  if (rows < 0 || cols <= 0 || cols % 8 || !aligned16(x) || !aligned16(bias))
    return set_error(AACC_ERR_INVALID, "bias_add: cols must be a multiple of 8, pointers 16-byte aligned");
  if (rows == 0) return AACC_OK;
  const int64_t n8 = rows * cols / 8;
  return check_launch("bias_add", launch_k(bias_add_kernel, dim3((unsigned)((n8 + 255) / 256)), dim3(256), 0, stream,
                                           (bf16*)x, (const bf16*)bias, n8, cols / 8));
}

int aacc_embed_rmsnorm(const int64_t* ids, const void* table, int64_t vocab, void* residual, const void* w, void* y,
                       int64_t rows, int64_t hidden, float eps, cudaStream_t stream) {
  int threads, V;
  int st = norm_shape(rows, hidden, "embed_rmsnorm", &threads, &V);
  if (st || rows == 0) return st;
  unsigned* err = device_error_ptr();
  AACC_NORM_DISPATCH(embed_rmsnorm_kernel, ids, (const bf16*)table, vocab, (bf16*)residual, (const bf16*)w, (bf16*)y,
                     (int)hidden, eps, err)
  return check_launch("embed_rmsnorm", le);
}

}  // extern "C"
