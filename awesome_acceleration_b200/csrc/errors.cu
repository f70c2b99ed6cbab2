// Host-side plumbing of the C ABI: status strings, the device error word and
// TMA tensor-map encoding.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "common.cuh"
#include "host.h"

namespace aacc {

__device__ unsigned g_device_error;

static thread_local char t_msg[512] = "ok";

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
  va_end(ap);
  return status;
}

static std::atomic<unsigned long long> g_launches{0};

int check_launch(const char* what, cudaError_t launch_status) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (launch_status != cudaSuccess) e = launch_status;
  if (e != cudaSuccess) return set_error(AACC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return AACC_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("AACC_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

static std::mutex g_mu;
static unsigned* g_err_ptr[64];

unsigned* device_error_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<unsigned*>(p);
  }
  return g_err_ptr[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int& c = cache[dev & 63];
  if (c == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    c = n;
  }
  return c;
}

static int load_encoder() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return set_error(AACC_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  return AACC_OK;
}

int make_tmap_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                 uint64_t stride2_bytes, uint32_t box0, uint32_t box1, uint32_t box2, bool swizzle128) {
  if (int st = load_encoder()) return st;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (stride1_bytes & 15) != 0 || (stride2_bytes & 15) != 0)
    return set_error(AACC_ERR_INVALID, "TMA operand must be 16-byte aligned (base %p, strides %llu %llu)", base,
                     (unsigned long long)stride1_bytes, (unsigned long long)stride2_bytes);
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(AACC_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu x %llu box %u x %u x %u",
                     (int)r, (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2, box0, box1, box2);
  return AACC_OK;
}

int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                 uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  if (int st = load_encoder()) return st;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (row_stride_bytes & 15) != 0)
    return set_error(AACC_ERR_INVALID, "TMA operand must be 16-byte aligned (base %p, row stride %llu)", base,
                     (unsigned long long)row_stride_bytes);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(AACC_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu box %u x %u", (int)r,
                     (unsigned long long)inner, (unsigned long long)outer, box_inner, box_outer);
  return AACC_OK;
}

}  // namespace aacc

extern "C" {

int aacc_version(void) { return 1; }

const char* aacc_last_error(void) { return aacc::t_msg; }

unsigned long long aacc_launch_count(void) { return aacc::g_launches.load(std::memory_order_relaxed); }

int aacc_get_device_error(unsigned* out) {
  if (!out) return aacc::set_error(AACC_ERR_INVALID, "null output");
  cudaError_t e = cudaMemcpyFromSymbol(out, aacc::g_device_error, sizeof(unsigned));
  if (e != cudaSuccess) return aacc::set_error(AACC_ERR_CUDA, "read device error: %s", cudaGetErrorString(e));
  return AACC_OK;
}

int aacc_get_device_error_async(unsigned* out, cudaStream_t stream) {
  if (!out) return aacc::set_error(AACC_ERR_INVALID, "null output");
  cudaError_t e = cudaMemcpyFromSymbolAsync(out, aacc::g_device_error, sizeof(unsigned), 0, cudaMemcpyDeviceToHost,
                                            stream);
  if (e != cudaSuccess) return aacc::set_error(AACC_ERR_CUDA, "read device error: %s", cudaGetErrorString(e));
  return AACC_OK;
}

int aacc_clear_device_error(void) {
  unsigned z = 0;
  cudaError_t e = cudaMemcpyToSymbol(aacc::g_device_error, &z, sizeof(unsigned));
  if (e != cudaSuccess) return aacc::set_error(AACC_ERR_CUDA, "clear device error: %s", cudaGetErrorString(e));
  return AACC_OK;
}

}  // extern "C"
