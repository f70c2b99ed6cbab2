// Host-only helpers shared by the C-ABI launchers.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace aacc {

// Encode a 2-D bf16 tensor map: `inner` contiguous elements per row, `outer`
// rows `row_stride_bytes` apart, box of box_inner x box_outer elements,
// optional 128-byte swizzle.  Out-of-bounds box elements read as zero.
int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                 uint32_t box_inner, uint32_t box_outer, bool swizzle128);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Raise a kernel's dynamic shared-memory limit once per device (the call is
// not a stream operation, so doing it once keeps it out of graph captures).
template <auto Kern>
inline cudaError_t set_smem_once(int bytes) {
  static unsigned long long done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (done & bit) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done |= bit;
  return e;
}

}  // namespace aacc
