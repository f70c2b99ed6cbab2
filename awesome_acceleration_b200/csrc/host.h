// Host-only helpers shared by the C-ABI launchers.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace aacc {

// Encode a 2-D bf16 tensor map: `inner` contiguous elements per row, `outer`
// rows `row_stride_bytes` apart, box of box_inner x box_outer elements,
// optional 128-byte swizzle.  Out-of-bounds box elements read as zero.
int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                 uint32_t box_inner, uint32_t box_outer, bool swizzle128);

// 3-D bf16 tensor map: d0 contiguous elements, d1 and d2 strided by
// stride1 / stride2 bytes; box of box0 x box1 x box2 elements, written to
// shared memory d0-fastest (row index = i2 * box1 + i1 when box0 fills a row).
int make_tmap_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                 uint64_t stride2_bytes, uint32_t box0, uint32_t box1, uint32_t box2, bool swizzle128);

// Streaming multiprocessors of the current device (cached per device).
int sm_count();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Programmatic dependent launch: every kernel of this library is launched with
// programmatic stream serialization, so its CTAs may start (shared memory,
// barriers, TMEM, weight prefetch) while the previous kernel drains; each
// kernel executes griddepcontrol.wait before touching data the previous
// kernel produced or consumed.  AACC_PDL=0 in the environment turns it off.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

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
