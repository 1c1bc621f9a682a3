// Host-side helpers shared by the C-ABI entry points (not part of the ABI).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace exk {

// Resolves cuTensorMapEncodeTiled through the runtime's driver entry point
// (no link-time dependency on libcuda) and encodes a 3-D tiled tensor map.
// dims/strides in elements / bytes; returns 0 or EXK_ETMAP / EXK_EDRIVER.
int make_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* ptr, uint64_t d0, uint64_t d1,
                 uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1,
                 uint32_t box2, CUtensorMapSwizzle swizzle);

// Makes `device` current for this library's runtime (the caller's framework
// keeps its own notion of the current device) and returns its SM count.
int use_device(int device, int* num_sms);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 0 if kernels may store through p: device or managed memory, or pinned host
// memory mapped into the device address space at the same address (an output
// written straight to the host over PCIe); EXK_EARG otherwise.
int device_reachable(const void* p);

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

}  // namespace exk
