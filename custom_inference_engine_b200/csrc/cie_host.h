// Host-side helpers shared by the C-ABI entry points (not part of the ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "cie_attention.h"

namespace cie {

// Records a formatted message for cie_last_error_message() and returns `status`.
int fail(int status, const char* fmt, ...);

// Number of SMs of the current device (cached per device).
int sm_count();

// Current device ordinal (cached CUDA call).
int current_device();

// Encodes a tiled TMA descriptor through the driver entry point
// cuTensorMapEncodeTiled (fetched once via cudaGetDriverEntryPoint).
// rank <= 5; dims / strides in elements / bytes as the driver expects
// (strides for dims 1..rank-1). Returns CIE_OK or a cie_status.
int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle);

// Sets the max dynamic shared memory attribute of `func` once per device.
int ensure_smem_attribute(const void* func, int bytes, int slot);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace cie
