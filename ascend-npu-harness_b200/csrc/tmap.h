// Host-side construction of TMA tensor maps (cuTensorMapEncodeTiled through the runtime's
// driver entry point, so the library links only against the CUDA runtime).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace hc {

// Encodes a row-major tensor of `rank` (2..3) dims, innermost first:
//   dims[0] elements contiguous, strides_bytes[i] = byte distance between consecutive
//   indices of dims[i+1].  `box` is the tile copied per TMA instruction.  Returns HC_OK or an
//   error status (message in hc_last_error_string()).
int encode_tmap(CUtensorMap* out, CUtensorMapDataType dtype, uint32_t rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

}  // namespace hc
