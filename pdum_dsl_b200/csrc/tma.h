// Host-side TMA tensor-map encoding (4-D, tiled).
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdint.h>

namespace pdb {
// dims / box are innermost-first; strides_bytes[i] is the byte stride of dim i+1.
int encode_tma_4d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[4],
                  const uint64_t strides_bytes[3], const uint32_t box[4], CUtensorMapSwizzle swizzle);
}  // namespace pdb
