// Host-side construction of TMA tensor maps (cuTensorMapEncodeTiled, reached
// through the runtime's driver entry point so the library needs no -lcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace faq {

// Encode a tiled tensor map of `rank` dims (dims[0] innermost, contiguous),
// `strides_bytes[i]` the byte stride of dim i+1, `box` the tile extent per dim.
// Returns FAQ_OK or an error code (with the message set).
int make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

}  // namespace faq
