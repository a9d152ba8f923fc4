// tmap.h -- creation of TMA tensor maps (cuTensorMapEncodeTiled, reached
// through the runtime's driver entry point so the library needs no -lcuda).
#pragma once

#include <cstdint>
#include <cuda.h>

namespace b200 {

// Tiled tensor map of rank 2 or 3.  dims/box are innermost first; strides
// are the byte strides of dims 1..rank-1.  Returns false if the driver
// rejects the map (alignment, box size) or the entry point is missing.
bool make_tmap(CUtensorMap *map, CUtensorMapDataType dt, const void *base, int rank, const uint64_t *dims,
               const uint64_t *strides, const uint32_t *box, CUtensorMapSwizzle sw);

}  // namespace b200
