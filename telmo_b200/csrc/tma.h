// tma.h -- host-side construction of TMA tensor maps (shared by the tcgen05 kernels).
#pragma once

#include <cuda.h>
#include <cstdint>

namespace telmo {

// A 2-D tensor map of `outer` rows of `inner` elements, rows `row_bytes` apart, copied in boxes
// of box_inner x box_outer elements. Reads outside the tensor fill zeros. False if the driver
// refuses the layout (alignment of the base or the stride, box sizes).
bool encode_map_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);

}  // namespace telmo
