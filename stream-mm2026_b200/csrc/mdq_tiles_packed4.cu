// mdq_tiles_packed4.cu - instantiations of the tiled step kernel for the
// packed4 code layout (one translation unit per layout, built in parallel).
#include "mdq_tiles.cuh"

namespace mdq {
MDQ_TILES_DEFINE(packed4, MDQ_LAYOUT_PACKED4)
}  // namespace mdq
