// mdq_tiles_m8v4.cu - instantiations of the tiled step kernel for the
// m8v4 code layout (one translation unit per layout, built in parallel).
#include "mdq_tiles.cuh"

namespace mdq {
MDQ_TILES_DEFINE(m8v4, MDQ_LAYOUT_M8V4)
}  // namespace mdq
