// mdq_tiles_s8u8.cu - instantiations of the tiled step kernel for the
// s8u8 code layout (one translation unit per layout, built in parallel).
#include "mdq_tiles.cuh"

namespace mdq {
MDQ_TILES_DEFINE(s8u8, MDQ_LAYOUT_S8U8)
}  // namespace mdq
