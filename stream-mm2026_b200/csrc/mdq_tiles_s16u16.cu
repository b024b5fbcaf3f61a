// mdq_tiles_s16u16.cu - instantiations of the tiled step kernel for the
// s16u16 code layout (one translation unit per layout, built in parallel).
#include "mdq_tiles.cuh"

namespace mdq {
MDQ_TILES_DEFINE(s16u16, MDQ_LAYOUT_S16U16)
}  // namespace mdq
