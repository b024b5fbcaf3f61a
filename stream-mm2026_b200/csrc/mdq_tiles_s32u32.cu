// mdq_tiles_s32u32.cu - instantiations of the tiled step kernel for the
// s32u32 code layout (one translation unit per layout, built in parallel).
#include "mdq_tiles.cuh"

namespace mdq {
MDQ_TILES_DEFINE(s32u32, MDQ_LAYOUT_S32U32)
}  // namespace mdq
