// mdq_blocks_s16u16.cu - instantiations of the warp-per-block step kernel for the
// s16u16 code layout (one translation unit per layout, built in parallel).
#include "mdq_blocks.cuh"

namespace mdq {
MDQ_BLOCKS_DEFINE(s16u16, MDQ_LAYOUT_S16U16)
}  // namespace mdq
