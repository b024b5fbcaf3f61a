// mdq_blocks_s8u8.cu - instantiations of the warp-per-block step kernel for the
// s8u8 code layout (one translation unit per layout, built in parallel).
#include "mdq_blocks.cuh"

namespace mdq {
MDQ_BLOCKS_DEFINE(s8u8, MDQ_LAYOUT_S8U8)
}  // namespace mdq
