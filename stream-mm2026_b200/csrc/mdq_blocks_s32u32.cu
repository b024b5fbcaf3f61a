// mdq_blocks_s32u32.cu - instantiations of the warp-per-block step kernel for the
// s32u32 code layout (one translation unit per layout, built in parallel).
#include "mdq_blocks.cuh"

namespace mdq {
MDQ_BLOCKS_DEFINE(s32u32, MDQ_LAYOUT_S32U32)
}  // namespace mdq
