// mdq_blocks_m8v4.cu - instantiations of the warp-per-block step kernel for the
// m8v4 code layout (one translation unit per layout, built in parallel).
#include "mdq_blocks.cuh"

namespace mdq {
MDQ_BLOCKS_DEFINE(m8v4, MDQ_LAYOUT_M8V4)
}  // namespace mdq
