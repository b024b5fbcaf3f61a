// mdq_blocks_packed4.cu - instantiations of the warp-per-block step kernel for the
// packed4 code layout (one translation unit per layout, built in parallel).
#include "mdq_blocks.cuh"

namespace mdq {
MDQ_BLOCKS_DEFINE(packed4, MDQ_LAYOUT_PACKED4)
}  // namespace mdq
