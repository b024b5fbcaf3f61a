// mdq_staged_packed4.cu - instantiations of the bulk-copy staged step kernel
// for packed 4-bit codes (blocks of 128 and 256 elements).
#include "mdq_staged.cuh"

namespace mdq {

template <int CAP>
mdq_status launch_staged_packed4(int gdt, const LaunchParams<CAP>& P, bool exact, int logb, int sms,
                              cudaStream_t s) {
#define MDQ_STAGED_CASE(L)                                                                   \
    case L:                                                                                  \
        if (gdt == MDQ_BF16)                                                                 \
            return exact ? launch_staged_t<MDQ_LAYOUT_PACKED4, __nv_bfloat16, true, CAP, L>(P, sms, s)            \
                         : launch_staged_t<MDQ_LAYOUT_PACKED4, __nv_bfloat16, false, CAP, L>(P, sms, s);          \
        return exact ? launch_staged_t<MDQ_LAYOUT_PACKED4, float, true, CAP, L>(P, sms, s)                        \
                     : launch_staged_t<MDQ_LAYOUT_PACKED4, float, false, CAP, L>(P, sms, s);
    switch (logb) {
        MDQ_STAGED_CASE(7)
        MDQ_STAGED_CASE(8)
    }
#undef MDQ_STAGED_CASE
    return mdq_fail(MDQ_ERR_INVALID_ARG, "staged kernel: block 2^%d", logb);
}

template mdq_status launch_staged_packed4<kCapSmall>(int, const LaunchParams<kCapSmall>&, bool, int,
                                                  int, cudaStream_t);
template mdq_status launch_staged_packed4<kCapLarge>(int, const LaunchParams<kCapLarge>&, bool, int,
                                                  int, cudaStream_t);

}  // namespace mdq
