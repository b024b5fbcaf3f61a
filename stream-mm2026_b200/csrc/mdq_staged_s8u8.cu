// mdq_staged_s8u8.cu - instantiations of the bulk-copy staged warp-per-block
// step kernel (int8/uint8 codes).
#include "mdq_staged.cuh"

namespace mdq {

template <int CAP>
mdq_status launch_staged_s8u8(int gdt, const LaunchParams<CAP>& P, bool exact, int logb, int sms,
                              cudaStream_t s) {
    if (gdt == MDQ_BF16) {
        if (logb == 10)
            return exact ? launch_staged_t<__nv_bfloat16, true, CAP, 10>(P, sms, s)
                         : launch_staged_t<__nv_bfloat16, false, CAP, 10>(P, sms, s);
        return exact ? launch_staged_t<__nv_bfloat16, true, CAP, 9>(P, sms, s)
                     : launch_staged_t<__nv_bfloat16, false, CAP, 9>(P, sms, s);
    }
    if (logb == 10)
        return exact ? launch_staged_t<float, true, CAP, 10>(P, sms, s)
                     : launch_staged_t<float, false, CAP, 10>(P, sms, s);
    return exact ? launch_staged_t<float, true, CAP, 9>(P, sms, s)
                 : launch_staged_t<float, false, CAP, 9>(P, sms, s);
}

template mdq_status launch_staged_s8u8<kCapSmall>(int, const LaunchParams<kCapSmall>&, bool, int,
                                                  int, cudaStream_t);
template mdq_status launch_staged_s8u8<kCapLarge>(int, const LaunchParams<kCapLarge>&, bool, int,
                                                  int, cudaStream_t);

}  // namespace mdq
