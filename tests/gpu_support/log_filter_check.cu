// Exhaustive checks of the two facts about logf the fused step relies on
// (test support, GPU; see mdq_math.cuh):
//   1. logf is monotone non-decreasing, so the block extremes of logf(x) are
//      logf of the extremes of x, and logf(1) = +0 (missing tail elements);
//   2. |approx_ln(x) - logf(x)| <= log_tol(approx_ln(x)), so v codes decided
//      from the approximation equal the reference's.
// Both are evaluated, exactly as the step evaluates them, on every float x
// from 1e-12f (the least value of v + 1e-12) to the largest float and +inf.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "mdq_math.cuh"

__global__ void check(uint32_t lo_bits, uint32_t hi_bits, unsigned long long* bad,
                      unsigned int* worst_ratio_bits, unsigned long long* nonmono) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    float worst = 0.0f;
    unsigned long long nbad = 0, nmono = 0;
    for (uint64_t b = lo_bits + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b <= hi_bits;
         b += stride) {
        const float x = __uint_as_float((uint32_t)b);
        const float a = mdq::approx_ln(x);
        const float l = logf(x);
        if (b < hi_bits && !(logf(__uint_as_float((uint32_t)b + 1)) >= l)) ++nmono;
        const double err = a == l ? 0.0 : fabs((double)a - (double)l);  // +inf == +inf
        const float tol = mdq::log_tol(a);
        if (!(err <= (double)tol)) ++nbad;  // NaN counts as bad
        else if (tol > 0.0f && isfinite(tol)) worst = fmaxf(worst, (float)(err / tol));
    }
    if (nbad) atomicAdd(bad, nbad);
    if (nmono) atomicAdd(nonmono, nmono);
    if (blockIdx.x == 0 && threadIdx.x == 0 && __float_as_uint(logf(1.0f)) != 0u)
        atomicAdd(nonmono, 1ull);
    atomicMax(worst_ratio_bits, __float_as_uint(worst));  // ratios are >= 0
}

// Returns 0 and fills out[0] = bound violations, out[1] = largest
// |a - l| / tol, out[2] = monotonicity violations (+1 if logf(1) != +0).
extern "C" int mdq_check_log_filter(double* out) {
    unsigned long long* bad = nullptr;
    unsigned long long* nonmono = nullptr;
    if (cudaMalloc(&nonmono, sizeof(*nonmono)) != cudaSuccess) return 1;
    cudaMemset(nonmono, 0, sizeof(*nonmono));
    unsigned int* worst = nullptr;
    if (cudaMalloc(&bad, sizeof(*bad)) != cudaSuccess) return 1;
    if (cudaMalloc(&worst, sizeof(*worst)) != cudaSuccess) return 1;
    cudaMemset(bad, 0, sizeof(*bad));
    cudaMemset(worst, 0, sizeof(*worst));
    const float lo = 1e-12f;
    uint32_t lo_bits, hi_bits = 0x7f800000u;  // through +inf
    memcpy(&lo_bits, &lo, 4);
    check<<<148 * 8, 256>>>(lo_bits, hi_bits, bad, worst, nonmono);
    unsigned long long h_bad = 0, h_mono = 0;
    cudaMemcpy(&h_mono, nonmono, sizeof(h_mono), cudaMemcpyDeviceToHost);
    unsigned int h_worst = 0;
    cudaMemcpy(&h_bad, bad, sizeof(h_bad), cudaMemcpyDeviceToHost);
    cudaMemcpy(&h_worst, worst, sizeof(h_worst), cudaMemcpyDeviceToHost);
    const cudaError_t e = cudaGetLastError();
    cudaFree(bad);
    cudaFree(worst);
    cudaFree(nonmono);
    if (e != cudaSuccess) return 2;
    float w;
    memcpy(&w, &h_worst, 4);
    out[0] = (double)h_bad;
    out[1] = (double)w;
    out[2] = (double)h_mono;
    return 0;
}
