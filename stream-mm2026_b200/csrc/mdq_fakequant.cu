// mdq_fakequant.cu - fused step of the reference's pure-PyTorch quantized
// AdamW (baseline/mdqbock_newhook.py:MDQAdamW), which keeps fp32 moments and
// updates the parameters with fake-quantised copies of them (see mdq.h,
// mdq_fq_desc).  The reference runs it as about twenty full-tensor torch
// operations per parameter and step (moment updates, padding, block views,
// log, max/min, round, clamp, exp, sqrt, divides); here one CTA reads a
// block's p, g, m and v once, reduces the block's extremes in registers and
// shared memory, and writes p, m and v once: 28 bytes per element with fp32
// gradients (26 with bf16), HBM-bound.
//
// Arithmetic follows the torch expression order of the reference, each torch
// operation rounded once, with what torch's own CUDA kernels do: fused
// multiply-adds for add(alpha=), addcmul (value * (t1 * t2) + self) and
// addcdiv, and a multiplication by the reciprocal (computed in double,
// rounded to float) for a tensor divided by a Python number; transcendentals are CUDA's logf / expf / sqrtf as
// torch's CUDA tensors compute them.  (Each of these was established by
// comparing candidate expressions with torch's results on a B200.)
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>

#include "mdq.h"

mdq_status mdq_fail(mdq_status s, const char* fmt, ...);
void mdq_clear_error();

namespace mdq_fq {

constexpr int kThreads = 256;
constexpr int kMaxBlock = 4096;
constexpr int kCap = 128;          // descriptors per launch

struct Desc {
    mdq_fq_desc d;
    int64_t unit_begin;            // first block of this descriptor in the launch
};

struct Params {
    int32_t n_desc;
    int64_t total_units;
    Desc d[kCap];
};

__device__ __forceinline__ int find_desc(const Params& P, int64_t u) {
    int lo = 0, hi = P.n_desc - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (P.d[mid].unit_begin <= u) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// torch.max / torch.min propagate NaN.
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float min_nan(float a, float b) {
    float r;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// Max |m|, max and min of log v over the CTA (fixed order not needed: max
// and min are exact).
__device__ __forceinline__ void cta_extremes(float& am, float& lmax, float& lmin, float4* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        am = max_nan(am, __shfl_xor_sync(0xffffffffu, am, o));
        lmax = max_nan(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
        lmin = min_nan(lmin, __shfl_xor_sync(0xffffffffu, lmin, o));
    }
    const int w = threadIdx.x >> 5;
    __syncthreads();  // the previous block's readers are done with `red`
    if ((threadIdx.x & 31) == 0) red[w] = make_float4(am, lmax, lmin, 0.0f);
    __syncthreads();
    float4 r = red[0];
#pragma unroll
    for (int k = 1; k < kThreads / 32; ++k) {
        const float4 o = red[k];
        r.x = max_nan(r.x, o.x);
        r.y = max_nan(r.y, o.y);
        r.z = min_nan(r.z, o.z);
    }
    am = r.x;
    lmax = r.y;
    lmin = r.z;
}

template <typename GT> __device__ __forceinline__ float load_g(const void* g, int64_t i);
template <> __device__ __forceinline__ float load_g<float>(const void* g, int64_t i) {
    return __ldcs(static_cast<const float*>(g) + i);
}
template <> __device__ __forceinline__ float load_g<__nv_bfloat16>(const void* g, int64_t i) {
    return __bfloat162float(static_cast<const __nv_bfloat16*>(g)[i]);
}

// One CTA per block unit; EPT elements per thread (thread t owns elements
// t + 256 k of the block, so each warp access is one 128-byte line).
template <typename GT, int EPT>
__global__ void __launch_bounds__(kThreads)
fq_step(const __grid_constant__ Params P) {
    __shared__ float4 red[kThreads / 32];
    const int tid = threadIdx.x;
    for (int64_t u = blockIdx.x; u < P.total_units; u += gridDim.x) {
        const Desc& D = P.d[find_desc(P, u)];
        const mdq_fq_desc& d = D.d;
        const int B = d.block;
        const int64_t e0 = (u - D.unit_begin) * (int64_t)B;
        const bool quant = d.bits < 31;
        const float eps = 1e-12f;
        float m[EPT], v[EPT], lv[EPT];
        float am = 0.0f, lmax = -INFINITY, lmin = INFINITY;
        bool first = true;
#pragma unroll
        for (int k = 0; k < EPT; ++k) {
            const int j = tid + kThreads * k;
            m[k] = 0.0f;
            v[k] = 0.0f;
            lv[k] = 0.0f;
            if (j >= B) continue;
            const int64_t i = e0 + j;
            if (i < d.n) {
                const float g = load_g<GT>(d.grad, i);
                // exp_avg.mul_(beta1).add_(grad, alpha=1-beta1)          (:159)
                m[k] = __fmaf_rn(d.one_minus_beta1, g, __fmul_rn(__ldcs(d.exp_avg + i), d.beta1));
                // exp_avg_sq.mul_(beta2).addcmul_(grad, grad, value=1-beta2) (:160):
                // torch's CUDA addcmul forms value * (t1 * t2) + self.
                v[k] = __fmaf_rn(d.one_minus_beta2, __fmul_rn(g, g),
                                 __fmul_rn(__ldcs(d.exp_avg_sq + i), d.beta2));
            }
            // Padding past the end of the tensor is a zero m and v (:63-66).
            if (quant) {
                lv[k] = logf(__fadd_rn(v[k], eps));
                const float a = fabsf(m[k]);
                am = first ? a : max_nan(am, a);
                lmax = first ? lv[k] : max_nan(lmax, lv[k]);
                lmin = first ? lv[k] : min_nan(lmin, lv[k]);
                first = false;
            }
        }
        float sm = 0.0f, dm = 1.0f, sv = 0.0f, dv = 1.0f, lo_m = 0.0f, hi_m = 0.0f, hi_v = 0.0f;
        if (quant) {
            cta_extremes(am, lmax, lmin, red);
            const float lm1 = (float)((1 << (d.bits - 1)) - 1);     // q_levels - 1
            const float lv1 = (float)((1u << d.bits) - 1u);         // 2^bits - 1
            // A tensor divided by a Python number: torch's CUDA kernel multiplies
            // by the reciprocal of the number, computed in double, as a float.
            sm = __fmul_rn(__fadd_rn(am, eps), (float)(1.0 / (double)lm1));  // (:80)
            dm = __fadd_rn(sm, eps);
            lo_m = -(float)(1 << (d.bits - 1));
            hi_m = lm1;
            sv = __fmul_rn(__fsub_rn(lmax, lmin), (float)(1.0 / (double)lv1));  // (:74)
            dv = __fadd_rn(sv, eps);
            hi_v = lv1;
        }
#pragma unroll
        for (int k = 0; k < EPT; ++k) {
            const int j = tid + kThreads * k;
            if (j >= B) continue;
            const int64_t i = e0 + j;
            if (i >= d.n) continue;
            float qm = m[k], qv = v[k];
            if (quant) {
                // torch.round(x / (scale + eps)).clamp(lo, hi) * scale
                const float rm = fminf(fmaxf(rintf(__fdiv_rn(m[k], dm)), lo_m), hi_m);
                qm = __fmul_rn(rm, sm);
                const float rv =
                    fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(lv[k], lmin), dv)), 0.0f), hi_v);
                qv = expf(__fadd_rn(__fmul_rn(rv, sv), lmin));        // (:76)
            }
            float p = d.p[i];
            if (d.apply_decay) p = __fmul_rn(p, d.decay);               // (:168)
            // denom = (q_v.sqrt() / sqrt(bc2)).add_(eps); p.addcdiv_(q_m, denom, value)
            const float denom = __fadd_rn(__fmul_rn(__fsqrt_rn(qv), d.inv_sqrt_bc2), d.eps);
            d.p[i] = __fmaf_rn(d.step_size, __fdiv_rn(qm, denom), p);
            __stcs(d.exp_avg + i, m[k]);
            __stcs(d.exp_avg_sq + i, v[k]);
        }
    }
}

template <typename GT, int EPT>
mdq_status launch_t(const Params& P, cudaStream_t s) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fq_step<GT, EPT>, kThreads, 0) !=
            cudaSuccess || occ < 1)
        occ = 1;
    int64_t grid = (int64_t)sms * occ;
    if (grid > P.total_units) grid = P.total_units;
    fq_step<GT, EPT><<<(unsigned)grid, kThreads, 0, s>>>(P);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return mdq_fail(MDQ_ERR_CUDA, "fake-quant launch: %s", cudaGetErrorString(e));
    return MDQ_OK;
}

mdq_status launch(const Params& P, int gdt, int max_block, cudaStream_t s) {
    const bool bf = gdt == MDQ_BF16;
    if (max_block <= 1024) return bf ? launch_t<__nv_bfloat16, 4>(P, s) : launch_t<float, 4>(P, s);
    if (max_block <= 2048) return bf ? launch_t<__nv_bfloat16, 8>(P, s) : launch_t<float, 8>(P, s);
    return bf ? launch_t<__nv_bfloat16, 16>(P, s) : launch_t<float, 16>(P, s);
}

}  // namespace mdq_fq

extern "C" mdq_status mdq_fakequant_adamw_multi(const mdq_fq_desc* descs, int32_t n_descs,
                                                cudaStream_t stream) {
    using namespace mdq_fq;
    mdq_clear_error();
    if (n_descs < 0 || (n_descs > 0 && descs == nullptr))
        return mdq_fail(MDQ_ERR_INVALID_ARG, "descs is null or n_descs negative");
    for (int i = 0; i < n_descs; ++i) {
        const mdq_fq_desc& d = descs[i];
        if (d.n < 0) return mdq_fail(MDQ_ERR_INVALID_ARG, "desc %d: negative n", i);
        if (d.n == 0) continue;
        if (!d.p || !d.grad || !d.exp_avg || !d.exp_avg_sq)
            return mdq_fail(MDQ_ERR_INVALID_ARG, "desc %d: null pointer", i);
        if (d.block < 1 || d.block > kMaxBlock)
            return mdq_fail(MDQ_ERR_UNSUPPORTED, "desc %d: block %d outside 1..%d", i, d.block,
                            kMaxBlock);
        if (d.bits < 1 || d.bits > 32)
            return mdq_fail(MDQ_ERR_UNSUPPORTED, "desc %d: bits %d outside 1..32", i, d.bits);
        if (d.grad_dtype != MDQ_F32 && d.grad_dtype != MDQ_BF16)
            return mdq_fail(MDQ_ERR_UNSUPPORTED, "desc %d: grad dtype must be MDQ_F32 or MDQ_BF16", i);
    }
    static thread_local Params P;
    // One launch per gradient dtype and up to kCap descriptors.
    for (int gdt = MDQ_F32; gdt <= MDQ_BF16; ++gdt) {
        int i = 0;
        while (i < n_descs) {
            P.n_desc = 0;
            P.total_units = 0;
            int max_block = 1;
            while (i < n_descs && P.n_desc < kCap) {
                const mdq_fq_desc& d = descs[i++];
                if (d.n == 0 || d.grad_dtype != gdt) continue;
                Desc& D = P.d[P.n_desc++];
                D.d = d;
                D.unit_begin = P.total_units;
                P.total_units += (d.n + d.block - 1) / d.block;
                if (d.block > max_block) max_block = d.block;
            }
            if (P.n_desc == 0) continue;
            const mdq_status st = launch(P, gdt, max_block, stream);
            if (st != MDQ_OK) return st;
        }
    }
    return MDQ_OK;
}
