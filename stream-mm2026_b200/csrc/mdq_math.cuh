// mdq_math.cuh - per-element arithmetic of the MDQ-AdamW step.
//
// Every expression here reproduces, operation for operation, the arithmetic of
// the reference kernel family (ruby320/STREAM-MM2026 CUDA/stquant_kernel.cu:
// 53-401) as its -O3 build evaluates it: nvcc contracts a*b+c into one fused
// multiply-add, so each contraction is written out with __fmaf_rn (which the
// compiler never re-associates) and every other operation with its correctly
// rounded intrinsic.  CUDA's own expf / logf / powf / sqrtf / pow are called,
// never re-derived, so the transcendental results are those of the reference.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mdq {

// Per-tensor constants, computed once per CTA when it starts a tensor.
struct StepConsts {
    float b1, omb1, b2, omb2;  // beta1, 1-beta1, beta2, 1-beta2
    float eps;
    float wd;                  // weight decay (0 disables the decay multiply)
    float decay;               // 1 - lr*wd                (contracted)
    float step_size;           // lr / bc1                 (IEEE divide)
    float sqrt_bc2;            // sqrtf(1 - beta2^step)    (IEEE sqrt)
    float inv_sqrt_bc2;        // 1 / sqrt_bc2             (fast p mode only)
    float lm_f, lv_f;          // (float)2^(m_bits-1), (float)(2^v_bits - 1)
    float inv_lm;              // 2^-(m_bits-1), exact
    double lm_d, lv_d;         // the same levels in double, for clamping
};

// CUDA/stquant_kernel.cu:88-89 (levels), :136-141 (bias correction, decay).
__device__ __forceinline__ StepConsts make_step_consts(float b1, float b2, float lr, float wd,
                                                       float eps, int step, int m_bits,
                                                       int v_bits) {
    StepConsts c;
    c.b1 = b1;
    c.b2 = b2;
    c.omb1 = __fsub_rn(1.0f, b1);
    c.omb2 = __fsub_rn(1.0f, b2);
    c.eps = eps;
    c.wd = wd;
    c.decay = __fmaf_rn(-lr, wd, 1.0f);
    const float bc1 = __fsub_rn(1.0f, powf(b1, (float)step));
    const float bc2 = __fsub_rn(1.0f, powf(b2, (float)step));
    c.step_size = __fdiv_rn(lr, bc1);
    c.sqrt_bc2 = __fsqrt_rn(bc2);
    c.inv_sqrt_bc2 = __frcp_rn(c.sqrt_bc2);
    c.lm_d = pow(2.0, m_bits - 1);
    c.lv_d = pow(2.0, v_bits) - 1.0;
    c.lm_f = (float)c.lm_d;
    c.lv_f = (float)c.lv_d;
    c.inv_lm = (float)(1.0 / c.lm_d);
    return c;
}

// Dequantised second moment: expf(q * sv + v_min)  (CUDA/stquant_kernel.cu:169).
__device__ __forceinline__ float dequant_v(float q, float sv, float vmin) {
    return expf(__fmaf_rn(q, sv, vmin));
}

// m = beta1*m + (1-beta1)*g  (CUDA/stquant_kernel.cu:175).
__device__ __forceinline__ float adam_m(float m, float g, const StepConsts& c) {
    return __fmaf_rn(c.b1, m, __fmul_rn(c.omb1, g));
}

// v = beta2*v + (1-beta2)*g*g  (CUDA/stquant_kernel.cu:176).
__device__ __forceinline__ float adam_v(float v, float g, const StepConsts& c) {
    return __fmaf_rn(c.b2, v, __fmul_rn(__fmul_rn(c.omb2, g), g));
}

// Parameter update with the unquantised moments (CUDA/stquant_kernel.cu:220-229).
template <bool EXACT>
__device__ __forceinline__ float update_p(float w, float m, float v, const StepConsts& c) {
    if (EXACT) {
        const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), c.sqrt_bc2), c.eps);
        if (c.wd != 0.0f) w = __fmul_rn(w, c.decay);
        return __fmaf_rn(-c.step_size, __fdiv_rn(m, denom), w);
    } else {
        // Hardware square root and reciprocal: a few ulp on the update term.
        float s, r;
        asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(s) : "f"(v));
        const float denom = __fmaf_rn(s, c.inv_sqrt_bc2, c.eps);
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(denom));
        if (c.wd != 0.0f) w = w * c.decay;
        return __fmaf_rn(-c.step_size, m * r, w);
    }
}

// ---------------------------------------------------------------------------
// Element pairs.  sm_100 issues two fp32 adds, multiplies or fused
// multiply-adds as one instruction on a register pair (add / mul / fma
// .rn.f32x2); each half is rounded to nearest exactly as the scalar
// __fadd_rn / __fmul_rn / __fmaf_rn, so the pair forms below return the same
// bits as their scalar counterparts, for half the issue slots.  Used only
// where no paired multiply feeds a paired add: ptxas (CUDA 12.9) was observed
// to fuse mul.rn.f32x2 followed by add.rn.f32x2 into one fused multiply-add,
// which changes the rounding (the magic-number rounding of the code checks
// stays scalar for that reason).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 bcast2(float a) { return make_float2(a, a); }

__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// m = beta1*m + (1-beta1)*g for two elements.
__device__ __forceinline__ float2 adam_m2(float2 m, float2 g, const StepConsts& c) {
    return fma2_rn(bcast2(c.b1), m, mul2_rn(bcast2(c.omb1), g));
}

// v = beta2*v + (1-beta2)*g*g for two elements.
__device__ __forceinline__ float2 adam_v2(float2 v, float2 g, const StepConsts& c) {
    return fma2_rn(bcast2(c.b2), v, mul2_rn(mul2_rn(bcast2(c.omb2), g), g));
}

// Parameter update of two elements (update_p).
template <bool EXACT>
__device__ __forceinline__ float2 update_p2(float2 w, float2 m, float2 v, const StepConsts& c) {
    if (EXACT) {
        return make_float2(update_p<true>(w.x, m.x, v.x, c), update_p<true>(w.y, m.y, v.y, c));
    } else {
        float2 s, r;
        asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(s.x) : "f"(v.x));
        asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(s.y) : "f"(v.y));
        const float2 denom = fma2_rn(s, bcast2(c.inv_sqrt_bc2), bcast2(c.eps));
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(denom.x));
        asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(denom.y));
        if (c.wd != 0.0f) w = mul2_rn(w, bcast2(c.decay));
        return fma2_rn(bcast2(-c.step_size), mul2_rn(m, r), w);
    }
}

// log(v + 1e-12)  (CUDA/stquant_kernel.cu:185).
__device__ __forceinline__ float log_v_of(float v) { return logf(__fadd_rn(v, 1e-12f)); }

// New block scales from the block reductions (CUDA/stquant_kernel.cu:192-195).
// Division by the power of two 2^(m_bits-1) is exact scaling, identical to the
// multiplication by its exact reciprocal.
__device__ __forceinline__ float scale_m_of(float max_abs_m, const StepConsts& c) {
    return __fmul_rn(__fadd_rn(max_abs_m, 1e-12f), c.inv_lm);
}

// Reciprocal estimate; the codes are verified exactly whatever its error.
__device__ __forceinline__ float rcp_estimate(float d) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
    return r;
}
__device__ __forceinline__ float scale_v_of(float max_lv, float min_lv, const StepConsts& c) {
    return __fdiv_rn(__fadd_rn(__fsub_rn(max_lv, min_lv), 1e-12f), c.lv_f);
}

// ---------------------------------------------------------------------------
// Requantisation.
//
// The reference computes q = round((double)x / (double)d) in double precision
// (round = half away from zero) and clamps in double (CUDA/stquant_kernel.cu:
// 205-215).  x and d are floats.  For |x/d| < 2^17 the double quotient never
// lands on, or crosses, a half-integer that the exact quotient does not, since
// a quotient of two floats that is not itself a half-integer stays at least
// 2^-26 away from every half-integer, while the double rounding error is below
// 2^-36; hence q = round_half_away(x/d) exactly.  The fast path computes
// y = |x| * RN(1/d) (relative error < 2^-22.9) and accepts rint(y) when y lies
// farther than y*2^-21 from the nearest half-integer; otherwise (and for NaN /
// Inf) it evaluates the reference's double expression itself.  Both branches
// therefore return the reference's code bit for bit.
// ---------------------------------------------------------------------------

// Reference expression for a signed (m) code, clamped to [-L, L-1].
static __device__ __noinline__ double requant_m_ref(float x, float d, double lm) {
    double q = round((double)x / (double)d);
    const double lo = -lm, hi = lm - 1.0;
    if (q < lo) q = lo;
    if (q > hi) q = hi;
    return q;
}

// Reference expression for an unsigned (v) code, clamped to [0, L].
static __device__ __noinline__ double requant_v_ref(float x, float d, double lv) {
    double q = round((double)x / (double)d);
    if (q < 0.0) q = 0.0;
    if (q > lv) q = lv;
    return q;
}

// ---------------------------------------------------------------------------
// Rounding.  The reference computes q = round((double)x / (double)d) with
// round-half-away-from-zero (CUDA/stquant_kernel.cu:205,212), x and d floats.
// For |x/d| < 2^17 the double quotient never lands on or crosses a
// half-integer the exact quotient does not (a quotient of floats that is not
// itself a half-integer stays >= 2^-26 from every half-integer, and the
// double rounding error is below 2^-36), so q is the integer nearest the
// exact x/d, with ties away from zero.
//
// Here r = rint(y) for an estimate y of x/d, computed without conversion
// instructions: for |y| <= 2^22, s = y + 1.5*2^23 rounds y to an integer r
// and has the bit pattern 0x4B400000 + r ("magic word").  r is then checked
// exactly: |x - r*d| < d/2 holds iff r is the nearest integer to x/d and x/d
// is not a tie; fma computes x - r*d with one rounding, which preserves a
// strict comparison with d/2 (a power-of-two multiple of d, exactly
// representable).  `round_checked` returns the magic word and |x - r*d|;
// with CORRECT it first moves r one step toward x/d when the remainder shows
// that y rounded to a neighbour (needed for 16-bit codes, where the estimate
// y = x * RN(1/d) can be off by more than the distance to a half-integer).
// A NaN operand gives a NaN remainder, which fails every comparison.
// ---------------------------------------------------------------------------
// Three-input max / min (sm_100): NaN operands are skipped as by fmaxf / fminf.
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
__device__ __forceinline__ float min3f(float a, float b, float c) {
    float r;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// BIAS (0..255) is added to the word: the magic constant 1.5 * 2^23 + BIAS
// rounds the same way (floats in [2^23, 2^24) are the integers).
template <bool CORRECT, int BIAS = 0>
__device__ __forceinline__ int round_checked(float y, float x, float d, float half_d, float& rem) {
    constexpr float kM = 12582912.0f + (float)BIAS;
    float s = __fadd_rn(y, kM);
    float r = __fsub_rn(s, kM);
    float e = __fmaf_rn(-r, d, x);
    if (CORRECT) {
        const float stp = e >= half_d ? 1.0f : (e <= -half_d ? -1.0f : 0.0f);
        s = __fadd_rn(s, stp);
        r = __fadd_rn(r, stp);
        e = __fmaf_rn(-r, d, x);
    }
    rem = fabsf(e);
    return __float_as_int(s);
}

// ---------------------------------------------------------------------------
// Logarithms.  The block statistics need max and min of logf(x), x = v + 1e-12,
// and each v code needs round((logf(x) - min) / d).
//  * Extremes: CUDA's logf is monotone non-decreasing on every float >= 1e-12
//    (a GPU test checks all of them), so max_i logf(x_i) = logf(max_i x_i):
//    the block reduces x and calls logf once.  fmaxf/fminf skip NaNs exactly
//    as the reference's reduction of fmaxf/fminf over logf values does, and a
//    missing tail element (log v taken as 0) enters as x = 1, logf(1) = +0.
//  * Codes: a = lg2.approx(x) * ln 2 approximates logf(x) within log_tol(a)
//    for every float x >= 1e-12 (checked exhaustively by the same GPU test);
//    a code is taken from the approximation only when it clears its rounding
//    boundary by more than that error, otherwise from logf itself.
// ---------------------------------------------------------------------------
constexpr float kLn2 = 0.693147182f;

// Flush-to-zero form: every argument here is a normal float >= 1e-12 (or NaN),
// where it equals the non-flushing one and needs no subnormal scaling.
__device__ __forceinline__ float approx_log2(float x) {
    float l2;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(l2) : "f"(x));
    return l2;
}

__device__ __forceinline__ float approx_ln(float x) { return __fmul_rn(approx_log2(x), kLn2); }

__device__ __forceinline__ float log_tol(float a) {
    return __fmaf_rn(fabsf(a), 0x1p-21f, 0x1p-20f);
}

}  // namespace mdq
