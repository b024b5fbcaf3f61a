// mdq_step.cu - B200 (sm_100a) fused quantized-AdamW step and its C ABI.
//
// Kernel design
// -------------
// The reference runs one thread per element and one CTA per quantisation block
// (CUDA/stquant_kernel.cu:61,421-422) with three shared-memory tree reductions
// per CTA and a double-precision divide per code.  Here a persistent grid of
// 256-thread CTAs (3 per SM) walks contiguous ranges of "tiles" of 2048
// consecutive elements of one tensor; each thread owns 8 consecutive elements,
// loaded and stored with 128-bit (p, g) and 32/64/128-bit (codes) streaming
// accesses.  A quantisation block of B elements (power of two, 8..2048) is
// owned by B/8 consecutive threads, so its max/min reductions are xor
// shuffles or one redux.sync (and, for B > 256, one shared-memory exchange).
// The block's log extremes come from one logf of the extreme v (logf is
// monotone), codes from a float estimate whose exactness is checked by an fma
// remainder, with the reference's double expression as the rare fallback.
// Tiles of all tensors of one layout / gradient dtype are scheduled in one
// launch from a descriptor table passed as a __grid_constant__ kernel
// parameter, so nothing is allocated and nothing is copied host-to-device per
// step.
//
// Block sizes that are not a power of two, or below 8, take a second kernel
// that keeps the reference's one-thread-per-element shape and reproduces its
// tree reduction (which, for a non-power-of-two CTA, folds only a subset of
// the elements; the codes depend on exactly that subset).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <math.h>
#include <algorithm>
#include <mutex>

#include "mdq.h"
#include "mdq_math.cuh"
#include "mdq_codes.cuh"

namespace mdq {

// Every launch walks 2048-element tiles: 256 threads x 8 elements (PT = 8,
// 3 CTAs per SM) or 128 threads x 16 elements (PT = 16, 4 CTAs per SM).
template <int PT> constexpr int threads_for() { return PT == 16 ? 128 : 256; }
constexpr int kThreads = 256;                  // PT = 8 CTA size
constexpr int kWarps = kThreads / 32;          // warps of the largest CTA
constexpr int kPerThread = 8;
constexpr int kTile = kThreads * kPerThread;  // 2048 elements for both shapes
constexpr int kLogTile = 11;
constexpr int kCapSmall = 8;                  // descriptors per launch, small table
constexpr int kCapLarge = 224;                // descriptors per launch, large table
constexpr int kProfSlots = 5;

#ifndef MDQ_USE_REDUX
#define MDQ_USE_REDUX 1
#endif
#ifndef MDQ_ENABLE_PT16
#define MDQ_ENABLE_PT16 1
#endif
#ifndef MDQ_MIN_CTAS_PT16
#define MDQ_MIN_CTAS_PT16 4
#endif
#ifndef MDQ_GROUP_BARRIER
#define MDQ_GROUP_BARRIER 1
#endif
#ifndef MDQ_USE_TABLES
#define MDQ_USE_TABLES 1
#endif
#ifndef MDQ_MIN_CTAS_PER_SM
#define MDQ_MIN_CTAS_PER_SM 3
#endif

// Device-side descriptor (one tensor or block-aligned tensor piece).
struct LaunchDesc {
    TensorPtrs t;
    int64_t n;
    int32_t tile_begin;  // first tile of this descriptor within the launch
    int32_t step;
    float lr, wd, eps, b1, b2;
    int8_t m_bits, v_bits, log2_block, vec;
};

template <int CAP>
struct LaunchParams {
    int32_t n_desc;
    int32_t total_tiles;
    unsigned long long* prof;
    LaunchDesc d[CAP];
};

// The tensor a CTA is working on, staged in shared memory by thread 0.
struct TileCtx {
    TensorPtrs t;
    int64_t n;
    int32_t tile_begin, tile_end;  // this tensor's tiles within the launch
    int32_t lb, vec;
    StepConsts C;
};

template <int CAP>
__device__ int find_desc(const LaunchParams<CAP>& P, int tile) {
    int lo = 0, hi = P.n_desc - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (P.d[mid].tile_begin <= tile) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// Max (bit k of MAXMASK set) or min of NV values over the `gthreads`
// consecutive threads that own one quantisation block (gthreads is uniform
// over the CTA, so the branches and the barrier are too).  Inside a warp:
// redux.sync when the block covers whole warps, xor shuffles otherwise; then
// one shared-memory exchange when a block spans several warps.  Every step is
// an fmaxf / fminf, which skip NaNs as the reference's reduction does.
template <unsigned MAXMASK, int NV>
__device__ __forceinline__ void group_reduce(float (&x)[NV], int gthreads, float4* red) {
    static_assert(NV <= 4, "partials are exchanged as one float4 per warp");
    if (MDQ_USE_REDUX && gthreads >= 32) {
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            float r;
            if ((MAXMASK >> k) & 1u)
                asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(x[k]));
            else
                asm volatile("redux.sync.min.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(x[k]));
            x[k] = r;
        }
    } else {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            if (o < gthreads) {
#pragma unroll
                for (int k = 0; k < NV; ++k) {
                    const float y = __shfl_xor_sync(0xffffffffu, x[k], o);
                    x[k] = ((MAXMASK >> k) & 1u) ? fmaxf(x[k], y) : fminf(x[k], y);
                }
            }
        }
    }
    if (gthreads > 32) {
        const int w = threadIdx.x >> 5;
        if ((threadIdx.x & 31) == 0) {
            float4 v;
            v.x = x[0];
            v.y = NV > 1 ? x[1 % NV] : 0.0f;
            v.z = NV > 2 ? x[2 % NV] : 0.0f;
            v.w = NV > 3 ? x[3 % NV] : 0.0f;
            red[w] = v;
        }
        // Only the warps of one block exchange partials: they meet at their
        // own named barrier (ids 1..), so other blocks' warps run on.
        if (MDQ_GROUP_BARRIER && gthreads < (int)blockDim.x)
            asm volatile("bar.sync %0, %1;" ::"r"(1 + w / (gthreads >> 5)), "r"(gthreads) : "memory");
        else
            __syncthreads();
        const int wpg = gthreads >> 5;
        const int w0 = (w / wpg) * wpg;
        for (int i = 0; i < wpg; ++i) {
            const float4 v = red[w0 + i];
            const float vals[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < NV; ++k)
                x[k] = ((MAXMASK >> k) & 1u) ? fmaxf(x[k], vals[k]) : fminf(x[k], vals[k]);
        }
    }
}

__device__ __forceinline__ void prof_mark(unsigned long long (&pc)[kProfSlots], int slot,
                                          unsigned long long& t0) {
    const unsigned long long t1 = clock64();
    pc[slot] += t1 - t0;
    t0 = t1;
}

// Dequantisation by table for 4-bit codes.  A 4-bit code has 16 values, so
// the 16 dequantised values of a block (v = expf(fma(q, sv, v_min)),
// m = q * sm: CUDA/stquant_kernel.cu:163-165) are computed once, entry k by
// lane k of each 16-lane half-warp, and every element fetches its value with
// one 16-wide shuffle indexed by the code's nibble (a 16-wide shuffle reads
// only the low four bits of the index, so the nibble needs no mask).  Every
// lane of a half-warp must lie in the same block: blocks of >= 16 * PT.
template <int LAYOUT> struct TableCodes;
template <> struct TableCodes<MDQ_LAYOUT_PACKED4> {
    struct Raw { uint2 w; };
    __device__ static void load8(const TensorPtrs& t, int64_t e, Raw& r) {
        r.w = __ldcs(reinterpret_cast<const uint2*>(static_cast<const uint8_t*>(t.m) + e));
    }
    // Byte j: q_m + 8 in the low nibble, q_v in the high one.
    __device__ static float m(const Raw& r, int j, float tm, float) {
        const unsigned w = j < 4 ? r.w.x : r.w.y;
        return __shfl_sync(0xffffffffu, tm, (int)(w >> (8 * (j & 3))), 16);
    }
    __device__ static float v(const Raw& r, int j, float tv) {
        const unsigned w = j < 4 ? r.w.x : r.w.y;
        return __shfl_sync(0xffffffffu, tv, (int)(w >> (8 * (j & 3) + 4)), 16);
    }
};
template <> struct TableCodes<MDQ_LAYOUT_M8V4> {
    struct Raw { uint2 w; unsigned vw; };
    __device__ static void load8(const TensorPtrs& t, int64_t e, Raw& r) {
        r.w = __ldcs(reinterpret_cast<const uint2*>(static_cast<const int8_t*>(t.m) + e));
        r.vw = __ldcs(reinterpret_cast<const unsigned*>(static_cast<const uint8_t*>(t.v) + (e >> 1)));
    }
    // int8 m codes have 256 values: converted directly.
    __device__ static float m(const Raw& r, int j, float, float sm) {
        const unsigned w = j < 4 ? r.w.x : r.w.y;
        const int q = (int)(int8_t)(uint8_t)(w >> (8 * (j & 3)));
        return __fmul_rn(small_int_to_float(q), sm);
    }
    __device__ static float v(const Raw& r, int j, float tv) {
        return __shfl_sync(0xffffffffu, tv, (int)(r.vw >> (4 * j)), 16);
    }
};
template <int LAYOUT> struct TableCodes { struct Raw {}; };

// One tile of 2048 elements.  FULL: every thread owns 8 in-range elements and
// all pointers allow vector access; otherwise element-wise guarded access.
// `red` is this tile's reduction scratch.
template <int LAYOUT, typename GT, bool EXACT_P, bool PROF, bool FULL, int PT, bool TBL>
__device__ __forceinline__ void tile_body(const TileCtx& X, int64_t tile_e0,
                                          float4* red,
                                          unsigned long long (&pc)[kProfSlots],
                                          unsigned long long& t0) {
    using CI = Codes<LAYOUT>;
    constexpr bool kApprox = CI::kApproxLog;
    constexpr bool kMagicC = CI::kMagicCodes;
    const float kNaN = __int_as_float(0x7fffffff);
    const int tid = threadIdx.x;
    const TensorPtrs T = X.t;
    const StepConsts& C = X.C;
    const int lb = X.lb;
    const int64_t n = X.n;
    const int64_t e0 = tile_e0 + tid * PT;
    const int64_t blk = e0 >> lb;
    int cnt = PT;
    if (!FULL) {
        const int64_t rem = n - e0;
        cnt = rem >= PT ? PT : (rem > 0 ? (int)rem : 0);
    }

    // ---- load ----------------------------------------------------------
    // TBL: 4-bit codes dequantised by table (full tiles only).
    constexpr bool kTab = TBL && FULL;
    using TC = TableCodes<LAYOUT>;
    float p[PT], g[PT];
    int qm[PT], qv[PT];
    typename TC::Raw raw[PT / 8];
    if (FULL) {
#pragma unroll
        for (int h = 0; h < PT / 8; ++h) {
            const float4* ps = reinterpret_cast<const float4*>(T.p + e0 + 8 * h);
            const float4 a = __ldcs(ps), b = __ldcs(ps + 1);
            p[8 * h + 0] = a.x; p[8 * h + 1] = a.y; p[8 * h + 2] = a.z; p[8 * h + 3] = a.w;
            p[8 * h + 4] = b.x; p[8 * h + 5] = b.y; p[8 * h + 6] = b.z; p[8 * h + 7] = b.w;
            float gg[8];
            Grad<GT>::load8(T.g, e0 + 8 * h, gg);
#pragma unroll
            for (int j = 0; j < 8; ++j) g[8 * h + j] = gg[j];
            if constexpr (kTab) {
                TC::load8(T, e0 + 8 * h, raw[h]);
            } else {
                int am[8], av[8];
                CI::load8(T, e0 + 8 * h, am, av);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    qm[8 * h + j] = am[j];
                    qv[8 * h + j] = av[j];
                }
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < PT; ++j) {
            p[j] = 0.0f; g[j] = 0.0f; qm[j] = 0; qv[j] = 0;
            if (j < cnt) {
                p[j] = T.p[e0 + j];
                g[j] = Grad<GT>::load1(T.g, e0 + j);
                CI::load1(T, e0 + j, qm[j], qv[j]);
            }
        }
    }
    float sm = 0.0f, sv = 0.0f, vmn = 0.0f;
    if (FULL || cnt > 0) { sm = T.sm[blk]; sv = T.sv[blk]; vmn = T.vmin[blk]; }

    // ---- dequantise, AdamW moments, parameter update -------------------
    // (CUDA/stquant_kernel.cu:163-177, 220-229)
    float m[PT], v[PT];
    if constexpr (kTab) {
        const float kf = small_int_to_float(tid & 15);
        const float tv = dequant_v(kf, sv, vmn);
        const float tm = __fmul_rn(__fsub_rn(kf, 8.0f), sm);
#pragma unroll
        for (int h = 0; h < PT / 8; ++h) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                m[8 * h + j] = TC::m(raw[h], j, tm, sm);
                v[8 * h + j] = TC::v(raw[h], j, tv);
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < PT; ++j) {
            const float qmf = kMagicC ? small_int_to_float(qm[j]) : (float)qm[j];
            m[j] = __fmul_rn(qmf, sm);
            const float qvf = kMagicC ? small_int_to_float(qv[j]) : (float)(unsigned)qv[j];
            v[j] = dequant_v(qvf, sv, vmn);
        }
    }
    if (PROF && tid == 0) prof_mark(pc, 0, t0);
#pragma unroll
    for (int j = 0; j < PT; ++j) {
        m[j] = adam_m(m[j], g[j], C);
        v[j] = adam_v(v[j], g[j], C);
    }
    if (PROF && tid == 0) prof_mark(pc, 1, t0);
#pragma unroll
    for (int j = 0; j < PT; ++j) p[j] = update_p<EXACT_P>(p[j], m[j], v[j], C);
    if (FULL) {
#pragma unroll
        for (int h = 0; h < PT / 8; ++h) {
            float4* pd = reinterpret_cast<float4*>(T.p + e0 + 8 * h);
            __stcs(pd, make_float4(p[8 * h + 0], p[8 * h + 1], p[8 * h + 2], p[8 * h + 3]));
            __stcs(pd + 1, make_float4(p[8 * h + 4], p[8 * h + 5], p[8 * h + 6], p[8 * h + 7]));
        }
    } else {
#pragma unroll
        for (int j = 0; j < PT; ++j)
            if (j < cnt) T.p[e0 + j] = p[j];
    }
    if (PROF && tid == 0) prof_mark(pc, 4, t0);

    // ---- block statistics (CUDA/stquant_kernel.cu:184-199) -------------
    // max |m|, and max / min of logf(x) as logf of max / min x (logf is
    // monotone).  NaN seeds make fmaxf/fminf skip only NaNs, as the
    // reference's reduction does; elements past the end enter as |m| = 0 and
    // x = 1 (log v = 0, :92-93).
    float x[PT];
#pragma unroll
    for (int j = 0; j < PT; ++j) x[j] = (FULL || j < cnt) ? __fadd_rn(v[j], 1e-12f) : 1.0f;
    const int gthreads = (1 << lb) / PT;
    float st[3] = {kNaN, kNaN, kNaN};
#pragma unroll
    for (int j = 0; j < PT; ++j) {
        const bool ok = FULL || j < cnt;
        st[0] = fmaxf(st[0], ok ? fabsf(m[j]) : 0.0f);
    }
#pragma unroll
    for (int j = 0; j < PT; j += 2) {
        st[1] = max3f(st[1], x[j], x[j + 1]);
        st[2] = min3f(st[2], x[j], x[j + 1]);
    }
    group_reduce<0b011u>(st, gthreads, red);
    const float lmax = logf(st[1]);
    const float lmin = logf(st[2]);
    const float new_sm = scale_m_of(st[0], C);
    const float new_sv = scale_v_of(lmax, lmin, C);
    if ((tid & (gthreads - 1)) == 0 && (FULL || (blk << lb) < n)) {
        T.sm[blk] = new_sm;
        T.sv[blk] = new_sv;
        T.vmin[blk] = lmin;
    }
    if (PROF && tid == 0) prof_mark(pc, 2, t0);

    // ---- requantise (CUDA/stquant_kernel.cu:204-216) --------------------
    const float dm = __fadd_rn(new_sm, 1e-12f), dv = __fadd_rn(new_sv, 1e-12f);
    const float rdm = rcp_estimate(dm), rdv = rcp_estimate(dv);
    const float half_dm = 0.5f * dm, half_dv = 0.5f * dv;
    // v codes from the approximate log see X' = RN(a - lmin) instead of the
    // reference's X = RN(logf(x) - lmin): |X' - X| <= log_tol + one ulp of a
    // difference of at most max(lmax - lmin, 1) (logs of floats >= 1e-12 lie
    // in [-27.7, 88.8]).  The remainder test absorbs that error.
    // X' is formed as RN(lg2(x) * ln2 - lmin) in one FMA: against the checked
    // a = RN(lg2(x) * ln2) that adds at most half an ulp of a, |a| 2^-24.
    float thr_v = half_dv;
    if (kApprox) {
        const float amax = fmaxf(fabsf(lmax), fabsf(lmin));
        const float errx = __fmaf_rn(fmaxf(__fsub_rn(lmax, lmin), 1.0f), 0x1p-22f,
                                     __fmaf_rn(amax, 0x1p-23f, log_tol(amax)));
        // (less one relative 2^-22 of d/2 for the rounding of the remainder)
        thr_v = __fmaf_rn(-errx, 1.001f, __fmul_rn(half_dv, 1.0f - 0x1p-22f));
    }
    // 16-bit codes can be mis-rounded by the reciprocal estimate; correct them.
    constexpr bool kCorrect = !kApprox;
    // The positive m extreme rounds to L and clamps to L - 1; every other
    // accepted code already lies in its level range (|m| <= max|m| bounds
    // m / dm by L (1 + 2^-22); accepted v codes have |X'/dv - r| < 1/2 with
    // X' in [-errx, lmax - lmin + errx]).
    constexpr int kB = CI::kMBias;
    const int mw_hi = kMagicBits + kB + (int)C.lm_f - 1;
    // Codes of all PT elements are formed and checked, then stored (forming
    // and storing them eight at a time measured slower).
    constexpr int G = PT;
#pragma unroll
    for (int h0 = 0; h0 < PT; h0 += G) {
        int mw[G], vw[G];
        float rem_m = 0.0f, rem_v = 0.0f;
#pragma unroll
        for (int j = 0; j < G; ++j) {
            const int k = h0 + j;
            float r;
            mw[j] = min(round_checked<kCorrect, kB>(__fmul_rn(m[k], rdm), m[k], dm, half_dm, r), mw_hi);
            rem_m = max_nan(rem_m, r);
            const float xv = kApprox ? __fmaf_rn(approx_log2(x[k]), kLn2, -lmin)
                                     : __fsub_rn(logf(x[k]), lmin);
            vw[j] = round_checked<kCorrect>(__fmul_rn(xv, rdv), xv, dv, half_dv, r);
            rem_v = max_nan(rem_v, r);
        }
        if (!kMagicC || !(rem_m < half_dm && rem_v < thr_v)) {
            // Rare: codes that fail their check take the reference's
            // double-precision expression (all of them for 32-bit codes).
#pragma unroll
            for (int j = 0; j < G; ++j) {
                const int k = h0 + j;
                float r;
                round_checked<kCorrect>(__fmul_rn(m[k], rdm), m[k], dm, half_dm, r);
                if (!kMagicC || !(r < half_dm)) mw[j] = CI::m_word(requant_m_ref(m[k], dm, C.lm_d));
                const float xv = kApprox ? __fmaf_rn(approx_log2(x[k]), kLn2, -lmin)
                                         : __fsub_rn(logf(x[k]), lmin);
                round_checked<kCorrect>(__fmul_rn(xv, rdv), xv, dv, half_dv, r);
                if (!kMagicC || !(r < thr_v))
                    vw[j] = CI::v_word(requant_v_ref(__fsub_rn(logf(x[k]), lmin), dv, C.lv_d));
            }
        }
        if (FULL) {
#pragma unroll
            for (int h = 0; h < G / 8; ++h) {
                int a[8], b[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) { a[j] = mw[8 * h + j]; b[j] = vw[8 * h + j]; }
                CI::store8(T, e0 + h0 + 8 * h, a, b);
            }
        } else {
            // One thread owns all its elements, so M8V4 nibble pairs never race.
#pragma unroll
            for (int j = 0; j < G; ++j)
                if (h0 + j < cnt) CI::store1(T, e0 + h0 + j, mw[j], vw[j]);
        }
    }
    if (PROF && tid == 0) prof_mark(pc, 3, t0);
}

// ---------------------------------------------------------------------------
// Tiled kernel: power-of-two blocks 8..2048.  Each CTA takes a contiguous
// range of tiles; the tensor it is in is staged in shared memory once, and
// CTA-wide barriers happen only at a tensor switch and, for blocks spanning
// several warps, inside the block reduction.
// ---------------------------------------------------------------------------
template <int LAYOUT, typename GT, bool EXACT_P, bool PROF, int CAP, int PT, bool TBL>
__global__ void __launch_bounds__(threads_for<PT>(), PT == 8 ? MDQ_MIN_CTAS_PER_SM : MDQ_MIN_CTAS_PT16)
mdq_step_tiles(const __grid_constant__ LaunchParams<CAP> P) {
    constexpr int kTileT = kTile;
    constexpr int kLogTileT = kLogTile;
    using CI = Codes<LAYOUT>;
    __shared__ float4 s_red[2][kWarps];  // per-warp partials, alternating by tile
    __shared__ TileCtx s_ctx;

    const int tid = threadIdx.x;
    unsigned long long pc[kProfSlots] = {0, 0, 0, 0, 0};
    const int64_t total = P.total_tiles;
    const int tile_lo = (int)(total * blockIdx.x / gridDim.x);
    const int tile_hi = (int)(total * (blockIdx.x + 1) / gridDim.x);
    int cur_end = -1;

    for (int tile = tile_lo; tile < tile_hi; ++tile) {
        if (tile >= cur_end) {
            __syncthreads();  // every thread is done with the previous tensor
            if (tid == 0) {
                const LaunchDesc& D = P.d[find_desc(P, tile)];
                s_ctx.t = D.t;
                s_ctx.n = D.n;
                s_ctx.tile_begin = D.tile_begin;
                s_ctx.tile_end = D.tile_begin + (int32_t)((D.n + kTileT - 1) >> kLogTileT);
                s_ctx.lb = D.log2_block;
                s_ctx.vec = D.vec;
                s_ctx.C = make_step_consts(D.b1, D.b2, D.lr, D.wd, D.eps, D.step, D.m_bits,
                                           D.v_bits);
            }
            __syncthreads();
            cur_end = s_ctx.tile_end;
        }
        unsigned long long t0 = 0;
        if (PROF && tid == 0) t0 = clock64();
        const int64_t n = s_ctx.n;
        const int64_t tile_e0 = (int64_t)(tile - s_ctx.tile_begin) << kLogTileT;

        float4* red = s_red[tile & 1];
        if (s_ctx.vec && tile_e0 + kTileT <= n)
            tile_body<LAYOUT, GT, EXACT_P, PROF, true, PT, TBL>(s_ctx, tile_e0, red, pc, t0);
        else
            tile_body<LAYOUT, GT, EXACT_P, PROF, false, PT, TBL>(s_ctx, tile_e0, red, pc, t0);
    }
    if (PROF && tid == 0 && P.prof != nullptr) {
        for (int k = 0; k < kProfSlots; ++k) atomicAdd(P.prof + k, pc[k]);
    }
}

// ---------------------------------------------------------------------------
// Tree kernel: any block 1..1024, one thread per element, one CTA per block,
// reductions folded exactly as the reference's shared-memory tree
// (CUDA/stquant_kernel.cu:27-50), which for a non-power-of-two CTA reads only
// the elements its halving schedule reaches.
// ---------------------------------------------------------------------------
template <int LAYOUT, typename GT, bool EXACT_P>
__global__ void mdq_step_tree(const LaunchDesc D, unsigned long long* prof) {
    using CI = Codes<LAYOUT>;
    extern __shared__ float s_tree[];  // 3 * blockDim.x
    const int T = blockDim.x;
    const int tid = threadIdx.x;
    const int64_t blk = blockIdx.x;
    const int64_t i = blk * T + tid;
    const bool ok = i < D.n;
    unsigned long long t0 = 0;
    unsigned long long pc[kProfSlots] = {0, 0, 0, 0, 0};
    if (prof && tid == 0) t0 = clock64();

    const StepConsts C = make_step_consts(D.b1, D.b2, D.lr, D.wd, D.eps, D.step, D.m_bits, D.v_bits);
    const float sm = D.t.sm[blk], sv = D.t.sv[blk], vmn = D.t.vmin[blk];
    float g = 0.0f, m = 0.0f, v = 0.0f;
    int qm = 0, qv = 0;
    if (ok) {
        g = Grad<GT>::load1(D.t.g, i);
        CI::load1(D.t, i, qm, qv);
        m = __fmul_rn(CI::kMagicCodes ? small_int_to_float(qm) : (float)qm, sm);
        v = dequant_v(CI::kMagicCodes ? small_int_to_float(qv) : (float)(unsigned)qv, sv, vmn);
        m = adam_m(m, g, C);
        v = adam_v(v, g, C);
    }
    if (prof && tid == 0) prof_mark(pc, 0, t0);

    const float lv = ok ? log_v_of(v) : 0.0f;
    float* r0 = s_tree;
    float* r1 = s_tree + T;
    float* r2 = s_tree + 2 * T;
    r0[tid] = ok ? fabsf(m) : 0.0f;
    r1[tid] = lv;
    r2[tid] = lv;
    __syncthreads();
    for (int s = T / 2; s > 0; s >>= 1) {
        if (tid < s) {
            r0[tid] = fmaxf(r0[tid], r0[tid + s]);
            r1[tid] = fmaxf(r1[tid], r1[tid + s]);
            r2[tid] = fminf(r2[tid], r2[tid + s]);
        }
        __syncthreads();
    }
    const float new_sm = scale_m_of(r0[0], C);
    const float new_sv = scale_v_of(r1[0], r2[0], C);
    const float new_vmin = r2[0];
    __syncthreads();  // every thread has read the folded values
    if (tid == 0) {
        D.t.sm[blk] = new_sm;
        D.t.sv[blk] = new_sv;
        D.t.vmin[blk] = new_vmin;
    }
    if (prof && tid == 0) prof_mark(pc, 2, t0);

    int mw = 0, vw = 0;
    if (ok) {
        const float dm = __fadd_rn(new_sm, 1e-12f), dv = __fadd_rn(new_sv, 1e-12f);
        mw = CI::m_word(requant_m_ref(m, dm, C.lm_d));
        vw = CI::v_word(requant_v_ref(__fsub_rn(lv, new_vmin), dv, C.lv_d));
        if (LAYOUT != MDQ_LAYOUT_M8V4) CI::store1(D.t, i, mw, vw);
    }
    if (LAYOUT == MDQ_LAYOUT_M8V4) {
        // Neighbouring elements share a byte (the block is even, so both lie
        // in this CTA): even elements write first, odd ones after a barrier.
        for (int par = 0; par < 2; ++par) {
            if (ok && (i & 1) == par) CI::store1(D.t, i, mw, vw);
            __syncthreads();
        }
    }
    if (prof && tid == 0) prof_mark(pc, 3, t0);
    if (ok) D.t.p[i] = update_p<EXACT_P>(D.t.p[i], m, v, C);
    if (prof && tid == 0) {
        prof_mark(pc, 4, t0);
        for (int k = 0; k < kProfSlots; ++k) atomicAdd(prof + k, pc[k]);
    }
}

}  // namespace mdq


// ===========================================================================
// Host side
// ===========================================================================
namespace {
thread_local char g_err[512] = "";
}  // namespace

// The library's per-thread error record, shared by every entry point.
mdq_status mdq_fail(mdq_status s, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return s;
}
void mdq_clear_error() { g_err[0] = '\0'; }

namespace {

mdq_status fail(mdq_status s, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return mdq_fail(s, "%s", buf);
}

int storage_bits_m(int layout) {
    switch (layout) {
        case MDQ_LAYOUT_PACKED4: return 4;
        case MDQ_LAYOUT_S8U8: return 8;
        case MDQ_LAYOUT_S16U16: return 16;
        case MDQ_LAYOUT_S32U32: return 32;
        case MDQ_LAYOUT_M8V4: return 8;
    }
    return 0;
}
int storage_bits_v(int layout) {
    switch (layout) {
        case MDQ_LAYOUT_PACKED4: return 4;
        case MDQ_LAYOUT_S8U8: return 8;
        case MDQ_LAYOUT_S16U16: return 16;
        case MDQ_LAYOUT_S32U32: return 32;
        case MDQ_LAYOUT_M8V4: return 4;
    }
    return 0;
}

bool aligned(const void* ptr, uintptr_t a) { return ((uintptr_t)ptr & (a - 1)) == 0; }

bool vec_ok(const mdq_tensor_desc& d) {
    if (!aligned(d.p, 16)) return false;
    if (!aligned(d.grad, 16)) return false;
    switch (d.layout) {
        case MDQ_LAYOUT_PACKED4: return aligned(d.exp_avg, 8);
        case MDQ_LAYOUT_S8U8: return aligned(d.exp_avg, 8) && aligned(d.exp_avg_sq, 8);
        case MDQ_LAYOUT_S16U16:
        case MDQ_LAYOUT_S32U32: return aligned(d.exp_avg, 16) && aligned(d.exp_avg_sq, 16);
        case MDQ_LAYOUT_M8V4: return aligned(d.exp_avg, 8) && aligned(d.exp_avg_sq, 4);
    }
    return false;
}

bool is_pow2(int x) { return x > 0 && (x & (x - 1)) == 0; }
int ilog2(int x) { int l = 0; while ((1 << l) < x) ++l; return l; }

bool fast_eligible(const mdq_tensor_desc& d) {
    return is_pow2(d.block) && d.block >= 8 && d.block <= mdq::kTile;
}

mdq_status validate(const mdq_tensor_desc& d, int idx) {
    if (d.n < 0) return fail(MDQ_ERR_INVALID_ARG, "desc %d: negative n", idx);
    if (d.n == 0) return MDQ_OK;
    if (d.layout < MDQ_LAYOUT_PACKED4 || d.layout > MDQ_LAYOUT_M8V4)
        return fail(MDQ_ERR_INVALID_ARG, "desc %d: bad layout %d", idx, d.layout);
    if (d.grad_dtype != MDQ_F32 && d.grad_dtype != MDQ_BF16)
        return fail(MDQ_ERR_UNSUPPORTED, "desc %d: grad dtype must be MDQ_F32 or MDQ_BF16", idx);
    if (!d.p || !d.grad || !d.exp_avg || !d.scale_m || !d.scale_v || !d.v_min)
        return fail(MDQ_ERR_INVALID_ARG, "desc %d: null pointer", idx);
    if (d.layout != MDQ_LAYOUT_PACKED4 && !d.exp_avg_sq)
        return fail(MDQ_ERR_INVALID_ARG, "desc %d: exp_avg_sq is null", idx);
    if (d.block < 1 || d.block > mdq::kTile)
        return fail(MDQ_ERR_UNSUPPORTED, "desc %d: block %d outside 1..%d", idx, d.block, mdq::kTile);
    if (!fast_eligible(d) && d.block > 1024)
        return fail(MDQ_ERR_UNSUPPORTED, "desc %d: block %d above 1024 must be a power of two",
                    idx, d.block);
    if (d.m_bits < 1 || d.m_bits > storage_bits_m(d.layout))
        return fail(MDQ_ERR_UNSUPPORTED, "desc %d: m_bits %d does not fit layout %d", idx,
                    d.m_bits, d.layout);
    if (d.v_bits < 1 || d.v_bits > storage_bits_v(d.layout))
        return fail(MDQ_ERR_UNSUPPORTED, "desc %d: v_bits %d does not fit layout %d", idx,
                    d.v_bits, d.layout);
    if (d.step < 0) return fail(MDQ_ERR_INVALID_ARG, "desc %d: negative step", idx);
    if (d.layout == MDQ_LAYOUT_M8V4 && (d.block & 1))
        return fail(MDQ_ERR_UNSUPPORTED, "desc %d: M8V4 needs an even block", idx);
    const int64_t tiles = (d.n + mdq::kTile - 1) / mdq::kTile;
    if (tiles > (int64_t)INT32_MAX / 2)
        return fail(MDQ_ERR_TOO_LARGE, "desc %d: n too large", idx);
    if (!fast_eligible(d) && (d.n + d.block - 1) / d.block > (int64_t)INT32_MAX)
        return fail(MDQ_ERR_TOO_LARGE, "desc %d: too many blocks", idx);
    return MDQ_OK;
}

mdq::LaunchDesc to_launch(const mdq_tensor_desc& d) {
    mdq::LaunchDesc L;
    L.t.p = d.p;
    L.t.g = d.grad;
    L.t.m = d.exp_avg;
    L.t.v = d.exp_avg_sq;
    L.t.sm = d.scale_m;
    L.t.sv = d.scale_v;
    L.t.vmin = d.v_min;
    L.n = d.n;
    L.tile_begin = 0;
    L.step = d.step;
    L.lr = d.lr;
    L.wd = d.weight_decay;
    L.eps = d.eps;
    L.b1 = d.beta1;
    L.b2 = d.beta2;
    L.m_bits = (int8_t)d.m_bits;
    L.v_bits = (int8_t)d.v_bits;
    L.log2_block = (int8_t)ilog2(d.block);
    L.vec = (int8_t)vec_ok(d);
    return L;
}

// Resident CTAs per SM for a kernel, cached per device.
struct DevInfo {
    int sms = 0;
};
std::mutex g_mu;
DevInfo g_dev[64];

mdq_status device_sms(int* sms) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(MDQ_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return fail(MDQ_ERR_CUDA, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_dev[dev].sms == 0) {
        int v = 0;
        e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess)
            return fail(MDQ_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
        g_dev[dev].sms = v;
    }
    *sms = g_dev[dev].sms;
    return MDQ_OK;
}

template <typename K>
int blocks_per_sm(K kernel, int threads) {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, threads, 0) != cudaSuccess ||
        b < 1)
        b = 1;
    return b;
}

template <int LAYOUT, typename GT, bool EXACT_P, bool PROF, int CAP, int PT, bool TBL>
mdq_status launch_tiles_t(const mdq::LaunchParams<CAP>& P, int sms, cudaStream_t stream) {
    auto k = mdq::mdq_step_tiles<LAYOUT, GT, EXACT_P, PROF, CAP, PT, TBL>;
    static int occ = 0;  // per instantiation; identical across B200 devices
    constexpr int kNT = mdq::threads_for<PT>();
    if (occ == 0) occ = blocks_per_sm(k, kNT);
    int grid = sms * occ;
    if (grid > P.total_tiles) grid = P.total_tiles;
    k<<<grid, kNT, 0, stream>>>(P);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MDQ_ERR_CUDA, "step launch: %s", cudaGetErrorString(e));
    return MDQ_OK;
}

template <int LAYOUT, typename GT, int CAP, int PT, bool TBL>
mdq_status launch_tiles_pt(const mdq::LaunchParams<CAP>& P, bool exact, bool prof, int sms,
                           cudaStream_t s) {
    if (exact) {
        return prof ? launch_tiles_t<LAYOUT, GT, true, true, CAP, PT, TBL>(P, sms, s)
                    : launch_tiles_t<LAYOUT, GT, true, false, CAP, PT, TBL>(P, sms, s);
    }
    return prof ? launch_tiles_t<LAYOUT, GT, false, true, CAP, PT, TBL>(P, sms, s)
                : launch_tiles_t<LAYOUT, GT, false, false, CAP, PT, TBL>(P, sms, s);
}

// Table dequantisation for 4-bit v codes when every 16-lane half-warp lies in
// one block (block >= 16 * PT).
template <int LAYOUT, typename GT, int CAP>
mdq_status launch_tiles_mode(const mdq::LaunchParams<CAP>& P, bool exact, bool prof, int sms,
                             int pt, int min_block, cudaStream_t s) {
    constexpr bool kV4 = LAYOUT == MDQ_LAYOUT_PACKED4 || LAYOUT == MDQ_LAYOUT_M8V4;
    if constexpr (kV4) {
        // (4-bit v layouts run PT = 16 whenever the block allows tables.)
        if (MDQ_USE_TABLES && pt == 16 && min_block >= 16 * pt)
            return launch_tiles_pt<LAYOUT, GT, CAP, 16, true>(P, exact, prof, sms, s);
    }
    return pt == 16 ? launch_tiles_pt<LAYOUT, GT, CAP, 16, false>(P, exact, prof, sms, s)
                    : launch_tiles_pt<LAYOUT, GT, CAP, 8, false>(P, exact, prof, sms, s);
}

template <int CAP>
mdq_status launch_tiles(int layout, int gdt, const mdq::LaunchParams<CAP>& P, bool exact, bool prof,
                        int sms, int pt, int min_block, cudaStream_t s) {
    const bool bf = gdt == MDQ_BF16;
    switch (layout) {
        case MDQ_LAYOUT_PACKED4:
            return bf ? launch_tiles_mode<MDQ_LAYOUT_PACKED4, __nv_bfloat16, CAP>(P, exact, prof, sms, pt, min_block, s)
                      : launch_tiles_mode<MDQ_LAYOUT_PACKED4, float, CAP>(P, exact, prof, sms, pt, min_block, s);
        case MDQ_LAYOUT_S8U8:
            return bf ? launch_tiles_mode<MDQ_LAYOUT_S8U8, __nv_bfloat16, CAP>(P, exact, prof, sms, pt, min_block, s)
                      : launch_tiles_mode<MDQ_LAYOUT_S8U8, float, CAP>(P, exact, prof, sms, pt, min_block, s);
        case MDQ_LAYOUT_S16U16:
            return bf ? launch_tiles_mode<MDQ_LAYOUT_S16U16, __nv_bfloat16, CAP>(P, exact, prof, sms, pt, min_block, s)
                      : launch_tiles_mode<MDQ_LAYOUT_S16U16, float, CAP>(P, exact, prof, sms, pt, min_block, s);
        case MDQ_LAYOUT_S32U32:
            return bf ? launch_tiles_mode<MDQ_LAYOUT_S32U32, __nv_bfloat16, CAP>(P, exact, prof, sms, pt, min_block, s)
                      : launch_tiles_mode<MDQ_LAYOUT_S32U32, float, CAP>(P, exact, prof, sms, pt, min_block, s);
        case MDQ_LAYOUT_M8V4:
            return bf ? launch_tiles_mode<MDQ_LAYOUT_M8V4, __nv_bfloat16, CAP>(P, exact, prof, sms, pt, min_block, s)
                      : launch_tiles_mode<MDQ_LAYOUT_M8V4, float, CAP>(P, exact, prof, sms, pt, min_block, s);
    }
    return fail(MDQ_ERR_INVALID_ARG, "bad layout %d", layout);
}

template <int LAYOUT, typename GT>
mdq_status launch_tree_t(const mdq::LaunchDesc& L, int block, bool exact,
                         unsigned long long* prof, cudaStream_t s) {
    const int64_t nblk = (L.n + block - 1) / block;
    const size_t smem = 3 * sizeof(float) * (size_t)block;
    if (exact)
        mdq::mdq_step_tree<LAYOUT, GT, true><<<(unsigned)nblk, block, smem, s>>>(L, prof);
    else
        mdq::mdq_step_tree<LAYOUT, GT, false><<<(unsigned)nblk, block, smem, s>>>(L, prof);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MDQ_ERR_CUDA, "tree launch: %s", cudaGetErrorString(e));
    return MDQ_OK;
}

mdq_status launch_tree(const mdq_tensor_desc& d, bool exact, unsigned long long* prof,
                       cudaStream_t s) {
    const mdq::LaunchDesc L = to_launch(d);
    const bool bf = d.grad_dtype == MDQ_BF16;
    switch (d.layout) {
        case MDQ_LAYOUT_PACKED4:
            return bf ? launch_tree_t<MDQ_LAYOUT_PACKED4, __nv_bfloat16>(L, d.block, exact, prof, s)
                      : launch_tree_t<MDQ_LAYOUT_PACKED4, float>(L, d.block, exact, prof, s);
        case MDQ_LAYOUT_S8U8:
            return bf ? launch_tree_t<MDQ_LAYOUT_S8U8, __nv_bfloat16>(L, d.block, exact, prof, s)
                      : launch_tree_t<MDQ_LAYOUT_S8U8, float>(L, d.block, exact, prof, s);
        case MDQ_LAYOUT_S16U16:
            return bf ? launch_tree_t<MDQ_LAYOUT_S16U16, __nv_bfloat16>(L, d.block, exact, prof, s)
                      : launch_tree_t<MDQ_LAYOUT_S16U16, float>(L, d.block, exact, prof, s);
        case MDQ_LAYOUT_S32U32:
            return bf ? launch_tree_t<MDQ_LAYOUT_S32U32, __nv_bfloat16>(L, d.block, exact, prof, s)
                      : launch_tree_t<MDQ_LAYOUT_S32U32, float>(L, d.block, exact, prof, s);
        case MDQ_LAYOUT_M8V4:
            return bf ? launch_tree_t<MDQ_LAYOUT_M8V4, __nv_bfloat16>(L, d.block, exact, prof, s)
                      : launch_tree_t<MDQ_LAYOUT_M8V4, float>(L, d.block, exact, prof, s);
    }
    return fail(MDQ_ERR_INVALID_ARG, "bad layout %d", d.layout);
}

// Packs the fast-path descriptors of one (layout, grad dtype) class into
// launches of at most CAP descriptors each.
template <int CAP>
mdq_status run_class(const mdq_tensor_desc* descs, const int* idx, int count, bool exact,
                     unsigned long long* prof, int sms, cudaStream_t s) {
    static thread_local mdq::LaunchParams<CAP> P;  // ~24 KB for CAP = 224
    // 16 elements per thread (4096-element tiles, 2 CTAs per SM) halve the
    // per-tile work; measured on B200 it pays for 4-bit v codes, and for
    // 8-bit codes only with blocks of 1024 or more.
    int min_block = mdq::kTile;
    for (int k = 0; k < count; ++k) min_block = std::min(min_block, (int)descs[idx[k]].block);
    const int layout = descs[idx[0]].layout;
    const bool v4 = layout == MDQ_LAYOUT_PACKED4 || layout == MDQ_LAYOUT_M8V4;
    const int pt = MDQ_ENABLE_PT16 && ((v4 && min_block >= 16) ||
                                       (layout == MDQ_LAYOUT_S8U8 && min_block >= 1024))
                       ? 16 : 8;
    const int64_t tile = mdq::kTile;
    int i = 0;
    while (i < count) {
        P.n_desc = 0;
        P.prof = prof;
        int64_t tiles = 0;
        while (i < count && P.n_desc < CAP) {
            const mdq_tensor_desc& d = descs[idx[i]];
            const int64_t t = (d.n + tile - 1) / tile;
            if (tiles + t > (int64_t)INT32_MAX && P.n_desc > 0) break;
            mdq::LaunchDesc L = to_launch(d);
            L.tile_begin = (int32_t)tiles;
            P.d[P.n_desc++] = L;
            tiles += t;
            ++i;
        }
        P.total_tiles = (int32_t)tiles;
        const mdq_tensor_desc& d0 = descs[idx[i - 1]];
        const mdq_status st = launch_tiles<CAP>(d0.layout, d0.grad_dtype, P, exact, prof != nullptr,
                                                sms, pt, min_block, s);
        if (st != MDQ_OK) return st;
    }
    return MDQ_OK;
}

}  // namespace

extern "C" {

mdq_status mdq_adamw_step_multi(const mdq_tensor_desc* descs, int32_t n_descs,
                                const mdq_step_options* opts, cudaStream_t stream) {
    g_err[0] = '\0';
    if (n_descs < 0 || (n_descs > 0 && descs == nullptr))
        return fail(MDQ_ERR_INVALID_ARG, "descs is null or n_descs negative");
    const bool exact = opts != nullptr && opts->p_mode == MDQ_P_EXACT;
    if (opts != nullptr && opts->p_mode != MDQ_P_FAST && opts->p_mode != MDQ_P_EXACT)
        return fail(MDQ_ERR_INVALID_ARG, "bad p_mode %d", opts->p_mode);
    unsigned long long* prof = opts ? opts->profile_cycles : nullptr;
    for (int i = 0; i < n_descs; ++i) {
        const mdq_status st = validate(descs[i], i);
        if (st != MDQ_OK) return st;
    }
    int sms = 0;
    bool any_work = false;
    for (int i = 0; i < n_descs; ++i) any_work |= descs[i].n > 0;
    if (any_work) {
        const mdq_status st = device_sms(&sms);
        if (st != MDQ_OK) return st;
    }
    // Group fast-path descriptors by (layout, grad dtype), keeping input order.
    constexpr int kClasses = 5 * 2;
    static thread_local int* order = nullptr;
    static thread_local int order_cap = 0;
    if (order_cap < n_descs) {
        delete[] order;
        order = new int[n_descs];
        order_cap = n_descs;
    }
    for (int c = 0; c < kClasses; ++c) {
        int cnt = 0;
        for (int i = 0; i < n_descs; ++i) {
            const mdq_tensor_desc& d = descs[i];
            if (d.n == 0 || !fast_eligible(d)) continue;
            if (d.layout * 2 + (d.grad_dtype == MDQ_BF16 ? 1 : 0) != c) continue;
            order[cnt++] = i;
        }
        if (cnt == 0) continue;
        const mdq_status st =
            cnt <= mdq::kCapSmall
                ? run_class<mdq::kCapSmall>(descs, order, cnt, exact, prof, sms, stream)
                : run_class<mdq::kCapLarge>(descs, order, cnt, exact, prof, sms, stream);
        if (st != MDQ_OK) return st;
    }
    for (int i = 0; i < n_descs; ++i) {
        const mdq_tensor_desc& d = descs[i];
        if (d.n == 0 || fast_eligible(d)) continue;
        const mdq_status st = launch_tree(d, exact, prof, stream);
        if (st != MDQ_OK) return st;
    }
    return MDQ_OK;
}

mdq_status mdq_fused_adamw(float* p, const void* grad, int32_t grad_dtype, void* exp_avg,
                           int32_t exp_avg_dtype, int64_t exp_avg_numel, void* exp_avg_sq,
                           int32_t exp_avg_sq_dtype, int64_t exp_avg_sq_numel, float* scale_m,
                           float* scale_v, float* v_min, int64_t n, float beta1, float beta2,
                           float lr, float weight_decay, float eps, int32_t step, int32_t bits,
                           int32_t block_size, unsigned long long* profile_cycles,
                           cudaStream_t stream) {
    g_err[0] = '\0';
    if (block_size < 1) return fail(MDQ_ERR_INVALID_ARG, "block_size must be >= 1");
    mdq_tensor_desc d;
    d.p = p;
    d.grad = grad;
    d.exp_avg = exp_avg;
    d.exp_avg_sq = exp_avg_sq;
    d.scale_m = scale_m;
    d.scale_v = scale_v;
    d.v_min = v_min;
    d.n = n;
    d.step = step;
    d.block = block_size > 1024 ? 1024 : block_size;  // CUDA/stquant_kernel.cu:421
    d.lr = lr;
    d.weight_decay = weight_decay;
    d.eps = eps;
    d.beta1 = beta1;
    d.beta2 = beta2;
    d.m_bits = bits;
    d.v_bits = bits;
    d.grad_dtype = grad_dtype;
    // Dispatch of CUDA/stquant_kernel.cu:430-463.
    if (bits == 4 && exp_avg_dtype == MDQ_U8 && exp_avg_sq_numel == 0) {
        if (exp_avg_numel != n)
            return fail(MDQ_ERR_INVALID_ARG, "packed4: exp_avg numel must match parameters");
        d.layout = MDQ_LAYOUT_PACKED4;
        d.exp_avg_sq = nullptr;
    } else if (exp_avg_dtype == MDQ_I8 && exp_avg_sq_dtype == MDQ_U8) {
        d.layout = MDQ_LAYOUT_S8U8;
    } else if (exp_avg_dtype == MDQ_I16 && exp_avg_sq_dtype == MDQ_U16) {
        d.layout = MDQ_LAYOUT_S16U16;
    } else if (exp_avg_dtype == MDQ_I32 && exp_avg_sq_dtype == MDQ_U32) {
        d.layout = MDQ_LAYOUT_S32U32;
    } else {
        return fail(MDQ_ERR_UNSUPPORTED,
                    "MDQ: state must be packed4 (uint8+empty), (int8,uint8), (int16,uint16) or "
                    "(int32,uint32), got dtypes %d / %d bits=%d",
                    exp_avg_dtype, exp_avg_sq_dtype, bits);
    }
    if (d.layout != MDQ_LAYOUT_PACKED4 && (exp_avg_numel < n || exp_avg_sq_numel < n))
        return fail(MDQ_ERR_INVALID_ARG, "exp_avg / exp_avg_sq hold fewer elements than p");
    mdq_step_options o;
    o.p_mode = MDQ_P_EXACT;
    o.profile_cycles = profile_cycles;
    return mdq_adamw_step_multi(&d, 1, &o, stream);
}

const char* mdq_last_error(void) { return g_err; }

int32_t mdq_abi_version(void) { return MDQ_ABI_VERSION; }

}  // extern "C"
