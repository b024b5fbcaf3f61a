// mdq_tiles.cuh - the tiled fused-step kernel (power-of-two blocks 8..2048)
// and its launch templates, shared by the per-layout translation units.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>

#include "mdq.h"
#include "mdq_math.cuh"
#include "mdq_codes.cuh"

// Error reporting of the library (thread-local message, mdq_last_error()).
mdq_status mdq_fail(mdq_status s, const char* fmt, ...);

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
#ifndef MDQ_V4_PT16_MIN_BLOCK
#define MDQ_V4_PT16_MIN_BLOCK 256
#endif
#ifndef MDQ_MIN_CTAS_PER_SM
#define MDQ_MIN_CTAS_PER_SM 3
#endif

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

// Device-side descriptor (one tensor or block-aligned tensor piece).
struct LaunchDesc {
    TensorPtrs t;
    int64_t n;
    int32_t tile_begin;  // first tile of this descriptor within the launch
    int32_t step;
    float lr, wd, eps, b1, b2;
    int8_t m_bits, v_bits, log2_block, vec;
};

// Other GPUs that receive copies of the updated parameters (mdq_step_options).
struct PeerSet {
    int32_t n;
    int64_t delta[7];
};

// Ranks whose gradient buffers are summed by the step (mdq_step_options).
struct GradRanks {
    int32_t n;
    float scale;
    int64_t delta[8];
};

template <int CAP>
struct LaunchParams {
    int32_t n_desc;
    int32_t total_tiles;
    unsigned long long* prof;
    PeerSet peers;
    GradRanks granks;
    LaunchDesc d[CAP];
};

// Store `val` at the same position of every peer's copy of the buffer that
// holds `local` (plain stores over NVLink into mapped peer memory).
template <typename V>
__device__ __forceinline__ void peer_store(const PeerSet& ps, V* local, const V& val) {
    for (int k = 0; k < ps.n; ++k)
        *reinterpret_cast<V*>(reinterpret_cast<char*>(local) + ps.delta[k]) = val;
}

// Four gradient values at element e: the local ones, or (GR: the launch has
// gradient ranks) scale * the fp32 sum over the ranks' buffers in rank
// order.  GR is a template parameter so that kernels without gradient ranks
// keep their register allocation.
template <typename GT, bool GR>
__device__ __forceinline__ void load_grad4(const void* g, int64_t e, float (&o)[4],
                                           const GradRanks& gr) {
    if constexpr (!GR) {
        Grad<GT>::load4(g, e, o);
    } else {
        float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int k = 0; k < gr.n; ++k) {
            float t[4];
            Grad<GT>::load4(static_cast<const char*>(g) + gr.delta[k], e, t);
#pragma unroll
            for (int j = 0; j < 4; ++j) s[j] = __fadd_rn(s[j], t[j]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = __fmul_rn(s[j], gr.scale);
    }
}

template <typename GT, bool GR>
__device__ __forceinline__ float load_grad1(const void* g, int64_t e, const GradRanks& gr) {
    if constexpr (!GR) {
        return Grad<GT>::load1(g, e);
    } else {
        float s = 0.0f;
        for (int k = 0; k < gr.n; ++k)
            s = __fadd_rn(s, Grad<GT>::load1(static_cast<const char*>(g) + gr.delta[k], e));
        return __fmul_rn(s, gr.scale);
    }
}

// Remote gradients staged ahead (gradient ranks, bf16 gradients, PT = 16):
// each thread copies its own elements of the next kStageDepth tiles from the
// other ranks (up to 7) into its own shared-memory slots with cp.async (plain
// 8-byte global-to-shared copies from mapped peer memory; the hardware's
// wait_group, no polling), so the NVLink latency of a tile overlaps the math
// of the tiles before it.  Other shapes load the peers' gradients directly.
constexpr int kStagedPeers = 7;
constexpr int kStageDepth = 2;   // tiles staged ahead
constexpr int kStageThreads = 128;
constexpr int kStageChunks = 4;

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
    const unsigned a = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(a), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The tensor a CTA is working on, staged in shared memory by thread 0.
struct TileCtx {
    PeerSet peers;
    GradRanks granks;
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
// lane of a half-warp must lie in the same block for each chunk: B >= 64.
template <int LAYOUT> struct TableCodes { struct Raw {}; };
template <> struct TableCodes<MDQ_LAYOUT_PACKED4> {
    struct Raw { unsigned w; };
    __device__ static void load4(const TensorPtrs& t, int64_t e, Raw& r) {
        r.w = __ldcs(reinterpret_cast<const unsigned*>(static_cast<const uint8_t*>(t.m) + e));
    }
    // Byte j: q_m + 8 in the low nibble, q_v in the high one.
    __device__ static float m(const Raw& r, int j, float tm, float) {
        return __shfl_sync(0xffffffffu, tm, (int)(r.w >> (8 * j)), 16);
    }
    __device__ static float v(const Raw& r, int j, float tv) {
        return __shfl_sync(0xffffffffu, tv, (int)(r.w >> (8 * j + 4)), 16);
    }
};
template <> struct TableCodes<MDQ_LAYOUT_M8V4> {
    struct Raw { unsigned w; unsigned vw; };
    __device__ static void load4(const TensorPtrs& t, int64_t e, Raw& r) {
        r.w = __ldcs(reinterpret_cast<const unsigned*>(static_cast<const int8_t*>(t.m) + e));
        r.vw = __ldcs(reinterpret_cast<const unsigned short*>(static_cast<const uint8_t*>(t.v) + (e >> 1)));
    }
    // int8 m codes have 256 values: converted directly.
    __device__ static float m(const Raw& r, int j, float, float sm) {
        const int q = (int)(int8_t)(uint8_t)(r.w >> (8 * j));
        return __fmul_rn(small_int_to_float(q), sm);
    }
    __device__ static float v(const Raw& r, int j, float tv) {
        return __shfl_sync(0xffffffffu, tv, (int)(r.vw >> (4 * j)), 16);
    }
};

// Requantisation constants of one block, from its reductions.
struct QConsts {
    float new_sm, new_sv, lmin;
    float dm, dv, rdm, rdv, half_dm, half_dv, thr_v;
    int mw_hi;
};

template <bool APPROX, int MBIAS>
__device__ __forceinline__ QConsts make_q(float max_abs_m, float xmax, float xmin, const StepConsts& C) {
    QConsts q;
    const float lmax = logf(xmax);
    q.lmin = logf(xmin);
    q.new_sm = scale_m_of(max_abs_m, C);
    q.new_sv = scale_v_of(lmax, q.lmin, C);
    q.dm = __fadd_rn(q.new_sm, 1e-12f);
    q.dv = __fadd_rn(q.new_sv, 1e-12f);
    q.rdm = rcp_estimate(q.dm);
    q.rdv = rcp_estimate(q.dv);
    q.half_dm = 0.5f * q.dm;
    q.half_dv = 0.5f * q.dv;
    // v codes from the approximate log see X' = RN(a - lmin) instead of the
    // reference's X = RN(logf(x) - lmin): |X' - X| <= log_tol + one ulp of a
    // difference of at most max(lmax - lmin, 1) (logs of floats >= 1e-12 lie
    // in [-27.7, 88.8]).  The remainder test absorbs that error.
    // X' is formed as RN(lg2(x) * ln2 - lmin) in one FMA: against the checked
    // a = RN(lg2(x) * ln2) that adds at most half an ulp of a, |a| 2^-24.
    q.thr_v = q.half_dv;
    if (APPROX) {
        const float amax = fmaxf(fabsf(lmax), fabsf(q.lmin));
        const float errx = __fmaf_rn(fmaxf(__fsub_rn(lmax, q.lmin), 1.0f), 0x1p-22f,
                                     __fmaf_rn(amax, 0x1p-23f, log_tol(amax)));
        // (less one relative 2^-22 of d/2 for the rounding of the remainder)
        q.thr_v = __fmaf_rn(-errx, 1.001f, __fmul_rn(q.half_dv, 1.0f - 0x1p-22f));
    }
    // The positive m extreme rounds to L and clamps to L - 1; every other
    // accepted code already lies in its level range (|m| <= max|m| bounds
    // m / dm by L (1 + 2^-22); accepted v codes have |X'/dv - r| < 1/2 with
    // X' in [-errx, lmax - lmin + errx]).
    q.mw_hi = kMagicBits + MBIAS + (int)C.lm_f - 1;
    return q;
}

// One tile of 2048 elements.  Thread layout ("stripes"): the L = min(32, B/PT)
// lanes that share a quantisation block own it interleaved in chunks of 4
// elements: lane r of a stripe owns elements 4*L*i + 4*r + (0..3), i < PT/4,
// of the stripe's span of L*PT elements.  Every element of a thread is thus in
// one block, and each warp-wide access covers whole 32-byte sectors (one or
// more 128-byte lines of parameters).  Stripes of 32 lanes cover one warp's
// 32*PT elements; a block of B > 32*PT elements spans B/(32*PT) warps.
// FULL: every element in range and all pointers allow vector access.
// `red` is this tile's cross-warp reduction scratch.
template <int LAYOUT, typename GT, bool EXACT_P, bool PROF, bool FULL, int PT, bool TBL, bool GR>
__device__ __forceinline__ void tile_body(const TileCtx& X, int64_t tile_e0,
                                          float4* red,
                                          unsigned long long (&pc)[kProfSlots],
                                          unsigned long long& t0,
                                          const uint2* stg = nullptr) {
    using CI = Codes<LAYOUT>;
    using TC = TableCodes<LAYOUT>;
    constexpr int NCH = PT / 4;
    constexpr int kLogPT = PT == 16 ? 4 : 3;
    constexpr int kSpan = 32 * PT;   // elements per warp and tile
    constexpr bool kApprox = CI::kApproxLog;
    constexpr bool kMagicC = CI::kMagicCodes;
    constexpr bool kTab = TBL && FULL;
    constexpr int kB = CI::kMBias;
    const float kNaN = __int_as_float(0x7fffffff);
    const int tid = threadIdx.x;
    const int lane = tid & 31, w = tid >> 5;
    const TensorPtrs T = X.t;
    const StepConsts& C = X.C;
    const int lb = X.lb;
    const int B = 1 << lb;
    const int64_t n = X.n;
    const int lgL = min(5, lb - kLogPT);  // lanes per stripe: L = 2^lgL
    const int L = 1 << lgL;
    const int r = lane & (L - 1);
    // Chunk i of this thread starts at e_first + 4*L*i.
    const int64_t e_first = tile_e0 + (int64_t)w * kSpan + ((lane >> lgL) << (lgL + kLogPT)) + 4 * r;
    const int cstride = 4 * L;
    const int64_t blk = e_first >> lb;
    int cnt[NCH];
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        cnt[i] = 4;
        if (!FULL) {
            const int64_t rem = n - (e_first + (int64_t)cstride * i);
            cnt[i] = rem >= 4 ? 4 : (rem > 0 ? (int)rem : 0);
        }
    }

    // ---- load ----------------------------------------------------------
    float p[PT], g[PT];
    int qm[PT], qv[PT];
    typename TC::Raw raw[NCH];
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int64_t e = e_first + (int64_t)cstride * i;
        if (FULL) {
            const float4 a = __ldcs(reinterpret_cast<const float4*>(T.p + e));
            p[4 * i + 0] = a.x; p[4 * i + 1] = a.y; p[4 * i + 2] = a.z; p[4 * i + 3] = a.w;
            float gg[4];
            if constexpr (GR && sizeof(GT) == 2 && PT == 16) {
                if (stg != nullptr) {
                    // This rank's values from memory, the others' from the
                    // staged copies; summed in rank order.
                    float sacc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    int slot = 0;
                    for (int k = 0; k < X.granks.n; ++k) {
                        uint2 w;
                        if (X.granks.delta[k] == 0) {
                            w = __ldcs(reinterpret_cast<const uint2*>(
                                static_cast<const __nv_bfloat16*>(T.g) + e));
                        } else {
                            w = stg[(slot * kStageChunks + i) * kStageThreads + threadIdx.x];
                            ++slot;
                        }
                        sacc[0] = __fadd_rn(sacc[0], __uint_as_float(w.x << 16));
                        sacc[1] = __fadd_rn(sacc[1], __uint_as_float(w.x & 0xffff0000u));
                        sacc[2] = __fadd_rn(sacc[2], __uint_as_float(w.y << 16));
                        sacc[3] = __fadd_rn(sacc[3], __uint_as_float(w.y & 0xffff0000u));
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) gg[j] = __fmul_rn(sacc[j], X.granks.scale);
                } else {
                    load_grad4<GT, GR>(T.g, e, gg, X.granks);
                }
            } else {
                load_grad4<GT, GR>(T.g, e, gg, X.granks);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) g[4 * i + j] = gg[j];
            if constexpr (kTab) {
                TC::load4(T, e, raw[i]);
            } else {
                int am[4], av[4];
                CI::load4(T, e, am, av);
#pragma unroll
                for (int j = 0; j < 4; ++j) { qm[4 * i + j] = am[j]; qv[4 * i + j] = av[j]; }
            }
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int k = 4 * i + j;
                p[k] = 0.0f; g[k] = 0.0f; qm[k] = 0; qv[k] = 0;
                if (j < cnt[i]) {
                    p[k] = T.p[e + j];
                    g[k] = load_grad1<GT, GR>(T.g, e + j, X.granks);
                    CI::load1(T, e + j, qm[k], qv[k]);
                }
            }
        }
    }
    // The block's scales (a block past the end is not read).
    float sm = 0.0f, sv = 0.0f, vmn = 0.0f;
    if (FULL || (blk << lb) < n) { sm = T.sm[blk]; sv = T.sv[blk]; vmn = T.vmin[blk]; }

    // ---- dequantise, AdamW moments, parameter update -------------------
    // (CUDA/stquant_kernel.cu:163-177, 220-229)
    float m[PT], v[PT];
    if constexpr (kTab) {
        const float kf = small_int_to_float(lane & 15);
        const float tv = dequant_v(kf, sv, vmn);
        const float tm = __fmul_rn(__fsub_rn(kf, 8.0f), sm);
#pragma unroll
        for (int i = 0; i < NCH; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                m[4 * i + j] = TC::m(raw[i], j, tm, sm);
                v[4 * i + j] = TC::v(raw[i], j, tv);
            }
    } else if constexpr (kMagicC) {
        // Element pairs: the magic-word subtraction, the scale multiply and
        // the exponent's fused multiply-add as paired instructions.
#pragma unroll
        for (int k = 0; k < PT; k += 2) {
            const float2 qmf = add2_rn(make_float2(__int_as_float(kMagicBits + qm[k]),
                                                   __int_as_float(kMagicBits + qm[k + 1])),
                                       bcast2(-kMagic));
            const float2 mm = mul2_rn(qmf, bcast2(sm));
            const float2 qvf = add2_rn(make_float2(__int_as_float(kMagicBits + qv[k]),
                                                   __int_as_float(kMagicBits + qv[k + 1])),
                                       bcast2(-kMagic));
            const float2 ev = fma2_rn(qvf, bcast2(sv), bcast2(vmn));
            m[k] = mm.x; m[k + 1] = mm.y;
            v[k] = expf(ev.x); v[k + 1] = expf(ev.y);
        }
    } else {
#pragma unroll
        for (int k = 0; k < PT; ++k) {
            m[k] = __fmul_rn((float)qm[k], sm);
            v[k] = dequant_v((float)(unsigned)qv[k], sv, vmn);
        }
    }
    if (PROF && tid == 0) prof_mark(pc, 0, t0);
    // AdamW moments and the parameter update on element pairs (mdq_math.cuh).
#pragma unroll
    for (int k = 0; k < PT; k += 2) {
        const float2 gg = make_float2(g[k], g[k + 1]);
        const float2 mm = adam_m2(make_float2(m[k], m[k + 1]), gg, C);
        const float2 vv = adam_v2(make_float2(v[k], v[k + 1]), gg, C);
        m[k] = mm.x; m[k + 1] = mm.y;
        v[k] = vv.x; v[k + 1] = vv.y;
    }
    if (PROF && tid == 0) prof_mark(pc, 1, t0);
#pragma unroll
    for (int k = 0; k < PT; k += 2) {
        const float2 pp = update_p2<EXACT_P>(make_float2(p[k], p[k + 1]), make_float2(m[k], m[k + 1]),
                                             make_float2(v[k], v[k + 1]), C);
        p[k] = pp.x; p[k + 1] = pp.y;
    }
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int64_t e = e_first + (int64_t)cstride * i;
        if (FULL) {
            __stcs(reinterpret_cast<float4*>(T.p + e),
                   make_float4(p[4 * i + 0], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]));
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < cnt[i]) T.p[e + j] = p[4 * i + j];
        }
    }
    if (T.p16 != nullptr) {
        // bf16 copy of the updated parameters (a sharded optimizer's
        // all-gather send buffer), round to nearest even; and the peers' copies.
#pragma unroll
        for (int i = 0; i < NCH; ++i) {
            const int64_t e = e_first + (int64_t)cstride * i;
            if (FULL) {
                const __nv_bfloat162 lo = __floats2bfloat162_rn(p[4 * i + 0], p[4 * i + 1]);
                const __nv_bfloat162 hi = __floats2bfloat162_rn(p[4 * i + 2], p[4 * i + 3]);
                uint2 w;
                w.x = *reinterpret_cast<const unsigned*>(&lo);
                w.y = *reinterpret_cast<const unsigned*>(&hi);
                __stcs(reinterpret_cast<uint2*>(T.p16 + e), w);
                peer_store(X.peers, reinterpret_cast<uint2*>(T.p16 + e), w);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j < cnt[i]) {
                        const __nv_bfloat16 b = __float2bfloat16_rn(p[4 * i + j]);
                        T.p16[e + j] = b;
                        peer_store(X.peers, T.p16 + e + j, b);
                    }
            }
        }
    } else if (X.peers.n > 0) {
        // fp32 parameters: the peers' copies of the updated values.
#pragma unroll
        for (int i = 0; i < NCH; ++i) {
            const int64_t e = e_first + (int64_t)cstride * i;
            if (FULL) {
                peer_store(X.peers, reinterpret_cast<float4*>(T.p + e),
                           make_float4(p[4 * i + 0], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]));
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j < cnt[i]) peer_store(X.peers, T.p + e + j, p[4 * i + j]);
            }
        }
    }
    if (PROF && tid == 0) prof_mark(pc, 4, t0);

    // ---- block statistics (CUDA/stquant_kernel.cu:184-199) -------------
    // max |m|, and max / min of logf(x) as logf of max / min x (logf is
    // monotone).  NaN seeds make fmaxf/fminf skip only NaNs, as the
    // reference's reduction does; elements past the end enter as |m| = 0 and
    // x = 1 (log v = 0, :92-93).
    float x[PT];
    if (FULL) {
#pragma unroll
        for (int k = 0; k < PT; k += 2) {
            const float2 xx = add2_rn(make_float2(v[k], v[k + 1]), bcast2(1e-12f));
            x[k] = xx.x; x[k + 1] = xx.y;
        }
    } else {
#pragma unroll
        for (int k = 0; k < PT; ++k) x[k] = (k & 3) < cnt[k / 4] ? __fadd_rn(v[k], 1e-12f) : 1.0f;
    }
    float s0 = kNaN, s1 = kNaN, s2 = kNaN;
#pragma unroll
    for (int k = 0; k < PT; k += 2) {
        const bool ok0 = FULL || (k & 3) < cnt[k / 4];
        const bool ok1 = FULL || ((k + 1) & 3) < cnt[k / 4];
        s0 = max3f(s0, ok0 ? fabsf(m[k]) : 0.0f, ok1 ? fabsf(m[k + 1]) : 0.0f);
    }
#pragma unroll
    for (int k = 0; k < PT; k += 2) {
        s1 = max3f(s1, x[k], x[k + 1]);
        s2 = min3f(s2, x[k], x[k + 1]);
    }
    if (L == 32) {
        asm volatile("redux.sync.max.f32 %0, %0, 0xffffffff;" : "+f"(s0));
        asm volatile("redux.sync.max.f32 %0, %0, 0xffffffff;" : "+f"(s1));
        asm volatile("redux.sync.min.f32 %0, %0, 0xffffffff;" : "+f"(s2));
        if (B > kSpan) {
            // One block spans B / kSpan warps: exchange one float4 per warp
            // among them, at a named barrier of only those warps (ids 1..).
            const int wpb = B / kSpan;
            if (lane == 0) red[w] = make_float4(s0, s1, s2, 0.0f);
            if (MDQ_GROUP_BARRIER && wpb < (int)(blockDim.x >> 5))
                asm volatile("bar.sync %0, %1;" ::"r"(1 + w / wpb), "r"(32 * wpb) : "memory");
            else
                __syncthreads();
            const int w0 = (w / wpb) * wpb;
            for (int k = 0; k < wpb; ++k) {
                const float4 o = red[w0 + k];
                s0 = fmaxf(s0, o.x);
                s1 = fmaxf(s1, o.y);
                s2 = fminf(s2, o.z);
            }
        }
    } else {
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) {
            if (o < L) {
                s0 = fmaxf(s0, __shfl_xor_sync(0xffffffffu, s0, o));
                s1 = fmaxf(s1, __shfl_xor_sync(0xffffffffu, s1, o));
                s2 = fminf(s2, __shfl_xor_sync(0xffffffffu, s2, o));
            }
        }
    }
    const QConsts Q = make_q<kApprox, kB>(s0, s1, s2, C);
    if ((e_first & (B - 1)) == 0 && e_first < n) {  // this thread starts the block
        T.sm[blk] = Q.new_sm;
        T.sv[blk] = Q.new_sv;
        T.vmin[blk] = Q.lmin;
    }
    if (PROF && tid == 0) prof_mark(pc, 2, t0);

    // ---- requantise (CUDA/stquant_kernel.cu:204-216) --------------------
    // 16-bit codes can be mis-rounded by the reciprocal estimate; correct them.
    constexpr bool kCorrect = !kApprox;
    int mw[PT], vw[PT];
    float rem_m = 0.0f, rem_v = 0.0f;
#pragma unroll
    for (int k = 0; k < PT; ++k) {
        float rr;
        mw[k] = min(round_checked<kCorrect, kB>(__fmul_rn(m[k], Q.rdm), m[k], Q.dm, Q.half_dm, rr),
                    Q.mw_hi);
        rem_m = max_nan(rem_m, rr);
        const float xv = kApprox ? __fmaf_rn(approx_log2(x[k]), kLn2, -Q.lmin)
                                 : __fsub_rn(logf(x[k]), Q.lmin);
        vw[k] = round_checked<kCorrect>(__fmul_rn(xv, Q.rdv), xv, Q.dv, Q.half_dv, rr);
        rem_v = max_nan(rem_v, rr);
    }
    if (!kMagicC || !(rem_m < Q.half_dm && rem_v < Q.thr_v)) {
        // Rare: codes that fail their check take the reference's
        // double-precision expression (all of them for 32-bit codes).
#pragma unroll
        for (int k = 0; k < PT; ++k) {
            float rr;
            round_checked<kCorrect>(__fmul_rn(m[k], Q.rdm), m[k], Q.dm, Q.half_dm, rr);
            if (!kMagicC || !(rr < Q.half_dm)) mw[k] = CI::m_word(requant_m_ref(m[k], Q.dm, C.lm_d));
            const float xv = kApprox ? __fmaf_rn(approx_log2(x[k]), kLn2, -Q.lmin)
                                     : __fsub_rn(logf(x[k]), Q.lmin);
            round_checked<kCorrect>(__fmul_rn(xv, Q.rdv), xv, Q.dv, Q.half_dv, rr);
            if (!kMagicC || !(rr < Q.thr_v))
                vw[k] = CI::v_word(requant_v_ref(__fsub_rn(logf(x[k]), Q.lmin), Q.dv, C.lv_d));
        }
    }
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
        const int64_t e = e_first + (int64_t)cstride * i;
        int a4[4], b4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) { a4[j] = mw[4 * i + j]; b4[j] = vw[4 * i + j]; }
        if (FULL) {
            CI::store4(T, e, a4, b4);
        } else {
            // One thread owns whole chunks, so M8V4 nibble pairs never race.
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (j < cnt[i]) CI::store1(T, e + j, a4[j], b4[j]);
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
template <int LAYOUT, typename GT, bool EXACT_P, bool PROF, int CAP, int PT, bool TBL, bool GR>
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
    constexpr bool kStage = GR && sizeof(GT) == 2 && PT == 16;
    // Staging slots (dynamic shared memory, sized by the launch for the
    // number of other ranks): [stage][rank slot][chunk][thread].
    extern __shared__ __align__(16) uint2 s_stage[];
    const int n_other = P.granks.n - 1;
    int next_issue = tile_lo;   // first tile whose copies are not issued yet

    for (int tile = tile_lo; tile < tile_hi; ++tile) {
        if (tile >= cur_end) {
            __syncthreads();  // every thread is done with the previous tensor
            if (tid == 0) {
                const LaunchDesc& D = P.d[find_desc(P, tile)];
                s_ctx.peers = P.peers;
                s_ctx.granks = P.granks;
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
        const bool full = s_ctx.vec && tile_e0 + kTileT <= n;
        const uint2* stg = nullptr;
        if constexpr (kStage) {
            const int np = s_ctx.granks.n - 1;       // other ranks
            if (np >= 1 && np <= kStagedPeers) {
                if (tile >= next_issue) next_issue = tile;   // (a new run of tiles)
                // Keep the copies of up to kStageDepth tiles ahead in flight,
                // one commit group per tile, within this tensor's full tiles.
                const int lgL = min(5, s_ctx.lb - 4);
                const int L = 1 << lgL;
                const int lane = tid & 31, w = tid >> 5;
                const int64_t within = (int64_t)w * 512 + ((lane >> lgL) << (lgL + 4)) +
                                       4 * (lane & (L - 1));
                while (next_issue <= tile + kStageDepth && next_issue < tile_hi &&
                       next_issue < cur_end) {
                    const int64_t e_t = (int64_t)(next_issue - s_ctx.tile_begin) << kLogTileT;
                    if (!(s_ctx.vec && e_t + kTileT <= n)) break;   // tail tile: loaded directly
                    const int slot_stage = next_issue % (kStageDepth + 1);
                    int slot = 0;
                    for (int k = 0; k < s_ctx.granks.n; ++k) {
                        if (s_ctx.granks.delta[k] == 0) continue;
                        const char* base = static_cast<const char*>(s_ctx.t.g) + s_ctx.granks.delta[k];
#pragma unroll
                        for (int i = 0; i < kStageChunks; ++i) {
                            const int64_t e = e_t + within + (int64_t)(4 * L) * i;
                            cp_async8(&s_stage[((slot_stage * n_other + slot) * kStageChunks + i) *
                                               kStageThreads + tid],
                                      base + 2 * e);
                        }
                        ++slot;
                    }
                    cp_async_commit();
                    ++next_issue;
                }
                if (tile < next_issue) {
                    // Groups committed after this tile's own may stay in flight.
                    const int after = next_issue - 1 - tile;
                    if (after >= 2) cp_async_wait<2>();
                    else if (after == 1) cp_async_wait<1>();
                    else cp_async_wait<0>();
                    if (full)
                        stg = &s_stage[(tile % (kStageDepth + 1)) * n_other * kStageChunks *
                                       kStageThreads];
                }
            }
        }
        if (full)
            tile_body<LAYOUT, GT, EXACT_P, PROF, true, PT, TBL, GR>(s_ctx, tile_e0, red, pc, t0, stg);
        else
            tile_body<LAYOUT, GT, EXACT_P, PROF, false, PT, TBL, GR>(s_ctx, tile_e0, red, pc, t0);
    }
    if (PROF && tid == 0 && P.prof != nullptr) {
        for (int k = 0; k < kProfSlots; ++k) atomicAdd(P.prof + k, pc[k]);
    }
}


}  // namespace mdq

namespace mdq {

template <typename K>
int blocks_per_sm(K kernel, int threads) {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, threads, 0) != cudaSuccess ||
        b < 1)
        b = 1;
    return b;
}

template <int LAYOUT, typename GT, bool EXACT_P, bool PROF, int CAP, int PT, bool TBL, bool GR>
mdq_status launch_tiles_t(const LaunchParams<CAP>& P, int sms, cudaStream_t stream) {
    auto k = mdq_step_tiles<LAYOUT, GT, EXACT_P, PROF, CAP, PT, TBL, GR>;
    constexpr int kNT = threads_for<PT>();
    constexpr bool kStage = GR && sizeof(GT) == 2 && PT == 16;
    int occ = 0;
    size_t smem = 0;
    if constexpr (kStage) {
        // Staging slots for the other ranks' gradients (up to 7 x 3 x 4 KB).
        const int n_other = P.granks.n - 1;
        if (n_other >= 1 && n_other <= kStagedPeers)
            smem = (size_t)(kStageDepth + 1) * n_other * kStageChunks * kStageThreads *
                   sizeof(uint2);
        // (set on every launch: the attribute is per device)
        const cudaError_t ea = cudaFuncSetAttribute(
            k, cudaFuncAttributeMaxDynamicSharedMemorySize,
            (int)((kStageDepth + 1) * kStagedPeers * kStageChunks * kStageThreads * sizeof(uint2)));
        if (ea != cudaSuccess)
            return mdq_fail(MDQ_ERR_CUDA, "staging smem attribute: %s", cudaGetErrorString(ea));
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kNT, smem) != cudaSuccess ||
            occ < 1)
            occ = 1;
    } else {
        static int occ_s = 0;  // per instantiation; identical across B200 devices
        if (occ_s == 0) occ_s = blocks_per_sm(k, kNT);
        occ = occ_s;
    }
    int grid = sms * occ;
    if (grid > P.total_tiles) grid = P.total_tiles;
    k<<<grid, kNT, smem, stream>>>(P);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return mdq_fail(MDQ_ERR_CUDA, "step launch: %s", cudaGetErrorString(e));
    return MDQ_OK;
}

template <int LAYOUT, typename GT, int CAP, int PT, bool TBL>
mdq_status launch_tiles_pt(const LaunchParams<CAP>& P, bool exact, bool prof, int sms,
                           cudaStream_t s) {
    // Launches that sum gradients over ranks take their own instantiation
    // (without the clock64 profiler).
    if (P.granks.n > 0) {
        return exact ? launch_tiles_t<LAYOUT, GT, true, false, CAP, PT, TBL, true>(P, sms, s)
                     : launch_tiles_t<LAYOUT, GT, false, false, CAP, PT, TBL, true>(P, sms, s);
    }
    if (exact) {
        return prof ? launch_tiles_t<LAYOUT, GT, true, true, CAP, PT, TBL, false>(P, sms, s)
                    : launch_tiles_t<LAYOUT, GT, true, false, CAP, PT, TBL, false>(P, sms, s);
    }
    return prof ? launch_tiles_t<LAYOUT, GT, false, true, CAP, PT, TBL, false>(P, sms, s)
                : launch_tiles_t<LAYOUT, GT, false, false, CAP, PT, TBL, false>(P, sms, s);
}

// Shapes instantiated per layout (chosen from B200 measurements): 4-bit-v
// layouts run PT = 16 for blocks of >= 256 elements, else PT = 8, with tables
// whenever every stripe has >= 16 lanes (B >= 16 * PT); all other layouts run
// PT = 8.  (A thread's PT elements lie in one block: B >= PT.)
template <int LAYOUT, typename GT, int CAP>
mdq_status launch_tiles_mode(const LaunchParams<CAP>& P, bool exact, bool prof, int sms,
                             int pt, int min_block, cudaStream_t s) {
    constexpr bool kV4 = LAYOUT == MDQ_LAYOUT_PACKED4 || LAYOUT == MDQ_LAYOUT_M8V4;
    if constexpr (kV4) {
        if (pt == 16) {
            // (PT = 16 runs only for blocks of >= 256: every stripe has 16+ lanes.)
            return launch_tiles_pt<LAYOUT, GT, CAP, 16, MDQ_USE_TABLES != 0>(P, exact, prof, sms, s);
        }
        if (MDQ_USE_TABLES && min_block >= 16 * 8)
            return launch_tiles_pt<LAYOUT, GT, CAP, 8, true>(P, exact, prof, sms, s);
        return launch_tiles_pt<LAYOUT, GT, CAP, 8, false>(P, exact, prof, sms, s);
    } else {
        return launch_tiles_pt<LAYOUT, GT, CAP, 8, false>(P, exact, prof, sms, s);
    }
}

// Per-layout entry points; each is defined in its own translation unit
// (mdq_tiles_<layout>.cu) so the kernel instantiations compile in parallel.
#define MDQ_TILES_SIG(NAME, CAP)                                                              \
    mdq_status launch_tiles_##NAME(int gdt, const LaunchParams<CAP>& P, bool exact, bool prof, \
                                   int sms, int pt, int min_block, cudaStream_t s)
#define MDQ_TILES_DECLARE(NAME)          \
    MDQ_TILES_SIG(NAME, kCapSmall);      \
    MDQ_TILES_SIG(NAME, kCapLarge);
#define MDQ_TILES_DEFINE_CAP(NAME, LAYOUT, CAP)                                                   \
    MDQ_TILES_SIG(NAME, CAP) {                                                                    \
        return gdt == MDQ_BF16                                                                    \
                   ? launch_tiles_mode<LAYOUT, __nv_bfloat16, CAP>(P, exact, prof, sms, pt, min_block, s) \
                   : launch_tiles_mode<LAYOUT, float, CAP>(P, exact, prof, sms, pt, min_block, s);        \
    }
#define MDQ_TILES_DEFINE(NAME, LAYOUT)                  \
    MDQ_TILES_DEFINE_CAP(NAME, LAYOUT, kCapSmall)       \
    MDQ_TILES_DEFINE_CAP(NAME, LAYOUT, kCapLarge)

MDQ_TILES_DECLARE(packed4)
MDQ_TILES_DECLARE(s8u8)
MDQ_TILES_DECLARE(s16u16)
MDQ_TILES_DECLARE(s32u32)
MDQ_TILES_DECLARE(m8v4)

}  // namespace mdq
