// mdq_blocks.cuh - the warp-per-block fused-step kernel for quantisation
// blocks of 512 or 1024 elements.
//
// In the tiled kernel (mdq_tiles.cuh) a block wider than one warp's span of
// 32 x PT elements is shared by several warps, which exchange their partial
// extremes through shared memory behind a named barrier on every tile, and
// every thread evaluates the block's requantisation constants (two logf, an
// IEEE divide, two reciprocals) for only PT elements.  Here one warp owns a
// whole block: it walks the block in S = B / 256 sub-tiles of 8 elements per
// lane (the stripe layout: lane r holds elements 128 i + 4 r + 0..3 of a
// sub-tile, i = 0, 1, so every warp access covers whole 32-byte sectors),
//   pass 1: loads p, g and the codes of a sub-tile, dequantises with the
//           block's old scales, applies AdamW, stores p, and parks the new m
//           and x = v + 1e-12 in the warp's slice of shared memory (each lane
//           reads back only what it wrote, so no barrier is needed);
//   then:   reduces max|m|, max x, min x over the warp with redux.sync and
//           computes the block's constants once per 32 S elements per lane;
//   pass 2: requantises the parked m and x and stores the codes.
// Warps work independently (no CTA barrier at all); a CTA of 8 warps takes 8
// consecutive blocks at a time, so it streams 8 B contiguous elements.
#pragma once

#include "mdq_tiles.cuh"

namespace mdq {

// Resident CTAs per SM: 1024-element blocks run 2 (128 registers per thread,
// no spills, 16 warps), 512-element blocks 3 (80 registers, 24 warps); both
// measured best on B200 for int8/uint8 codes.
template <int LOGB> constexpr int blk_min_ctas() { return LOGB >= 10 ? 2 : 3; }

constexpr int kBlkWarps = 8;
constexpr int kBlkThreads = 32 * kBlkWarps;

// Shared-memory bytes of one CTA for blocks of 2^LOGB elements.
template <int LOGB> constexpr int blocks_smem_bytes() {
    return kBlkWarps * (2 << LOGB) * (int)sizeof(float);
}

// Raw (undecoded) gradient words of 4 elements, so that a sub-tile's loads
// can be issued one sub-tile ahead and decoded later.
template <typename GT> struct GradRaw;
template <> struct GradRaw<float> {
    using T = float4;
    __device__ static T load(const void* g, int64_t e) {
        return __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(g) + e));
    }
    __device__ static void decode(const T& w, float* o) { o[0] = w.x; o[1] = w.y; o[2] = w.z; o[3] = w.w; }
};
template <> struct GradRaw<__nv_bfloat16> {
    using T = uint2;
    __device__ static T load(const void* g, int64_t e) {
        return __ldcs(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(g) + e));
    }
    __device__ static void decode(const T& w, float* o) {
        o[0] = __uint_as_float(w.x << 16);
        o[1] = __uint_as_float(w.x & 0xffff0000u);
        o[2] = __uint_as_float(w.y << 16);
        o[3] = __uint_as_float(w.y & 0xffff0000u);
    }
};

// Loads of one sub-tile, issued ahead of their use: p, g and the code words
// (one byte per element of m codes or of packed 4-bit pairs, and of v codes
// when the layout has a separate v array).
template <typename GT> struct PreLoads {
    float4 p[2];
    typename GradRaw<GT>::T g[2];
    unsigned m[2], v[2];
    bool valid;
    __device__ void load(const TensorPtrs& T, int64_t e_sub, int lane) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int64_t e = e_sub + 128 * i + 4 * lane;
            p[i] = __ldcs(reinterpret_cast<const float4*>(T.p + e));
            g[i] = GradRaw<GT>::load(T.g, e);
            m[i] = __ldcs(reinterpret_cast<const unsigned*>(static_cast<const uint8_t*>(T.m) + e));
            if (T.v != nullptr)
                v[i] = __ldcs(reinterpret_cast<const unsigned*>(static_cast<const uint8_t*>(T.v) + e));
        }
        valid = true;
    }
};

// Where pass 1 parks a lane's m and x = v + 1e-12 for pass 2: elements
// 256 s + 128 i + 4 lane + (0..3) of the block, as one float4 each.
struct ParkSplit {
    float* wm;
    float* wx;
    __device__ float* m(int s, int i, int lane) const { return wm + 256 * s + 128 * i + 4 * lane; }
    __device__ float* x(int s, int i, int lane) const { return wx + 256 * s + 128 * i + 4 * lane; }
};

// Pass 2 of a block (CUDA/stquant_kernel.cu:204-216): requantises the parked
// m and x of the block at e0 with the block's new constants Q and stores the
// codes.  Each lane reads back only what it parked itself.
template <int LAYOUT, bool FULL, int LOGB, typename PARK>
__device__ __forceinline__ void requant_block(const TileCtx& X, int64_t e0, const QConsts& Q,
                                              const PARK& park) {
    using CI = Codes<LAYOUT>;
    constexpr int S = (1 << LOGB) / 256;
    constexpr bool kApprox = CI::kApproxLog;
    constexpr bool kMagicC = CI::kMagicCodes;
    constexpr int kB = CI::kMBias;
    const int lane = threadIdx.x & 31;
    const TensorPtrs T = X.t;
    const StepConsts& C = X.C;
    const int64_t n = X.n;
    constexpr bool kCorrect = !kApprox;
#pragma unroll 1
    for (int s = 0; s < S; ++s) {
        float m[8], x[8];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float4 a = *reinterpret_cast<const float4*>(park.m(s, i, lane));
            const float4 b = *reinterpret_cast<const float4*>(park.x(s, i, lane));
            m[4 * i + 0] = a.x; m[4 * i + 1] = a.y; m[4 * i + 2] = a.z; m[4 * i + 3] = a.w;
            x[4 * i + 0] = b.x; x[4 * i + 1] = b.y; x[4 * i + 2] = b.z; x[4 * i + 3] = b.w;
        }
        int mw[8], vw[8];
        float rem_m = 0.0f, rem_v = 0.0f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            float rr;
            mw[k] = min(round_checked<kCorrect, kB>(__fmul_rn(m[k], Q.rdm), m[k], Q.dm,
                                                    Q.half_dm, rr), Q.mw_hi);
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
            for (int k = 0; k < 8; ++k) {
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
        for (int i = 0; i < 2; ++i) {
            const int64_t e = e0 + 256 * s + 128 * i + 4 * lane;
            int a4[4], b4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) { a4[j] = mw[4 * i + j]; b4[j] = vw[4 * i + j]; }
            if (FULL) {
                CI::store4(T, e, a4, b4);
            } else {
                const int64_t rem = n - e;
                const int c = rem >= 4 ? 4 : (rem > 0 ? (int)rem : 0);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j < c) CI::store1(T, e + j, a4[j], b4[j]);
            }
        }
    }
}

// One quantisation block (unit) of the tensor in X, starting at element e0.
// FULL: all B elements in range and all pointers allow vector access.
template <int LAYOUT, typename GT, bool EXACT_P, bool FULL, int LOGB, bool TBL, bool GR>
__device__ __forceinline__ void block_body(const TileCtx& X, int64_t e0, float* wm, float* wx,
                                           PreLoads<GT>& pre, int64_t next_e0) {
    using CI = Codes<LAYOUT>;
    using TC = TableCodes<LAYOUT>;
    constexpr int B = 1 << LOGB;
    constexpr int S = B / 256;
    constexpr bool kApprox = CI::kApproxLog;
    constexpr bool kMagicC = CI::kMagicCodes;
    constexpr bool kTab = TBL && FULL;
    constexpr int kB = CI::kMBias;
    const float kNaN = __int_as_float(0x7fffffff);
    const int lane = threadIdx.x & 31;
    const TensorPtrs T = X.t;
    const StepConsts& C = X.C;
    const int64_t n = X.n;
    const int64_t blk = e0 >> LOGB;

    const float sm = T.sm[blk], sv = T.sv[blk], vmn = T.vmin[blk];
    float tv = 0.0f, tm = 0.0f;
    if constexpr (kTab) {
        const float kf = small_int_to_float(lane & 15);
        tv = dequant_v(kf, sv, vmn);
        tm = __fmul_rn(__fsub_rn(kf, 8.0f), sm);
    }
    float s0 = kNaN, s1 = kNaN, s2 = kNaN;

    // ---- pass 1: dequantise, AdamW, parameter update ---------------------
    // (Sub-tile loops are not unrolled: the unrolled body overflows the
    // instruction cache, measured as the dominant "no instruction" stall.)
    // int8/uint8 codes, full blocks: one sub-tile of loads in flight ahead;
    // during the last sub-tile, the first sub-tile of the warp's next block
    // (next_e0 >= 0: same tensor, full) is loaded.
    constexpr bool kPre = FULL && (LAYOUT == MDQ_LAYOUT_S8U8 ||
                                   (LAYOUT == MDQ_LAYOUT_PACKED4 && kTab));
    if constexpr (kPre) {
        if (!pre.valid) pre.load(T, e0, lane);
    }
#pragma unroll 1
    for (int s = 0; s < S; ++s) {
        int cnt[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            cnt[i] = 4;
            if (!FULL) {
                const int64_t rem = n - (e0 + 256 * s + 128 * i + 4 * lane);
                cnt[i] = rem >= 4 ? 4 : (rem > 0 ? (int)rem : 0);
            }
        }
        float p[8], g[8], m[8], v[8];
        int qm[8], qv[8];
        typename TC::Raw raw[2];
        if constexpr (kPre) {
            // Decode the words loaded during the previous sub-tile, then
            // issue the next sub-tile's loads so they fly during this one.
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                p[4 * i + 0] = pre.p[i].x; p[4 * i + 1] = pre.p[i].y;
                p[4 * i + 2] = pre.p[i].z; p[4 * i + 3] = pre.p[i].w;
                GradRaw<GT>::decode(pre.g[i], g + 4 * i);
                if constexpr (GR) {   // gradients summed over ranks: load them now
                    float gg[4];
                    load_grad4<GT, GR>(T.g, e0 + 256 * s + 128 * i + 4 * lane, gg, X.granks);
#pragma unroll
                    for (int j = 0; j < 4; ++j) g[4 * i + j] = gg[j];
                }
                if constexpr (LAYOUT == MDQ_LAYOUT_PACKED4) {
                    raw[i].w = pre.m[i];   // the packed byte pairs, decoded by table
                } else {
                    // int8/uint8 code bytes (the only prefetched plain layout)
                    const unsigned mw = pre.m[i] ^ 0x80808080u;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        m[4 * i + j] = __fmul_rn(byte_as_float_s8(mw, j), sm);
                        v[4 * i + j] = dequant_v(byte_as_float_u8(pre.v[i], j), sv, vmn);
                    }
                }
            }
            pre.valid = false;
            if (s + 1 < S)
                pre.load(T, e0 + 256 * (s + 1), lane);
            else if (next_e0 >= 0)
                pre.load(T, next_e0, lane);
        } else {
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int64_t e = e0 + 256 * s + 128 * i + 4 * lane;
                if (FULL) {
                    const float4 a = __ldcs(reinterpret_cast<const float4*>(T.p + e));
                    p[4 * i + 0] = a.x; p[4 * i + 1] = a.y; p[4 * i + 2] = a.z; p[4 * i + 3] = a.w;
                    float gg[4];
                    load_grad4<GT, GR>(T.g, e, gg, X.granks);
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
        }
        if constexpr (kTab) {
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    m[4 * i + j] = TC::m(raw[i], j, tm, sm);
                    v[4 * i + j] = TC::v(raw[i], j, tv);
                }
        } else if constexpr (kPre) {
            // (dequantised above, from the prefetched code bytes)
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float qmf = kMagicC ? small_int_to_float(qm[k]) : (float)qm[k];
                m[k] = __fmul_rn(qmf, sm);
                const float qvf = kMagicC ? small_int_to_float(qv[k]) : (float)(unsigned)qv[k];
                v[k] = dequant_v(qvf, sv, vmn);
            }
        }
        if constexpr (EXACT_P) {
            // (scalar: measured faster than pairs with the IEEE divides)
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                m[k] = adam_m(m[k], g[k], C);
                v[k] = adam_v(v[k], g[k], C);
                p[k] = update_p<true>(p[k], m[k], v[k], C);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 8; k += 2) {   // element pairs (mdq_math.cuh)
                const float2 gg = make_float2(g[k], g[k + 1]);
                const float2 mm = adam_m2(make_float2(m[k], m[k + 1]), gg, C);
                const float2 vv = adam_v2(make_float2(v[k], v[k + 1]), gg, C);
                const float2 pp = update_p2<false>(make_float2(p[k], p[k + 1]), mm, vv, C);
                m[k] = mm.x; m[k + 1] = mm.y;
                v[k] = vv.x; v[k + 1] = vv.y;
                p[k] = pp.x; p[k + 1] = pp.y;
            }
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int64_t e = e0 + 256 * s + 128 * i + 4 * lane;
            if (FULL) {
                const float4 pv = make_float4(p[4 * i + 0], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
                __stcs(reinterpret_cast<float4*>(T.p + e), pv);
                if (T.p16 != nullptr) {
                    const __nv_bfloat162 lo = __floats2bfloat162_rn(p[4 * i + 0], p[4 * i + 1]);
                    const __nv_bfloat162 hi = __floats2bfloat162_rn(p[4 * i + 2], p[4 * i + 3]);
                    uint2 w;
                    w.x = *reinterpret_cast<const unsigned*>(&lo);
                    w.y = *reinterpret_cast<const unsigned*>(&hi);
                    __stcs(reinterpret_cast<uint2*>(T.p16 + e), w);
                    peer_store(X.peers, reinterpret_cast<uint2*>(T.p16 + e), w);
                } else {
                    peer_store(X.peers, reinterpret_cast<float4*>(T.p + e), pv);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j < cnt[i]) {
                        T.p[e + j] = p[4 * i + j];
                        if (T.p16 != nullptr) {
                            const __nv_bfloat16 b = __float2bfloat16_rn(p[4 * i + j]);
                            T.p16[e + j] = b;
                            peer_store(X.peers, T.p16 + e + j, b);
                        } else {
                            peer_store(X.peers, T.p + e + j, p[4 * i + j]);
                        }
                    }
            }
        }
        // Block statistics (CUDA/stquant_kernel.cu:184-199): |m|, and x =
        // v + 1e-12 whose logf extremes are logf of its extremes; elements
        // past the end enter as |m| = 0 and x = 1 (log v = 0, :92-93).
        float x[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const bool ok = FULL || (k & 3) < cnt[k / 4];
            x[k] = ok ? __fadd_rn(v[k], 1e-12f) : 1.0f;
            if (!ok) m[k] = 0.0f;
        }
#pragma unroll
        for (int k = 0; k < 8; k += 2) {
            s0 = max3f(s0, fabsf(m[k]), fabsf(m[k + 1]));
            s1 = max3f(s1, x[k], x[k + 1]);
            s2 = min3f(s2, x[k], x[k + 1]);
        }
        // Park m and x for pass 2 (this lane's own slots).
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int o = 256 * s + 128 * i + 4 * lane;
            *reinterpret_cast<float4*>(wm + o) =
                make_float4(m[4 * i + 0], m[4 * i + 1], m[4 * i + 2], m[4 * i + 3]);
            *reinterpret_cast<float4*>(wx + o) =
                make_float4(x[4 * i + 0], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
        }
    }

    asm volatile("redux.sync.max.f32 %0, %0, 0xffffffff;" : "+f"(s0));
    asm volatile("redux.sync.max.f32 %0, %0, 0xffffffff;" : "+f"(s1));
    asm volatile("redux.sync.min.f32 %0, %0, 0xffffffff;" : "+f"(s2));
    const QConsts Q = make_q<kApprox, kB>(s0, s1, s2, C);
    if (lane == 0) {
        T.sm[blk] = Q.new_sm;
        T.sv[blk] = Q.new_sv;
        T.vmin[blk] = Q.lmin;
    }

    // ---- pass 2: requantise (CUDA/stquant_kernel.cu:204-216) ---------------
    requant_block<LAYOUT, FULL, LOGB>(X, e0, Q, ParkSplit{wm, wx});
}

// Partial or unaligned blocks (a tensor's tail) take an out-of-line copy of
// the body, so the hot loop's code stays small.
template <int LAYOUT, typename GT, bool EXACT_P, int LOGB, bool TBL, bool GR>
__device__ __noinline__ void block_body_tail(const TileCtx& X, int64_t e0, float* wm, float* wx) {
    PreLoads<GT> none;
    none.valid = false;
    block_body<LAYOUT, GT, EXACT_P, false, LOGB, TBL, GR>(X, e0, wm, wx, none, -1);
}

// Persistent grid: CTA c takes units [total c / grid, total (c+1) / grid),
// warp w the units lo + w, lo + w + 8, ...; `tile_begin` of a descriptor
// counts units (blocks) here.  Each warp stages the tensor it works on in its
// own shared-memory slot.
template <int LAYOUT, typename GT, bool EXACT_P, int CAP, int LOGB, bool TBL, bool GR>
__global__ void __launch_bounds__(kBlkThreads, blk_min_ctas<LOGB>())
mdq_step_blocks(const __grid_constant__ LaunchParams<CAP> P) {
    extern __shared__ __align__(16) float s_park[];
    __shared__ TileCtx s_wctx[kBlkWarps];
    const int w = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    float* wm = s_park + (size_t)w * (2 << LOGB);
    float* wx = wm + (1 << LOGB);
    TileCtx& X = s_wctx[w];
    const int64_t total = P.total_tiles;
    const int lo = (int)(total * blockIdx.x / gridDim.x);
    const int hi = (int)(total * (blockIdx.x + 1) / gridDim.x);
    int cur_end = -1;
    PreLoads<GT> pre;
    pre.valid = false;
    for (int u = lo + w; u < hi; u += kBlkWarps) {
        if (u >= cur_end) {
            pre.valid = false;
            __syncwarp();
            if (lane == 0) {
                const LaunchDesc& D = P.d[find_desc(P, u)];
                X.peers = P.peers;
                X.granks = P.granks;
                X.t = D.t;
                X.n = D.n;
                X.tile_begin = D.tile_begin;
                X.tile_end = D.tile_begin + (int32_t)((D.n + (1 << LOGB) - 1) >> LOGB);
                X.lb = LOGB;
                X.vec = D.vec;
                X.C = make_step_consts(D.b1, D.b2, D.lr, D.wd, D.eps, D.step, D.m_bits,
                                       D.v_bits);
            }
            __syncwarp();
            cur_end = X.tile_end;
        }
        const int64_t e0 = (int64_t)(u - X.tile_begin) << LOGB;
        if (X.vec && e0 + (1 << LOGB) <= X.n) {
            // The warp's next block, when it is a full block of this tensor.
            const int u2 = u + kBlkWarps;
            const int64_t e2 = (int64_t)(u2 - X.tile_begin) << LOGB;
            const int64_t next_e0 = (u2 < hi && u2 < cur_end && e2 + (1 << LOGB) <= X.n) ? e2 : -1;
            block_body<LAYOUT, GT, EXACT_P, true, LOGB, TBL, GR>(X, e0, wm, wx, pre, next_e0);
        } else {
            pre.valid = false;
            block_body_tail<LAYOUT, GT, EXACT_P, LOGB, TBL, GR>(X, e0, wm, wx);
        }
    }
}

template <int LAYOUT, typename GT, bool EXACT_P, int CAP, int LOGB, bool TBL, bool GR>
mdq_status launch_blocks_t(const LaunchParams<CAP>& P, int sms, cudaStream_t stream) {
    auto k = mdq_step_blocks<LAYOUT, GT, EXACT_P, CAP, LOGB, TBL, GR>;
    constexpr int kSmem = blocks_smem_bytes<LOGB>();
    // The shared-memory attribute is per device: set on every launch.
    {
        const cudaError_t e =
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
        if (e != cudaSuccess)
            return mdq_fail(MDQ_ERR_CUDA, "block kernel smem attribute: %s", cudaGetErrorString(e));
    }
    static int occ = 0;  // per instantiation; identical across B200 devices
    if (occ == 0) {
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k, kBlkThreads, kSmem) != cudaSuccess ||
            b < 1)
            b = 1;
        occ = b;
    }
    int64_t grid = (int64_t)sms * occ;
    const int64_t ctas_needed = (P.total_tiles + kBlkWarps - 1) / kBlkWarps;
    if (grid > ctas_needed) grid = ctas_needed;
    if (grid < 1) grid = 1;
    k<<<(unsigned)grid, kBlkThreads, kSmem, stream>>>(P);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return mdq_fail(MDQ_ERR_CUDA, "block step launch: %s", cudaGetErrorString(e));
    return MDQ_OK;
}

// Blocks of 2^LOGB (9 or 10) elements; tables for 4-bit v codes.
template <int LAYOUT, typename GT, int CAP>
mdq_status launch_blocks_mode(const LaunchParams<CAP>& P, bool exact, int logb, int sms,
                              cudaStream_t s) {
    constexpr bool kV4 = LAYOUT == MDQ_LAYOUT_PACKED4 || LAYOUT == MDQ_LAYOUT_M8V4;
    constexpr bool kT = kV4 && MDQ_USE_TABLES != 0;
    if (P.granks.n > 0) {
        if (logb == 10)
            return exact ? launch_blocks_t<LAYOUT, GT, true, CAP, 10, kT, true>(P, sms, s)
                         : launch_blocks_t<LAYOUT, GT, false, CAP, 10, kT, true>(P, sms, s);
        return exact ? launch_blocks_t<LAYOUT, GT, true, CAP, 9, kT, true>(P, sms, s)
                     : launch_blocks_t<LAYOUT, GT, false, CAP, 9, kT, true>(P, sms, s);
    }
    if (logb == 10)
        return exact ? launch_blocks_t<LAYOUT, GT, true, CAP, 10, kT, false>(P, sms, s)
                     : launch_blocks_t<LAYOUT, GT, false, CAP, 10, kT, false>(P, sms, s);
    return exact ? launch_blocks_t<LAYOUT, GT, true, CAP, 9, kT, false>(P, sms, s)
                 : launch_blocks_t<LAYOUT, GT, false, CAP, 9, kT, false>(P, sms, s);
}

#define MDQ_BLOCKS_SIG(NAME, CAP)                                                               \
    mdq_status launch_blocks_##NAME(int gdt, const LaunchParams<CAP>& P, bool exact, int logb, \
                                    int sms, cudaStream_t s)
#define MDQ_BLOCKS_DECLARE(NAME)     \
    MDQ_BLOCKS_SIG(NAME, kCapSmall); \
    MDQ_BLOCKS_SIG(NAME, kCapLarge);
#define MDQ_BLOCKS_DEFINE_CAP(NAME, LAYOUT, CAP)                                                 \
    MDQ_BLOCKS_SIG(NAME, CAP) {                                                                  \
        return gdt == MDQ_BF16                                                                   \
                   ? launch_blocks_mode<LAYOUT, __nv_bfloat16, CAP>(P, exact, logb, sms, s)      \
                   : launch_blocks_mode<LAYOUT, float, CAP>(P, exact, logb, sms, s);             \
    }
#define MDQ_BLOCKS_DEFINE(NAME, LAYOUT)             \
    MDQ_BLOCKS_DEFINE_CAP(NAME, LAYOUT, kCapSmall)  \
    MDQ_BLOCKS_DEFINE_CAP(NAME, LAYOUT, kCapLarge)

MDQ_BLOCKS_DECLARE(packed4)
MDQ_BLOCKS_DECLARE(s8u8)
MDQ_BLOCKS_DECLARE(s16u16)
MDQ_BLOCKS_DECLARE(s32u32)
MDQ_BLOCKS_DECLARE(m8v4)

}  // namespace mdq
