// mdq_staged.cuh - warp-per-block fused step with bulk-copy (TMA) staging,
// for int8/uint8 codes and quantisation blocks of 128 to 1024 elements.
//
// The warp-per-block kernel (mdq_blocks.cuh) loads each sub-tile with plain
// per-lane loads one sub-tile ahead; with 16 warps per SM that keeps about
// 32 KB per SM in flight, and global-load latency (long_scoreboard) is one of
// its first stalls.  Here every warp owns a ring of NS chunk slots in shared
// memory; a chunk is 512 consecutive elements' inputs:
//
//   chunk = p (4 B/elt) | g (2 or 4 B/elt) | m codes (1 B/elt) | v codes (1 B/elt)
//
// A block of B elements takes CPB = B / 512 consecutive ring slots and the
// ring has NS = CPB + 1 of them.  When the warp starts a block it issues the
// first chunk of the next block it will take into the free slot; when it
// finishes the block, the remaining chunks of the next block go into the
// slots it has just freed.  The copies are cp.async.bulk global -> shared
// (the bulk-copy engine, no per-lane load instructions, no multicast), each
// completing on its slot's mbarrier.  Pass 1 parks the new m and
// x = v + 1e-12 in the chunk it has just consumed (8 B per element, the size
// of the inputs with bf16 or fp32 gradients), so there is no separate park
// buffer: 8 KB per warp at 512-element blocks, 12 KB at 1024 (bf16
// gradients), and 16 warps per SM.  The arithmetic is that of mdq_blocks.cuh,
// operation for operation (CUDA/stquant_kernel.cu:149-231); pass 2 is shared
// with it (requant_block).
#pragma once

#include "mdq_blocks.cuh"

namespace mdq {

constexpr int kChunkLog = 9;                 // 512-element chunks
constexpr int kChunk = 1 << kChunkLog;

// A warp's unit of work: one block of 2^LOGB elements (LOGB >= 9), or, for
// blocks of 128 or 256 elements, 1024 elements (8 or 4 whole blocks).
template <int LOGB> __host__ __device__ constexpr int stg_logu() { return LOGB >= 9 ? LOGB : 10; }
template <int LOGB> __host__ __device__ constexpr int stg_cpb() { return 1 << (stg_logu<LOGB>() - kChunkLog); }
template <int LOGB> __host__ __device__ constexpr int stg_ns() { return stg_cpb<LOGB>() + 1; }
template <typename GT> __host__ __device__ constexpr int stg_chunk_bytes() {
    return (4 + (int)sizeof(GT) + 2) * kChunk;
}
// Bytes a chunk's copies bring: int8/uint8 codes two arrays, packed 4-bit
// codes one (the slot keeps room for two: the park needs 8 B per element).
template <typename GT, int LAYOUT> __host__ __device__ constexpr int stg_copy_bytes() {
    return (4 + (int)sizeof(GT) + (LAYOUT == MDQ_LAYOUT_PACKED4 ? 1 : 2)) * kChunk;
}
// Blocks of a unit; with small blocks a unit's first chunk slot also holds
// the blocks' old scales (sm, sv, v_min: three 32-byte areas behind it).
template <int LOGB> __host__ __device__ constexpr int stg_nbu() { return 1 << (stg_logu<LOGB>() - LOGB); }
template <typename GT, int LOGB> __host__ __device__ constexpr int stg_slot_bytes() {
    return stg_chunk_bytes<GT>() + (LOGB >= 9 ? 0 : 128);
}
// Warps per CTA and resident CTAs per SM: 8 warps and 2 CTAs (16 warps per
// SM at up to 128 registers) when the ring fits twice per SM, else 4 warps
// and 3 CTAs (fp32 gradients at 1024-element units: 15 KB per warp).
template <typename GT, int LOGB> __host__ __device__ constexpr int stg_warps() {
    return 8 * stg_ns<LOGB>() * stg_slot_bytes<GT, LOGB>() <= 100 * 1024 ? 8 : 4;
}
template <typename GT, int LOGB> __host__ __device__ constexpr int stg_min_ctas() {
    return stg_warps<GT, LOGB>() == 8 ? 2 : 3;
}
template <typename GT, int LOGB> __host__ __device__ constexpr int stg_smem_bytes() {
    return stg_warps<GT, LOGB>() * stg_ns<LOGB>() * stg_slot_bytes<GT, LOGB>();
}

// Iteration limit of a wait on a slot's mbarrier.  A bulk copy of a few KB
// lands in microseconds; the limit (several hundred milliseconds at least)
// only keeps a lost completion from hanging the GPU.
constexpr int kStageWaitLimit = 1 << 22;

// Count of staged-kernel waits that ran out (a warp stops at the first).
__device__ unsigned int g_stage_timeouts;

__device__ __forceinline__ int lane_id() { return (int)(threadIdx.x & 31); }

__device__ __forceinline__ unsigned smem_u32(const void* p) {
    return (unsigned)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(unsigned bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}

// True once the barrier's phase `parity` has completed; false after
// kStageWaitLimit unsuccessful probes.
__device__ __forceinline__ bool mbar_wait(unsigned bar, unsigned parity) {
    for (int it = 0; it < kStageWaitLimit; ++it) {
        unsigned done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// One global -> shared bulk copy whose bytes complete on `bar`; the source
// lines are marked evict-first in L2 (each is read once).
__device__ __forceinline__ void bulk_load(unsigned dst, const void* src, unsigned bytes, unsigned bar,
                                          unsigned long long policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}

// Issues the copies of the chunk at element e0 of tensor T into the slot at
// shared address `dst` (lane 0 only); with `nsc` > 0 also the old scales of
// the nsc blocks from block blk0 on, behind the chunk (32-byte areas).  Every
// lane must have finished its accesses of the slot and fenced them against
// the async proxy before.
template <typename GT, int LAYOUT = MDQ_LAYOUT_S8U8>
__device__ __forceinline__ void stage_chunk(const TensorPtrs& T, int64_t e0, unsigned dst,
                                            unsigned bar, unsigned long long policy,
                                            int64_t blk0 = 0, int nsc = 0) {
    constexpr unsigned C = kChunk;
    constexpr unsigned kG = (unsigned)sizeof(GT) * C;
    const unsigned sb = 4u * (unsigned)nsc;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                 "r"((unsigned)stg_copy_bytes<GT, LAYOUT>() + 3 * sb)
                 : "memory");
    bulk_load(dst, T.p + e0, 4 * C, bar, policy);
    bulk_load(dst + 4 * C, static_cast<const GT*>(T.g) + e0, kG, bar, policy);
    bulk_load(dst + 4 * C + kG, static_cast<const int8_t*>(T.m) + e0, C, bar, policy);
    if (LAYOUT != MDQ_LAYOUT_PACKED4)
        bulk_load(dst + 5 * C + kG, static_cast<const uint8_t*>(T.v) + e0, C, bar, policy);
    if (nsc > 0) {
        const unsigned so = (unsigned)stg_chunk_bytes<GT>();
        bulk_load(dst + so, T.sm + blk0, sb, bar, policy);
        bulk_load(dst + so + 32, T.sv + blk0, sb, bar, policy);
        bulk_load(dst + so + 64, T.vmin + blk0, sb, bar, policy);
    }
}

// Park addresses inside consumed chunks; sub-tile s of the block lies in
// chunk s / 2 as its local sub-tile s % 2.  m of an element goes where its p
// was.  x goes where its gradient was (fp32 gradients); with bf16 gradients
// the gradient area of a local sub-tile t holds 128 floats, so elements
// 256 t + 4 lane + (0..3) (i = 0) park there and elements
// 256 t + 128 + 4 lane + (0..3) (i = 1) in the sub-tile's m-code bytes
// (lanes 0-15) or v-code bytes (lanes 16-31), 64 floats each.  Every position
// was read, by some lane, before it is overwritten; a __syncwarp separates
// the two.
template <typename GT, int CPB>
struct ParkRing {
    char* ch[CPB];
    // ch[c] by selects (a dynamic index would put the array in local memory)
    __device__ char* chunk(int c) const {
        char* r = ch[0];
#pragma unroll
        for (int k = 1; k < CPB; ++k) r = c == k ? ch[k] : r;
        return r;
    }
    __device__ float* m(int s, int i, int lane) const {
        return reinterpret_cast<float*>(chunk(s >> 1)) + 256 * (s & 1) + 128 * i + 4 * lane;
    }
    __device__ float* x(int s, int i, int lane) const {
        constexpr int C = kChunk;
        const int t = s & 1;
        char* base = chunk(s >> 1);
        float* g = reinterpret_cast<float*>(base + 4 * C);
        if constexpr (sizeof(GT) == 4) {
            return g + 256 * t + 128 * i + 4 * lane;
        } else {
            if (i == 0) return g + 128 * t + 4 * lane;
            float* codes = reinterpret_cast<float*>(base + 6 * C + (lane >= 16 ? C : 0));
            return codes + 64 * t + 4 * (lane & 15);
        }
    }
};

// One full, staged quantisation block whose chunks lie in park.ch[]: pass 1
// from the chunks (waiting for chunk c's barrier bars[c] / parity par[c]
// before its first sub-tile), pass 2 shared with mdq_blocks.cuh.  Returns
// false when a wait ran out (nothing written for this block then).
template <typename GT, bool EXACT_P, int LOGB>
__device__ __forceinline__ bool staged_block_body(const TileCtx& X, int64_t e0,
                                                  const ParkRing<GT, stg_cpb<LOGB>()>& park,
                                                  const unsigned (&bars)[stg_cpb<LOGB>()],
                                                  const unsigned (&par)[stg_cpb<LOGB>()]) {
    using CI = Codes<MDQ_LAYOUT_S8U8>;
    constexpr int B = 1 << LOGB;
    constexpr int S = B / 256;
    constexpr int C = kChunk;
    constexpr int kG = (int)sizeof(GT) * C;
    const float kNaN = __int_as_float(0x7fffffff);
    const int lane = threadIdx.x & 31;
    const TensorPtrs T = X.t;
    const StepConsts& Cs = X.C;
    const int64_t blk = e0 >> LOGB;
    const float sm = T.sm[blk], sv = T.sv[blk], vmn = T.vmin[blk];
    float s0 = kNaN, s1 = kNaN, s2 = kNaN;

    // ---- pass 1: dequantise, AdamW, parameter update (:163-181) ----------
#pragma unroll 1
    for (int s = 0; s < S; ++s) {
        if ((s & 1) == 0) {
            unsigned bar = bars[0], ph = par[0];
#pragma unroll
            for (int c = 1; c < stg_cpb<LOGB>(); ++c)
                if ((s >> 1) == c) { bar = bars[c]; ph = par[c]; }
            if (!mbar_wait(bar, ph)) return false;
        }
        const char* chunk = park.chunk(s >> 1);
        const int t = s & 1;
        // Elements 4 i + 2 h + (0, 1) of the lane form pair 2 i + h.
        float2 p[4], g[4], m[4], v[4];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int k = 256 * t + 128 * i + 4 * lane;
            const float4 a = *reinterpret_cast<const float4*>(chunk + 4 * k);
            p[2 * i] = make_float2(a.x, a.y);
            p[2 * i + 1] = make_float2(a.z, a.w);
            float gg[4];
            const typename GradRaw<GT>::T gw =
                *reinterpret_cast<const typename GradRaw<GT>::T*>(chunk + 4 * C + (int)sizeof(GT) * k);
            GradRaw<GT>::decode(gw, gg);
            g[2 * i] = make_float2(gg[0], gg[1]);
            g[2 * i + 1] = make_float2(gg[2], gg[3]);
            const unsigned mw = *reinterpret_cast<const unsigned*>(chunk + 4 * C + kG + k) ^ 0x80808080u;
            const unsigned vw = *reinterpret_cast<const unsigned*>(chunk + 5 * C + kG + k);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                // Code bytes as exact floats (the magic-word subtraction paired).
                const float2 qm = add2_rn(
                    make_float2(__int_as_float((int)__byte_perm(mw, (unsigned)kMagicBits, 0x7650u + 2 * h)),
                                __int_as_float((int)__byte_perm(mw, (unsigned)kMagicBits, 0x7651u + 2 * h))),
                    bcast2(-(kMagic + 128.0f)));
                const float2 qv = add2_rn(
                    make_float2(__int_as_float((int)__byte_perm(vw, (unsigned)kMagicBits, 0x7650u + 2 * h)),
                                __int_as_float((int)__byte_perm(vw, (unsigned)kMagicBits, 0x7651u + 2 * h))),
                    bcast2(-kMagic));
                m[2 * i + h] = mul2_rn(qm, bcast2(sm));
                const float2 ev = fma2_rn(qv, bcast2(sv), bcast2(vmn));
                v[2 * i + h] = make_float2(expf(ev.x), expf(ev.y));
            }
        }
        // Every lane's reads of this sub-tile precede the park writes below.
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            m[k] = adam_m2(m[k], g[k], Cs);
            v[k] = adam_v2(v[k], g[k], Cs);
            p[k] = update_p2<EXACT_P>(p[k], m[k], v[k], Cs);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int64_t e = e0 + 256 * s + 128 * i + 4 * lane;
            const float4 pv = make_float4(p[2 * i].x, p[2 * i].y, p[2 * i + 1].x, p[2 * i + 1].y);
            __stcs(reinterpret_cast<float4*>(T.p + e), pv);
            if (T.p16 != nullptr) {
                const __nv_bfloat162 lo = __floats2bfloat162_rn(pv.x, pv.y);
                const __nv_bfloat162 hi = __floats2bfloat162_rn(pv.z, pv.w);
                uint2 w;
                w.x = *reinterpret_cast<const unsigned*>(&lo);
                w.y = *reinterpret_cast<const unsigned*>(&hi);
                __stcs(reinterpret_cast<uint2*>(T.p16 + e), w);
            }
        }
        // Block statistics (:184-199): |m| and x = v + 1e-12 (a full block).
        float2 x[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            x[k] = add2_rn(v[k], bcast2(1e-12f));
            s0 = max3f(s0, fabsf(m[k].x), fabsf(m[k].y));
            s1 = max3f(s1, x[k].x, x[k].y);
            s2 = min3f(s2, x[k].x, x[k].y);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            *reinterpret_cast<float4*>(park.m(s, i, lane)) =
                make_float4(m[2 * i].x, m[2 * i].y, m[2 * i + 1].x, m[2 * i + 1].y);
            *reinterpret_cast<float4*>(park.x(s, i, lane)) =
                make_float4(x[2 * i].x, x[2 * i].y, x[2 * i + 1].x, x[2 * i + 1].y);
        }
    }
    // Parks of other lanes (the bf16 x areas mix lanes) before any read back.
    __syncwarp();
    asm volatile("redux.sync.max.f32 %0, %0, 0xffffffff;" : "+f"(s0));
    asm volatile("redux.sync.max.f32 %0, %0, 0xffffffff;" : "+f"(s1));
    asm volatile("redux.sync.min.f32 %0, %0, 0xffffffff;" : "+f"(s2));
    const QConsts Q = make_q<CI::kApproxLog, CI::kMBias>(s0, s1, s2, Cs);
    if (lane == 0) {
        T.sm[blk] = Q.new_sm;
        T.sv[blk] = Q.new_sv;
        T.vmin[blk] = Q.lmin;
    }
    // ---- pass 2: requantise (:204-216) ------------------------------------
    requant_block<MDQ_LAYOUT_S8U8, true, LOGB>(X, e0, Q, park);
    return true;
}

// One full, staged unit of 1024 elements holding NBU = 1024 / B whole blocks
// of B = 128 or 256 elements.  Sub-tile s (256 elements) holds blocks
// (2 s, 2 s + 1) (B = 128: its halves i = 0, 1) or block s (B = 256); every
// lane has 4 elements of each block it touches.  Pass 1 runs as for large
// blocks, with the block's old scales read from the unit's staged scale areas;
// each block's three extremes are reduced over the warp right after its
// sub-tile and kept by lane b = block index.  Then every lane evaluates the
// requantisation constants of block `lane` (one evaluation per lane covers
// all NBU blocks, instead of one per lane and block), lanes < NBU store the
// new scales, and pass 2 takes each block's constants from lane b by shuffle.
// Returns false when a wait ran out.
template <int LAYOUT, typename GT, bool EXACT_P, int LOGB>
__device__ __forceinline__ bool staged_small_body(const TileCtx& X, int64_t e0,
                                                  const ParkRing<GT, 2>& park,
                                                  const unsigned (&bars)[2],
                                                  const unsigned (&par)[2]) {
    using CI = Codes<LAYOUT>;
    constexpr int C = kChunk;
    constexpr int kG = (int)sizeof(GT) * C;
    constexpr int NBU = stg_nbu<LOGB>();
    constexpr bool kPacked = LAYOUT == MDQ_LAYOUT_PACKED4;
    const float kf = small_int_to_float(lane_id() & 15);   // table entry of this lane
    const float kNaN = __int_as_float(0x7fffffff);
    const int lane = threadIdx.x & 31;
    const TensorPtrs T = X.t;
    const StepConsts& Cs = X.C;
    const int64_t blk0 = e0 >> LOGB;
    const float* scl = reinterpret_cast<const float*>(park.ch[0] + stg_chunk_bytes<GT>());
    float R0 = kNaN, R1 = kNaN, R2 = kNaN;   // this lane's block (lane < NBU): extremes

    // ---- pass 1 (:163-199) -------------------------------------------------
#pragma unroll 1
    for (int s = 0; s < 4; ++s) {
        if ((s & 1) == 0) {
            const unsigned bar = s == 0 ? bars[0] : bars[1];
            const unsigned ph = s == 0 ? par[0] : par[1];
            if (!mbar_wait(bar, ph)) return false;
        }
        const char* chunk = park.chunk(s >> 1);
        const int t = s & 1;
        float2 p[4], g[4], m[4], v[4];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int b = LOGB == 7 ? 2 * s + i : s;          // block within the unit
            const float sm = scl[b], sv = scl[8 + b], vmn = scl[16 + b];
            const int k = 256 * t + 128 * i + 4 * lane;
            const float4 a = *reinterpret_cast<const float4*>(chunk + 4 * k);
            p[2 * i] = make_float2(a.x, a.y);
            p[2 * i + 1] = make_float2(a.z, a.w);
            float gg[4];
            const typename GradRaw<GT>::T gw =
                *reinterpret_cast<const typename GradRaw<GT>::T*>(chunk + 4 * C + (int)sizeof(GT) * k);
            GradRaw<GT>::decode(gw, gg);
            g[2 * i] = make_float2(gg[0], gg[1]);
            g[2 * i + 1] = make_float2(gg[2], gg[3]);
            if constexpr (kPacked) {
                // 16-entry tables of the block's dequantised values
                // (CUDA/stquant_kernel.cu:163-169), entry lane % 16, read
                // with one 16-wide shuffle per value indexed by the nibble.
                const float tv = dequant_v(kf, sv, vmn);
                const float tm = __fmul_rn(__fsub_rn(kf, 8.0f), sm);
                const unsigned cw = *reinterpret_cast<const unsigned*>(chunk + 4 * C + kG + k);
                float mv[4], vv[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    mv[j] = __shfl_sync(0xffffffffu, tm, (int)(cw >> (8 * j)), 16);
                    vv[j] = __shfl_sync(0xffffffffu, tv, (int)(cw >> (8 * j + 4)), 16);
                }
                m[2 * i] = make_float2(mv[0], mv[1]);
                m[2 * i + 1] = make_float2(mv[2], mv[3]);
                v[2 * i] = make_float2(vv[0], vv[1]);
                v[2 * i + 1] = make_float2(vv[2], vv[3]);
                continue;
            }
            const unsigned mw = *reinterpret_cast<const unsigned*>(chunk + 4 * C + kG + k) ^ 0x80808080u;
            const unsigned vw = *reinterpret_cast<const unsigned*>(chunk + 5 * C + kG + k);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float2 qm = add2_rn(
                    make_float2(__int_as_float((int)__byte_perm(mw, (unsigned)kMagicBits, 0x7650u + 2 * h)),
                                __int_as_float((int)__byte_perm(mw, (unsigned)kMagicBits, 0x7651u + 2 * h))),
                    bcast2(-(kMagic + 128.0f)));
                const float2 qv = add2_rn(
                    make_float2(__int_as_float((int)__byte_perm(vw, (unsigned)kMagicBits, 0x7650u + 2 * h)),
                                __int_as_float((int)__byte_perm(vw, (unsigned)kMagicBits, 0x7651u + 2 * h))),
                    bcast2(-kMagic));
                m[2 * i + h] = mul2_rn(qm, bcast2(sm));
                const float2 ev = fma2_rn(qv, bcast2(sv), bcast2(vmn));
                v[2 * i + h] = make_float2(expf(ev.x), expf(ev.y));
            }
        }
        __syncwarp();   // every lane's reads of this sub-tile precede the parks
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            m[k] = adam_m2(m[k], g[k], Cs);
            v[k] = adam_v2(v[k], g[k], Cs);
            p[k] = update_p2<EXACT_P>(p[k], m[k], v[k], Cs);
        }
        float2 x[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) x[k] = add2_rn(v[k], bcast2(1e-12f));
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int64_t e = e0 + 256 * s + 128 * i + 4 * lane;
            const float4 pv = make_float4(p[2 * i].x, p[2 * i].y, p[2 * i + 1].x, p[2 * i + 1].y);
            __stcs(reinterpret_cast<float4*>(T.p + e), pv);
            if (T.p16 != nullptr) {
                const __nv_bfloat162 lo = __floats2bfloat162_rn(pv.x, pv.y);
                const __nv_bfloat162 hi = __floats2bfloat162_rn(pv.z, pv.w);
                uint2 w;
                w.x = *reinterpret_cast<const unsigned*>(&lo);
                w.y = *reinterpret_cast<const unsigned*>(&hi);
                __stcs(reinterpret_cast<uint2*>(T.p16 + e), w);
            }
            *reinterpret_cast<float4*>(park.m(s, i, lane)) =
                make_float4(m[2 * i].x, m[2 * i].y, m[2 * i + 1].x, m[2 * i + 1].y);
            *reinterpret_cast<float4*>(park.x(s, i, lane)) =
                make_float4(x[2 * i].x, x[2 * i].y, x[2 * i + 1].x, x[2 * i + 1].y);
        }
        // Block extremes (:184-199), reduced over the warp per block.
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            if (LOGB == 8 && i == 1) break;
            const int k0 = LOGB == 7 ? 2 * i : 0, k1 = LOGB == 7 ? 2 * i + 2 : 4;
            float a0 = kNaN, a1 = kNaN, a2 = kNaN;
#pragma unroll
            for (int k = k0; k < k1; ++k) {
                a0 = max3f(a0, fabsf(m[k].x), fabsf(m[k].y));
                a1 = max3f(a1, x[k].x, x[k].y);
                a2 = min3f(a2, x[k].x, x[k].y);
            }
            asm volatile("redux.sync.max.f32 %0, %0, 0xffffffff;" : "+f"(a0));
            asm volatile("redux.sync.max.f32 %0, %0, 0xffffffff;" : "+f"(a1));
            asm volatile("redux.sync.min.f32 %0, %0, 0xffffffff;" : "+f"(a2));
            const int b = LOGB == 7 ? 2 * s + i : s;
            if (lane == b) { R0 = a0; R1 = a1; R2 = a2; }
        }
    }
    __syncwarp();   // parks of other lanes (the bf16 x areas mix lanes)
    // Constants of block `lane` (lanes >= NBU evaluate a NaN block, unused).
    const QConsts Q = make_q<CI::kApproxLog, CI::kMBias>(R0, R1, R2, Cs);
    if (lane < NBU) {
        T.sm[blk0 + lane] = Q.new_sm;
        T.sv[blk0 + lane] = Q.new_sv;
        T.vmin[blk0 + lane] = Q.lmin;
    }

    // ---- pass 2: requantise (:204-216) -------------------------------------
#pragma unroll 1
    for (int s = 0; s < 4; ++s) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int b = LOGB == 7 ? 2 * s + i : s;
            QConsts q;
            q.rdm = __shfl_sync(0xffffffffu, Q.rdm, b);
            q.dm = __shfl_sync(0xffffffffu, Q.dm, b);
            q.half_dm = __shfl_sync(0xffffffffu, Q.half_dm, b);
            q.lmin = __shfl_sync(0xffffffffu, Q.lmin, b);
            q.rdv = __shfl_sync(0xffffffffu, Q.rdv, b);
            q.dv = __shfl_sync(0xffffffffu, Q.dv, b);
            q.half_dv = __shfl_sync(0xffffffffu, Q.half_dv, b);
            q.thr_v = __shfl_sync(0xffffffffu, Q.thr_v, b);
            q.mw_hi = Q.mw_hi;   // the same for every block
            const float4 am = *reinterpret_cast<const float4*>(park.m(s, i, lane));
            const float4 ax = *reinterpret_cast<const float4*>(park.x(s, i, lane));
            const float mm[4] = {am.x, am.y, am.z, am.w};
            const float xx[4] = {ax.x, ax.y, ax.z, ax.w};
            int mw[4], vw[4];
            float rem_m = 0.0f, rem_v = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float rr;
                mw[j] = min(round_checked<false, CI::kMBias>(__fmul_rn(mm[j], q.rdm), mm[j], q.dm,
                                                              q.half_dm, rr), q.mw_hi);
                rem_m = max_nan(rem_m, rr);
                const float xv = __fmaf_rn(approx_log2(xx[j]), kLn2, -q.lmin);
                vw[j] = round_checked<false>(__fmul_rn(xv, q.rdv), xv, q.dv, q.half_dv, rr);
                rem_v = max_nan(rem_v, rr);
            }
            if (!(rem_m < q.half_dm && rem_v < q.thr_v)) {
                // Rare: codes that fail their check take the reference's
                // double-precision expression.
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float rr;
                    round_checked<false>(__fmul_rn(mm[j], q.rdm), mm[j], q.dm, q.half_dm, rr);
                    if (!(rr < q.half_dm)) mw[j] = CI::m_word(requant_m_ref(mm[j], q.dm, Cs.lm_d));
                    const float xv = __fmaf_rn(approx_log2(xx[j]), kLn2, -q.lmin);
                    round_checked<false>(__fmul_rn(xv, q.rdv), xv, q.dv, q.half_dv, rr);
                    if (!(rr < q.thr_v))
                        vw[j] = CI::v_word(requant_v_ref(__fsub_rn(logf(xx[j]), q.lmin), q.dv, Cs.lv_d));
                }
            }
            CI::store4(T, e0 + 256 * s + 128 * i + 4 * lane, mw, vw);
        }
    }
    return true;
}

// Persistent grid: CTA c takes units (one block, or 1024 elements of small
// blocks) [total c / grid,
// total (c + 1) / grid), warp w the units lo + w, lo + w + W, ...  A unit is
// staged when its tensor allows bulk copies (16-byte aligned bases, bit 1 of
// `vec`) and the block is full.  The chunks of unit u sit at ring positions
// base + c (mod NS); the next unit's chunk c at base + CPB + c.  A staged
// unit whose chunks were not issued ahead (the warp's first unit of a
// tensor) issues them at once.  Other units (tails, unaligned tensors) run
// the direct-load body of mdq_blocks.cuh, parking in the ring.
template <int LAYOUT, typename GT, bool EXACT_P, int CAP, int LOGB>
__global__ void __launch_bounds__(32 * stg_warps<GT, LOGB>(), stg_min_ctas<GT, LOGB>())
mdq_step_staged(const __grid_constant__ LaunchParams<CAP> P) {
    constexpr int W = stg_warps<GT, LOGB>();
    constexpr int CPB = stg_cpb<LOGB>();
    constexpr int NS = stg_ns<LOGB>();
    constexpr int kCh = stg_slot_bytes<GT, LOGB>();
    constexpr int B = 1 << LOGB;
    constexpr int LOGU = stg_logu<LOGB>();
    constexpr int U = 1 << LOGU;              // elements of a unit
    constexpr int NBU = stg_nbu<LOGB>();
    constexpr bool kSmall = LOGB < 9;
    static_assert(kSmall || NS * kCh >= 2 * B * (int)sizeof(float),
                  "the ring holds a direct-path park");
    static_assert(kSmall || LAYOUT == MDQ_LAYOUT_S8U8, "packed 4-bit codes: small blocks only");
    extern __shared__ __align__(128) char s_ring[];
    __shared__ TileCtx s_wctx[W];
    __shared__ __align__(8) unsigned long long s_bar[W][NS];
    const int w = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    char* ring = s_ring + (size_t)w * NS * kCh;
    const unsigned ring_s = smem_u32(ring);
    const unsigned bar0 = smem_u32(&s_bar[w][0]);
    TileCtx& X = s_wctx[w];
    unsigned long long policy = 0;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    if (lane == 0) {
#pragma unroll
        for (int k = 0; k < NS; ++k) mbar_init(bar0 + 8 * k);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncwarp();

    const int64_t total = P.total_tiles;
    const int lo = (int)(total * blockIdx.x / gridDim.x);
    const int hi = (int)(total * (blockIdx.x + 1) / gridDim.x);
    int cur_end = -1;
    // Per slot: unit * CPB + chunk whose copy was issued into it (-1: none),
    // and the parity of its barrier's current phase (bit k of `parity`).
    // Slots are indexed by a run-time position, so both live in registers
    // through unrolled selects rather than indexed arrays.
    int held[NS];
    unsigned parity = 0u;
#pragma unroll
    for (int k = 0; k < NS; ++k) held[k] = -1;
    auto held_at = [&](int k) {
        int r = held[0];
#pragma unroll
        for (int j = 1; j < NS; ++j) r = k == j ? held[j] : r;
        return r;
    };
    auto set_held = [&](int k, int val) {
#pragma unroll
        for (int j = 0; j < NS; ++j) if (k == j) held[j] = val;
    };
    int base = 0;
    for (int u = lo + w; u < hi; u += W) {
        if (u >= cur_end) {
            __syncwarp();
            if (lane == 0) {
                const LaunchDesc& D = P.d[find_desc(P, u)];
                X.peers = P.peers;
                X.granks = P.granks;
                X.t = D.t;
                X.n = D.n;
                X.tile_begin = D.tile_begin;
                X.tile_end = D.tile_begin + (int32_t)((D.n + U - 1) >> LOGU);
                X.lb = LOGB;
                X.vec = D.vec;
                X.C = make_step_consts(D.b1, D.b2, D.lr, D.wd, D.eps, D.step, D.m_bits,
                                       D.v_bits);
            }
            __syncwarp();
            cur_end = X.tile_end;
        }
        const bool bulk = (X.vec & 2) != 0;
        const int64_t e0 = (int64_t)(u - X.tile_begin) << LOGU;
        const bool stage_cur = bulk && e0 + U <= X.n;
        const int u2 = u + W;
        const int64_t e2 = (int64_t)(u2 - X.tile_begin) << LOGU;
        const bool stage_next = bulk && u2 < hi && u2 < cur_end && e2 + U <= X.n;
        // Every lane is done with the free slots (earlier units); order those
        // generic accesses before the copy engine writes them.
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        int pos[CPB];
        unsigned bars[CPB], par[CPB];
        ParkRing<GT, CPB> park;
#pragma unroll
        for (int c = 0; c < CPB; ++c) {
            pos[c] = base + c >= NS ? base + c - NS : base + c;
            park.ch[c] = ring + pos[c] * kCh;
            bars[c] = bar0 + 8 * pos[c];
            par[c] = (parity >> pos[c]) & 1u;
            if (stage_cur && held_at(pos[c]) != u * CPB + c) {
                if (lane == 0)
                    stage_chunk<GT, LAYOUT>(X.t, e0 + c * kChunk, ring_s + pos[c] * kCh, bars[c], policy,
                                    e0 >> LOGB, kSmall && c == 0 ? NBU : 0);
                set_held(pos[c], u * CPB + c);
            }
        }
        const int fpos = base + CPB >= NS ? base + CPB - NS : base + CPB;   // the free slot
        if (stage_next) {
            if (lane == 0)
                stage_chunk<GT, LAYOUT>(X.t, e2, ring_s + fpos * kCh, bar0 + 8 * fpos, policy, e2 >> LOGB,
                                kSmall ? NBU : 0);
            set_held(fpos, u2 * CPB);
        }
        if (stage_cur) {
            bool ok;
            if constexpr (kSmall)
                ok = staged_small_body<LAYOUT, GT, EXACT_P, LOGB>(X, e0, park, bars, par);
            else
                ok = staged_block_body<GT, EXACT_P, LOGB>(X, e0, park, bars, par);
            if (!ok) {
                if (lane == 0) atomicAdd(&g_stage_timeouts, 1u);
                // Wait, again bounded, for every copy still owed to this
                // warp's slots before the warp gives up.
#pragma unroll
                for (int k = 0; k < NS; ++k)
                    if (held[k] >= 0) mbar_wait(bar0 + 8 * k, (parity >> k) & 1u);
                return;
            }
#pragma unroll
            for (int c = 0; c < CPB; ++c) {
                parity ^= 1u << pos[c];
                set_held(pos[c], -1);
            }
        } else if constexpr (!kSmall) {
            // Tails and tensors whose bases do not allow bulk copies (rare):
            // the out-of-line direct-load body, parking at the start of the
            // warp's ring (2 B floats <= NS chunks).  No copy is in flight
            // then: the next unit is not staged either (a later unit of a
            // tail or of an unaligned tensor).
            float* wm = reinterpret_cast<float*>(ring);
            block_body_tail<MDQ_LAYOUT_S8U8, GT, EXACT_P, LOGB, false, false>(
                X, e0, wm, wm + B);
        }
        // (Small blocks: the host passes only whole, bulk-aligned units; the
        // rest of a tensor goes to the tiled kernel.)
        // The remaining chunks of the next unit go into this unit's first
        // slots, now free.
        if (stage_next && CPB > 1) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
#pragma unroll
            for (int c = 1; c < CPB; ++c) {
                if (lane == 0)
                    stage_chunk<GT, LAYOUT>(X.t, e2 + c * kChunk, ring_s + pos[c - 1] * kCh,
                                    bar0 + 8 * pos[c - 1], policy);
                set_held(pos[c - 1], u2 * CPB + c);
            }
        }
        base = base + CPB >= NS ? base + CPB - NS : base + CPB;
    }
}

template <int LAYOUT, typename GT, bool EXACT_P, int CAP, int LOGB>
mdq_status launch_staged_t(const LaunchParams<CAP>& P, int sms, cudaStream_t stream) {
    auto k = mdq_step_staged<LAYOUT, GT, EXACT_P, CAP, LOGB>;
    constexpr int W = stg_warps<GT, LOGB>();
    constexpr int kSmem = stg_smem_bytes<GT, LOGB>();
    {
        const cudaError_t e =
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
        if (e != cudaSuccess)
            return mdq_fail(MDQ_ERR_CUDA, "staged kernel smem attribute: %s", cudaGetErrorString(e));
    }
    static int occ = 0;  // per instantiation; identical across B200 devices
    if (occ == 0) {
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, k, 32 * W, kSmem) != cudaSuccess || b < 1)
            b = 1;
        occ = b;
    }
    int64_t grid = (int64_t)sms * occ;
    const int64_t ctas_needed = (P.total_tiles + W - 1) / W;
    if (grid > ctas_needed) grid = ctas_needed;
    if (grid < 1) grid = 1;
    k<<<(unsigned)grid, 32 * W, kSmem, stream>>>(P);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return mdq_fail(MDQ_ERR_CUDA, "staged step launch: %s", cudaGetErrorString(e));
    return MDQ_OK;
}

// Blocks of 2^logb elements, no peers and no gradient ranks: int8/uint8
// codes with logb 7..10, packed 4-bit codes with logb 7 or 8.
template <int CAP>
mdq_status launch_staged_s8u8(int gdt, const LaunchParams<CAP>& P, bool exact, int logb, int sms,
                              cudaStream_t s);
template <int CAP>
mdq_status launch_staged_packed4(int gdt, const LaunchParams<CAP>& P, bool exact, int logb, int sms,
                                 cudaStream_t s);

}  // namespace mdq
