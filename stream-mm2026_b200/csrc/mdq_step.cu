// mdq_step.cu - B200 (sm_100a) fused quantized-AdamW step and its C ABI.
//
// Kernel design
// -------------
// The reference runs one thread per element and one CTA per quantisation block
// (CUDA/stquant_kernel.cu:61,421-422) with three shared-memory tree reductions
// per CTA.  Here a persistent grid of 256-thread CTAs walks "tiles" of 2048
// consecutive elements of one tensor; each thread owns 8 consecutive elements,
// loaded and stored with 128-bit (p, g) and 32/64/128-bit (codes) accesses.  A
// quantisation block of B elements (power of two, 8..2048) is owned by B/8
// consecutive threads, so the block max/min reductions are warp shuffles (and,
// for B > 256, one shared-memory exchange).  For 4-bit v codes (and 8-bit v
// codes with B >= 512) the 2^k possible dequantised v values of each block are
// tabulated once in shared memory, replacing one expf per element by a shared
// load of the identical value.  Tiles of all tensors of one layout / gradient
// dtype are scheduled in one launch from a descriptor table passed as a
// __grid_constant__ kernel parameter, so nothing is allocated and nothing is
// copied host-to-device per step.
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
#include <mutex>

#include "mdq.h"
#include "mdq_math.cuh"

namespace mdq {

constexpr int kThreads = 256;
constexpr int kPerThread = 8;
constexpr int kTile = kThreads * kPerThread;  // 2048 elements
constexpr int kLogTile = 11;
constexpr int kTblMax = 1024;                 // floats of dequantised-v table per tile
constexpr int kCapSmall = 8;                  // descriptors per launch, small table
constexpr int kCapLarge = 224;                // descriptors per launch, large table
constexpr int kProfSlots = 5;

// Device-side descriptor (one tensor or block-aligned tensor piece).
struct LaunchDesc {
    float* p;
    const void* g;
    void* m;
    void* v;
    float* sm;
    float* sv;
    float* vmin;
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

// ---------------------------------------------------------------------------
// Code storage per layout.  qm holds the signed m code value, qv the unsigned
// v code value (for PACKED4 the m nibble minus 8, as the reference unpacks it).
// ---------------------------------------------------------------------------
template <int LAYOUT> struct Codes;

template <> struct Codes<MDQ_LAYOUT_PACKED4> {
    static constexpr int kTblBits = 4;
    __device__ static void load8(const LaunchDesc& d, int64_t e, int (&qm)[8], unsigned (&qv)[8]) {
        const uint2 w = __ldcs(reinterpret_cast<const uint2*>(static_cast<const uint8_t*>(d.m) + e));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const unsigned b = ((j < 4 ? w.x : w.y) >> (8 * (j & 3))) & 0xffu;
            qm[j] = (int)(b & 15u) - 8;
            qv[j] = b >> 4;
        }
    }
    __device__ static void load1(const LaunchDesc& d, int64_t e, int& qm, unsigned& qv) {
        const unsigned b = static_cast<const uint8_t*>(d.m)[e];
        qm = (int)(b & 15u) - 8;
        qv = b >> 4;
    }
    // CUDA/stquant_kernel.cu:118-130: nibble clamps after the level clamps.
    __device__ static unsigned pack(int mi, int vi) {
        int mu = mi + 8;
        mu = mu < 0 ? 0 : (mu > 15 ? 15 : mu);
        vi = vi < 0 ? 0 : (vi > 15 ? 15 : vi);
        return ((unsigned)vi << 4) | ((unsigned)mu & 15u);
    }
    __device__ static void store8(const LaunchDesc& d, int64_t e, const int (&mi)[8], const int (&vi)[8]) {
        uint2 w = make_uint2(0u, 0u);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const unsigned b = pack(mi[j], vi[j]);
            if (j < 4) w.x |= b << (8 * j); else w.y |= b << (8 * (j - 4));
        }
        __stcs(reinterpret_cast<uint2*>(static_cast<uint8_t*>(d.m) + e), w);
    }
    __device__ static void store1(const LaunchDesc& d, int64_t e, int mi, int vi) {
        static_cast<uint8_t*>(d.m)[e] = (uint8_t)pack(mi, vi);
    }
    // Integer conversion of a double-path code, as CUDA/stquant_kernel.cu:118,126.
    __device__ static int m_int(double q) { return (int)q; }
    __device__ static int v_int(double q) { return (int)q; }
};

template <typename MT, typename VT> struct CodesPlain {
    // 8 codes of MT / VT: 8, 16 or 32 bytes each.
    template <typename T>
    __device__ static void ld8(const T* src, T (&o)[8]) {
        if constexpr (sizeof(T) == 1) {
            const uint2 w = __ldcs(reinterpret_cast<const uint2*>(src));
            const T* b = reinterpret_cast<const T*>(&w);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = b[j];
        } else if constexpr (sizeof(T) == 2) {
            const uint4 w = __ldcs(reinterpret_cast<const uint4*>(src));
            const T* b = reinterpret_cast<const T*>(&w);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = b[j];
        } else {
            const uint4 w0 = __ldcs(reinterpret_cast<const uint4*>(src));
            const uint4 w1 = __ldcs(reinterpret_cast<const uint4*>(src) + 1);
            const T* b0 = reinterpret_cast<const T*>(&w0);
            const T* b1 = reinterpret_cast<const T*>(&w1);
#pragma unroll
            for (int j = 0; j < 4; ++j) { o[j] = b0[j]; o[j + 4] = b1[j]; }
        }
    }
    template <typename T>
    __device__ static void st8(T* dst, const T (&o)[8]) {
        if constexpr (sizeof(T) == 1) {
            uint2 w;
            T* b = reinterpret_cast<T*>(&w);
#pragma unroll
            for (int j = 0; j < 8; ++j) b[j] = o[j];
            __stcs(reinterpret_cast<uint2*>(dst), w);
        } else if constexpr (sizeof(T) == 2) {
            uint4 w;
            T* b = reinterpret_cast<T*>(&w);
#pragma unroll
            for (int j = 0; j < 8; ++j) b[j] = o[j];
            __stcs(reinterpret_cast<uint4*>(dst), w);
        } else {
            uint4 w0, w1;
            T* b0 = reinterpret_cast<T*>(&w0);
            T* b1 = reinterpret_cast<T*>(&w1);
#pragma unroll
            for (int j = 0; j < 4; ++j) { b0[j] = o[j]; b1[j] = o[j + 4]; }
            __stcs(reinterpret_cast<uint4*>(dst), w0);
            __stcs(reinterpret_cast<uint4*>(dst) + 1, w1);
        }
    }
    __device__ static void load8(const LaunchDesc& d, int64_t e, int (&qm)[8], unsigned (&qv)[8]) {
        MT a[8];
        VT b[8];
        ld8(static_cast<const MT*>(d.m) + e, a);
        ld8(static_cast<const VT*>(d.v) + e, b);
#pragma unroll
        for (int j = 0; j < 8; ++j) { qm[j] = (int)a[j]; qv[j] = (unsigned)b[j]; }
    }
    __device__ static void load1(const LaunchDesc& d, int64_t e, int& qm, unsigned& qv) {
        qm = (int)static_cast<const MT*>(d.m)[e];
        qv = (unsigned)static_cast<const VT*>(d.v)[e];
    }
    __device__ static void store8(const LaunchDesc& d, int64_t e, const int (&mi)[8], const int (&vi)[8]) {
        MT a[8];
        VT b[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) { a[j] = (MT)mi[j]; b[j] = (VT)(unsigned)vi[j]; }
        st8(static_cast<MT*>(d.m) + e, a);
        st8(static_cast<VT*>(d.v) + e, b);
    }
    __device__ static void store1(const LaunchDesc& d, int64_t e, int mi, int vi) {
        static_cast<MT*>(d.m)[e] = (MT)mi;
        static_cast<VT*>(d.v)[e] = (VT)(unsigned)vi;
    }
    // Conversions of a double-path code as the reference's stores perform
    // them (CUDA/stquant_kernel.cu:210,215 and the 16/32-bit twins).
    __device__ static int m_int(double q) { return (int)(MT)q; }
    __device__ static int v_int(double q) { return (int)(unsigned)(VT)q; }
};

template <> struct Codes<MDQ_LAYOUT_S8U8> : CodesPlain<int8_t, uint8_t> {
    static constexpr int kTblBits = 8;
};
template <> struct Codes<MDQ_LAYOUT_S16U16> : CodesPlain<int16_t, uint16_t> {
    static constexpr int kTblBits = 0;
};
template <> struct Codes<MDQ_LAYOUT_S32U32> : CodesPlain<int32_t, uint32_t> {
    static constexpr int kTblBits = 0;
};

// int8 m codes + v nibbles packed two per byte.
template <> struct Codes<MDQ_LAYOUT_M8V4> {
    static constexpr int kTblBits = 4;
    __device__ static void load8(const LaunchDesc& d, int64_t e, int (&qm)[8], unsigned (&qv)[8]) {
        const uint2 w = __ldcs(reinterpret_cast<const uint2*>(static_cast<const int8_t*>(d.m) + e));
        const unsigned vw = __ldcs(reinterpret_cast<const unsigned*>(static_cast<const uint8_t*>(d.v) + (e >> 1)));
        const int8_t* b = reinterpret_cast<const int8_t*>(&w);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            qm[j] = b[j];
            qv[j] = (vw >> (4 * j)) & 15u;
        }
    }
    __device__ static void load1(const LaunchDesc& d, int64_t e, int& qm, unsigned& qv) {
        qm = static_cast<const int8_t*>(d.m)[e];
        qv = (static_cast<const uint8_t*>(d.v)[e >> 1] >> (4 * (e & 1))) & 15u;
    }
    __device__ static unsigned nib(int vi) { return (unsigned)(vi < 0 ? 0 : (vi > 15 ? 15 : vi)); }
    __device__ static void store8(const LaunchDesc& d, int64_t e, const int (&mi)[8], const int (&vi)[8]) {
        uint2 w;
        int8_t* b = reinterpret_cast<int8_t*>(&w);
        unsigned vw = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            b[j] = (int8_t)mi[j];
            vw |= nib(vi[j]) << (4 * j);
        }
        __stcs(reinterpret_cast<uint2*>(static_cast<int8_t*>(d.m) + e), w);
        __stcs(reinterpret_cast<unsigned*>(static_cast<uint8_t*>(d.v) + (e >> 1)), vw);
    }
    // Single elements share a byte with their neighbour: only used by the
    // owner of a whole tail, which writes each byte once (see store_tail).
    __device__ static void store1(const LaunchDesc& d, int64_t e, int mi, int vi) {
        static_cast<int8_t*>(d.m)[e] = (int8_t)mi;
        uint8_t* vb = static_cast<uint8_t*>(d.v) + (e >> 1);
        const unsigned sh = 4 * (unsigned)(e & 1);
        *vb = (uint8_t)((*vb & ~(15u << sh)) | (nib(vi) << sh));
    }
    __device__ static int m_int(double q) { return (int)(int8_t)q; }
    __device__ static int v_int(double q) { return (int)q; }
};

// Gradient element loads.
template <typename GT> struct Grad;
template <> struct Grad<float> {
    __device__ static void load8(const void* g, int64_t e, float (&o)[8]) {
        const float4* s = reinterpret_cast<const float4*>(static_cast<const float*>(g) + e);
        const float4 a = __ldcs(s), b = __ldcs(s + 1);
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
        o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    }
    __device__ static float load1(const void* g, int64_t e) { return static_cast<const float*>(g)[e]; }
};
template <> struct Grad<__nv_bfloat16> {
    __device__ static void load8(const void* g, int64_t e, float (&o)[8]) {
        const uint4 w = __ldcs(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(g) + e));
        const unsigned u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            o[2 * j] = __uint_as_float(u[j] << 16);
            o[2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
        }
    }
    __device__ static float load1(const void* g, int64_t e) {
        return __bfloat162float(static_cast<const __nv_bfloat16*>(g)[e]);
    }
};

__device__ __forceinline__ unsigned long long prof_now() { return clock64(); }

template <int CAP>
__device__ __forceinline__ int find_desc(const LaunchParams<CAP>& P, int tile) {
    int lo = 0, hi = P.n_desc - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (P.d[mid].tile_begin <= tile) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// ---------------------------------------------------------------------------
// Fast kernel: power-of-two blocks 8..2048, tiles of 2048 elements.
// ---------------------------------------------------------------------------
template <int LAYOUT, typename GT, bool EXACT_P, bool PROF, int CAP>
__global__ void __launch_bounds__(kThreads)
mdq_step_tiles(const __grid_constant__ LaunchParams<CAP> P) {
    using CI = Codes<LAYOUT>;
    constexpr bool kAllDouble = (LAYOUT == MDQ_LAYOUT_S32U32);
    __shared__ float s_tbl[kTblMax];
    __shared__ float s_red[3][kThreads / 32];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    int cur = -1;
    StepConsts C;
    unsigned long long pc[kProfSlots] = {0, 0, 0, 0, 0};

    for (int tile = blockIdx.x; tile < P.total_tiles; tile += gridDim.x) {
        const int t = find_desc(P, tile);
        const LaunchDesc& D = P.d[t];
        if (t != cur) {
            C = make_step_consts(D.b1, D.b2, D.lr, D.wd, D.eps, D.step, D.m_bits, D.v_bits);
            cur = t;
        }
        unsigned long long t0 = 0;
        if (PROF && tid == 0) t0 = prof_now();

        const int lb = D.log2_block;
        const int64_t n = D.n;
        const int64_t tile_e0 = (int64_t)(tile - D.tile_begin) << kLogTile;
        const int64_t e0 = tile_e0 + tid * kPerThread;
        const int64_t rem = n - e0;
        const int cnt = rem >= kPerThread ? kPerThread : (rem > 0 ? (int)rem : 0);
        const int64_t nblk = (n + ((int64_t)1 << lb) - 1) >> lb;
        const int64_t blk = e0 >> lb;

        // Dequantised-v table: entries (local block, code) of this tile.
        constexpr int kTB = CI::kTblBits;
        const bool use_tbl = kTB > 0 && ((kTile >> lb) << kTB) <= kTblMax;
        __syncthreads();  // previous tile's readers of s_tbl / s_red are done
        if (use_tbl) {
            const int entries = (kTile >> lb) << kTB;
            const int64_t blk0 = tile_e0 >> lb;
            for (int j = tid; j < entries; j += kThreads) {
                const int64_t b = blk0 + (j >> kTB);
                float val = 0.0f;
                if (b < nblk) val = dequant_v((float)(j & ((1 << kTB) - 1)), D.sv[b], D.vmin[b]);
                s_tbl[j] = val;
            }
            __syncthreads();
        }

        float p[8], g[8];
        int qm[8];
        unsigned qv[8];
        if (cnt == kPerThread && D.vec) {
            const float4* ps = reinterpret_cast<const float4*>(D.p + e0);
            const float4 a = __ldcs(ps), b = __ldcs(ps + 1);
            p[0] = a.x; p[1] = a.y; p[2] = a.z; p[3] = a.w;
            p[4] = b.x; p[5] = b.y; p[6] = b.z; p[7] = b.w;
            Grad<GT>::load8(D.g, e0, g);
            CI::load8(D, e0, qm, qv);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                p[j] = 0.0f; g[j] = 0.0f; qm[j] = 0; qv[j] = 0;
                if (j < cnt) {
                    p[j] = D.p[e0 + j];
                    g[j] = Grad<GT>::load1(D.g, e0 + j);
                    CI::load1(D, e0 + j, qm[j], qv[j]);
                }
            }
        }
        float sm = 0.0f, sv = 0.0f, vmn = 0.0f;
        if (cnt > 0) { sm = D.sm[blk]; sv = D.sv[blk]; vmn = D.vmin[blk]; }

        // Dequantise (CUDA/stquant_kernel.cu:163-169).
        float m[8], v[8];
        const int tbl_base = use_tbl ? (((tid * kPerThread) >> lb) << kTB) : 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            m[j] = __fmul_rn((float)qm[j], sm);
            v[j] = use_tbl ? s_tbl[tbl_base + (int)qv[j]] : dequant_v((float)qv[j], sv, vmn);
        }
        if (PROF && tid == 0) { const auto t1 = prof_now(); pc[0] += t1 - t0; t0 = t1; }

        // AdamW moments (CUDA/stquant_kernel.cu:174-177).
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            m[j] = adam_m(m[j], g[j], C);
            v[j] = adam_v(v[j], g[j], C);
        }
        if (PROF && tid == 0) { const auto t1 = prof_now(); pc[1] += t1 - t0; t0 = t1; }

        // Parameter update from the unquantised moments (CUDA/stquant_kernel.cu:220-229).
#pragma unroll
        for (int j = 0; j < 8; ++j) p[j] = update_p<EXACT_P>(p[j], m[j], v[j], C);
        if (cnt == kPerThread && D.vec) {
            float4* pd = reinterpret_cast<float4*>(D.p + e0);
            __stcs(pd, make_float4(p[0], p[1], p[2], p[3]));
            __stcs(pd + 1, make_float4(p[4], p[5], p[6], p[7]));
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (j < cnt) D.p[e0 + j] = p[j];
        }
        if (PROF && tid == 0) { const auto t1 = prof_now(); pc[4] += t1 - t0; t0 = t1; }

        // Block statistics.  NaN seeds make fmaxf/fminf ignore nothing but
        // NaNs, exactly as the reference's tree over fmaxf/fminf does; missing
        // tail elements enter as 0 (CUDA/stquant_kernel.cu:92-97).
        float lv[8];
        float amax = __int_as_float(0x7fffffff), lmax = amax, lmin = amax;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            lv[j] = log_v_of(v[j]);
            const bool ok = j < cnt;
            amax = fmaxf(amax, ok ? fabsf(m[j]) : 0.0f);
            lmax = fmaxf(lmax, ok ? lv[j] : 0.0f);
            lmin = fminf(lmin, ok ? lv[j] : 0.0f);
        }
        const int gthreads = (1 << lb) >> 3;  // threads per quantisation block
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            if (o < gthreads) {
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
                lmin = fminf(lmin, __shfl_xor_sync(0xffffffffu, lmin, o));
            }
        }
        if (gthreads > 32) {  // CTA-uniform
            const int w = tid >> 5;
            if (lane == 0) { s_red[0][w] = amax; s_red[1][w] = lmax; s_red[2][w] = lmin; }
            __syncthreads();
            const int wpg = gthreads >> 5;
            const int w0 = (w / wpg) * wpg;
            amax = s_red[0][w0]; lmax = s_red[1][w0]; lmin = s_red[2][w0];
            for (int k = 1; k < wpg; ++k) {
                amax = fmaxf(amax, s_red[0][w0 + k]);
                lmax = fmaxf(lmax, s_red[1][w0 + k]);
                lmin = fminf(lmin, s_red[2][w0 + k]);
            }
        }
        const float new_sm = scale_m_of(amax, C);
        const float new_sv = scale_v_of(lmax, lmin, C);
        if ((tid & (gthreads - 1)) == 0 && blk < nblk) {
            D.sm[blk] = new_sm;
            D.sv[blk] = new_sv;
            D.vmin[blk] = lmin;
        }
        if (PROF && tid == 0) { const auto t1 = prof_now(); pc[2] += t1 - t0; t0 = t1; }

        // Requantise (CUDA/stquant_kernel.cu:204-216).
        const float dm = __fadd_rn(new_sm, 1e-12f), dv = __fadd_rn(new_sv, 1e-12f);
        const float rdm = __frcp_rn(dm), rdv = __frcp_rn(dv);
        int mi[8], vi[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float xm = m[j];
            const float xv = __fsub_rn(lv[j], lmin);
            bool ok_m = false, ok_v = false;
            float rm = 0.0f, rv = 0.0f;
            if (!kAllDouble) {
                rm = round_ratio_fast(xm, rdm, ok_m);
                rv = round_ratio_fast(xv, rdv, ok_v);
            }
            if (ok_m) {
                rm = fminf(fmaxf(rm, -C.lm_f), __fsub_rn(C.lm_f, 1.0f));
                mi[j] = (int)rm;
            } else {
                mi[j] = CI::m_int(requant_m_ref(xm, dm, C.lm_d));
            }
            if (ok_v) {
                rv = fminf(fmaxf(rv, 0.0f), C.lv_f);
                vi[j] = (int)rv;
            } else {
                vi[j] = CI::v_int(requant_v_ref(xv, dv, C.lv_d));
            }
        }
        if (cnt == kPerThread && D.vec) {
            CI::store8(D, e0, mi, vi);
        } else {
            // One thread owns all 8 elements, so M8V4 nibble pairs never race.
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (j < cnt) CI::store1(D, e0 + j, mi[j], vi[j]);
        }
        if (PROF && tid == 0) { const auto t1 = prof_now(); pc[3] += t1 - t0; }
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
    if (prof && tid == 0) t0 = prof_now();

    const StepConsts C = make_step_consts(D.b1, D.b2, D.lr, D.wd, D.eps, D.step, D.m_bits, D.v_bits);
    const float sm = D.sm[blk], sv = D.sv[blk], vmn = D.vmin[blk];
    float g = 0.0f, m = 0.0f, v = 0.0f;
    int qm = 0;
    unsigned qv = 0;
    if (ok) {
        g = Grad<GT>::load1(D.g, i);
        CI::load1(D, i, qm, qv);
        m = __fmul_rn((float)qm, sm);
        v = dequant_v((float)qv, sv, vmn);
    }
    if (prof && tid == 0) { const auto t1 = prof_now(); pc[0] += t1 - t0; t0 = t1; }
    if (ok) {
        m = adam_m(m, g, C);
        v = adam_v(v, g, C);
    }
    if (prof && tid == 0) { const auto t1 = prof_now(); pc[1] += t1 - t0; t0 = t1; }

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
        D.sm[blk] = new_sm;
        D.sv[blk] = new_sv;
        D.vmin[blk] = new_vmin;
    }
    if (prof && tid == 0) { const auto t1 = prof_now(); pc[2] += t1 - t0; t0 = t1; }

    int code_m = 0, code_v = 0;
    if (ok) {
        const float dm = __fadd_rn(new_sm, 1e-12f), dv = __fadd_rn(new_sv, 1e-12f);
        const int mi = CI::m_int(requant_m_ref(m, dm, C.lm_d));
        const int vi = CI::v_int(requant_v_ref(__fsub_rn(lv, new_vmin), dv, C.lv_d));
        if (LAYOUT != MDQ_LAYOUT_M8V4) CI::store1(D, i, mi, vi);
        code_m = mi;
        code_v = vi;
    }
    if (LAYOUT == MDQ_LAYOUT_M8V4) {
        // Neighbouring elements share a byte (the block is even, so both lie
        // in this CTA): even elements write first, odd ones after a barrier.
        for (int par = 0; par < 2; ++par) {
            if (ok && (i & 1) == par) CI::store1(D, i, code_m, code_v);
            __syncthreads();
        }
    }
    if (prof && tid == 0) { const auto t1 = prof_now(); pc[3] += t1 - t0; t0 = t1; }
    if (ok) {
        D.p[i] = update_p<EXACT_P>(D.p[i], m, v, C);
    }
    if (prof && tid == 0) {
        pc[4] += prof_now() - t0;
        for (int k = 0; k < kProfSlots; ++k) atomicAdd(prof + k, pc[k]);
    }
}

}  // namespace mdq

// ===========================================================================
// Host side
// ===========================================================================
namespace {

thread_local char g_err[512] = "";

mdq_status fail(mdq_status s, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return s;
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
    L.p = d.p;
    L.g = d.grad;
    L.m = d.exp_avg;
    L.v = d.exp_avg_sq;
    L.sm = d.scale_m;
    L.sv = d.scale_v;
    L.vmin = d.v_min;
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
int blocks_per_sm(K kernel) {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, mdq::kThreads, 0) != cudaSuccess ||
        b < 1)
        b = 1;
    return b;
}

template <int LAYOUT, typename GT, bool EXACT_P, bool PROF, int CAP>
mdq_status launch_tiles_t(const mdq::LaunchParams<CAP>& P, int sms, cudaStream_t stream) {
    auto k = mdq::mdq_step_tiles<LAYOUT, GT, EXACT_P, PROF, CAP>;
    static int occ = 0;  // per instantiation; identical across B200 devices
    if (occ == 0) occ = blocks_per_sm(k);
    int grid = sms * occ;
    if (grid > P.total_tiles) grid = P.total_tiles;
    k<<<grid, mdq::kThreads, 0, stream>>>(P);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(MDQ_ERR_CUDA, "step launch: %s", cudaGetErrorString(e));
    return MDQ_OK;
}

template <int LAYOUT, typename GT, int CAP>
mdq_status launch_tiles_mode(const mdq::LaunchParams<CAP>& P, bool exact, bool prof, int sms,
                             cudaStream_t s) {
    if (exact) {
        return prof ? launch_tiles_t<LAYOUT, GT, true, true, CAP>(P, sms, s)
                    : launch_tiles_t<LAYOUT, GT, true, false, CAP>(P, sms, s);
    }
    return prof ? launch_tiles_t<LAYOUT, GT, false, true, CAP>(P, sms, s)
                : launch_tiles_t<LAYOUT, GT, false, false, CAP>(P, sms, s);
}

template <int CAP>
mdq_status launch_tiles(int layout, int gdt, const mdq::LaunchParams<CAP>& P, bool exact, bool prof,
                        int sms, cudaStream_t s) {
    const bool bf = gdt == MDQ_BF16;
    switch (layout) {
        case MDQ_LAYOUT_PACKED4:
            return bf ? launch_tiles_mode<MDQ_LAYOUT_PACKED4, __nv_bfloat16, CAP>(P, exact, prof, sms, s)
                      : launch_tiles_mode<MDQ_LAYOUT_PACKED4, float, CAP>(P, exact, prof, sms, s);
        case MDQ_LAYOUT_S8U8:
            return bf ? launch_tiles_mode<MDQ_LAYOUT_S8U8, __nv_bfloat16, CAP>(P, exact, prof, sms, s)
                      : launch_tiles_mode<MDQ_LAYOUT_S8U8, float, CAP>(P, exact, prof, sms, s);
        case MDQ_LAYOUT_S16U16:
            return bf ? launch_tiles_mode<MDQ_LAYOUT_S16U16, __nv_bfloat16, CAP>(P, exact, prof, sms, s)
                      : launch_tiles_mode<MDQ_LAYOUT_S16U16, float, CAP>(P, exact, prof, sms, s);
        case MDQ_LAYOUT_S32U32:
            return bf ? launch_tiles_mode<MDQ_LAYOUT_S32U32, __nv_bfloat16, CAP>(P, exact, prof, sms, s)
                      : launch_tiles_mode<MDQ_LAYOUT_S32U32, float, CAP>(P, exact, prof, sms, s);
        case MDQ_LAYOUT_M8V4:
            return bf ? launch_tiles_mode<MDQ_LAYOUT_M8V4, __nv_bfloat16, CAP>(P, exact, prof, sms, s)
                      : launch_tiles_mode<MDQ_LAYOUT_M8V4, float, CAP>(P, exact, prof, sms, s);
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
    int i = 0;
    while (i < count) {
        P.n_desc = 0;
        P.prof = prof;
        int64_t tiles = 0;
        while (i < count && P.n_desc < CAP) {
            const mdq_tensor_desc& d = descs[idx[i]];
            const int64_t t = (d.n + mdq::kTile - 1) / mdq::kTile;
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
                                                sms, s);
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
