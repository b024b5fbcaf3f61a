// mdq_step.cu - B200 (sm_100a) fused quantized-AdamW step and its C ABI.
//
// Kernel design
// -------------
// The reference runs one thread per element and one CTA per quantisation block
// (CUDA/stquant_kernel.cu:61,421-422) with three shared-memory tree reductions
// per CTA and a double-precision divide per code.  Here a persistent grid
// walks contiguous ranges of "tiles" of 2048 consecutive elements of one
// tensor (mdq_tiles.cuh), PT = 8 or 16 elements per thread.  The L = B/PT
// lanes (at most 32) that share a quantisation block of B elements own it
// interleaved in 4-element chunks, so every warp-wide load and store covers
// whole 32-byte sectors, a thread's elements lie in one block, and the
// block's max/min reductions are xor shuffles or one redux.sync (plus, for
// blocks wider than a warp's span, one shared-memory exchange).
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
#include <stddef.h>
#include <algorithm>
#include <mutex>
#include <vector>

#include "mdq.h"
#include "mdq_math.cuh"
#include "mdq_codes.cuh"

#include "mdq_tiles.cuh"
#include "mdq_blocks.cuh"

namespace mdq {
// Bulk-copy staged warp-per-block kernel, int8/uint8 codes (mdq_staged_s8u8.cu).
template <int CAP>
mdq_status launch_staged_s8u8(int gdt, const LaunchParams<CAP>& P, bool exact, int logb, int sms,
                              cudaStream_t s);
// The same for packed 4-bit codes at 128/256-element blocks (mdq_staged_packed4.cu).
template <int CAP>
mdq_status launch_staged_packed4(int gdt, const LaunchParams<CAP>& P, bool exact, int logb, int sms,
                                 cudaStream_t s);
}  // namespace mdq

// The C layout the Python mirror (mdq_b200/kernels.py, _lib.py) packs.
static_assert(offsetof(mdq_tensor_desc, grad_dtype) == 104, "mdq_tensor_desc layout");
static_assert(offsetof(mdq_tensor_desc, p_bf16) == 112, "mdq_tensor_desc layout");
static_assert(sizeof(mdq_tensor_desc) == 120, "mdq_tensor_desc layout");
static_assert(offsetof(mdq_step_options, n_peers) == 16, "mdq_step_options layout");
static_assert(offsetof(mdq_step_options, peer_delta) == 24, "mdq_step_options layout");
static_assert(offsetof(mdq_step_options, n_grad_ranks) == 80, "mdq_step_options layout");
static_assert(offsetof(mdq_step_options, grad_delta) == 88, "mdq_step_options layout");
static_assert(sizeof(mdq_step_options) == 152, "mdq_step_options layout");

namespace mdq {

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
    if (ok) {
        const float pn = update_p<EXACT_P>(D.t.p[i], m, v, C);
        D.t.p[i] = pn;
        if (D.t.p16 != nullptr) D.t.p16[i] = __float2bfloat16_rn(pn);
    }
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
    if (d.p_bf16 != nullptr && !aligned(d.p_bf16, 8)) return false;
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

// Bit 1 of LaunchDesc::vec: every streamed array starts on a 16-byte
// boundary, as bulk copies into shared memory need (int8/uint8 and packed
// 4-bit codes).
bool bulk_ok(const mdq_tensor_desc& d) {
    if (!(aligned(d.p, 16) && aligned(d.grad, 16) && aligned(d.exp_avg, 16))) return false;
    if (d.layout == MDQ_LAYOUT_S8U8) return aligned(d.exp_avg_sq, 16);
    return d.layout == MDQ_LAYOUT_PACKED4;
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
    L.t.p16 = static_cast<__nv_bfloat16*>(d.p_bf16);
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
    L.vec = (int8_t)(vec_ok(d) ? (bulk_ok(d) ? 3 : 1) : 0);
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

template <int CAP>
mdq_status launch_blocks(int layout, int gdt, const mdq::LaunchParams<CAP>& P, bool exact, int logb,
                         int sms, cudaStream_t s) {
    switch (layout) {
        case MDQ_LAYOUT_PACKED4: return mdq::launch_blocks_packed4(gdt, P, exact, logb, sms, s);
        case MDQ_LAYOUT_S8U8: return mdq::launch_blocks_s8u8(gdt, P, exact, logb, sms, s);
        case MDQ_LAYOUT_S16U16: return mdq::launch_blocks_s16u16(gdt, P, exact, logb, sms, s);
        case MDQ_LAYOUT_S32U32: return mdq::launch_blocks_s32u32(gdt, P, exact, logb, sms, s);
        case MDQ_LAYOUT_M8V4: return mdq::launch_blocks_m8v4(gdt, P, exact, logb, sms, s);
    }
    return fail(MDQ_ERR_INVALID_ARG, "bad layout %d", layout);
}

// Which kernel takes a class whose blocks all have 512 or 1024 elements.
// Measured on B200 (2^30 elements, bf16 gradients, Gparams/s, tiled vs
// warp-per-block, fast p / exact p):
//   int8/uint8 codes, 1024: 285 vs 316-322 / 252 vs 286-292
//   packed 4-bit,     1024: 435 vs 402 / 293 vs 329
// so the warp-per-block kernel takes the int8/uint8 layout, and packed 4-bit
// codes in exact p mode at 1024-element blocks; the tiled kernel the rest.
// MDQ_BLOCK_KERNEL=1 / =0 forces the choice for every eligible class
// (measurement).  Read once.
bool use_block_kernel(int layout, int block, bool exact) {
    static int mode = -2;
    if (mode == -2) {
        const char* e = getenv("MDQ_BLOCK_KERNEL");
        mode = e == nullptr ? -1 : (e[0] == '1' ? 1 : 0);
    }
    if (mode >= 0) return mode == 1;
    return layout == MDQ_LAYOUT_S8U8 || (layout == MDQ_LAYOUT_PACKED4 && exact && block == 1024);
}

// Whether int8/uint8 classes on the warp-per-block path take the bulk-copy
// staged variant (mdq_staged.cuh); it serves launches without peers or
// gradient ranks.  Measured on B200 (2^30 elements, bf16 gradients,
// Gparams/s, staged vs direct loads, fast p / exact p):
//   512-element blocks:  341 vs 239 / 240 vs 187
//   1024-element blocks: 356 vs 330 / 251 vs 255
// and, against the tiled kernel, for 128 / 256-element blocks (1024-element
// units of whole blocks):
//   128-element blocks:  314 vs 303 / 224 vs 238
//   256-element blocks:  325 vs 306 / 226 vs 244
// so exact p at 128, 256 and 1024-element blocks stays on the other kernels.
// MDQ_STAGED=0 / =1 forces the choice (measurement).  Read once.
bool use_staged_kernel(int layout, int block, bool exact, const mdq::PeerSet& peers,
                       const mdq::GradRanks& granks) {
    static int mode = -2;
    if (mode == -2) {
        const char* e = getenv("MDQ_STAGED");
        mode = e == nullptr ? -1 : (e[0] == '1' ? 1 : 0);
    }
    if (peers.n != 0 || granks.n != 0) return false;
    if (layout == MDQ_LAYOUT_PACKED4) {
        // Packed 4-bit codes, fast p (staged vs tiled, Gparams/s): 128-element
        // blocks 404 vs 359, 256-element blocks 423 vs 422; the tiled kernel's
        // tables serve the larger blocks.  MDQ_STAGED=1 also takes 256.
        if (exact || block > 256) return false;
        if (mode >= 0) return mode == 1;
        return block == 128;
    }
    if (layout != MDQ_LAYOUT_S8U8) return false;
    if (mode >= 0) return mode == 1;
    return !(exact && (block == 1024 || block <= 256));
}

template <int CAP>
mdq_status launch_tiles(int layout, int gdt, const mdq::LaunchParams<CAP>& P, bool exact, bool prof,
                        int sms, int pt, int min_block, cudaStream_t s) {
    switch (layout) {
        case MDQ_LAYOUT_PACKED4: return mdq::launch_tiles_packed4(gdt, P, exact, prof, sms, pt, min_block, s);
        case MDQ_LAYOUT_S8U8: return mdq::launch_tiles_s8u8(gdt, P, exact, prof, sms, pt, min_block, s);
        case MDQ_LAYOUT_S16U16: return mdq::launch_tiles_s16u16(gdt, P, exact, prof, sms, pt, min_block, s);
        case MDQ_LAYOUT_S32U32: return mdq::launch_tiles_s32u32(gdt, P, exact, prof, sms, pt, min_block, s);
        case MDQ_LAYOUT_M8V4: return mdq::launch_tiles_m8v4(gdt, P, exact, prof, sms, pt, min_block, s);
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
// Small-block staging (blocks of 128 / 256 elements, mdq_staged.cuh) takes
// whole 1024-element units of tensors whose arrays, scales included, all
// start on 16-byte boundaries.
bool bulk_ok_small(const mdq_tensor_desc& d) {
    return bulk_ok(d) && aligned(d.scale_m, 16) && aligned(d.scale_v, 16) && aligned(d.v_min, 16);
}

// The same tensor from element `off` on (a multiple of its block).
mdq_tensor_desc desc_from(const mdq_tensor_desc& d, int64_t off) {
    mdq_tensor_desc r = d;
    const int64_t gsz = d.grad_dtype == MDQ_BF16 ? 2 : 4;
    r.p = d.p + off;
    r.grad = static_cast<const char*>(d.grad) + off * gsz;
    // (packed 4-bit codes: one byte per element, both nibbles)
    const int64_t mbytes = d.layout == MDQ_LAYOUT_PACKED4 ? 8 : storage_bits_m(d.layout);
    r.exp_avg = static_cast<char*>(d.exp_avg) + off * mbytes / 8;
    if (d.exp_avg_sq != nullptr)
        r.exp_avg_sq = static_cast<char*>(d.exp_avg_sq) + off * storage_bits_v(d.layout) / 8;
    r.scale_m = d.scale_m + off / d.block;
    r.scale_v = d.scale_v + off / d.block;
    r.v_min = d.v_min + off / d.block;
    if (d.p_bf16 != nullptr) r.p_bf16 = static_cast<uint16_t*>(d.p_bf16) + off;
    r.n = d.n - off;
    return r;
}

template <int CAP>
mdq_status run_class(const mdq_tensor_desc* descs, const int* idx, int count, bool exact,
                     unsigned long long* prof, const mdq::PeerSet& peers,
                     const mdq::GradRanks& granks, int sms, cudaStream_t s,
                     bool allow_small_staged = true) {
    static thread_local mdq::LaunchParams<CAP> P;  // ~24 KB for CAP = 224
    P.peers = peers;
    P.granks = granks;
    // 16 elements per thread (4096-element tiles, 2 CTAs per SM) halve the
    // per-tile work; measured on B200 it pays for 4-bit v codes, and for
    // 8-bit codes only with blocks of 1024 or more.
    int min_block = mdq::kTile, max_block = 0;
    for (int k = 0; k < count; ++k) {
        min_block = std::min(min_block, (int)descs[idx[k]].block);
        max_block = std::max(max_block, (int)descs[idx[k]].block);
    }
    const int layout = descs[idx[0]].layout;
    if (allow_small_staged && min_block == max_block && (min_block == 128 || min_block == 256) &&
        prof == nullptr && use_staged_kernel(layout, min_block, exact, peers, granks)) {
        // Whole 1024-element units of aligned tensors: the staged kernel;
        // the rest (each tensor's last n mod 1024 elements, which start on a
        // block boundary, and unaligned tensors): the tiled kernel.
        constexpr int64_t kUnit = 1024;
        const int logb = min_block == 128 ? 7 : 8;
        std::vector<mdq_tensor_desc> rest;
        std::vector<int> staged;
        for (int k = 0; k < count; ++k) {
            const mdq_tensor_desc& d = descs[idx[k]];
            const int64_t whole = d.n / kUnit * kUnit;
            if (whole > 0 && bulk_ok_small(d)) {
                staged.push_back(idx[k]);
                if (d.n > whole) rest.push_back(desc_from(d, whole));
            } else {
                rest.push_back(d);
            }
        }
        size_t i = 0;
        while (i < staged.size()) {
            P.n_desc = 0;
            P.prof = nullptr;
            int64_t units = 0;
            while (i < staged.size() && P.n_desc < CAP) {
                const mdq_tensor_desc& d = descs[staged[i]];
                const int64_t u = d.n / kUnit;
                if (units + u > (int64_t)INT32_MAX && P.n_desc > 0) break;
                mdq::LaunchDesc L = to_launch(d);
                L.n = u * kUnit;
                L.tile_begin = (int32_t)units;
                P.d[P.n_desc++] = L;
                units += u;
                ++i;
            }
            P.total_tiles = (int32_t)units;
            const int gdt = descs[staged[0]].grad_dtype;
            const mdq_status st =
                layout == MDQ_LAYOUT_PACKED4
                    ? mdq::launch_staged_packed4<CAP>(gdt, P, exact, logb, sms, s)
                    : mdq::launch_staged_s8u8<CAP>(gdt, P, exact, logb, sms, s);
            if (st != MDQ_OK) return st;
        }
        if (rest.empty()) return MDQ_OK;
        std::vector<int> ridx(rest.size());
        for (size_t k = 0; k < rest.size(); ++k) ridx[k] = (int)k;
        return run_class<CAP>(rest.data(), ridx.data(), (int)rest.size(), exact, prof, peers,
                              granks, sms, s, false);
    }
    if (min_block == max_block && (min_block == 512 || min_block == 1024) && prof == nullptr &&
        use_block_kernel(layout, min_block, exact)) {
        // Warp-per-block kernel: a launch's units are quantisation blocks.
        const int logb = min_block == 1024 ? 10 : 9;
        int i = 0;
        while (i < count) {
            P.n_desc = 0;
            P.prof = nullptr;
            int64_t units = 0;
            while (i < count && P.n_desc < CAP) {
                const mdq_tensor_desc& d = descs[idx[i]];
                const int64_t u = (d.n + min_block - 1) / min_block;
                if (units + u > (int64_t)INT32_MAX && P.n_desc > 0) break;
                mdq::LaunchDesc L = to_launch(d);
                L.tile_begin = (int32_t)units;
                P.d[P.n_desc++] = L;
                units += u;
                ++i;
            }
            P.total_tiles = (int32_t)units;
            const mdq_tensor_desc& d0 = descs[idx[i - 1]];
            const mdq_status st =
                use_staged_kernel(d0.layout, min_block, exact, peers, granks)
                    ? mdq::launch_staged_s8u8<CAP>(d0.grad_dtype, P, exact, logb, sms, s)
                    : launch_blocks<CAP>(d0.layout, d0.grad_dtype, P, exact, logb, sms, s);
            if (st != MDQ_OK) return st;
        }
        return MDQ_OK;
    }
    const bool v4 = layout == MDQ_LAYOUT_PACKED4 || layout == MDQ_LAYOUT_M8V4;
    const int pt = MDQ_ENABLE_PT16 && v4 && min_block >= MDQ_V4_PT16_MIN_BLOCK ? 16 : 8;
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
    mdq::PeerSet peers{};
    if (opts != nullptr && opts->n_peers != 0) {
        if (opts->n_peers < 0 || opts->n_peers > 7)
            return fail(MDQ_ERR_INVALID_ARG, "n_peers %d outside 0..7", opts->n_peers);
        peers.n = opts->n_peers;
        for (int k = 0; k < peers.n; ++k) {
            if (opts->peer_delta[k] == 0 || (opts->peer_delta[k] & 15) != 0)
                return fail(MDQ_ERR_INVALID_ARG, "peer_delta[%d] must be a non-zero multiple of 16",
                            k);
            peers.delta[k] = opts->peer_delta[k];
        }
    }
    mdq::GradRanks granks{};
    granks.scale = 1.0f;
    if (opts != nullptr && opts->n_grad_ranks != 0) {
        if (opts->n_grad_ranks < 0 || opts->n_grad_ranks > 8)
            return fail(MDQ_ERR_INVALID_ARG, "n_grad_ranks %d outside 0..8", opts->n_grad_ranks);
        granks.n = opts->n_grad_ranks;
        granks.scale = opts->grad_scale;
        for (int k = 0; k < granks.n; ++k) {
            if ((opts->grad_delta[k] & 15) != 0)
                return fail(MDQ_ERR_INVALID_ARG, "grad_delta[%d] must be a multiple of 16", k);
            granks.delta[k] = opts->grad_delta[k];
        }
    }
    for (int i = 0; i < n_descs; ++i) {
        const mdq_status st = validate(descs[i], i);
        if (st != MDQ_OK) return st;
        if (granks.n > 0 && descs[i].n > 0 && !fast_eligible(descs[i]))
            return fail(MDQ_ERR_UNSUPPORTED,
                        "desc %d: block %d needs the per-element kernel, which has no gradient "
                        "reduction", i, descs[i].block);
        if (peers.n > 0 && descs[i].n > 0 && !fast_eligible(descs[i]))
            return fail(MDQ_ERR_UNSUPPORTED,
                        "desc %d: block %d needs the per-element kernel, which has no peer copies",
                        i, descs[i].block);
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
                ? run_class<mdq::kCapSmall>(descs, order, cnt, exact, prof, peers, granks, sms,
                                            stream)
                : run_class<mdq::kCapLarge>(descs, order, cnt, exact, prof, peers, granks, sms,
                                            stream);
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
    mdq_tensor_desc d = {};  // every field not set below (p_bf16) stays zero
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
    mdq_step_options o = {};  // no peers
    o.p_mode = MDQ_P_EXACT;
    o.profile_cycles = profile_cycles;
    return mdq_adamw_step_multi(&d, 1, &o, stream);
}

const char* mdq_last_error(void) { return g_err; }

int32_t mdq_abi_version(void) { return MDQ_ABI_VERSION; }

}  // extern "C"
