// mdq_stats.cu - fused per-tensor gradient statistics for the MDQ bit policy.
//
// The policy scores each tensor from n_l = RMS(g), r_l = std(g) / mean|g| and
// v_l = mean(g^2) (reference CUDA/stquant_opt_simple.py:94-98: three torch
// reductions per tensor, each a full pass over the gradient).  Here one launch
// reads every gradient once and produces, per tensor, the float64 sums
// (sum g, sum g^2, sum |g|, count) from which all three follow.
//
// Determinism: each tensor is cut into chunks of kChunk elements; pass 1
// writes one partial record (three doubles) per chunk into a caller-provided
// workspace, pass 2 folds each tensor's records in a fixed order.  No atomics,
// so repeated calls give identical bits.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <mutex>

#include "mdq.h"

namespace mdq_stats {

constexpr int kThreads = 256;
constexpr int kChunk = 1 << 16;  // elements per partial record
constexpr int kCap = 256;        // tensors per launch

struct Params {
    int32_t n;
    int32_t total_chunks;
    const void* g[kCap];
    int64_t count[kCap];
    int32_t chunk_begin[kCap + 1];
};

__device__ __forceinline__ int find_tensor(const Params& P, int c) {
    int lo = 0, hi = P.n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (P.chunk_begin[mid] <= c) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ void acc(float x, float& s, float& s2, float& sa) {
    s += x;
    s2 = fmaf(x, x, s2);
    sa += fabsf(x);
}

// Sum over the CTA in a fixed order (shuffle tree, then warp 0 over warps).
__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    double r = 0.0;
    if (threadIdx.x == 0)
        for (int i = 0; i < kThreads / 32; ++i) r += red[i];
    __syncthreads();
    return r;
}

// Pass 1: one chunk per CTA iteration -> partial[c] = (sum g, sum g^2, sum |g|).
template <typename GT>
__global__ void __launch_bounds__(kThreads) chunk_sums(const __grid_constant__ Params P,
                                                       double* partial) {
    __shared__ double red[kThreads / 32];
    for (int c = blockIdx.x; c < P.total_chunks; c += gridDim.x) {
        const int t = find_tensor(P, c);
        const int64_t n = P.count[t];
        const int64_t e0 = (int64_t)(c - P.chunk_begin[t]) * kChunk;
        const int64_t e1 = min(e0 + (int64_t)kChunk, n);
        const GT* g = static_cast<const GT*>(P.g[t]);
        // Per-thread float sums over <= 256 elements, then float64.
        float s = 0.0f, s2 = 0.0f, sa = 0.0f;
        const bool vec = ((uintptr_t)(g + e0) & 15) == 0;
        constexpr int kV = 16 / sizeof(GT);
        // Vector loads over whole rows of kThreads * kV elements, the rest
        // element by element.
        const int64_t done = vec ? ((e1 - e0) / ((int64_t)kThreads * kV)) * kThreads * kV : 0;
        if (vec) {
            for (int64_t i = e0 + (int64_t)threadIdx.x * kV; i < e0 + done;
                 i += (int64_t)kThreads * kV) {
                const uint4 w = __ldcs(reinterpret_cast<const uint4*>(g + i));
                if constexpr (sizeof(GT) == 4) {
                    acc(__uint_as_float(w.x), s, s2, sa);
                    acc(__uint_as_float(w.y), s, s2, sa);
                    acc(__uint_as_float(w.z), s, s2, sa);
                    acc(__uint_as_float(w.w), s, s2, sa);
                } else {
                    const unsigned u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        acc(__uint_as_float(u[k] << 16), s, s2, sa);
                        acc(__uint_as_float(u[k] & 0xffff0000u), s, s2, sa);
                    }
                }
            }
        }
        for (int64_t j = e0 + done + threadIdx.x; j < e1; j += kThreads) {
            float x;
            if constexpr (sizeof(GT) == 4) x = reinterpret_cast<const float*>(g)[j];
            else x = __bfloat162float(g[j]);
            acc(x, s, s2, sa);
        }
        const double a = block_sum((double)s, red);
        const double b = block_sum((double)s2, red);
        const double d = block_sum((double)sa, red);
        if (threadIdx.x == 0) {
            partial[3 * (int64_t)c + 0] = a;
            partial[3 * (int64_t)c + 1] = b;
            partial[3 * (int64_t)c + 2] = d;
        }
    }
}

// Pass 2: one CTA per tensor folds its chunk records in a fixed order.
__global__ void __launch_bounds__(kThreads) tensor_sums(const __grid_constant__ Params P,
                                                        const double* partial, double* out) {
    __shared__ double red[kThreads / 32];
    const int t = blockIdx.x;
    double s = 0.0, s2 = 0.0, sa = 0.0;
    for (int c = P.chunk_begin[t] + threadIdx.x; c < P.chunk_begin[t + 1]; c += kThreads) {
        s += partial[3 * (int64_t)c + 0];
        s2 += partial[3 * (int64_t)c + 1];
        sa += partial[3 * (int64_t)c + 2];
    }
    s = block_sum(s, red);
    s2 = block_sum(s2, red);
    sa = block_sum(sa, red);
    if (threadIdx.x == 0) {
        out[4 * t + 0] = s;
        out[4 * t + 1] = s2;
        out[4 * t + 2] = sa;
        out[4 * t + 3] = (double)P.count[t];
    }
}

}  // namespace mdq_stats

// The library's error record (mdq_step.cu).
mdq_status mdq_fail(mdq_status s, const char* fmt, ...);
void mdq_clear_error();

namespace {

// ceil(n / kChunk) without forming n + kChunk - 1 (no overflow near INT64_MAX).
int64_t chunks_of(int64_t n) {
    return n / mdq_stats::kChunk + (n % mdq_stats::kChunk != 0 ? 1 : 0);
}

// Checks every argument and every launch group before anything is launched,
// so a failing call leaves `out` untouched.  Returns the total number of
// partial records (chunks) the call needs.
mdq_status validate_stats_call(const void* const* grads, const int64_t* counts, int32_t n_tensors,
                               int64_t* total_chunks) {
    using mdq_stats::kCap;
    int64_t total = 0;
    for (int b = 0; b < n_tensors; b += kCap) {
        const int cnt = n_tensors - b < kCap ? n_tensors - b : kCap;
        int64_t c = 0;
        for (int i = 0; i < cnt; ++i) {
            const int64_t n = counts[b + i];
            if (n < 0) return mdq_fail(MDQ_ERR_INVALID_ARG, "tensor %d: negative count", b + i);
            if (grads != nullptr && n > 0 && grads[b + i] == nullptr)
                return mdq_fail(MDQ_ERR_INVALID_ARG, "tensor %d: null gradient", b + i);
            c += chunks_of(n);  // <= 2^47 per tensor: no overflow across 256 tensors
            if (c > INT32_MAX)
                return mdq_fail(MDQ_ERR_TOO_LARGE, "too many elements in one call");
        }
        total += c;
        if (total > INT32_MAX) return mdq_fail(MDQ_ERR_TOO_LARGE, "too many elements in one call");
    }
    *total_chunks = total;
    return MDQ_OK;
}

}  // namespace

extern "C" {

mdq_status mdq_grad_stats_workspace_bytes(const int64_t* counts, int32_t n_tensors,
                                          int64_t* bytes) {
    mdq_clear_error();
    if (n_tensors < 0 || (n_tensors > 0 && counts == nullptr) || bytes == nullptr)
        return mdq_fail(MDQ_ERR_INVALID_ARG, "bad arguments");
    int64_t chunks = 0;
    const mdq_status st = validate_stats_call(nullptr, counts, n_tensors, &chunks);
    if (st != MDQ_OK) return st;
    *bytes = chunks * 3 * (int64_t)sizeof(double);
    return MDQ_OK;
}

mdq_status mdq_grad_stats_multi(const void* const* grads, const int64_t* counts,
                                int32_t n_tensors, int32_t grad_dtype, double* out,
                                void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
    using namespace mdq_stats;
    mdq_clear_error();
    if (n_tensors < 0 || (n_tensors > 0 && (grads == nullptr || counts == nullptr || out == nullptr)))
        return mdq_fail(MDQ_ERR_INVALID_ARG, "null argument");
    if (grad_dtype != MDQ_F32 && grad_dtype != MDQ_BF16)
        return mdq_fail(MDQ_ERR_UNSUPPORTED, "grad dtype must be MDQ_F32 or MDQ_BF16");
    int64_t chunks = 0;
    mdq_status st = validate_stats_call(grads, counts, n_tensors, &chunks);
    if (st != MDQ_OK) return st;
    const int64_t need = chunks * 3 * (int64_t)sizeof(double);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
        return mdq_fail(MDQ_ERR_INVALID_ARG, "workspace holds %lld bytes, %lld needed",
                    (long long)workspace_bytes, (long long)need);
    if (((uintptr_t)workspace & 7) != 0) return mdq_fail(MDQ_ERR_INVALID_ARG, "workspace misaligned");
    static thread_local Params P;
    int64_t chunk_base = 0;
    for (int b = 0; b < n_tensors; b += kCap) {
        const int cnt = n_tensors - b < kCap ? n_tensors - b : kCap;
        P.n = cnt;
        int64_t c = 0;
        for (int i = 0; i < cnt; ++i) {  // (validated above)
            P.g[i] = grads[b + i];
            P.count[i] = counts[b + i];
            P.chunk_begin[i] = (int32_t)c;
            c += chunks_of(counts[b + i]);
        }
        P.chunk_begin[cnt] = (int32_t)c;
        P.total_chunks = (int32_t)c;
        double* part = static_cast<double*>(workspace) + 3 * chunk_base;
        if (c > 0) {
            const int grid = c < 148 * 8 ? (int)c : 148 * 8;
            if (grad_dtype == MDQ_F32)
                chunk_sums<float><<<grid, kThreads, 0, stream>>>(P, part);
            else
                chunk_sums<__nv_bfloat16><<<grid, kThreads, 0, stream>>>(P, part);
        }
        tensor_sums<<<cnt, kThreads, 0, stream>>>(P, part, out + 4 * (int64_t)b);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return mdq_fail(MDQ_ERR_CUDA, "grad stats launch: %s", cudaGetErrorString(e));
        chunk_base += c;
    }
    return MDQ_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot allocate device memory for the workspace: a host
// program that binds the C ABI directly (cgo, JNI, ...) and owns no device
// allocator, or a training step that must not call cudaMalloc (which can
// synchronise the device) in the middle of its work.  For them the
// partial-sum records live in a fixed array in this library's device memory:
// kNoAllocRecords records of three doubles (1.5 MiB), held on every GPU that
// loads the library until the process exits.  One record covers up to
// kChunk = 65536 elements of one tensor, so a call accepts at most
// kNoAllocRecords records in total (sum over tensors of ceil(count / 65536),
// about 4.29e9 elements when tensors are large).
// ---------------------------------------------------------------------------
namespace {

constexpr int64_t kNoAllocRecords = 65536;
static __device__ __align__(256) double g_noalloc_partials[kNoAllocRecords * 3];

// Device address of g_noalloc_partials per device.  The host-side name of the
// array is only a stand-in; its device address comes from
// cudaGetSymbolAddress, looked up with that device current.  The address
// belongs to the device's current context: it is cached together with that
// context's unique id and looked up again when the id changes (for instance
// after the caller reset the device, which destroys the context).
typedef int (*CtxGetCurrentFn)(void** ctx);
typedef int (*CtxGetIdFn)(void* ctx, unsigned long long* id);

struct NoallocSlot {
    void* addr;
    unsigned long long ctx_id;
};
std::mutex g_noalloc_mu;
NoallocSlot g_noalloc_slot[64] = {};
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;
bool g_ctx_fns_looked_up = false;

// Unique id of the calling thread's current context, 0 when the driver cannot
// tell (then the cached address is trusted as is).
unsigned long long current_ctx_id() {
    if (!g_ctx_fns_looked_up) {
        g_ctx_fns_looked_up = true;
        void* f1 = nullptr;
        void* f2 = nullptr;
        cudaDriverEntryPointQueryResult q1, q2;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) == cudaSuccess &&
            cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) == cudaSuccess &&
            q1 == cudaDriverEntryPointSuccess && q2 == cudaDriverEntryPointSuccess) {
            g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
            g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f2);
        }
    }
    if (g_ctx_get_current == nullptr || g_ctx_get_id == nullptr) return 0;
    void* ctx = nullptr;
    unsigned long long id = 0;
    if (g_ctx_get_current(&ctx) != 0 || ctx == nullptr || g_ctx_get_id(ctx, &id) != 0) return 0;
    return id;
}

mdq_status noalloc_scratch(void** ptr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return mdq_fail(MDQ_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return mdq_fail(MDQ_ERR_CUDA, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    const unsigned long long id = current_ctx_id();
    NoallocSlot& slot = g_noalloc_slot[dev];
    if (slot.addr == nullptr || (id != 0 && id != slot.ctx_id)) {
        void* a = nullptr;
        e = cudaGetSymbolAddress(&a, g_noalloc_partials);
        if (e != cudaSuccess || a == nullptr)
            return mdq_fail(MDQ_ERR_CUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        slot.addr = a;
        slot.ctx_id = current_ctx_id();  // the lookup may have created the context
    }
    *ptr = slot.addr;
    return MDQ_OK;
}

}  // namespace

extern "C" mdq_status mdq_grad_stats_multi_noalloc(const void* const* grads, const int64_t* counts,
                                                   int32_t n_tensors, int32_t grad_dtype,
                                                   double* out, cudaStream_t stream) {
    mdq_clear_error();
    int64_t need = 0;
    mdq_status st = mdq_grad_stats_workspace_bytes(counts, n_tensors, &need);
    if (st != MDQ_OK) return st;
    const int64_t cap = kNoAllocRecords * 3 * (int64_t)sizeof(double);
    if (need > cap)
        return mdq_fail(MDQ_ERR_TOO_LARGE,
                        "mdq_grad_stats_multi_noalloc: %lld partial records needed, the built-in "
                        "scratch holds %lld (one per 65536 elements of each tensor)",
                        (long long)(need / (3 * (int64_t)sizeof(double))),
                        (long long)kNoAllocRecords);
    void* scratch = nullptr;
    st = noalloc_scratch(&scratch);
    if (st != MDQ_OK) return st;
    // Every record pass 2 reads is written by pass 1 of the same call, so the
    // scratch needs no clearing; calls that overlap on the GPU share it and race.
    return mdq_grad_stats_multi(grads, counts, n_tensors, grad_dtype, out, scratch, cap, stream);
}

