/*
 * mdq.h - C ABI of the B200-native fused quantized-AdamW ("MDQ") optimizer step.
 *
 * One call performs, in a single HBM pass per element: dequantise the Adam
 * moments m and v from their low-bit codes and per-block scales, apply AdamW
 * (moment update, decoupled weight decay, bias correction), write the fp32
 * parameters, and requantise m and v with fresh per-block scales.
 *
 * Semantics follow the reference kernel family
 *   ruby320/STREAM-MM2026  CUDA/stquant_kernel.cu:53-401
 * and its launcher CUDA/stquant_kernel.cu:414-465.  Codes and block scales are
 * bit-identical to that kernel (same rounding: double-precision divide and
 * round-half-away-from-zero; same CUDA libm calls; same tail-block handling).
 *
 * Plain pointers and sizes only: no exceptions cross this boundary, every entry
 * point returns an mdq_status and mdq_last_error() describes the last failure
 * of the calling thread.  All device pointers are owned by the caller; nothing
 * here allocates device memory.  Work is enqueued asynchronously on `stream`.
 */
#ifndef MDQ_H_
#define MDQ_H_

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MDQ_ABI_VERSION 3

typedef enum mdq_status {
    MDQ_OK = 0,
    MDQ_ERR_INVALID_ARG = 1,   /* null pointer, negative size, bad enum value   */
    MDQ_ERR_UNSUPPORTED = 2,   /* dtype / layout / bits combination not handled */
    MDQ_ERR_CUDA = 3,          /* a CUDA runtime call failed                     */
    MDQ_ERR_TOO_LARGE = 4      /* size exceeds a documented limit                */
} mdq_status;

/* Element types, used where the reference dispatches on tensor dtype. */
typedef enum mdq_dtype {
    MDQ_F32 = 0,
    MDQ_BF16 = 1,
    MDQ_I8 = 2,
    MDQ_U8 = 3,
    MDQ_I16 = 4,
    MDQ_U16 = 5,
    MDQ_I32 = 6,
    MDQ_U32 = 7
} mdq_dtype;

/*
 * Storage layout of the moment codes.
 *   PACKED4 : one byte per element, low nibble = q_m + 8, high nibble = q_v
 *             (CUDA/stquant_kernel.cu:52,130); exp_avg_sq unused.
 *   S8U8    : int8 m codes, uint8 v codes (CUDA/stquant_kernel.cu:148-231).
 *   S16U16  : int16 / uint16 (CUDA/stquant_kernel.cu:233-316).
 *   S32U32  : int32 / uint32 (CUDA/stquant_kernel.cu:318-401).
 *   M8V4    : int8 m codes; v codes packed two per byte (element 2i in the low
 *             nibble of byte i).  No reference counterpart: the "8-bit m and
 *             4-bit v" configuration.  m and v never depend on one another in
 *             the step, so its m codes equal an all-8-bit run's and its v codes
 *             an all-4-bit run's.
 */
typedef enum mdq_layout {
    MDQ_LAYOUT_PACKED4 = 0,
    MDQ_LAYOUT_S8U8 = 1,
    MDQ_LAYOUT_S16U16 = 2,
    MDQ_LAYOUT_S32U32 = 3,
    MDQ_LAYOUT_M8V4 = 4
} mdq_layout;

/* Parameter-update arithmetic.  Codes and scales are bit-exact in both modes. */
typedef enum mdq_p_mode {
    MDQ_P_FAST = 0,   /* hardware sqrt/reciprocal; p within a few ulp per step */
    MDQ_P_EXACT = 1   /* the reference's IEEE expression, p bit-identical      */
} mdq_p_mode;

/*
 * One tensor (or one block-aligned piece of a tensor) to update.
 * `block` is the quantisation block in elements; scale_m / scale_v / v_min
 * hold ceil(n / block) floats each and are read and rewritten in place.
 * A tensor's last block may be partial: its missing elements take part in the
 * block reductions as |m| = 0 and log v = 0, as in the reference
 * (CUDA/stquant_kernel.cu:92-97).
 */
typedef struct mdq_tensor_desc {
    float* p;              /* fp32 parameters [n], updated in place            */
    const void* grad;      /* gradient [n], grad_dtype                         */
    void* exp_avg;         /* m codes (or PACKED4 bytes)                       */
    void* exp_avg_sq;      /* v codes (NULL for PACKED4)                       */
    float* scale_m;        /* [ceil(n/block)] */
    float* scale_v;        /* [ceil(n/block)] */
    float* v_min;          /* [ceil(n/block)] */
    int64_t n;             /* elements                                         */
    int32_t step;          /* bias-correction step (already incremented)       */
    int32_t block;         /* quantisation block, 1..2048                      */
    float lr, weight_decay, eps, beta1, beta2;
    int32_t m_bits;        /* 1..32, at most the m storage width               */
    int32_t v_bits;        /* 1..32, at most the v storage width               */
    int32_t layout;        /* mdq_layout                                       */
    int32_t grad_dtype;    /* MDQ_F32 or MDQ_BF16                              */
    void* p_bf16;          /* NULL, or bf16 [n]: the updated parameters rounded
                              to bfloat16 (round to nearest even) are also
                              written here.  No reference counterpart: the
                              step writes a sharded optimizer's bf16
                              all-gather send buffer itself (ABI version 2)  */
} mdq_tensor_desc;

typedef struct mdq_step_options {
    int32_t p_mode;                    /* mdq_p_mode                               */
    unsigned long long* profile_cycles;/* NULL, or device uint64[5]: clock64 sums
                                          per phase (dequant, adam_mv,
                                          scale_reduce, quant, update_p) added by
                                          one thread per CTA; reference
                                          CUDA/stquant_kernel.cu:8-24,403-412     */
    /* Peer copies (ABI version 3; no reference counterpart): the step also
     * stores every updated parameter into n_peers other GPUs' memory, at the
     * address of its local copy plus peer_delta[k] bytes.  The local copy is
     * p_bf16 when a descriptor sets it (bf16 stores), else p (fp32 stores).
     * For buffers mapped at the same layout on every GPU (symmetric memory),
     * so that a sharded optimizer's step is also its parameter all-gather.
     * 0..7 peers; block sizes that need the one-thread-per-element kernel
     * (not a power of two, or below 8) are refused when n_peers > 0.        */
    int32_t n_peers;
    int32_t reserved;
    int64_t peer_delta[7];
    /* Gradient reduction in the step (ABI version 3; no reference
     * counterpart): with n_grad_ranks > 0 the gradient of an element is
     * grad_scale * (sum over k < n_grad_ranks, in k order, of the value at
     * the descriptor's grad address plus grad_delta[k] bytes), summed in fp32.
     * With symmetric gradient buffers and one delta per rank in rank order
     * (0 for the calling rank), this is the average over ranks that a
     * reduce-scatter would have delivered to the shard's owner.  1..8 ranks;
     * deltas multiples of 16.                                                */
    int32_t n_grad_ranks;
    float grad_scale;
    int64_t grad_delta[8];
} mdq_step_options;

/*
 * Multi-tensor step: every tensor in `descs` is updated by as few launches as
 * the mix of layouts and gradient dtypes allows (one per layout/dtype pair and
 * up to 224 tensors per launch).  Replaces the reference's one launch and two
 * host synchronisations per parameter (CUDA/stquant_opt_simple.py:242-266,
 * CUDA/stquant_opt_fused_io.py:56-79).  `opts` may be NULL (fast p mode, no
 * profiling).  Tensors with n == 0 are skipped.
 */
mdq_status mdq_adamw_step_multi(const mdq_tensor_desc* descs, int32_t n_descs,
                                const mdq_step_options* opts, cudaStream_t stream);

/*
 * Single-tensor entry point with the reference launcher's argument list:
 * replaces launch_fused_mdq_adamw (CUDA/stquant_kernel.cu:414-418), bound to
 * Python as stquant_timetest_cpp.fused_mdq_adamw (CUDA/stquant_core.cpp:3-15).
 * Because pointers carry no dtype, the dtypes the reference reads from its
 * tensors are passed explicitly, together with the element counts its dispatch
 * inspects (CUDA/stquant_kernel.cu:430-463):
 *   bits == 4, exp_avg U8 and exp_avg_sq_numel == 0  -> PACKED4
 *   exp_avg I8  / exp_avg_sq U8                      -> S8U8
 *   exp_avg I16 / exp_avg_sq U16                     -> S16U16
 *   exp_avg I32 / exp_avg_sq U32                     -> S32U32
 * anything else fails with MDQ_ERR_UNSUPPORTED, as the reference's TORCH_CHECK
 * does.  The quantisation block is min(block_size, 1024), the reference's CTA
 * size (CUDA/stquant_kernel.cu:421).  grad_dtype may be MDQ_F32 (the
 * reference's only choice) or MDQ_BF16.  The parameter update uses the
 * reference's exact IEEE expression (MDQ_P_EXACT).
 */
mdq_status mdq_fused_adamw(float* p, const void* grad, int32_t grad_dtype,
                           void* exp_avg, int32_t exp_avg_dtype, int64_t exp_avg_numel,
                           void* exp_avg_sq, int32_t exp_avg_sq_dtype, int64_t exp_avg_sq_numel,
                           float* scale_m, float* scale_v, float* v_min,
                           int64_t n,
                           float beta1, float beta2, float lr, float weight_decay, float eps,
                           int32_t step, int32_t bits, int32_t block_size,
                           unsigned long long* profile_cycles, cudaStream_t stream);

/*
 * Per-tensor gradient statistics for the bit-width policy in one fused pass:
 * out[4*i .. 4*i+3] = (sum g, sum g^2, sum |g|, count) in float64 for
 * grads[i] (counts[i] elements of grad_dtype, MDQ_F32 or MDQ_BF16).  Replaces
 * the three torch reductions per tensor of _compute_grad_stats
 * (CUDA/stquant_opt_simple.py:94-98); n_l, r_l and v_l follow from the sums.
 * `workspace` is caller-owned device memory of at least the size reported by
 * mdq_grad_stats_workspace_bytes; results are deterministic (fixed summation
 * order, no atomics).  `out` is device memory and is overwritten.
 */
mdq_status mdq_grad_stats_workspace_bytes(const int64_t* counts, int32_t n_tensors,
                                          int64_t* bytes);
mdq_status mdq_grad_stats_multi(const void* const* grads, const int64_t* counts,
                                int32_t n_tensors, int32_t grad_dtype, double* out,
                                void* workspace, int64_t workspace_bytes, cudaStream_t stream);

/*
 * mdq_grad_stats_multi without a caller workspace, for callers that cannot
 * allocate device memory (a host binding the C ABI directly with no device
 * allocator of its own, or a step that must not call cudaMalloc, which can
 * synchronise the device).  No counterpart in the reference.  The scratch is
 * a fixed 1.5 MiB array inside this library, resident on every GPU that loads
 * it until the process exits; a call may need at most 65536 partial records,
 * one per 65536 elements of each tensor (sum over tensors of
 * ceil(count / 65536)), and larger calls fail with MDQ_ERR_TOO_LARGE.  The
 * first call on each device looks up the array's device address (with that
 * device current); make that first call before any stream capture.  The
 * address is kept per device together with the id of the context it belongs
 * to, and looked up again when that context has been replaced (a device
 * reset).  Calls share the array: calls that overlap on the GPU race.
 * Allocates nothing.
 */
mdq_status mdq_grad_stats_multi_noalloc(const void* const* grads, const int64_t* counts,
                                        int32_t n_tensors, int32_t grad_dtype, double* out,
                                        cudaStream_t stream);

/*
 * The reference's pure-PyTorch quantized AdamW (baseline/mdqbock_newhook.py:
 * MDQAdamW.step, :86-175, with robust_quantize :58-83) as one fused pass per
 * quantisation block.  That optimizer keeps fp32 moments and updates the
 * parameters with fake-quantised copies of them:
 *   m = beta1 m + (1-beta1) g;  v = beta2 v + (1-beta2) g^2       (:159-160)
 *   m~ = q(m) * s_m,  s_m = (max|m| + 1e-12) / (2^(b-1) - 1),
 *        q(m) = clamp(rint(m / (s_m + 1e-12)), -2^(b-1), 2^(b-1)-1)     (:78-82)
 *   v~ = exp(q(v) * s_v + min log(v+1e-12)),  s_v = (max - min of log(v+1e-12))
 *        / (2^b - 1),  q(v) = clamp(rint((log(v+1e-12) - min) / (s_v + 1e-12)),
 *        0, 2^b - 1)                                                   (:70-76)
 *   p *= decay (if apply_decay);  p += step_size * m~ / (sqrt(v~) * inv_sqrt_bc2 + eps)
 * over blocks of `block` elements, the last one padded with zeros that take
 * part in the block's extremes (:63-66); bits >= 31 uses m and v unquantised
 * (:59).  rint is round-half-to-even, as torch.round.  The scalars are the
 * reference's Python doubles rounded to float, as torch uses them:
 * one_minus_beta1 = 1 - beta1, decay = 1 - lr * weight_decay, step_size =
 * -lr / (1 - beta1^step), inv_sqrt_bc2 = 1 / sqrt(1 - beta2^step) (torch
 * divides a tensor by a Python number by multiplying with the reciprocal,
 * computed in double and rounded to float).
 * No counterpart in the reference's CUDA code.
 */
typedef struct mdq_fq_desc {
    float* p;              /* fp32 [n], updated in place                       */
    const void* grad;      /* [n], grad_dtype (MDQ_F32 or MDQ_BF16)            */
    float* exp_avg;        /* fp32 m [n], updated in place                     */
    float* exp_avg_sq;     /* fp32 v [n], updated in place                     */
    int64_t n;
    int32_t block;         /* 1..4096                                          */
    int32_t bits;          /* 1..32 (>= 31: no quantisation)                   */
    int32_t grad_dtype;
    int32_t apply_decay;   /* weight_decay != 0                                */
    float beta1, one_minus_beta1, beta2, one_minus_beta2;
    float decay, step_size, inv_sqrt_bc2, eps;
} mdq_fq_desc;

mdq_status mdq_fakequant_adamw_multi(const mdq_fq_desc* descs, int32_t n_descs,
                                     cudaStream_t stream);

/* Message describing the calling thread's most recent failure ("" if none). */
const char* mdq_last_error(void);

/* MDQ_ABI_VERSION of the loaded library. */
int32_t mdq_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MDQ_H_ */
