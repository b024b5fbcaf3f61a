/*
 * mdq_oracle.c - CPU restatement of the reference's fused MDQ-AdamW kernels.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for tests/, __graft_entry__.smoke()
 * and the CPU-baseline leg of bench.py.  Nothing in the product links it.
 *
 * Follows ruby320/STREAM-MM2026 CUDA/stquant_kernel.cu, element for element:
 *   dequantise           :163-169 (packed4 :71-75)
 *   AdamW moments        :174-177
 *   |m|, log(v + 1e-12)  :184-185, invalid tail elements as 0 (:92-93)
 *   block max/min        :187-189 with the shared-memory tree of :27-50,
 *                        reproduced slot by slot (for a CTA size that is not a
 *                        power of two the tree folds only part of the block)
 *   scales               :192-199
 *   requantise (double)  :204-216 (packed4 :112-130)
 *   parameter update     :220-229
 * One CTA of the reference = one quantisation block of T elements.
 *
 * The reference is compiled by nvcc with FMA contraction enabled; the
 * contractions it forms (a*b + c -> fma) are written here with fmaf, and this
 * file is compiled with -ffp-contract=off so the C compiler forms no others.
 * Transcendentals come from the host libm (expf, logf, powf): CUDA's versions
 * may differ from these by an ulp, so against the GPU this oracle agrees
 * bit-for-bit only where those calls agree.  The GPU tests therefore pin the
 * CUDA kernel against the reference's own compiled kernel, and compare this
 * oracle with committed outputs of that kernel under a stated ulp tolerance.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>

enum { L_PACKED4 = 0, L_S8U8 = 1, L_S16U16 = 2, L_S32U32 = 3, L_M8V4 = 4 };

/* Code read: signed m code value and unsigned v code value of element i. */
static void load_codes(int layout, const void* mc, const void* vc, int64_t i, int* qm,
                       uint32_t* qv) {
    switch (layout) {
        case L_PACKED4: {
            const uint8_t b = ((const uint8_t*)mc)[i];
            *qm = (int)(b & 15) - 8;
            *qv = (uint32_t)(b >> 4);
            return;
        }
        case L_S8U8:
            *qm = ((const int8_t*)mc)[i];
            *qv = ((const uint8_t*)vc)[i];
            return;
        case L_S16U16:
            *qm = ((const int16_t*)mc)[i];
            *qv = ((const uint16_t*)vc)[i];
            return;
        case L_S32U32:
            *qm = ((const int32_t*)mc)[i];
            *qv = ((const uint32_t*)vc)[i];
            return;
        case L_M8V4:
            *qm = ((const int8_t*)mc)[i];
            *qv = (uint32_t)((((const uint8_t*)vc)[i >> 1] >> (4 * (i & 1))) & 15);
            return;
    }
}

static int clampi(int x, int lo, int hi) { return x < lo ? lo : (x > hi ? hi : x); }

/* Code write from the clamped double codes, with the reference's casts. */
static void store_codes(int layout, void* mc, void* vc, int64_t i, double qm, double qv) {
    switch (layout) {
        case L_PACKED4: {
            const int mu = clampi((int)qm + 8, 0, 15);
            const int vi = clampi((int)qv, 0, 15);
            ((uint8_t*)mc)[i] = (uint8_t)((vi << 4) | (mu & 15));
            return;
        }
        case L_S8U8:
            ((int8_t*)mc)[i] = (int8_t)qm;
            ((uint8_t*)vc)[i] = (uint8_t)qv;
            return;
        case L_S16U16:
            ((int16_t*)mc)[i] = (int16_t)qm;
            ((uint16_t*)vc)[i] = (uint16_t)qv;
            return;
        case L_S32U32:
            ((int32_t*)mc)[i] = (int32_t)qm;
            ((uint32_t*)vc)[i] = (uint32_t)qv;
            return;
        case L_M8V4: {
            ((int8_t*)mc)[i] = (int8_t)qm;
            uint8_t* b = (uint8_t*)vc + (i >> 1);
            const int sh = 4 * (int)(i & 1);
            const int vi = clampi((int)qv, 0, 15);
            *b = (uint8_t)((*b & ~(15 << sh)) | (vi << sh));
            return;
        }
    }
}

/* The reference's halving tree over T slots (CUDA/stquant_kernel.cu:27-50). */
static float tree_max(float* s, int T) {
    for (int h = T / 2; h > 0; h >>= 1)
        for (int t = 0; t < h; ++t) s[t] = fmaxf(s[t], s[t + h]);
    return s[0];
}
static float tree_min(float* s, int T) {
    for (int h = T / 2; h > 0; h >>= 1)
        for (int t = 0; t < h; ++t) s[t] = fminf(s[t], s[t + h]);
    return s[0];
}

typedef struct {
    float* p;
    const float* grad;
    int layout;
    void* m_codes;
    void* v_codes;
    float* scale_m;
    float* scale_v;
    float* v_min;
    int64_t n;
    int T;
    float beta1, beta2, lr, weight_decay, eps;
    int step;
    double lm, lv;
    int64_t b_begin, b_end;
} job_t;

/* Blocks [b_begin, b_end) of one tensor; each block is one reference CTA. */
static void* run_blocks(void* arg) {
    const job_t* J = (const job_t*)arg;
    const int T = J->T;
    const float omb1 = 1.0f - J->beta1, omb2 = 1.0f - J->beta2;
    const float bc1 = 1.0f - powf(J->beta1, (float)J->step);
    const float bc2 = 1.0f - powf(J->beta2, (float)J->step);
    float* mm = (float*)malloc(sizeof(float) * 5 * (size_t)T);
    if (mm == NULL) return (void*)1;
    float* vv = mm + T;
    float* ra = mm + 2 * T;
    float* rmax = mm + 3 * T;
    float* rmin = mm + 4 * T;
    for (int64_t b = J->b_begin; b < J->b_end; ++b) {
        const float sm = J->scale_m[b], sv = J->scale_v[b], vmn = J->v_min[b];
        for (int t = 0; t < T; ++t) {
            const int64_t i = b * T + t;
            const int ok = i < J->n;
            float m = 0.0f, v = 0.0f;
            if (ok) {
                int qm = 0;
                uint32_t qv = 0;
                load_codes(J->layout, J->m_codes, J->v_codes, i, &qm, &qv);
                const float g = J->grad[i];
                m = (float)qm * sm;
                v = expf(fmaf((float)qv, sv, vmn));
                m = fmaf(J->beta1, m, omb1 * g);
                v = fmaf(J->beta2, v, (omb2 * g) * g);
            }
            mm[t] = m;
            vv[t] = v;
            const float lgv = ok ? logf(v + 1e-12f) : 0.0f;
            ra[t] = ok ? fabsf(m) : 0.0f;
            rmax[t] = lgv;
            rmin[t] = lgv;
        }
        /* The trees overwrite their slots; log v is recomputed below by the
           same call, giving the same value. */
        const float max_m = tree_max(ra, T);
        const float max_lv = tree_max(rmax, T);
        const float min_lv = tree_min(rmin, T);
        const float s_sm = (max_m + 1e-12f) / (float)J->lm;
        const float s_sv = (max_lv - min_lv + 1e-12f) / (float)J->lv;
        J->scale_m[b] = s_sm;
        J->scale_v[b] = s_sv;
        J->v_min[b] = min_lv;

        for (int t = 0; t < T; ++t) {
            const int64_t i = b * T + t;
            if (i >= J->n) break;
            const float m = mm[t], v = vv[t];
            const float lgv = logf(v + 1e-12f);
            double qm = round((double)m / (double)(s_sm + 1e-12f));
            if (qm < -J->lm) qm = -J->lm;
            if (qm > J->lm - 1.0) qm = J->lm - 1.0;
            double qv = round((double)(lgv - min_lv) / (double)(s_sv + 1e-12f));
            if (qv < 0.0) qv = 0.0;
            if (qv > J->lv) qv = J->lv;
            store_codes(J->layout, J->m_codes, J->v_codes, i, qm, qv);

            const float denom = (sqrtf(v) / sqrtf(bc2)) + J->eps;
            float w = J->p[i];
            if (J->weight_decay != 0.0f) w *= fmaf(-J->lr, J->weight_decay, 1.0f);
            w = fmaf(-(J->lr / bc1), m / denom, w);
            J->p[i] = w;
        }
    }
    free(mm);
    return NULL;
}

/*
 * One step over one tensor.  grad is fp32 (a bf16 gradient is widened exactly
 * by the caller).  block is the CTA size T of the reference (it clamps the
 * requested block to 1024 before launch; the caller applies that clamp).
 * Blocks are spread over n_threads host threads (<= 1: the calling thread).
 * M8V4 needs an even block so no byte of nibbles spans two threads' blocks.
 * Returns 0, or -1 on a bad argument / failed allocation.
 */
int mdq_oracle_step(float* p, const float* grad, int layout, void* m_codes, void* v_codes,
                    float* scale_m, float* scale_v, float* v_min, int64_t n, int block,
                    float beta1, float beta2, float lr, float weight_decay, float eps,
                    int step, int m_bits, int v_bits, int n_threads) {
    if (n < 0 || block < 1 || block > 4096 || layout < 0 || layout > 4) return -1;
    if (layout == L_M8V4 && (block & 1)) return -1;
    if (n == 0) return 0;
    const int64_t nblk = (n + block - 1) / block;
    job_t base;
    base.p = p;
    base.grad = grad;
    base.layout = layout;
    base.m_codes = m_codes;
    base.v_codes = v_codes;
    base.scale_m = scale_m;
    base.scale_v = scale_v;
    base.v_min = v_min;
    base.n = n;
    base.T = block;
    base.beta1 = beta1;
    base.beta2 = beta2;
    base.lr = lr;
    base.weight_decay = weight_decay;
    base.eps = eps;
    base.step = step;
    base.lm = pow(2.0, m_bits - 1);
    base.lv = pow(2.0, v_bits) - 1.0;
    int nt = n_threads < 1 ? 1 : n_threads;
    if (nt > 256) nt = 256;
    if ((int64_t)nt > nblk) nt = (int)nblk;
    job_t jobs[256];
    pthread_t th[256];
    int rc = 0;
    for (int k = 0; k < nt; ++k) {
        jobs[k] = base;
        jobs[k].b_begin = nblk * k / nt;
        jobs[k].b_end = nblk * (k + 1) / nt;
    }
    for (int k = 1; k < nt; ++k)
        if (pthread_create(&th[k], NULL, run_blocks, &jobs[k]) != 0) return -1;
    if (run_blocks(&jobs[0]) != NULL) rc = -1;
    for (int k = 1; k < nt; ++k) {
        void* r = NULL;
        pthread_join(th[k], &r);
        if (r != NULL) rc = -1;
    }
    return rc;
}

/*
 * Per-tensor gradient statistics of the bit-width policy as partial sums:
 * out[0..3] = sum g, sum g^2, sum |g|, count (double accumulation).
 */
void mdq_oracle_grad_sums(const float* g, int64_t n, double* out) {
    double s = 0.0, s2 = 0.0, sa = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        const double x = g[i];
        s += x;
        s2 += x * x;
        sa += fabs(x);
    }
    out[0] = s;
    out[1] = s2;
    out[2] = sa;
    out[3] = (double)n;
}

#include <unistd.h>

int mdq_oracle_max_threads(void) {
    const long c = sysconf(_SC_NPROCESSORS_ONLN);
    return c < 1 ? 1 : (int)c;
}
