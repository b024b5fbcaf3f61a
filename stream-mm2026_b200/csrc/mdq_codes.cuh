// mdq_codes.cuh - moment-code storage layouts and gradient loads.
//
// Every layout exposes the same per-thread interface over 4 consecutive
// elements (vectorised) or one element (scalar):
//   load4 / load1   -> signed m code values, unsigned v code values
//   store4 / store1 <- codes as "magic" words (see below)
//   m_word / v_word    the reference's integer conversion of a code computed on
//                      the double path, as a magic word
//
// Magic words.  For |q| < 2^22 the float q + 1.5*2^23 has the bit pattern
// 0x4B400000 + q, so adding that constant to a rounded float yields the code's
// integer with no conversion instruction, and since 0x4B400000 has zero low 16
// bits the code's low byte / half-word is the word's low byte / half-word.
// Layouts whose codes need more than 22 bits (S32U32) store plain integers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "mdq.h"

namespace mdq {

constexpr int kMagicBits = 0x4B400000;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23

// Low bytes of four words packed into one word (PRMT).
__device__ __forceinline__ unsigned pack_low_bytes(unsigned a, unsigned b, unsigned c, unsigned d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// 16 * hi_word + lo_word in one integer multiply-add: since 17 * 0x4B400000
// has a zero low byte, its low byte is 16 * qhi + qlo (mod 256) for the codes
// qhi, qlo of two magic words: the packed nibble pair when both are in [0, 15].
__device__ __forceinline__ unsigned nibble_pair(int hi_word, int lo_word) {
    return (unsigned)hi_word * 16u + (unsigned)lo_word;
}

// Exact float of a small integer (|q| < 2^22) without an I2F instruction.
__device__ __forceinline__ float small_int_to_float(int q) {
    return __fsub_rn(__int_as_float(kMagicBits + q), kMagic);
}

// The four byte codes of a word as exact floats, one byte permute each: a
// byte u placed in the low byte of kMagicBits (whose low byte is zero) is the
// float 1.5 * 2^23 + u.  int8 codes are biased to u = q + 128 first (one xor
// per word) and unbiased in the subtraction.
__device__ __forceinline__ float byte_as_float_u8(unsigned w, int j) {
    return __fsub_rn(__int_as_float((int)__byte_perm(w, (unsigned)kMagicBits, 0x7650u + (unsigned)j)),
                     kMagic);
}
__device__ __forceinline__ float byte_as_float_s8(unsigned w_xor80, int j) {
    return __fsub_rn(__int_as_float((int)__byte_perm(w_xor80, (unsigned)kMagicBits, 0x7650u + (unsigned)j)),
                     kMagic + 128.0f);
}

// Pointers of the tensor a CTA is working on.
struct TensorPtrs {
    float* p;
    const void* g;
    void* m;
    void* v;
    float* sm;
    float* sv;
    float* vmin;
    __nv_bfloat16* p16;  // optional bf16 copy of the updated parameters
};

template <int LAYOUT> struct Codes;

// One byte per element: low nibble q_m + 8, high nibble q_v
// (CUDA/stquant_kernel.cu:52,71-73,130).
template <> struct Codes<MDQ_LAYOUT_PACKED4> {
    static constexpr bool kApproxLog = true;
    static constexpr bool kMagicCodes = true;
    // m words carry the nibble bias: kMagicBits + q_m + 8 (rounding adds
    // 1.5 * 2^23 + 8), so the word's low nibble is the stored nibble.
    static constexpr int kMBias = 8;
    __device__ static void load4(const TensorPtrs& t, int64_t e, int (&qm)[4], int (&qv)[4]) {
        const unsigned w = __ldcs(reinterpret_cast<const unsigned*>(static_cast<const uint8_t*>(t.m) + e));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const unsigned b = w >> (8 * j);
            qm[j] = (int)(b & 15u) - 8;
            qv[j] = (int)((b >> 4) & 15u);
        }
    }
    __device__ static void load1(const TensorPtrs& t, int64_t e, int& qm, int& qv) {
        const unsigned b = static_cast<const uint8_t*>(t.m)[e];
        qm = (int)(b & 15u) - 8;
        qv = (int)(b >> 4);
    }
    // Codes are within [-8, 7] and [0, 15] once clamped to their levels
    // (m_bits, v_bits <= 4), so the reference's nibble clamps
    // (CUDA/stquant_kernel.cu:120-128) never bind and masking suffices.
    __device__ static unsigned byte_of(int mw, int vw) {
        return (((unsigned)vw & 15u) << 4) | ((unsigned)mw & 15u);
    }
    // Byte = 16 q_v + (q_m + 8), one multiply-add of the two words, gathered
    // with byte permutes.
    __device__ static void store4(const TensorPtrs& t, int64_t e, const int (&mw)[4], const int (&vw)[4]) {
        __stcs(reinterpret_cast<unsigned*>(static_cast<uint8_t*>(t.m) + e),
               pack_low_bytes(nibble_pair(vw[0], mw[0]), nibble_pair(vw[1], mw[1]),
                              nibble_pair(vw[2], mw[2]), nibble_pair(vw[3], mw[3])));
    }
    __device__ static void store1(const TensorPtrs& t, int64_t e, int mw, int vw) {
        static_cast<uint8_t*>(t.m)[e] = (uint8_t)byte_of(mw, vw);
    }
    // (int)q as CUDA/stquant_kernel.cu:118,126, as a magic word.  A NaN code
    // (NaN or infinite gradients) leaves the reference build's nibble at 0,
    // i.e. q = -8: its integer conversion of NaN lands below the nibble clamp.
    __device__ static int m_word(double q) { return kMagicBits + kMBias + (isnan(q) ? -8 : (int)q); }
    __device__ static int v_word(double q) { return kMagicBits + (int)q; }
};

template <typename MT, typename VT, bool MAGIC> struct CodesPlain {
    static constexpr bool kMagicCodes = MAGIC;
    static constexpr int kMBias = 0;
    template <typename T>
    __device__ static void ld4(const T* src, int (&o)[4]) {
        if constexpr (sizeof(T) == 1) {
            const unsigned w = __ldcs(reinterpret_cast<const unsigned*>(src));
            const T* b = reinterpret_cast<const T*>(&w);
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] = (int)b[j];
        } else if constexpr (sizeof(T) == 2) {
            const uint2 w = __ldcs(reinterpret_cast<const uint2*>(src));
            const T* b = reinterpret_cast<const T*>(&w);
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] = (int)b[j];
        } else {
            const uint4 w = __ldcs(reinterpret_cast<const uint4*>(src));
            const T* b = reinterpret_cast<const T*>(&w);
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] = (int)b[j];
        }
    }
    template <typename T>
    __device__ static void st4(T* dst, const int (&o)[4]) {
        if constexpr (sizeof(T) == 1) {
            __stcs(reinterpret_cast<unsigned*>(dst), pack_low_bytes(o[0], o[1], o[2], o[3]));
        } else if constexpr (sizeof(T) == 2) {
            __stcs(reinterpret_cast<uint2*>(dst),
                   make_uint2(__byte_perm(o[0], o[1], 0x5410), __byte_perm(o[2], o[3], 0x5410)));
        } else {
            __stcs(reinterpret_cast<uint4*>(dst),
                   make_uint4((unsigned)o[0], (unsigned)o[1], (unsigned)o[2], (unsigned)o[3]));
        }
    }
    __device__ static void load4(const TensorPtrs& t, int64_t e, int (&qm)[4], int (&qv)[4]) {
        ld4(static_cast<const MT*>(t.m) + e, qm);
        ld4(static_cast<const VT*>(t.v) + e, qv);
    }
    __device__ static void load1(const TensorPtrs& t, int64_t e, int& qm, int& qv) {
        qm = (int)static_cast<const MT*>(t.m)[e];
        qv = (int)static_cast<const VT*>(t.v)[e];
    }
    __device__ static void store4(const TensorPtrs& t, int64_t e, const int (&mw)[4], const int (&vw)[4]) {
        st4(static_cast<MT*>(t.m) + e, mw);
        st4(static_cast<VT*>(t.v) + e, vw);
    }
    // Magic words and plain integers both truncate to the stored code.
    __device__ static void store1(const TensorPtrs& t, int64_t e, int mw, int vw) {
        static_cast<MT*>(t.m)[e] = (MT)mw;
        static_cast<VT*>(t.v)[e] = (VT)(unsigned)vw;
    }
    // The reference's conversions of a double-path code
    // (CUDA/stquant_kernel.cu:210,215 and the 16/32-bit twins).
    __device__ static int m_word(double q) { return (MAGIC ? kMagicBits : 0) + (int)(MT)q; }
    __device__ static int v_word(double q) { return (MAGIC ? kMagicBits : 0) + (int)(unsigned)(VT)q; }
};

template <> struct Codes<MDQ_LAYOUT_S8U8> : CodesPlain<int8_t, uint8_t, true> {
    static constexpr bool kApproxLog = true;
};
template <> struct Codes<MDQ_LAYOUT_S16U16> : CodesPlain<int16_t, uint16_t, true> {
    static constexpr bool kApproxLog = false;
};
template <> struct Codes<MDQ_LAYOUT_S32U32> : CodesPlain<int32_t, uint32_t, false> {
    static constexpr bool kApproxLog = false;
};

// int8 m codes + v nibbles packed two per byte (element 2i in the low nibble).
template <> struct Codes<MDQ_LAYOUT_M8V4> {
    static constexpr bool kApproxLog = true;
    static constexpr bool kMagicCodes = true;
    static constexpr int kMBias = 0;
    __device__ static void load4(const TensorPtrs& t, int64_t e, int (&qm)[4], int (&qv)[4]) {
        const unsigned w = __ldcs(reinterpret_cast<const unsigned*>(static_cast<const int8_t*>(t.m) + e));
        const unsigned vw = __ldcs(reinterpret_cast<const unsigned short*>(static_cast<const uint8_t*>(t.v) + (e >> 1)));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            qm[j] = (int)(int8_t)(uint8_t)(w >> (8 * j));
            qv[j] = (int)((vw >> (4 * j)) & 15u);
        }
    }
    __device__ static void load1(const TensorPtrs& t, int64_t e, int& qm, int& qv) {
        qm = static_cast<const int8_t*>(t.m)[e];
        qv = (int)((static_cast<const uint8_t*>(t.v)[e >> 1] >> (4 * (e & 1))) & 15u);
    }
    __device__ static void store4(const TensorPtrs& t, int64_t e, const int (&mw)[4], const int (&vw)[4]) {
        __stcs(reinterpret_cast<unsigned*>(static_cast<int8_t*>(t.m) + e),
               pack_low_bytes(mw[0], mw[1], mw[2], mw[3]));
        // v codes are within [0, 15] (4-bit levels), so pairs pack exactly.
        const unsigned nib = __byte_perm(nibble_pair(vw[1], vw[0]), nibble_pair(vw[3], vw[2]), 0x0040);
        __stcs(reinterpret_cast<unsigned short*>(static_cast<uint8_t*>(t.v) + (e >> 1)), (unsigned short)nib);
    }
    // Neighbouring elements share a byte: callers give each byte one owner.
    __device__ static void store1(const TensorPtrs& t, int64_t e, int mw, int vw) {
        static_cast<int8_t*>(t.m)[e] = (int8_t)mw;
        uint8_t* vb = static_cast<uint8_t*>(t.v) + (e >> 1);
        const unsigned sh = 4 * (unsigned)(e & 1);
        *vb = (uint8_t)((*vb & ~(15u << sh)) | (((unsigned)vw & 15u) << sh));
    }
    __device__ static int m_word(double q) { return kMagicBits + (int)(int8_t)q; }
    // A 4-bit v code, clamped into its nibble as the packed4 layout does.
    __device__ static int v_word(double q) {
        int vi = (int)q;
        vi = vi < 0 ? 0 : (vi > 15 ? 15 : vi);
        return kMagicBits + vi;
    }
};

// Gradient loads (fp32, or bf16 widened exactly).
template <typename GT> struct Grad;
template <> struct Grad<float> {
    __device__ static void load4(const void* g, int64_t e, float (&o)[4]) {
        const float4 a = __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(g) + e));
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    }
    __device__ static float load1(const void* g, int64_t e) { return static_cast<const float*>(g)[e]; }
};
template <> struct Grad<__nv_bfloat16> {
    __device__ static void load4(const void* g, int64_t e, float (&o)[4]) {
        const uint2 w = __ldcs(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(g) + e));
        o[0] = __uint_as_float(w.x << 16);
        o[1] = __uint_as_float(w.x & 0xffff0000u);
        o[2] = __uint_as_float(w.y << 16);
        o[3] = __uint_as_float(w.y & 0xffff0000u);
    }
    __device__ static float load1(const void* g, int64_t e) {
        return __bfloat162float(static_cast<const __nv_bfloat16*>(g)[e]);
    }
};

}  // namespace mdq
