// Deterministic scalar math shared by the CUDA kernels and by the CPU oracle.
//
// Tile intersection must be bit-identical between the GPU kernel and its CPU
// checker. Every float operation on that path therefore goes through the helpers
// below: explicitly rounded IEEE add/mul/div/sqrt (no FMA contraction on either
// side) and a natural logarithm built only from those operations, so that gcc and
// nvcc produce the same bits.
//
// det_logf: range reduction x = m * 2^e with m in [sqrt(1/2), sqrt(2)), then
// log(m) = 2 atanh(s), s = (m - 1) / (m + 1), summed as the odd Taylor series
// 2 (s + s^3/3 + s^5/5 + s^7/7 + s^9/9 + s^11/11). |s| <= 0.1716 so the first
// omitted term is below 2^-30 relative. Accuracy is within 3 ulp of the true
// logarithm for normal positive inputs (checked against libm in the tests).
// Inputs <= 0, NaN or inf are not used on the hot path; they return NaN / -inf /
// inf like logf.
#pragma once

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define GSB_HD __host__ __device__ __forceinline__
#else
#define GSB_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define DET_ADD(a, b) __fadd_rn((a), (b))
#define DET_SUB(a, b) __fsub_rn((a), (b))
#define DET_MUL(a, b) __fmul_rn((a), (b))
#define DET_DIV(a, b) __fdiv_rn((a), (b))
#define DET_SQRT(a) __fsqrt_rn((a))
#else
#include <math.h>
#define DET_ADD(a, b) ((float)((float)(a) + (float)(b)))
#define DET_SUB(a, b) ((float)((float)(a) - (float)(b)))
#define DET_MUL(a, b) ((float)((float)(a) * (float)(b)))
#define DET_DIV(a, b) ((float)((float)(a) / (float)(b)))
#define DET_SQRT(a) sqrtf((a))
#endif

GSB_HD uint32_t det_f2u(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
#endif
}

GSB_HD float det_u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}

// Float -> int32 with truncation toward zero, NaN -> 0 and saturation at the
// int32 range: the semantics of the GPU's cvt.rzi.s32.f32 (and of a C cast in
// device code), reproduced for the host where a plain cast of NaN is undefined.
GSB_HD int det_f2i_rz(float f) {
#if defined(__CUDA_ARCH__)
    return __float2int_rz(f);
#else
    if (f != f) return 0;
    if (f >= 2147483648.0f) return 2147483647;
    if (f <= -2147483648.0f) return (int)(-2147483647 - 1);
    return (int)f;
#endif
}

// fminf/fmaxf semantics (a NaN operand yields the other operand) on both sides.
GSB_HD float det_fmin(float a, float b) {
    if (a != a) return b;
    if (b != b) return a;
    return a < b ? a : b;
}
GSB_HD float det_fmax(float a, float b) {
    if (a != a) return b;
    if (b != b) return a;
    return a > b ? a : b;
}

GSB_HD float det_logf(float x) {
    if (!(x > 0.f)) return (x == 0.f) ? det_u2f(0xff800000u) : det_u2f(0x7fc00000u);
    uint32_t u = det_f2u(x);
    if (u >= 0x7f800000u) return x; // +inf or NaN
    int e = 0;
    if (u < 0x00800000u) { // subnormal: scale by 2^23
        x = DET_MUL(x, 8388608.0f);
        u = det_f2u(x);
        e = -23;
    }
    e += (int)((u >> 23) & 0xffu) - 127;
    float m = det_u2f((u & 0x007fffffu) | 0x3f800000u); // [1, 2)
    if (m > 1.41421356f) {
        m = DET_MUL(m, 0.5f);
        e += 1;
    }
    const float s = DET_DIV(DET_SUB(m, 1.0f), DET_ADD(m, 1.0f));
    const float s2 = DET_MUL(s, s);
    // Horner form of 1 + s2/3 + s2^2/5 + s2^3/7 + s2^4/9 + s2^5/11
    float p = 0.0909090909f;                    // 1/11
    p = DET_ADD(DET_MUL(p, s2), 0.111111111f);  // 1/9
    p = DET_ADD(DET_MUL(p, s2), 0.142857143f);  // 1/7
    p = DET_ADD(DET_MUL(p, s2), 0.2f);          // 1/5
    p = DET_ADD(DET_MUL(p, s2), 0.333333333f);  // 1/3
    p = DET_ADD(DET_MUL(p, s2), 1.0f);
    const float logm = DET_MUL(DET_MUL(2.0f, s), p);
    // ln 2 split into a head exactly representable with 16 fraction bits and a tail
    const float ln2_hi = 0.693145751953125f;
    const float ln2_lo = 1.42860682030941723212e-6f;
    const float fe = (float)e;
    return DET_ADD(DET_ADD(DET_MUL(fe, ln2_hi), logm), DET_MUL(fe, ln2_lo));
}
