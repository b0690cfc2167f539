/* rad_types.h -- the data half of the radiance engine's kernel-plugin ABI (ABI 17), restated for this
 * repository: element types, the tensor record every operand travels in, the status codes, and the small
 * helpers a plugin uses to read them.
 *
 * The engine's own headers are not shipped with radiance-exl3; this file declares exactly the names the
 * EXL3 plugins use (kernels/exl3ref/ref.c, kernels/exl3ref/rows.c, include/exl3_abi.h,
 * include/exl3_encoding.h, tests/ref/exl3ref_run.cpp), with the meanings those files give them. It is
 * source-compatible by construction; binary compatibility with a real ABI-17 engine is not verifiable
 * without that engine. Element-type numbers are the ones the reference's harness writes
 * (tests/ref/test_exl3ref.py:45-46) and status codes the ones it reads (test_exl3ref.py:44).
 *
 * Plain C99, header-only. */
#ifndef RAD_TYPES_H
#define RAD_TYPES_H

#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <stdio.h>
#include <math.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ element types */
enum {
    RAD_DT_INVALID = 0,
    RAD_F32 = 1,
    RAD_F16 = 2,
    RAD_BF16 = 3,
    RAD_I8 = 4,
    RAD_I16 = 5,
    RAD_I64 = 6,
    RAD_U8 = 9,
    RAD_I32 = 11,
    RAD_U4 = 19,
    RAD_U2 = 20,
    RAD_U1 = 22,
    RAD_U3 = 24,
    RAD_U5 = 26,
    RAD_U6 = 28,
    RAD_U7 = 30,
    /* Types at or above this are a plugin's own stored forms; their size comes from its layout hook. */
    RAD_DT_PLUGIN_BASE = 1024
};

/* Bits one element of `dt` occupies; 0 for an unknown or plugin type. */
static inline int rad_dtype_bits(uint32_t dt) {
    switch (dt) {
    case RAD_F32: case RAD_I32: return 32;
    case RAD_F16: case RAD_BF16: case RAD_I16: return 16;
    case RAD_I64: return 64;
    case RAD_I8: case RAD_U8: return 8;
    case RAD_U1: return 1;
    case RAD_U2: return 2;
    case RAD_U3: return 3;
    case RAD_U4: return 4;
    case RAD_U5: return 5;
    case RAD_U6: return 6;
    case RAD_U7: return 7;
    default: return 0;
    }
}

/* Bytes of `n` densely packed elements of `dt` (sub-byte types round up to a whole byte). */
static inline int64_t rad_dtype_bytes(uint32_t dt, int64_t n) {
    return (n * rad_dtype_bits(dt) + 7) / 8;
}

/* ------------------------------------------------------------------ status codes */
enum {
    RAD_OK = 0,
    RAD_E_SHAPE = -1,
    RAD_E_DTYPE = -2,
    RAD_E_ALIGN = -3,
    RAD_E_STRIDE = -4,
    RAD_E_SCRATCH = -5,
    RAD_E_DEVICE = -6,
    RAD_E_NOMEM = -7,
    RAD_E_FORMAT = -8,
    RAD_E_SCHEMA = -9,
    RAD_E_UNSUPPORTED = -10,
    RAD_E_INVAL = -12
};

/* ------------------------------------------------------------------ the tensor record */
#define RAD_MAX_RANK 6

/* One operand. Extents and strides are in ELEMENTS. A weight table has stride[0] == 0 when `data` is the
 * engine's array of per-entry pointers, or a real leading stride for the stacked form. A null `data`
 * marks an absent optional operand. */
typedef struct RadTensor {
    void*    data;
    uint32_t dtype;
    uint32_t rank;
    int64_t  shape[RAD_MAX_RANK];
    int64_t  stride[RAD_MAX_RANK];
} RadTensor;

static inline int64_t rad_tensor_numel(const RadTensor* t) {
    int64_t n = 1;
    for (uint32_t r = 0; r < t->rank; ++r) n *= t->shape[r];
    return n;
}
/* Rows of a matrix view: the product of every extent but the last. */
static inline int64_t rad_tensor_rows(const RadTensor* t) {
    int64_t n = 1;
    for (uint32_t r = 0; r + 1 < t->rank; ++r) n *= t->shape[r];
    return n;
}
static inline int64_t rad_tensor_lastdim(const RadTensor* t) {
    return t->rank ? t->shape[t->rank - 1] : 1;
}
/* Elements between consecutive rows of the matrix view. */
static inline int64_t rad_tensor_row_pitch(const RadTensor* t) {
    return t->rank >= 2 ? t->stride[t->rank - 2] : rad_tensor_lastdim(t);
}
/* Dense row-major strides for the current extents. */
static inline void rad_tensor_pack(RadTensor* t) {
    int64_t s = 1;
    for (int r = (int)t->rank - 1; r >= 0; --r) {
        t->stride[r] = s;
        s *= t->shape[r];
    }
}
static inline int rad_tensor_is_contiguous(const RadTensor* t) {
    int64_t s = 1;
    for (int r = (int)t->rank - 1; r >= 0; --r) {
        if (t->shape[r] != 1 && t->stride[r] != s) return 0;
        s *= t->shape[r];
    }
    return 1;
}
static inline int rad_ptr_aligned(const void* p, int64_t align) {
    return align <= 1 || ((uintptr_t)p % (uintptr_t)align) == 0;
}

/* ------------------------------------------------------------------ narrowing (round to nearest even) */
static inline float rad_f16_to_f32(uint16_t h) {
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16;
    const int e = (h >> 10) & 0x1F;
    const uint32_t m = h & 0x3FFu;
    uint32_t u;
    float f;
    if (e == 0) {                                  /* zero or subnormal: m * 2^-24, exact in f32 */
        f = (float)m * 5.9604644775390625e-8f;
        return s ? -f : f;
    }
    if (e == 31) u = s | 0x7F800000u | (m << 13);  /* inf / nan */
    else u = s | ((uint32_t)(e + 112) << 23) | (m << 13);
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t rad_f32_to_f16(float f) {
    uint32_t u, s, a;
    memcpy(&u, &f, 4);
    s = (u >> 16) & 0x8000u;
    a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return (uint16_t)(s | 0x7E00u);          /* nan */
    if (a >= 0x477FF000u) return (uint16_t)(s | 0x7C00u);         /* >= 65520: inf */
    if (a < 0x38800000u) {                                        /* below 2^-14: subnormal or zero */
        /* value = a_f * 2^24 units of 2^-24, rounded to nearest even by the f32 add of 0.5 ulp trick */
        float af;
        memcpy(&af, &a, 4);
        {
            const double units = (double)af * 16777216.0;         /* exact: af < 2^-14 */
            double r = floor(units);
            const double rem = units - r;
            if (rem > 0.5 || (rem == 0.5 && fmod(r, 2.0) != 0.0)) r += 1.0;
            return (uint16_t)(s | (uint32_t)r);
        }
    }
    {
        const uint32_t mant = a & 0x7FFFFFu, exp = (a >> 23) - 112;
        uint32_t h = (exp << 10) | (mant >> 13);
        const uint32_t rem = mant & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;   /* carries into the exponent correctly */
        return (uint16_t)(s | h);
    }
}

static inline float rad_bf16_to_f32(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Round to nearest even; a NaN stays a quiet NaN with its sign. */
static inline uint16_t rad_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* RAD_TYPES_H */
