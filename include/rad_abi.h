/* rad_abi.h -- the call half of the radiance engine's kernel-plugin ABI (ABI 17), restated: parameters,
 * the argument block a row's launch receives, operand schemas, selection constraints and the row record.
 *
 * Declares the names the EXL3 plugins use, with the meanings they give them:
 *   RadParam / rad_param_*        include/exl3_abi.h:700-749, 757-781; tests/ref/exl3ref_run.cpp:250-262
 *   RadArgs / rad_arg_in          kernels/exl3ref/ref.c:88-139, 235-276; exl3ref_run.cpp:401-414
 *   RadOpSchema and its specs     include/exl3_abi.h:372-627
 *   RadConstraint / RAD_C*        kernels/exl3ref/rows.c:148-157; kernels/exl3r4d/rows.c:250-318;
 *                                 exl3ref_run.cpp:150-172 (how selection evaluates one)
 *   RadOpdDesc                    kernels/exl3ref/rows.c:27-86
 *   RadKernelInfo                 kernels/exl3ref/rows.c:159-239; kernels/exl3r4d/rows.c:369-520
 * Source-compatible with those files; the real engine's binary layout is not available to check. */
#ifndef RAD_ABI_H
#define RAD_ABI_H

#include "rad_types.h"
#include "rad_encoding.h"

#ifdef __cplusplus
extern "C" {
#endif

#define RAD_ABI_VERSION 17u

/* A stream handle: the device library's cudaStream_t; ignored by a host row. */
typedef void* RadStream;

/* ------------------------------------------------------------------ parameters */
enum { RAD_P_INT = 1, RAD_P_STR = 2, RAD_P_F64 = 3 };
enum { RAD_OPTIONAL = 0, RAD_REQUIRED = 1 };
enum { RAD_PROLE_NONE = 0 };

/* One resolved parameter. An integer parameter that was declared over a range (the op's M) carries its
 * low bound in `ival` and its high bound in `ihi` (0 when it is a single value). */
typedef struct RadParam {
    const char* key;
    int32_t     kind;
    int64_t     ival;
    int64_t     ihi;
    const char* sval;
    double      dval;
} RadParam;

#define RAD_INT(k, v) { (k), RAD_P_INT, (int64_t)(v), 0, 0, 0.0 }
#define RAD_STR(k, s) { (k), RAD_P_STR, 0, 0, (s), 0.0 }

static inline const RadParam* rad_param_find(const RadParam* p, int n, const char* key) {
    for (int i = 0; p && key && i < n; ++i)
        if (p[i].key && strcmp(p[i].key, key) == 0) return &p[i];
    return 0;
}
static inline int64_t rad_param_geti(const RadParam* p, int n, const char* key, int64_t dflt) {
    const RadParam* f = rad_param_find(p, n, key);
    return f && f->kind == RAD_P_INT ? f->ival : dflt;
}
static inline const char* rad_param_gets(const RadParam* p, int n, const char* key, const char* dflt) {
    const RadParam* f = rad_param_find(p, n, key);
    return f && f->kind == RAD_P_STR ? f->sval : dflt;
}
/* A dimension parameter: a range's high bound, else its value. */
static inline int64_t rad_param_getdim(const RadParam* p, int n, const char* key, int64_t dflt) {
    const RadParam* f = rad_param_find(p, n, key);
    if (!f || f->kind != RAD_P_INT) return dflt;
    return f->ihi > f->ival ? f->ihi : f->ival;
}

/* ------------------------------------------------------------------ the launch's argument block */
typedef struct RadArgs {
    const RadTensor* t;
    int              n_t;
    const RadParam*  p;
    int              n_p;
    void*            scratch;          /* the slice the row's scratch hook asked for, device memory */
    int64_t          scratch_bytes;
    void*            instance;         /* what the row's init returned */
    int              rank, world_size;
} RadArgs;

/* Operand i when it is present (in range and with data), else null. */
static inline const RadTensor* rad_arg_in(const RadArgs* a, int i) {
    if (!a || i < 0 || i >= a->n_t || !a->t[i].data) return 0;
    return &a->t[i];
}

/* ------------------------------------------------------------------ schemas */
enum { RAD_OPD_IN = 1, RAD_OPD_OUT = 2, RAD_OPD_WTAB = 3, RAD_OPD_WEIGHT = 4 };

typedef struct RadParamSpec {
    const char* key;
    int32_t     type;       /* RAD_P_* */
    int32_t     required;   /* RAD_REQUIRED / RAD_OPTIONAL */
    int32_t     role;       /* RAD_PROLE_* */
} RadParamSpec;

typedef struct RadOperandSpec {
    const char* name;
    int32_t     role;       /* RAD_OPD_* */
    int32_t     optional;
} RadOperandSpec;

typedef struct RadOpSchema {
    const char*           op;
    const RadParamSpec*   params;
    int                   n_params;
    const RadOperandSpec* operands;
    int                   n_operands;
    const char*           doc;
} RadOpSchema;

/* ------------------------------------------------------------------ operand descriptions (shape hook) */
enum { RAD_OPD_F_ABSENT = 1, RAD_OPD_F_IDX_CU = 4 };
enum { RAD_FILL_NONE = 0, RAD_FILL_NORMAL = 1, RAD_FILL_INDEX = 2, RAD_FILL_ZERO = 3 };

typedef struct RadOpdDesc {
    uint32_t dtype;
    uint32_t rank;
    int64_t  shape[RAD_MAX_RANK];
    uint32_t flags;
    uint32_t fill;
    int64_t  idx_max;
    int64_t  idx_const;
} RadOpdDesc;

/* ------------------------------------------------------------------ selection constraints */
enum { RAD_C_IN = 1, RAD_C_EQ = 2, RAD_C_LE = 3, RAD_C_GE = 4, RAD_C_DIV = 5 };
/* Keys with this prefix name a machine fact rather than a parameter. */
#define RAD_DEVICE_FACT_PREFIX "device."

typedef struct RadConstraint {
    const char* key;
    int32_t     op;
    int64_t     ival;
    const char* sval;
} RadConstraint;

#define RAD_CIN(k, s)  { (k), RAD_C_IN, 0, (s) }
#define RAD_CEQ(k, v)  { (k), RAD_C_EQ, (int64_t)(v), 0 }
#define RAD_CLE(k, v)  { (k), RAD_C_LE, (int64_t)(v), 0 }
#define RAD_CGE(k, v)  { (k), RAD_C_GE, (int64_t)(v), 0 }
#define RAD_CDIV(k, v) { (k), RAD_C_DIV, (int64_t)(v), 0 }

/* ------------------------------------------------------------------ the row */
enum { RAD_DOMAIN_HOST = 1, RAD_DOMAIN_DEVICE = 2 };

typedef int     (*RadLaunchFn)(const RadArgs* a, RadStream s);
typedef int     (*RadOpdShapeFn)(const RadParam* p, int n_p, int operand, RadOpdDesc* out);
typedef int64_t (*RadScratchFn)(const RadArgs* a);
typedef int     (*RadInitFn)(const RadParam* p, int n_p, int rank, int world_size, void** inst);
typedef void    (*RadFiniFn)(void* inst);
typedef int     (*RadLayoutFn)(const RadParam* p, int n_p, int operand, const RadEncoding* enc,
                               const int* sel, const RadTensor* planes, int n_planes, RadLayout* out);
typedef int     (*RadRelayoutFn)(const RadParam* p, int n_p, int operand, const RadEncoding* enc,
                                 const int* sel, const RadTensor* planes, int n_planes, void* dst,
                                 int64_t dst_bytes);
typedef int     (*RadUnrelayoutFn)(const RadParam* p, int n_p, int operand, const RadEncoding* enc,
                                   const int* sel, const void* src, int64_t src_bytes,
                                   const RadTensor* planes, int n_planes);

typedef struct RadKernelInfo {
    const char*          name;
    const char*          op;
    const char*          family;
    const char*          computes;
    const char*          shape;
    const char*          dtypes;
    int32_t              domain;
    int32_t              priority;
    const RadConstraint* constraints;
    int                  n_constraints;
    RadLaunchFn          launch;
    RadOpdShapeFn        opd_shape;
    RadScratchFn         scratch;
    RadInitFn            init;
    RadFiniFn            fini;
    RadLayoutFn          layout;
    RadRelayoutFn        relayout;
    RadUnrelayoutFn      unrelayout;
} RadKernelInfo;

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* RAD_ABI_H */
