/* exl3b200_dev.h -- the argument records the C host side hands the CUDA side. Plain C structs of device
 * pointers and sizes, passed by value as kernel parameters; no CUDA or torch type appears here, so the
 * C files include it without the CUDA headers. */
#ifndef EXL3B200_DEV_H
#define EXL3B200_DEV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { EXL3B_MAX_CLS = 4 };
enum { EXL3B_OP_DOWN = 0, EXL3B_OP_GATE_UP = 1, EXL3B_OP_PREP_GU = 2 };

/* One plane table of one class: entry j at `base` + j * stride_bytes (the stacked form), or, with
 * stride_bytes == 0, at ((const void* const*)base)[j] (the engine's pointer table). */
typedef struct Exl3bTab {
    const void* base;
    int64_t     stride_bytes;
} Exl3bTab;

/* One class of experts: class c holds experts e with e % n_class == c, at entry e / n_class. `codes` is
 * the STORED form: the tile-stream record (gate's then up's for a stacked gate_up). */
typedef struct Exl3bClass {
    int64_t  rows, cols;
    Exl3bTab codes, suh, suh1, svh, dn_suh;
} Exl3bClass;

/* One launch of gate_up, down or prep_gu over the routing contract. */
typedef struct Exl3bOp {
    int32_t        op;                  /* EXL3B_OP_* */
    int32_t        bits, codebook, h_rot, a_rot, n_class;
    int32_t        x_bf16;              /* the input rows are bf16 (token rows only) */
    int32_t        out_f16;             /* down only: the output rows are f16 instead of bf16 */
    int64_t        T, n_expert, top_k;
    int64_t        x_pitch, x_rows;     /* elements */
    int64_t        y_pitch, y_cols;     /* elements */
    int64_t        x_cols;              /* max class cols */
    const void*    x;
    void*          y;
    const int32_t* sorted_tok;
    const int32_t* expert_offset;
    int32_t*       err;                 /* device word: set nonzero when a bounded wait gives up */
    const uint64_t* row_dst;            /* optional (down): output row i is written at row_dst[i], not y + i*pitch */
    int32_t        live_only;           /* 1: rows outside the runs are left untouched, not zeroed */
    Exl3bClass     cls[EXL3B_MAX_CLS];
} Exl3bOp;

/* Launch shape the host chose for the decode-band GEMM. */
typedef struct Exl3bPlan {
    int32_t ksplit;       /* CTAs of a cluster, each a K range of the same output block */
    int32_t mch;          /* 16-row chunks a unit holds in registers (rows a unit = 16 * mch) */
    int32_t clusters;     /* persistent clusters */
    int32_t smem_bytes;
} Exl3bPlan;

#ifdef __cplusplus
}
#endif

#endif /* EXL3B200_DEV_H */
