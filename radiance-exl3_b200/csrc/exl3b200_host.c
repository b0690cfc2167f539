/* exl3b200_host.c -- the host side of libexl3b200.so: the plugin's identity and rows, the shape, scratch and
 * layout hooks, and the launch adapters that turn a RadArgs into the kernels' argument records.
 *
 * Plain C against the plugin ABI. A launch reads everything off the operands and the parameters; it
 * allocates nothing, synchronises nothing and reads no environment (the rule of
 * kernels/exl3r4d/launch.c:1-3). It refuses, before anything is written, exactly what the reference refuses
 * (kernels/exl3ref/ref.c:64-139, 278-305; docs/OPS-exl3.md:292-301), and in addition what the device code
 * needs: the codes tables in this library's stored form (the record its layout hook declared), 16-byte
 * aligned. Routing VALUES live in device memory and are not read here; the kernels clamp every run and
 * token index instead, so malformed routing gives wrong rows, never a stray access. */
#include "exl3b200.h"
#include "exl3b200_abi.h"
#include "exl3b200_dev.h"

#include <stdlib.h>
#include <string.h>

/* The CUDA side (exl3b200_kernels.cu, exl3b200_moe.cu, exl3b200_tc.cu). */
int     exl3b_cuda_decode_what(const void* record, int64_t rows, int64_t cols, int bits, int codebook, void* out,
                               void* stream);
int     exl3b_cuda_prep(const Exl3bOp* op, void* dst, int64_t dst_pitch, void* stream);
int     exl3b_cuda_gemm_tc(const Exl3bOp* op, const void* xin, int64_t xin_pitch, int sm_count, void* stream);
int64_t exl3b_tc_smem_bytes(int bits);
int     exl3b_plan_skinny(const Exl3bOp* op, int sm_count, Exl3bPlan* p);
int     exl3b_cuda_gemm_skinny(const Exl3bOp* op, const Exl3bPlan* p, void* stream);
int     exl3b_cuda_device_info(int* sm_count, int32_t** err_word);
int     exl3b_cuda_read_error(int clear, int32_t* value);

/* The stored dtype of a codes table: the tile-stream record (plugin-private, sized by the layout hook). */
enum { EXL3B_DT_RECORD = RAD_DT_PLUGIN_BASE + 0x3B2 };
#define EXL3B_RECORD_TAG "exl3b200.record"

/* ------------------------------------------------------------------ operand checks */

/* Entry j of a table on the host side is not read (the entries may be device memory); only the stacked
 * form's base is checked for alignment. */
static int check_table(const RadTensor* t, int p, int bits, int64_t rows, int64_t cols, int64_t need) {
    int64_t pr, pc, numel = 1, acc = 1;
    exl3b_plane_extents(rows, cols, p, &pr, &pc);
    const int codes = p == EXL3B_P_CODES || p == EXL3B_P_DN_CODES;
    if (codes) {
        if (t->dtype == exl3b_codes_dtype(bits)) return RAD_E_DTYPE;   /* canonical plane: not re-laid */
        if (t->dtype != EXL3B_DT_RECORD) return RAD_E_DTYPE;
    } else if (t->dtype != RAD_F16) {
        return RAD_E_DTYPE;
    }
    if (t->rank < 2 || t->shape[0] < need) return RAD_E_SHAPE;
    for (uint32_t r = 1; r < t->rank; ++r) numel *= t->shape[r];
    if (numel != pr * pc) return RAD_E_SHAPE;
    if (codes) {
        if (t->rank != 3 || t->shape[1] != pr || t->shape[2] != pc) return RAD_E_SHAPE;
        if (t->stride[0] != 0) return RAD_E_STRIDE;                    /* a stored form is a pointer table */
        return RAD_OK;
    }
    for (int r = (int)t->rank - 1; r >= 1; --r) {
        if (t->shape[r] != 1 && t->stride[r] != acc) return RAD_E_STRIDE;
        acc *= t->shape[r];
    }
    if (t->stride[0] != 0) {
        if (t->stride[0] < numel) return RAD_E_STRIDE;
        if (!rad_ptr_aligned(t->data, 2)) return RAD_E_ALIGN;
    }
    return RAD_OK;
}

static Exl3bTab tab_of(const RadTensor* t, int64_t elem_bytes) {
    Exl3bTab x;
    x.base = t ? t->data : 0;
    x.stride_bytes = t ? t->stride[0] * elem_bytes : 0;
    return x;
}

/* gate_up / down / prep_gu (two- or four-class): the refusals, then the kernels' argument record. `y_f16`: down
 * writes f16 rows instead of bf16 (the f16-output linear; the op itself writes bf16). */
static int build_op_ex(const RadArgs* a, int op, Exl3bGeom* g, Exl3bOp* k, int y_f16) {
    const Exl3bPositions* at = exl3b_positions(op);
    if (a->n_t < at->n_opd) return RAD_E_INVAL;
    if (!rad_arg_in(a, at->x) || !rad_arg_in(a, at->sorted) || !rad_arg_in(a, at->offset) || !rad_arg_in(a, at->y))
        return RAD_E_INVAL;
    int odd = 0, odd_planes = 0;
    for (int p = EXL3B_P_CODES; p <= EXL3B_P_SVH; ++p) {
        if (at->plane[0][p] < 0) continue;
        for (int c = 0; c < (at->n_cls == 4 ? 4 : 1); ++c)
            if (!rad_arg_in(a, at->plane[c][p])) return RAD_E_INVAL;
        ++odd_planes;
        odd += rad_arg_in(a, at->plane[1][p]) != 0;
    }
    if (odd != 0 && odd != odd_planes) return RAD_E_INVAL;
    int rc = exl3b_geom_parse(a->p, a->n_p, op, odd != 0, g);
    if (rc != RAD_OK) return rc;
    if (g->op == EXL3B_GATE_UP && g->h_rot)
        for (int c = 0; c < g->n_class; ++c)
            if (!rad_arg_in(a, at->plane[c][EXL3B_P_DN_SUH])) return RAD_E_INVAL;

    const RadTensor* x = rad_arg_in(a, at->x);
    const RadTensor* y = rad_arg_in(a, at->y);
    const RadTensor* st = rad_arg_in(a, at->sorted);
    const RadTensor* off = rad_arg_in(a, at->offset);
    const int token_rows = g->gate_up && !g->a_rot;
    if (token_rows ? x->dtype != RAD_F16 && x->dtype != RAD_BF16 : x->dtype != RAD_F16) return RAD_E_DTYPE;
    if (y_f16 && g->op != EXL3B_DOWN) return RAD_E_INVAL;
    if (y->dtype != (g->op == EXL3B_DOWN && !y_f16 ? (uint32_t)RAD_BF16 : (uint32_t)RAD_F16)) return RAD_E_DTYPE;
    if (st->dtype != RAD_I32 || off->dtype != RAD_I32) return RAD_E_DTYPE;
    if (!rad_tensor_is_contiguous(st) || !rad_tensor_is_contiguous(off)) return RAD_E_STRIDE;
    if (x->rank < 2 || y->rank < 2) return RAD_E_SHAPE;
    if (x->stride[x->rank - 1] != 1 || y->stride[y->rank - 1] != 1) return RAD_E_STRIDE;
    const int64_t T = rad_tensor_rows(y), x_rows = rad_tensor_rows(x);
    if (rad_tensor_lastdim(y) != g->y_cols || rad_tensor_lastdim(x) < (g->a_rot ? 2 * g->x_cols : g->x_cols))
        return RAD_E_SHAPE;
    if (rad_tensor_numel(st) < T || rad_tensor_numel(off) < g->n_expert + 1) return RAD_E_SHAPE;
    if (!token_rows && x_rows < T) return RAD_E_SHAPE;
    for (int c = 0; c < g->n_class; ++c)
        for (int p = 0; p < EXL3B_N_P; ++p) {
            if (at->plane[c][p] < 0) continue;
            const RadTensor* t = rad_arg_in(a, at->plane[c][p]);
            if (!t || (p == EXL3B_P_DN_SUH && !g->h_rot)) continue;
            rc = check_table(t, p, g->bits, g->rows[c], g->cols[c], exl3b_class_entries(g, c));
            if (rc != RAD_OK) return rc;
        }

    memset(k, 0, sizeof *k);
    k->op = g->op == EXL3B_DOWN ? EXL3B_OP_DOWN : g->op == EXL3B_PREP_GU ? EXL3B_OP_PREP_GU : EXL3B_OP_GATE_UP;
    k->bits = g->bits;
    k->codebook = g->codebook;
    k->h_rot = g->h_rot;
    k->a_rot = g->a_rot;
    k->n_class = g->n_class;
    k->x_bf16 = x->dtype == RAD_BF16;
    k->out_f16 = y_f16 != 0;
    k->T = T;
    k->n_expert = g->n_expert;
    k->top_k = g->top_k;
    k->x_pitch = rad_tensor_row_pitch(x);
    k->x_rows = x_rows;
    k->y_pitch = rad_tensor_row_pitch(y);
    k->y_cols = g->y_cols;
    k->x_cols = g->x_cols;
    k->x = x->data;
    k->y = y->data;
    k->sorted_tok = (const int32_t*)st->data;
    k->expert_offset = (const int32_t*)off->data;
    for (int c = 0; c < EXL3B_MAX_CLASS; ++c) {
        const int cc = c < g->n_class ? c : 0;
        Exl3bClass* cl = &k->cls[c];
        cl->rows = g->rows[cc];
        cl->cols = g->cols[cc];
        const int* pl = at->plane[cc];
        cl->codes = tab_of(pl[EXL3B_P_CODES] >= 0 ? rad_arg_in(a, pl[EXL3B_P_CODES]) : 0, 0);
        cl->suh = tab_of(pl[EXL3B_P_SUH] >= 0 ? rad_arg_in(a, pl[EXL3B_P_SUH]) : 0, 2);
        cl->suh1 = tab_of(pl[EXL3B_P_SUH1] >= 0 ? rad_arg_in(a, pl[EXL3B_P_SUH1]) : 0, 2);
        cl->svh = tab_of(pl[EXL3B_P_SVH] >= 0 ? rad_arg_in(a, pl[EXL3B_P_SVH]) : 0, 2);
        cl->dn_suh = tab_of(pl[EXL3B_P_DN_SUH] >= 0 && g->h_rot ? rad_arg_in(a, pl[EXL3B_P_DN_SUH]) : 0, 2);
    }
    return RAD_OK;
}

static int build_op(const RadArgs* a, int op, Exl3bGeom* g, Exl3bOp* k) { return build_op_ex(a, op, g, k, 0); }

/* The band choice. The tensor-core path decodes each expert's weights once for up to 64 of its rows and pays its
 * input-rotation pass (the prep kernel into scratch) once per row; the decode-band path re-rotates per output block
 * and holds at most 64 rows in registers, but splits K over clusters so that a few live experts still spread over
 * the GPU. The tensor-core path is taken when the pass makes at least EXL3B_TC_MIN_UNITS of its units (64-row groups
 * of each live expert's rows x 256-row output pairs, estimated as (live experts + rows / 64) x pairs), or when the live
 * experts average at least EXL3B_TC_MIN_ROWS rows and make at least EXL3B_TC_FEW_UNITS units (fewer leave nearly every
 * SM idle: a lone expert of 16 rows 2048 -> 512 is two units), provided every class's output is a whole number of
 * 256-row unit pairs and its input rows can be read by a 16-byte-aligned tensor map;
 * otherwise the decode-band path serves the launch (the two agree within the ops' tolerance, not bit for bit:
 * their f32 accumulations run in different orders). */
#ifndef EXL3B_TC_MIN_ROWS
#define EXL3B_TC_MIN_ROWS 16
#endif
#ifndef EXL3B_TC_FEW_UNITS
#define EXL3B_TC_FEW_UNITS 8
#endif
#ifndef EXL3B_TC_MIN_UNITS
#define EXL3B_TC_MIN_UNITS 64
#endif
static int tc_band(const Exl3bOp* k) {
    if (k->op == EXL3B_OP_PREP_GU || k->T <= 0) return 0;
    const int64_t live = k->n_expert < k->T ? k->n_expert : k->T;
    if (live <= 0) return 0;
    int64_t pairs = 0;
    for (int c = 0; c < k->n_class; ++c) {
        if (k->cls[c].cols % 128) return 0;
        if (k->op == EXL3B_OP_DOWN && k->cls[c].rows % 256) return 0;
        if (k->cls[c].rows / 256 > pairs) pairs = k->cls[c].rows / 256;
    }
    const int64_t units = (live + k->T / 64) * pairs;
    if (units < EXL3B_TC_MIN_UNITS && (k->T / live < EXL3B_TC_MIN_ROWS || units < EXL3B_TC_FEW_UNITS)) return 0;
    if ((k->n_expert + 1) * 4 > 16384) return 0;
    /* the kernel's shared memory (rings by bitrate + the unit prefix) must fit a CTA */
    if (exl3b_tc_smem_bytes(k->bits) + ((k->n_expert + 1) * 4 + 15) / 16 * 16 + 16 + 4096 > 227 * 1024) return 0;
    return 1;
}

/* Scratch the tensor-core path needs: the rotated input rows when the op's input is not already rotated. */
static int64_t tc_scratch_bytes(const Exl3bOp* k) {
    if (!tc_band(k)) return 0;
    if (k->op == EXL3B_OP_GATE_UP && !k->a_rot) return (k->T * 2 * k->x_cols * 2 + 255) / 256 * 256;
    if (k->op == EXL3B_OP_DOWN && !k->h_rot) return (k->T * k->x_cols * 2 + 255) / 256 * 256;
    return 0;
}

static int run_op(Exl3bOp* k, void* scratch, int64_t scratch_bytes, void* stream) {
    int sm = 0;
    int32_t* err = 0;
    if (exl3b_cuda_device_info(&sm, &err) != 0) return RAD_E_DEVICE;
    k->err = err;
    if (k->op == EXL3B_OP_PREP_GU) return exl3b_cuda_prep(k, k->y, k->y_pitch, stream) == 0 ? RAD_OK : RAD_E_DEVICE;
    if (k->T == 0) return RAD_OK;
    if (tc_band(k)) {
        const int64_t need = tc_scratch_bytes(k);
        const void* xin = 0;
        int64_t pitch = 0;
        if (need == 0) {
            xin = k->x;
            pitch = k->x_pitch;
            if (!rad_ptr_aligned(xin, 16) || (pitch * 2) % 16) xin = 0;
        } else if (scratch && scratch_bytes >= need && rad_ptr_aligned(scratch, 256)) {
            pitch = k->op == EXL3B_OP_GATE_UP ? 2 * k->x_cols : k->x_cols;
            if (exl3b_cuda_prep(k, scratch, pitch, stream) != 0) return RAD_E_DEVICE;
            xin = scratch;
        }
        if (xin) return exl3b_cuda_gemm_tc(k, xin, pitch, sm, stream) == 0 ? RAD_OK : RAD_E_DEVICE;
    }
    Exl3bPlan plan;
    if (exl3b_plan_skinny(k, sm, &plan) != 0) return RAD_E_SHAPE;
    return exl3b_cuda_gemm_skinny(k, &plan, stream) == 0 ? RAD_OK : RAD_E_DEVICE;
}

static int launch_op(const RadArgs* a, RadStream s, int op) {
    Exl3bGeom g;
    Exl3bOp k;
    const int rc = build_op(a, op, &g, &k);
    if (rc != RAD_OK) return rc;
    return run_op(&k, a->scratch, a->scratch_bytes, s);
}

/* moe_exl3_down whose output row i is written at row_dst[i] (a device table of row addresses) instead of y + i*pitch:
 * the expert-parallel combine fused into down -- each pair's row goes straight into its source rank's memory. The
 * RadArgs are the down row's, checked the same way (the y operand still names the rows' dtype and width). */
int exl3b200_moe_down_rows(const RadArgs* a, const uint64_t* row_dst, void* stream) {
    Exl3bGeom g;
    Exl3bOp k;
    if (!a || !row_dst) return RAD_E_INVAL;
    const int rc = build_op(a, EXL3B_DOWN, &g, &k);
    if (rc != RAD_OK) return rc;
    k.row_dst = row_dst;
    return run_op(&k, a->scratch, a->scratch_bytes, stream);
}

/* moe_exl3_down with f16 output rows (config 1's single linear, [M, K] f16 -> [M, N] f16): the down row's operands,
 * checks and arithmetic, the f32 result times svh rounded once to f16 instead of bf16. */
int exl3b200_moe_down_f16(const RadArgs* a, void* stream) {
    Exl3bGeom g;
    Exl3bOp k;
    if (!a) return RAD_E_INVAL;
    const int rc = build_op_ex(a, EXL3B_DOWN, &g, &k, 1);
    if (rc != RAD_OK) return rc;
    return run_op(&k, a->scratch, a->scratch_bytes, stream);
}

/* The scratch exl3b200_moe_down_f16 uses for these arguments (the rotated input rows of the tensor-core band), 0 when
 * it needs none or the arguments are refused. The down row's own scratch hook refuses an f16 y. */
int64_t exl3b200_moe_down_f16_scratch(const RadArgs* a) {
    Exl3bGeom g;
    Exl3bOp k;
    if (!a || build_op_ex(a, EXL3B_DOWN, &g, &k, 1) != RAD_OK) return 0;
    return tc_scratch_bytes(&k);
}

/* moe_exl3_gate_up (down = 0) or moe_exl3_down (down = 1) over the live rows only: rows outside the runs are left
 * untouched instead of zeroed, so a caller may pass a capacity-sized sorted_tok whose live count is known only on the
 * device (expert_offset[n_expert]). down may also write through a row-address table (row_dst, else NULL). */
int exl3b200_moe_op_live(const RadArgs* a, int down, const uint64_t* row_dst, void* stream) {
    Exl3bGeom g;
    Exl3bOp k;
    if (!a || (row_dst && !down)) return RAD_E_INVAL;
    const int rc = build_op(a, down ? EXL3B_DOWN : EXL3B_GATE_UP, &g, &k);
    if (rc != RAD_OK) return rc;
    k.live_only = 1;
    k.row_dst = row_dst;
    return run_op(&k, a->scratch, a->scratch_bytes, stream);
}

static int64_t op_scratch(const RadArgs* a, int op) {
    Exl3bGeom g;
    Exl3bOp k;
    if (build_op(a, op, &g, &k) != RAD_OK) return 0;
    return tc_scratch_bytes(&k);
}

/* gate_up_down: its two halves, h in the launch's scratch (docs/OPS-exl3.md:177-191). */
static int64_t gd_h_bytes(const RadArgs* a, int mod4) {
    const Exl3bPositions* gd = exl3b_positions(mod4 ? EXL3B_GU_DN4 : EXL3B_GU_DN);
    const RadTensor* y = rad_arg_in(a, gd->y);
    static const char* const nq[4] = { "N", "N_1", "N_2", "N_3" };
    const int64_t N = rad_param_geti(a->p, a->n_p, "N", 0);
    int64_t W = 0;
    if (mod4) {
        for (int c = 0; c < 4; ++c) {
            const int64_t n = rad_param_geti(a->p, a->n_p, nq[c], N) / 2;
            if (n > W) W = n;
        }
    } else {
        const int64_t No = rad_param_geti(a->p, a->n_p, "N_odd", N);
        W = (N > No ? N : No) / 2;
    }
    const int64_t T = y ? rad_tensor_rows(y) : rad_param_getdim(a->p, a->n_p, "M", 0) * rad_param_geti(a->p, a->n_p, "top_k", 0);
    return T > 0 && W > 0 ? (T * W * 2 + 255) / 256 * 256 : 0;
}

/* Build the two halves' argument records; h at `h_data` (the launch's scratch, or a placeholder for sizing). */
static int gd_halves(const RadArgs* a, int mod4, void* h_data, Exl3bOp* k1, Exl3bOp* k2) {
    const Exl3bPositions* gd = exl3b_positions(mod4 ? EXL3B_GU_DN4 : EXL3B_GU_DN);
    if (a->n_t < gd->n_opd || !rad_arg_in(a, gd->y)) return RAD_E_INVAL;
    RadParam pg[16], pd[16];
    int ng = 0, nd = 0;
    exl3b_gd_params(a->p, a->n_p, mod4, pg, &ng, pd, &nd);
    const int64_t T = rad_tensor_rows(rad_arg_in(a, gd->y));
    static const char* const nq[4] = { "N", "N_1", "N_2", "N_3" };
    const int64_t N = rad_param_geti(a->p, a->n_p, "N", 0);
    int64_t W = 0;
    for (int c = 0; c < (mod4 ? 4 : 2); ++c) {
        const int64_t n = (mod4 ? rad_param_geti(a->p, a->n_p, nq[c], N)
                                : (c ? rad_param_geti(a->p, a->n_p, "N_odd", N) : N)) / 2;
        if (n > W) W = n;
    }
    if (T < 0 || W <= 0) return RAD_E_SHAPE;
    RadTensor h;
    memset(&h, 0, sizeof h);
    h.data = h_data;
    h.dtype = RAD_F16;
    h.rank = 2;
    h.shape[0] = T;
    h.shape[1] = W;
    rad_tensor_pack(&h);
    RadTensor tg[24], td[16];
    exl3b_gd_operands(a->t, &h, mod4, tg, td);
    RadArgs ag = *a, ad = *a;
    ag.t = tg;
    ag.n_t = exl3b_positions(mod4 ? EXL3B_GATE_UP4 : EXL3B_GATE_UP)->n_opd;
    ag.p = pg;
    ag.n_p = ng;
    ad.t = td;
    ad.n_t = exl3b_positions(mod4 ? EXL3B_DOWN4 : EXL3B_DOWN)->n_opd;
    ad.p = pd;
    ad.n_p = nd;
    Exl3bGeom g1, g2;
    int rc = build_op(&ag, mod4 ? EXL3B_GATE_UP4 : EXL3B_GATE_UP, &g1, k1);
    if (rc != RAD_OK) return rc;
    return build_op(&ad, mod4 ? EXL3B_DOWN4 : EXL3B_DOWN, &g2, k2);
}

static int launch_gd(const RadArgs* a, RadStream s, int mod4) {
    const Exl3bPositions* gd = exl3b_positions(mod4 ? EXL3B_GU_DN4 : EXL3B_GU_DN);
    if (a->n_t < gd->n_opd || !rad_arg_in(a, gd->y)) return RAD_E_INVAL;
    const int64_t need = gd_h_bytes(a, mod4);
    if (need <= 0) return RAD_E_SHAPE;
    if (!a->scratch || a->scratch_bytes < need) return RAD_E_SCRATCH;
    /* both halves are checked before either is launched: a refusal writes nothing */
    Exl3bOp k1, k2;
    const int rc = gd_halves(a, mod4, a->scratch, &k1, &k2);
    if (rc != RAD_OK) return rc;
    uint8_t* rest = (uint8_t*)a->scratch + need;
    const int r1 = run_op(&k1, rest, a->scratch_bytes - need, s);
    if (r1 != RAD_OK) return r1;
    return run_op(&k2, 0, 0, s);
}

static int64_t gd_scratch_of(const RadArgs* a, int mod4) {
    const int64_t h = gd_h_bytes(a, mod4);
    Exl3bOp k1, k2;
    static uint16_t placeholder[8];
    if (h <= 0 || gd_halves(a, mod4, placeholder, &k1, &k2) != RAD_OK) return h;
    return h + tc_scratch_bytes(&k1);
}

static int64_t gd_scratch(const RadArgs* a) { return gd_scratch_of(a, 0); }
static int64_t gd4_scratch(const RadArgs* a) { return gd_scratch_of(a, 1); }
static int64_t gu_scratch(const RadArgs* a) { return op_scratch(a, EXL3B_GATE_UP); }
static int64_t dn_scratch(const RadArgs* a) { return op_scratch(a, EXL3B_DOWN); }
static int64_t gu4_scratch(const RadArgs* a) { return op_scratch(a, EXL3B_GATE_UP4); }
static int64_t dn4_scratch(const RadArgs* a) { return op_scratch(a, EXL3B_DOWN4); }

static int gu_launch(const RadArgs* a, RadStream s)  { return launch_op(a, s, EXL3B_GATE_UP); }
static int dn_launch(const RadArgs* a, RadStream s)  { return launch_op(a, s, EXL3B_DOWN); }
static int pg_launch(const RadArgs* a, RadStream s)  { return launch_op(a, s, EXL3B_PREP_GU); }
static int gd_launch(const RadArgs* a, RadStream s)  { return launch_gd(a, s, 0); }
static int gu4_launch(const RadArgs* a, RadStream s) { return launch_op(a, s, EXL3B_GATE_UP4); }
static int dn4_launch(const RadArgs* a, RadStream s) { return launch_op(a, s, EXL3B_DOWN4); }
static int pg4_launch(const RadArgs* a, RadStream s) { return launch_op(a, s, EXL3B_PREP_GU4); }
static int gd4_launch(const RadArgs* a, RadStream s) { return launch_gd(a, s, 1); }

/* ------------------------------------------------------------------ the shape hook
 * Every operand described from the parameters alone, as the reference library describes it
 * (kernels/exl3ref/rows.c:16-134): the canonical planes, stacked; what the layout hook then stores is this
 * library's business. */
static void desc(RadOpdDesc* d, uint32_t dt, uint32_t rank, const int64_t* shape, uint32_t fill) {
    memset(d, 0, sizeof *d);
    d->dtype = dt;
    d->rank = rank;
    for (uint32_t r = 0; r < rank; ++r) d->shape[r] = shape[r];
    d->fill = fill;
    d->idx_const = -1;
}

static int shape_of(const RadParam* p, int n_p, int op, int operand, RadOpdDesc* out) {
    Exl3bGeom g;
    const Exl3bPositions* at = exl3b_positions(op);
    if (exl3b_geom_parse(p, n_p, op, exl3b_geom_two_classes(p, n_p), &g) != RAD_OK) return RAD_E_UNSUPPORTED;
    if (operand < 0 || operand >= at->n_opd || !out) return RAD_E_SHAPE;
    const int64_t T = g.M * g.top_k;
    RadOpdDesc v[24];
    memset(v, 0, sizeof v);
    const int64_t x_rows = g.gate_up && !g.a_rot ? g.M : T, x_cols = g.a_rot ? 2 * g.x_cols : g.x_cols;
    desc(&v[at->x], RAD_F16, 2, (int64_t[]){ x_rows, x_cols }, RAD_FILL_NORMAL);
    for (int c = 0; c < at->n_cls; ++c)
        for (int pl = 0; pl < EXL3B_N_P; ++pl) {
            const int k = at->plane[c][pl];
            if (k < 0) continue;
            if (c >= g.n_class || (pl == EXL3B_P_DN_SUH && !g.h_rot)) {
                memset(&v[k], 0, sizeof v[k]);
                v[k].idx_const = -1;
                v[k].flags = RAD_OPD_F_ABSENT;
                continue;
            }
            int64_t r, cl;
            exl3b_plane_extents(g.rows[c], g.cols[c], pl, &r, &cl);
            const int64_t ext[3] = { exl3b_class_entries(&g, c), r, cl };
            if (pl == EXL3B_P_CODES) {
                desc(&v[k], exl3b_codes_dtype(g.bits), 3, ext, RAD_FILL_INDEX);
                v[k].idx_max = (int64_t)1 << g.bits;
            } else {
                desc(&v[k], RAD_F16, 3, ext, RAD_FILL_NORMAL);
            }
        }
    desc(&v[at->sorted], RAD_I32, 1, (int64_t[]){ T }, RAD_FILL_INDEX);
    v[at->sorted].idx_max = T;
    desc(&v[at->offset], RAD_I32, 1, (int64_t[]){ g.n_expert + 1 }, RAD_FILL_INDEX);
    v[at->offset].flags = RAD_OPD_F_IDX_CU;
    desc(&v[at->y], g.op == EXL3B_DOWN ? RAD_BF16 : RAD_F16, 2, (int64_t[]){ T, g.y_cols }, RAD_FILL_NORMAL);
    if (at->ids >= 0) {
        desc(&v[at->ids], RAD_I32, 2, (int64_t[]){ g.M, g.top_k }, RAD_FILL_INDEX);
        v[at->ids].idx_max = g.n_expert;
    }
    for (int k = 0; k < at->n_opd; ++k) {
        if (v[k].flags & RAD_OPD_F_ABSENT) continue;
        for (uint32_t r = 0; r < v[k].rank; ++r)
            if (v[k].shape[r] <= 0) return RAD_E_UNSUPPORTED;
    }
    *out = v[operand];
    return RAD_OK;
}

static int gd_shape_of(const RadParam* p, int n_p, int mod4, int operand, RadOpdDesc* out) {
    const int gop = mod4 ? EXL3B_GATE_UP4 : EXL3B_GATE_UP, dop = mod4 ? EXL3B_DOWN4 : EXL3B_DOWN;
    const Exl3bPositions* gd = exl3b_positions(mod4 ? EXL3B_GU_DN4 : EXL3B_GU_DN);
    const Exl3bPositions* gu = exl3b_positions(gop);
    const Exl3bPositions* dn = exl3b_positions(dop);
    RadParam pg[16], pd[16];
    int ng = 0, nd = 0;
    exl3b_gd_params(p, n_p, mod4, pg, &ng, pd, &nd);
    if (operand == gd->x) return shape_of(pg, ng, gop, gu->x, out);
    if (operand == gd->sorted) return shape_of(pg, ng, gop, gu->sorted, out);
    if (operand == gd->offset) return shape_of(pg, ng, gop, gu->offset, out);
    if (operand == gd->y) return shape_of(pd, nd, dop, dn->y, out);
    for (int c = 0; c < gd->n_cls; ++c) {
        for (int q = EXL3B_P_CODES; q <= EXL3B_P_DN_SUH; ++q)
            if (operand == gd->plane[c][q]) return shape_of(pg, ng, gop, gu->plane[c][q], out);
        if (operand == gd->plane[c][EXL3B_P_DN_CODES]) return shape_of(pd, nd, dop, dn->plane[c][EXL3B_P_CODES], out);
        if (operand == gd->plane[c][EXL3B_P_DN_SVH]) return shape_of(pd, nd, dop, dn->plane[c][EXL3B_P_SVH], out);
    }
    return RAD_E_SHAPE;
}

static int gu_shape(const RadParam* p, int n, int o, RadOpdDesc* d)  { return shape_of(p, n, EXL3B_GATE_UP, o, d); }
static int dn_shape(const RadParam* p, int n, int o, RadOpdDesc* d)  { return shape_of(p, n, EXL3B_DOWN, o, d); }
static int pg_shape(const RadParam* p, int n, int o, RadOpdDesc* d)  { return shape_of(p, n, EXL3B_PREP_GU, o, d); }
static int gd_shape(const RadParam* p, int n, int o, RadOpdDesc* d)  { return gd_shape_of(p, n, 0, o, d); }
static int gu4_shape(const RadParam* p, int n, int o, RadOpdDesc* d) { return shape_of(p, n, EXL3B_GATE_UP4, o, d); }
static int dn4_shape(const RadParam* p, int n, int o, RadOpdDesc* d) { return shape_of(p, n, EXL3B_DOWN4, o, d); }
static int pg4_shape(const RadParam* p, int n, int o, RadOpdDesc* d) { return shape_of(p, n, EXL3B_PREP_GU4, o, d); }
static int gd4_shape(const RadParam* p, int n, int o, RadOpdDesc* d) { return gd_shape_of(p, n, 1, o, d); }

/* ------------------------------------------------------------------ the layout hooks
 * A codes table is stored as the tile-stream record (gate's record then up's for a stacked weight); every
 * other plane is read as it is (RAD_E_UNSUPPORTED). The geometry of the operand is its class's
 * (kernels/exl3r4d/layout.c:1-25 describes the same choice for the gfx1201 library). */
typedef struct LayoutWhat {
    int64_t rows, cols;   /* the plane's [rows, cols] */
    int     bits, stacked;
} LayoutWhat;

static int layout_what(int op, const RadParam* p, int n_p, int operand, const RadEncoding* enc, const int* sel,
                       const RadTensor* planes, int n_planes, LayoutWhat* w) {
    Exl3bGeom g;
    const int mod4 = (op & EXL3B_MOD4) != 0, base = exl3b_op_base(op);
    int gop = op;
    RadParam pg[16], pd[16];
    int ng = 0, nd = 0;
    const RadParam* pp = p;
    int npp = n_p, plane = -1, cls = -1, rc;
    if (base == EXL3B_PREP_GU) return RAD_E_UNSUPPORTED;
    const Exl3bPositions* at = exl3b_positions(op);
    for (int c = 0; c < at->n_cls; ++c)
        for (int q = 0; q < EXL3B_N_P; ++q)
            if (at->plane[c][q] == operand) { plane = q; cls = c; }
    if (plane != EXL3B_P_CODES && plane != EXL3B_P_DN_CODES) return RAD_E_UNSUPPORTED;
    if (base == EXL3B_GU_DN) {
        exl3b_gd_params(p, n_p, mod4, pg, &ng, pd, &nd);
        if (plane == EXL3B_P_CODES) { pp = pg; npp = ng; gop = mod4 ? EXL3B_GATE_UP4 : EXL3B_GATE_UP; }
        else { pp = pd; npp = nd; gop = mod4 ? EXL3B_DOWN4 : EXL3B_DOWN; }
    }
    rc = exl3b_geom_parse(pp, npp, gop, exl3b_geom_two_classes(pp, npp), &g);
    if (rc != RAD_OK) return rc;
    if (cls >= g.n_class) return RAD_E_SHAPE;
    int bits = -1, cb = -1, stacked = 0;
    {
        /* the encoding must be exactly the canonical exl3 one of this K and codebook */
        RadEncoding want;
        const int gate = exl3b_op_base(gop) == EXL3B_GATE_UP;
        if (!enc || exl3b_encoding_make(g.bits, g.codebook, gate, &want) != RAD_OK || !rad_enc_equal(enc, &want))
            return RAD_E_DTYPE;
        bits = g.bits;
        cb = g.codebook;
        stacked = gate;
    }
    (void)cb;
    if (!sel || *sel != 0 || !planes || n_planes != 1) return RAD_E_SHAPE;
    const RadTensor* t = &planes[0];
    if (t->dtype != exl3b_codes_dtype(bits) || t->rank != 2 || t->shape[0] != g.rows[cls] || t->shape[1] != g.cols[cls])
        return RAD_E_SHAPE;
    w->rows = g.rows[cls];
    w->cols = g.cols[cls];
    w->bits = bits;
    w->stacked = stacked;
    return RAD_OK;
}

static int do_layout(int op, const RadParam* p, int n_p, int o, const RadEncoding* e, const int* sel,
                     const RadTensor* pl, int n, RadLayout* out) {
    LayoutWhat w;
    const int rc = layout_what(op, p, n_p, o, e, sel, pl, n, &w);
    if (rc != RAD_OK) return rc;
    out->dtype = EXL3B_DT_RECORD;
    out->bytes = w.rows * w.cols * w.bits / 8;
    out->align = 256;
    out->tag = EXL3B_RECORD_TAG;
    return RAD_OK;
}

static int do_relayout(int op, const RadParam* p, int n_p, int o, const RadEncoding* e, const int* sel,
                       const RadTensor* pl, int n, void* dst, int64_t bytes) {
    LayoutWhat w;
    const int rc = layout_what(op, p, n_p, o, e, sel, pl, n, &w);
    if (rc != RAD_OK) return rc;
    if (!dst || bytes < w.rows * w.cols * w.bits / 8) return RAD_E_SHAPE;
    const int64_t rb = (w.cols * w.bits + 7) / 8;
    const uint8_t* codes = (const uint8_t*)pl[0].data;
    if (!w.stacked) return exl3b200_codes_to_record(codes, rb, w.rows, w.cols, w.bits, (uint16_t*)dst) ? RAD_E_SHAPE : RAD_OK;
    const int64_t half = w.rows / 2, half_elems = half * w.cols * w.bits / 16;
    if (exl3b200_codes_to_record(codes, rb, half, w.cols, w.bits, (uint16_t*)dst)) return RAD_E_SHAPE;
    if (exl3b200_codes_to_record(codes + half * rb, rb, half, w.cols, w.bits, (uint16_t*)dst + half_elems))
        return RAD_E_SHAPE;
    return RAD_OK;
}

static int do_unrelayout(int op, const RadParam* p, int n_p, int o, const RadEncoding* e, const int* sel,
                         const void* src, int64_t bytes, const RadTensor* pl, int n) {
    LayoutWhat w;
    const int rc = layout_what(op, p, n_p, o, e, sel, pl, n, &w);
    if (rc != RAD_OK) return rc;
    if (!src || bytes < w.rows * w.cols * w.bits / 8) return RAD_E_SHAPE;
    const int64_t rb = (w.cols * w.bits + 7) / 8;
    uint8_t* codes = (uint8_t*)pl[0].data;
    if (!w.stacked) return exl3b200_record_to_codes((const uint16_t*)src, w.rows, w.cols, w.bits, codes, rb) ? RAD_E_SHAPE : RAD_OK;
    const int64_t half = w.rows / 2, half_elems = half * w.cols * w.bits / 16;
    if (exl3b200_record_to_codes((const uint16_t*)src, half, w.cols, w.bits, codes, rb)) return RAD_E_SHAPE;
    if (exl3b200_record_to_codes((const uint16_t*)src + half_elems, half, w.cols, w.bits, codes + half * rb, rb))
        return RAD_E_SHAPE;
    return RAD_OK;
}

#define HOOKS(nm, OP)                                                                                              \
    static int nm##_layout(const RadParam* p, int n_p, int o, const RadEncoding* e, const int* sel,                \
                           const RadTensor* pl, int n, RadLayout* out) {                                           \
        return do_layout(OP, p, n_p, o, e, sel, pl, n, out);                                                       \
    }                                                                                                              \
    static int nm##_relayout(const RadParam* p, int n_p, int o, const RadEncoding* e, const int* sel,              \
                             const RadTensor* pl, int n, void* dst, int64_t b) {                                   \
        return do_relayout(OP, p, n_p, o, e, sel, pl, n, dst, b);                                                  \
    }                                                                                                              \
    static int nm##_unrelayout(const RadParam* p, int n_p, int o, const RadEncoding* e, const int* sel,            \
                               const void* src, int64_t b, const RadTensor* pl, int n) {                           \
        return do_unrelayout(OP, p, n_p, o, e, sel, src, b, pl, n);                                                \
    }
HOOKS(gu, EXL3B_GATE_UP)
HOOKS(dn, EXL3B_DOWN)
HOOKS(gd, EXL3B_GU_DN)
HOOKS(gu4, EXL3B_GATE_UP4)
HOOKS(dn4, EXL3B_DOWN4)
HOOKS(gd4, EXL3B_GU_DN4)
#undef HOOKS

/* ------------------------------------------------------------------ the rows */
#define DTYPES RAD_CIN("dtype", "exl3k2 exl3k3 exl3k4 exl3k5 exl3k6 exl3k7 exl3k8")
#define CODEBOOKS RAD_CIN("codebook", "mul1 mcg 3inst")
static const RadConstraint c_gu[] = { DTYPES, CODEBOOKS, RAD_CIN("h_rot", "0 1"), RAD_CIN("a_rot", "0 1"),
                                      RAD_CDIV("K", 128), RAD_CDIV("N", 256), RAD_CLE("n_expert", 1 << 20) };
static const RadConstraint c_dn[] = { DTYPES, CODEBOOKS, RAD_CIN("h_rot", "0 1"), RAD_CDIV("K", 128),
                                      RAD_CDIV("N", 128), RAD_CLE("n_expert", 1 << 20) };
static const RadConstraint c_pg[] = { DTYPES, RAD_CDIV("K", 128), RAD_CLE("n_expert", 1 << 20) };
static const RadConstraint c_gd[] = { DTYPES, CODEBOOKS, RAD_CDIV("K", 128), RAD_CDIV("N", 256),
                                      RAD_CLE("n_expert", 1 << 20) };
#define N_OF(a) (int)(sizeof(a) / sizeof((a)[0]))

static const RadKernelInfo k_rows[] = {
    { "exl3b200_moe_gate_up", "moe_exl3_gate_up", "moe",
      "EXL3 routed experts, gate and up, f16 h: input rotation in the kernel's prologue (a_rot 1: prep_gu's xr read "
      "as it is), trellis decode in registers into tensor-core fragments, the output rotation, svh, SiLU(gate)*up, "
      "h_rot's down rotation (sm_100a)",
      "any M; K % 128, N % 256 (each class); up to four classes in one grid",
      "exl3k2..exl3k8; mul1, mcg, 3inst; a f16 or bf16; h f16", RAD_DOMAIN_DEVICE, 10, c_gu, N_OF(c_gu),
      gu_launch, gu_shape, gu_scratch, 0, 0, gu_layout, gu_relayout, gu_unrelayout },
    { "exl3b200_moe_down", "moe_exl3_down", "moe",
      "EXL3 routed experts, down, bf16 y: input rotation (h_rot 0), trellis decode in registers into tensor-core "
      "fragments, the output rotation and svh (sm_100a)",
      "any M; K % 128, N % 128 (each class); up to four classes in one grid",
      "exl3k2..exl3k8; mul1, mcg, 3inst; h f16; y bf16", RAD_DOMAIN_DEVICE, 10, c_dn, N_OF(c_dn),
      dn_launch, dn_shape, dn_scratch, 0, 0, dn_layout, dn_relayout, dn_unrelayout },
    { "exl3b200_moe_prep_gu", "moe_exl3_prep_gu", "moe",
      "EXL3 routed experts, gate_up's input rotation as an op: every sorted row of every run, a[token] x suh and "
      "x suh.1, each 128-block Hadamard-rotated, side by side in xr (sm_100a)",
      "any M; K % 128 (each class)", "exl3k2..exl3k8; a f16 or bf16; xr f16", RAD_DOMAIN_DEVICE, 10, c_pg, N_OF(c_pg),
      pg_launch, pg_shape, 0, 0, 0, 0, 0, 0 },
    { "exl3b200_moe_gate_up_down", "moe_exl3_gate_up_down", "moe",
      "EXL3 routed experts, the decode chain as one op: gate_up (a_rot 0, h_rot 1) into the launch's scratch, then "
      "down (h_rot 1); the separate ops' bits (sm_100a)",
      "any M; K % 128, N % 256 (each class)", "exl3k2..exl3k8; mul1, mcg, 3inst; a f16 or bf16; y bf16",
      RAD_DOMAIN_DEVICE, 10, c_gd, N_OF(c_gd), gd_launch, gd_shape, gd_scratch, 0, 0, gd_layout, gd_relayout,
      gd_unrelayout },
    { "exl3b200_moe_gate_up_mod4", "moe_exl3_gate_up_mod4", "moe",
      "EXL3 routed experts, gate and up, four classes by number mod 4: the gate_up kernels (sm_100a)",
      "any M; K % 128, N % 256 (each class); four classes in one grid",
      "exl3k2..exl3k8; mul1, mcg, 3inst; a f16 or bf16; h f16", RAD_DOMAIN_DEVICE, 10, c_gu, N_OF(c_gu),
      gu4_launch, gu4_shape, gu4_scratch, 0, 0, gu4_layout, gu4_relayout, gu4_unrelayout },
    { "exl3b200_moe_down_mod4", "moe_exl3_down_mod4", "moe",
      "EXL3 routed experts, down, four classes by number mod 4: the down kernels (sm_100a)",
      "any M; K % 128, N % 128 (each class); four classes in one grid",
      "exl3k2..exl3k8; mul1, mcg, 3inst; h f16; y bf16", RAD_DOMAIN_DEVICE, 10, c_dn, N_OF(c_dn),
      dn4_launch, dn4_shape, dn4_scratch, 0, 0, dn4_layout, dn4_relayout, dn4_unrelayout },
    { "exl3b200_moe_prep_gu_mod4", "moe_exl3_prep_gu_mod4", "moe",
      "EXL3 routed experts, gate_up's input rotation as an op, four classes by number mod 4 (sm_100a)",
      "any M; K % 128 (each class)", "exl3k2..exl3k8; a f16 or bf16; xr f16", RAD_DOMAIN_DEVICE, 10, c_pg,
      N_OF(c_pg), pg4_launch, pg4_shape, 0, 0, 0, 0, 0, 0 },
    { "exl3b200_moe_gate_up_down_mod4", "moe_exl3_gate_up_down_mod4", "moe",
      "EXL3 routed experts, the decode chain as one op, four classes by number mod 4 (sm_100a)",
      "any M; K % 128, N % 256 (each class)", "exl3k2..exl3k8; mul1, mcg, 3inst; a f16 or bf16; y bf16",
      RAD_DOMAIN_DEVICE, 10, c_gd, N_OF(c_gd), gd4_launch, gd4_shape, gd4_scratch, 0, 0, gd4_layout, gd4_relayout,
      gd4_unrelayout },
};

static const RadPluginInfo k_info = {
    RAD_PLUGIN_KERNEL, "exl3b200", "0.1.0",
    "EXL3 routed-expert GEMMs (moe_exl3_gate_up, moe_exl3_down, moe_exl3_prep_gu, moe_exl3_gate_up_down, and their "
    "_mod4 forms) on NVIDIA B200: trellis decode fused into the expert GEMMs",
    "sm_100a",
};

uint32_t             rad_plugin_abi_version(void) { return RAD_ABI_VERSION; }
const RadPluginInfo* rad_plugin_info(void) { return &k_info; }
int                  rad_kernel_schema_count(void) { return exl3b_schema_count(); }
const RadOpSchema*   rad_kernel_schema_at(int i) { return exl3b_schema_at(i); }
int                  rad_kernel_count(void) { return N_OF(k_rows); }
const RadKernelInfo* rad_kernel_at(int i) { return i >= 0 && i < N_OF(k_rows) ? &k_rows[i] : 0; }
int                  rad_kernel_concurrent(int i) { return i >= 0 && i < N_OF(k_rows); }

/* ------------------------------------------------------------------ direct entry points */
int exl3b200_decode_what(const void* record, int64_t rows, int64_t cols, int bits, int codebook, void* w_hat,
                         void* stream) {
    if (!record || !w_hat || bits < 1 || bits > 8 || codebook < 0 || codebook > 2) return RAD_E_INVAL;
    if (rows <= 0 || cols <= 0 || rows % 16 || cols % 16) return RAD_E_SHAPE;
    if (!rad_ptr_aligned(record, 4) || !rad_ptr_aligned(w_hat, 4)) return RAD_E_ALIGN;
    return exl3b_cuda_decode_what(record, rows, cols, bits, codebook, w_hat, stream) == 0 ? RAD_OK : RAD_E_DEVICE;
}

int exl3b200_read_error(int clear, int32_t* value) {
    return exl3b_cuda_read_error(clear, value) == 0 ? RAD_OK : RAD_E_DEVICE;
}
