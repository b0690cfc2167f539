/* exl3b200_abi.c -- the EXL3 routed-expert op interface (include/exl3b200_abi.h): operand positions, the
 * eight schemas, the geometry parse and the fused op's two halves.
 *
 * These are interface facts that must equal the reference's for the library to be a drop-in beside it
 * (include/exl3_abi.h; the engine's loader refuses a second library whose schemas differ,
 * include/exl3_abi.h:5-9). Operand tables are written out per op; the schema documentation strings are the
 * reference's text, because the loader compares schemas field for field. */
#include "exl3b200_abi.h"

#include <stdio.h>
#include <string.h>

/* ------------------------------------------------------------------ operand positions
 * include/exl3_abi.h:313-346. Per op: x, sorted, offset, y, operand count, classes, then per class the
 * operand of codes, suh, suh1, svh, dn_suh, dn_codes, dn_svh (-1 none), then the optional ids. */
#define NOC { -1, -1, -1, -1, -1, -1, -1 }
static const Exl3bPositions k_dn = { 0, 4, 5, 9, 10, 2, { { 1, 2, -1, 3, -1, -1, -1 }, { 6, 7, -1, 8, -1, -1, -1 }, NOC, NOC }, -1 };
static const Exl3bPositions k_gu = { 0, 6, 7, 13, 14, 2, { { 1, 2, 3, 4, 5, -1, -1 }, { 8, 9, 10, 11, 12, -1, -1 }, NOC, NOC }, -1 };
static const Exl3bPositions k_pg = { 0, 3, 4, 7, 8, 2, { { -1, 1, 2, -1, -1, -1, -1 }, { -1, 5, 6, -1, -1, -1, -1 }, NOC, NOC }, -1 };
static const Exl3bPositions k_gd = { 0, 8, 9, 17, 18, 2, { { 1, 2, 3, 4, 5, 6, 7 }, { 10, 11, 12, 13, 14, 15, 16 }, NOC, NOC }, -1 };
static const Exl3bPositions k_dn4 = { 0, 4, 5, 15, 16, 4,
                                      { { 1, 2, -1, 3, -1, -1, -1 }, { 6, 7, -1, 8, -1, -1, -1 },
                                        { 9, 10, -1, 11, -1, -1, -1 }, { 12, 13, -1, 14, -1, -1, -1 } }, -1 };
static const Exl3bPositions k_gu4 = { 0, 6, 7, 23, 24, 4,
                                      { { 1, 2, 3, 4, 5, -1, -1 }, { 8, 9, 10, 11, 12, -1, -1 },
                                        { 13, 14, 15, 16, 17, -1, -1 }, { 18, 19, 20, 21, 22, -1, -1 } }, -1 };
static const Exl3bPositions k_pg4 = { 0, 3, 4, 11, 13, 4,
                                      { { -1, 1, 2, -1, -1, -1, -1 }, { -1, 5, 6, -1, -1, -1, -1 },
                                        { -1, 7, 8, -1, -1, -1, -1 }, { -1, 9, 10, -1, -1, -1, -1 } }, 12 };
static const Exl3bPositions k_gd4 = { 0, 8, 9, 31, 32, 4,
                                      { { 1, 2, 3, 4, 5, 6, 7 }, { 10, 11, 12, 13, 14, 15, 16 },
                                        { 17, 18, 19, 20, 21, 22, 23 }, { 24, 25, 26, 27, 28, 29, 30 } }, -1 };
#undef NOC

const Exl3bPositions* exl3b_positions(int op) {
    switch (op) {
    case EXL3B_GATE_UP:  return &k_gu;
    case EXL3B_PREP_GU:  return &k_pg;
    case EXL3B_GU_DN:    return &k_gd;
    case EXL3B_DOWN4:    return &k_dn4;
    case EXL3B_GATE_UP4: return &k_gu4;
    case EXL3B_PREP_GU4: return &k_pg4;
    case EXL3B_GU_DN4:   return &k_gd4;
    default:             return &k_dn;
    }
}

static const char* const k_names[8] = {
    "moe_exl3_down", "moe_exl3_gate_up", "moe_exl3_prep_gu", "moe_exl3_gate_up_down",
    "moe_exl3_down_mod4", "moe_exl3_gate_up_mod4", "moe_exl3_prep_gu_mod4", "moe_exl3_gate_up_down_mod4",
};
int exl3b_op_of(const char* name) {
    for (int i = 0; name && i < 8; ++i)
        if (!strcmp(name, k_names[i])) return i;
    return -1;
}
const char* exl3b_op_name(int op) { return op >= 0 && op < 8 ? k_names[op] : 0; }

/* ------------------------------------------------------------------ schemas (include/exl3_abi.h:366-627) */
#define PI(k) { k, RAD_P_INT, RAD_REQUIRED, RAD_PROLE_NONE }
#define PS(k) { k, RAD_P_STR, RAD_REQUIRED, RAD_PROLE_NONE }
#define PO(k) { k, RAD_P_INT, RAD_OPTIONAL, RAD_PROLE_NONE }
static const RadParamSpec p_gu[] = { PI("M"), PI("N"), PI("K"), PI("n_expert"), PI("top_k"), PS("dtype"),
                                     PS("codebook"), PO("N_odd"), PO("K_odd"), PI("h_rot"), PI("a_rot") };
static const RadParamSpec p_dn[] = { PI("M"), PI("N"), PI("K"), PI("n_expert"), PI("top_k"), PS("dtype"),
                                     PS("codebook"), PO("N_odd"), PO("K_odd"), PI("h_rot") };
static const RadParamSpec p_pg[] = { PI("M"), PI("K"), PI("n_expert"), PI("top_k"), PS("dtype"), PO("K_odd") };
static const RadParamSpec p_gd[] = { PI("M"), PI("N"), PI("K"), PI("n_expert"), PI("top_k"), PS("dtype"),
                                     PS("codebook"), PO("N_odd"), PO("K_odd") };
static const RadParamSpec p_gu4[] = { PI("M"), PI("N"), PI("K"), PI("n_expert"), PI("top_k"), PS("dtype"),
                                      PS("codebook"), PO("N_1"), PO("K_1"), PO("N_2"), PO("K_2"), PO("N_3"),
                                      PO("K_3"), PI("h_rot"), PI("a_rot") };
static const RadParamSpec p_dn4[] = { PI("M"), PI("N"), PI("K"), PI("n_expert"), PI("top_k"), PS("dtype"),
                                      PS("codebook"), PO("N_1"), PO("K_1"), PO("N_2"), PO("K_2"), PO("N_3"),
                                      PO("K_3"), PI("h_rot") };
static const RadParamSpec p_pg4[] = { PI("M"), PI("K"), PI("n_expert"), PI("top_k"), PS("dtype"), PO("K_1"),
                                      PO("K_2"), PO("K_3") };
static const RadParamSpec p_gd4[] = { PI("M"), PI("N"), PI("K"), PI("n_expert"), PI("top_k"), PS("dtype"),
                                      PS("codebook"), PO("N_1"), PO("K_1"), PO("N_2"), PO("K_2"), PO("N_3"),
                                      PO("K_3") };
#undef PI
#undef PS
#undef PO

#define IN(n) { n, RAD_OPD_IN, 0 }
#define INO(n) { n, RAD_OPD_IN, 1 }
#define OUT(n) { n, RAD_OPD_OUT, 0 }
#define WT(n) { n, RAD_OPD_WTAB, 0 }
#define WTO(n) { n, RAD_OPD_WTAB, 1 }
static const RadOperandSpec o_gu[14] = { IN("a"), WT("codes"), WT("suh"), WT("suh1"), WT("svh"), WTO("dn_suh"),
                                         IN("sorted_tok"), IN("expert_offset"), WTO("codes_odd"), WTO("suh_odd"),
                                         WTO("suh1_odd"), WTO("svh_odd"), WTO("dn_suh_odd"), OUT("h") };
static const RadOperandSpec o_dn[10] = { IN("h"), WT("codes"), WT("suh"), WT("svh"), IN("sorted_tok"),
                                         IN("expert_offset"), WTO("codes_odd"), WTO("suh_odd"), WTO("svh_odd"),
                                         OUT("y") };
static const RadOperandSpec o_gd[18] = { IN("a"), WT("codes"), WT("suh"), WT("suh1"), WT("svh"), WT("dn_suh"),
                                         WT("dn_codes"), WT("dn_svh"), IN("sorted_tok"), IN("expert_offset"),
                                         WTO("codes_odd"), WTO("suh_odd"), WTO("suh1_odd"), WTO("svh_odd"),
                                         WTO("dn_suh_odd"), WTO("dn_codes_odd"), WTO("dn_svh_odd"), OUT("y") };
static const RadOperandSpec o_pg[8] = { IN("a"), WT("suh"), WT("suh1"), IN("sorted_tok"), IN("expert_offset"),
                                        WTO("suh_odd"), WTO("suh1_odd"), OUT("xr") };
#define GUC(q) WT("codes_" q), WT("suh_" q), WT("suh1_" q), WT("svh_" q), WTO("dn_suh_" q)
static const RadOperandSpec o_gu4[24] = { IN("a"), WT("codes"), WT("suh"), WT("suh1"), WT("svh"), WTO("dn_suh"),
                                          IN("sorted_tok"), IN("expert_offset"), GUC("1"), GUC("2"), GUC("3"),
                                          OUT("h") };
#define DNC(q) WT("codes_" q), WT("suh_" q), WT("svh_" q)
static const RadOperandSpec o_dn4[16] = { IN("h"), WT("codes"), WT("suh"), WT("svh"), IN("sorted_tok"),
                                          IN("expert_offset"), DNC("1"), DNC("2"), DNC("3"), OUT("y") };
#define PGC(q) WT("suh_" q), WT("suh1_" q)
static const RadOperandSpec o_pg4[13] = { IN("a"), WT("suh"), WT("suh1"), IN("sorted_tok"), IN("expert_offset"),
                                          PGC("1"), PGC("2"), PGC("3"), OUT("xr"), INO("topk_ids") };
#define GDC(q) WT("codes_" q), WT("suh_" q), WT("suh1_" q), WT("svh_" q), WT("dn_suh_" q), WT("dn_codes_" q), \
               WT("dn_svh_" q)
static const RadOperandSpec o_gd4[32] = { IN("a"), WT("codes"), WT("suh"), WT("suh1"), WT("svh"), WT("dn_suh"),
                                          WT("dn_codes"), WT("dn_svh"), IN("sorted_tok"), IN("expert_offset"),
                                          GDC("1"), GDC("2"), GDC("3"), OUT("y") };
#undef IN
#undef INO
#undef OUT
#undef WT
#undef WTO
#undef GUC
#undef DNC
#undef PGC
#undef GDC

#define N_OF(a) (int)(sizeof(a) / sizeof((a)[0]))
static const RadOpSchema k_schemas[8] = {
    { "moe_exl3_gate_up", p_gu, N_OF(p_gu), o_gu, 14,
      "EXL3 routed experts, gate and up: per sorted row, a[sorted_tok/top_k] scaled by suh "
      "(suh.1 for up) and rotated, times W_hat, rotated back and scaled by svh, then "
      "f16(silu(gate) * up); with h_rot = 1 that then scaled by down's suh (dn_suh) and "
      "rotated, which is down's first step; with a_rot = 1 `a` is moe_exl3_prep_gu's xr and "
      "the input rotation is not redone. One weight table a plane a parity class, expert e "
      "at entry e/2; rows past expert_offset[n_expert] are zero. expert_w is not applied. "
      "docs/OPS-exl3.md." },
    { "moe_exl3_down", p_dn, N_OF(p_dn), o_dn, 10,
      "EXL3 routed experts, down: per sorted row, h[i] scaled by suh and rotated (with h_rot = "
      "1: h[i] as gate_up already rotated it), times W_hat, rotated back and scaled by svh, "
      "bf16. One weight table a plane a parity class, expert e at entry e/2; rows past "
      "expert_offset[n_expert] are zero. expert_w is not applied. docs/OPS-exl3.md." },
    { "moe_exl3_prep_gu", p_pg, N_OF(p_pg), o_pg, 8,
      "EXL3 routed experts, gate_up's input rotation as an op: per sorted row, "
      "a[sorted_tok/top_k] scaled by suh and rotated, then by suh.1 and rotated, side by side "
      "(xr, f16 [T, 2*max(K, K_odd)]) -- what moe_exl3_gate_up with a_rot = 1 reads. Rows "
      "past expert_offset[n_expert] are zero. docs/OPS-exl3.md." },
    { "moe_exl3_gate_up_down", p_gd, N_OF(p_gd), o_gd, 18,
      "EXL3 routed experts, the decode chain as one op: y = moe_exl3_down(h_rot = 1) of "
      "moe_exl3_gate_up(a_rot = 0, h_rot = 1) of a, on the same routing; dn_suh / dn_codes / dn_svh "
      "are down's planes ([K, N/2]); h and the rotated input are scratch. Rows past "
      "expert_offset[n_expert] are zero. docs/OPS-exl3.md." },
    { "moe_exl3_gate_up_mod4", p_gu4, N_OF(p_gu4), o_gu4, 24,
      "moe_exl3_gate_up over FOUR classes of experts by number mod 4 (moe_gemm_q_mod4's): class q at "
      "[N_q, K_q], expert e at entry e/4 of class e%4; otherwise moe_exl3_gate_up. docs/OPS-exl3.md." },
    { "moe_exl3_down_mod4", p_dn4, N_OF(p_dn4), o_dn4, 16,
      "moe_exl3_down over FOUR classes of experts by number mod 4 (moe_gemm_q_mod4's): class q at "
      "[N_q, K_q], expert e at entry e/4 of class e%4; otherwise moe_exl3_down. docs/OPS-exl3.md." },
    { "moe_exl3_prep_gu_mod4", p_pg4, N_OF(p_pg4), o_pg4, 13,
      "moe_exl3_prep_gu over FOUR classes of experts by number mod 4: class q's input width K_q, "
      "expert e at entry e/4 of class e%4; xr f16 [T, 2*max(K_q)]; otherwise moe_exl3_prep_gu. "
      "topk_ids (optional, i32 [M, top_k]): the router's expert of each (token, slot), the sort's input -- "
      "a speed hint only, the output does not depend on it. docs/OPS-exl3.md." },
    { "moe_exl3_gate_up_down_mod4", p_gd4, N_OF(p_gd4), o_gd4, 32,
      "moe_exl3_gate_up_down over FOUR classes of experts by number mod 4: y = moe_exl3_down_mod4(h_rot = 1) of "
      "moe_exl3_gate_up_mod4(a_rot = 0, h_rot = 1) of a; class q at [N_q, K_q], expert e at entry e/4 of class "
      "e%4; otherwise moe_exl3_gate_up_down. docs/OPS-exl3.md." },
};

int exl3b_schema_count(void) { return 8; }
const RadOpSchema* exl3b_schema_at(int i) { return i >= 0 && i < 8 ? &k_schemas[i] : 0; }

/* ------------------------------------------------------------------ encoding names */
uint32_t exl3b_codes_dtype(int bits) {
    static const uint32_t dt[9] = { RAD_DT_INVALID, RAD_U1, RAD_U2, RAD_U3, RAD_U4, RAD_U5, RAD_U6, RAD_U7, RAD_U8 };
    return bits >= 1 && bits <= 8 ? dt[bits] : (uint32_t)RAD_DT_INVALID;
}
int exl3b_bits_of_dtype(uint32_t dtype) {
    for (int k = 1; k <= 8; ++k)
        if (exl3b_codes_dtype(k) == dtype) return k;
    return -1;
}
int exl3b_gemm_bits(const char* dtype) {
    if (!dtype || strncmp(dtype, "exl3k", 5) != 0 || dtype[5] < '2' || dtype[5] > '8' || dtype[6] != 0) return -1;
    return dtype[5] - '0';
}
const char* exl3b_codebook_name(int cb) {
    return cb == EXL3B_CB_3INST ? "3inst" : cb == EXL3B_CB_MCG ? "mcg" : cb == EXL3B_CB_MUL1 ? "mul1" : 0;
}
int exl3b_codebook_from_name(const char* name) {
    for (int cb = 0; name && cb < 3; ++cb)
        if (!strcmp(name, exl3b_codebook_name(cb))) return cb;
    return -1;
}
/* The canonical encoding of a K-bit weight (include/exl3_encoding.h:84-98): scheme "exl3", transform
 * "<codebook>/h128", planes codes uK [1x1], suh f16 [0x1], svh f16 [1x0], and suh.1 f16 [0x1] when stacked. */
int exl3b_encoding_make(int bits, int codebook, int stacked, RadEncoding* out) {
    char t[RAD_ENC_STR];
    const char* cb = exl3b_codebook_name(codebook);
    const uint32_t dt = exl3b_codes_dtype(bits);
    if (!out || !cb || dt == RAD_DT_INVALID) return RAD_E_INVAL;
    rad_enc_clear(out);
    rad_enc_copy_str(out->scheme, "exl3");
    snprintf(t, sizeof t, "%s/%s", cb, "h128");
    rad_enc_copy_str(out->transform, t);
    rad_enc_add_plane(out, "codes", dt, 1, 1);
    rad_enc_add_plane(out, "suh", RAD_F16, 0, 1);
    rad_enc_add_plane(out, "svh", RAD_F16, 1, 0);
    if (stacked) rad_enc_add_plane(out, "suh.1", RAD_F16, 0, 1);
    return RAD_OK;
}

/* ------------------------------------------------------------------ geometry (include/exl3_abi.h:687-749) */
int exl3b_geom_two_classes(const RadParam* p, int n_p) {
    return rad_param_find(p, n_p, "N_odd") != 0 || rad_param_find(p, n_p, "K_odd") != 0;
}

int exl3b_geom_parse(const RadParam* p, int n_p, int op_in, int two_classes, Exl3bGeom* g) {
    static const char* const nq[4] = { "N", "N_1", "N_2", "N_3" };
    static const char* const kq[4] = { "K", "K_1", "K_2", "K_3" };
    static const char* const need_all[] = { "M", "K", "n_expert", "top_k", "dtype" };
    const int mod4 = (op_in & EXL3B_MOD4) != 0, op = exl3b_op_base(op_in);
    const int prep = op == EXL3B_PREP_GU, gd = op == EXL3B_GU_DN;
    const int gate_up = op == EXL3B_GATE_UP || prep || gd;
    memset(g, 0, sizeof *g);
    for (int i = 0; i < 5; ++i)
        if (!rad_param_find(p, n_p, need_all[i])) return RAD_E_SCHEMA;
    if (!prep) {
        if (!rad_param_find(p, n_p, "N") || !rad_param_find(p, n_p, "codebook")) return RAD_E_SCHEMA;
        if (!gd && !rad_param_find(p, n_p, "h_rot")) return RAD_E_SCHEMA;
    }
    if (op == EXL3B_GATE_UP && !rad_param_find(p, n_p, "a_rot")) return RAD_E_SCHEMA;
    const char* dt = rad_param_gets(p, n_p, "dtype", 0);
    const char* cb = rad_param_gets(p, n_p, "codebook", 0);
    if (!dt || (!prep && !cb)) return RAD_E_SCHEMA;
    const int64_t N = rad_param_geti(p, n_p, "N", 0), K = rad_param_geti(p, n_p, "K", 0);
    const int64_t No = rad_param_geti(p, n_p, "N_odd", N), Ko = rad_param_geti(p, n_p, "K_odd", K);
    g->op = op;
    g->gate_up = gate_up;
    g->M = rad_param_getdim(p, n_p, "M", 0);
    g->n_expert = rad_param_geti(p, n_p, "n_expert", 0);
    g->top_k = rad_param_geti(p, n_p, "top_k", 0);
    g->h_rot = prep ? 0 : gd ? 1 : (int)rad_param_geti(p, n_p, "h_rot", -1);
    g->a_rot = op == EXL3B_GATE_UP ? (int)rad_param_geti(p, n_p, "a_rot", -1) : 0;
    g->bits = exl3b_gemm_bits(dt);
    g->codebook = prep ? -1 : exl3b_codebook_from_name(cb);
    if (g->bits < 0 || (!prep && g->codebook < 0)) return RAD_E_DTYPE;
    if ((g->h_rot != 0 && g->h_rot != 1) || (g->a_rot != 0 && g->a_rot != 1)) return RAD_E_INVAL;
    if (g->M < 1 || g->n_expert < 1 || g->top_k < 1) return RAD_E_SHAPE;
    if (!mod4 && !two_classes && ((!prep && No != N) || Ko != K)) return RAD_E_SHAPE;
    g->n_class = mod4 ? 4 : two_classes ? 2 : 1;
    for (int c = 0; c < EXL3B_MAX_CLASS; ++c) {
        const int has = mod4 || c == 1;   /* two-class ops: class 1 is the odd class; 2 and 3 repeat class 0 */
        g->rows[c] = prep ? 0 : !has ? N : mod4 ? rad_param_geti(p, n_p, nq[c], N) : No;
        g->cols[c] = !has ? K : mod4 ? rad_param_geti(p, n_p, kq[c], K) : Ko;
    }
    const int64_t rows_mult = gate_up ? 256 : 128;
    g->x_cols = g->y_cols = 0;
    for (int c = 0; c < EXL3B_MAX_CLASS; ++c) {
        if (g->cols[c] <= 0 || g->cols[c] % 128 || (!prep && (g->rows[c] <= 0 || g->rows[c] % rows_mult)))
            return RAD_E_SHAPE;
        if (g->cols[c] > g->x_cols) g->x_cols = g->cols[c];
        if (g->rows[c] > g->y_cols) g->y_cols = g->rows[c];
    }
    g->y_cols = prep ? 2 * g->x_cols : gd ? g->x_cols : g->y_cols / (gate_up ? 2 : 1);
    return RAD_OK;
}

void exl3b_plane_extents(int64_t rows, int64_t cols, int p, int64_t* r, int64_t* c) {
    if (p == EXL3B_P_DN_CODES || p == EXL3B_P_DN_SVH) {
        *r = cols;
        *c = p == EXL3B_P_DN_SVH ? 1 : rows / 2;
        return;
    }
    *r = (p == EXL3B_P_SUH || p == EXL3B_P_SUH1 || p == EXL3B_P_DN_SUH) ? 1 : rows;
    *c = p == EXL3B_P_SVH ? 1 : p == EXL3B_P_DN_SUH ? rows / 2 : cols;
}

/* ------------------------------------------------------------------ gate_up_down as its halves */
void exl3b_gd_params(const RadParam* p, int n_p, int mod4, RadParam* pg, int* n_pg, RadParam* pd, int* n_pd) {
    static const char* const nq[4] = { "N", "N_1", "N_2", "N_3" };
    static const char* const kq[4] = { "K", "K_1", "K_2", "K_3" };
    const RadParam h1 = RAD_INT("h_rot", 1), a0 = RAD_INT("a_rot", 0);
    const int64_t N = rad_param_geti(p, n_p, "N", 0), K = rad_param_geti(p, n_p, "K", 0);
    const int max_g = mod4 ? 13 : 9, max_d = mod4 ? 5 : 6;
    int ng = 0, nd = 0;
    for (int i = 0; i < n_p; ++i) {
        const char* k = p[i].key;
        if (!strcmp(k, "h_rot") || !strcmp(k, "a_rot")) continue;
        if (ng < max_g) pg[ng++] = p[i];
        int shape = 0;
        if (mod4) {
            for (int c = 0; c < 4; ++c) shape |= !strcmp(k, nq[c]) || !strcmp(k, kq[c]);
        } else {
            shape = !strcmp(k, "N") || !strcmp(k, "K") || !strcmp(k, "N_odd") || !strcmp(k, "K_odd");
        }
        if (!shape && nd < max_d) pd[nd++] = p[i];   /* M, n_expert, top_k, dtype, codebook */
    }
    pg[ng++] = h1;
    pg[ng++] = a0;
    if (mod4) {
        for (int c = 0; c < 4; ++c) {
            RadParam a = RAD_INT(nq[c], rad_param_geti(p, n_p, kq[c], K));
            RadParam b = RAD_INT(kq[c], rad_param_geti(p, n_p, nq[c], N) / 2);
            pd[nd++] = a;
            pd[nd++] = b;
        }
    } else {
        const int64_t No = rad_param_geti(p, n_p, "N_odd", N), Ko = rad_param_geti(p, n_p, "K_odd", K);
        RadParam a = RAD_INT("N", K), b = RAD_INT("K", N / 2);
        pd[nd++] = a;
        pd[nd++] = b;
        if (exl3b_geom_two_classes(p, n_p)) {
            RadParam c = RAD_INT("N_odd", Ko), d = RAD_INT("K_odd", No / 2);
            pd[nd++] = c;
            pd[nd++] = d;
        }
    }
    pd[nd++] = h1;
    *n_pg = ng;
    *n_pd = nd;
}

void exl3b_gd_operands(const RadTensor* t, const RadTensor* h, int mod4, RadTensor* tg, RadTensor* td) {
    const Exl3bPositions* gd = exl3b_positions(mod4 ? EXL3B_GU_DN4 : EXL3B_GU_DN);
    const Exl3bPositions* gu = exl3b_positions(mod4 ? EXL3B_GATE_UP4 : EXL3B_GATE_UP);
    const Exl3bPositions* dn = exl3b_positions(mod4 ? EXL3B_DOWN4 : EXL3B_DOWN);
    memset(tg, 0, (size_t)gu->n_opd * sizeof *tg);
    memset(td, 0, (size_t)dn->n_opd * sizeof *td);
    for (int c = 0; c < gd->n_cls; ++c) {
        for (int q = EXL3B_P_CODES; q <= EXL3B_P_DN_SUH; ++q)
            if (gu->plane[c][q] >= 0) tg[gu->plane[c][q]] = t[gd->plane[c][q]];
        td[dn->plane[c][EXL3B_P_CODES]] = t[gd->plane[c][EXL3B_P_DN_CODES]];
        td[dn->plane[c][EXL3B_P_SUH]] = t[gd->plane[c][EXL3B_P_DN_SUH]];
        td[dn->plane[c][EXL3B_P_SVH]] = t[gd->plane[c][EXL3B_P_DN_SVH]];
    }
    tg[gu->x] = t[gd->x];
    tg[gu->sorted] = td[dn->sorted] = t[gd->sorted];
    tg[gu->offset] = td[dn->offset] = t[gd->offset];
    tg[gu->y] = td[dn->x] = *h;
    td[dn->y] = t[gd->y];
}
