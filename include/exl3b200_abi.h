/* exl3b200_abi.h -- the EXL3 routed-expert op interface as this library implements it: the eight op
 * schemas, where each operand sits, how the parameters parse into a geometry, and the fused op read as its
 * two halves. The interface is the reference's (include/exl3_abi.h, EXL3_IFACE_VERSION 7): the same op
 * names, parameter keys, operand names and positions, refusal codes and geometry rules, so that this
 * library's rows and the reference library's rows are interchangeable behind the radiance plugin ABI.
 * The code is this repository's own; each declaration cites the reference line it matches.
 *
 * Plain C; the definitions are in radiance-exl3_b200/csrc/exl3b200_abi.c. */
#ifndef EXL3B200_ABI_H
#define EXL3B200_ABI_H

#include "rad_abi.h"
#include "rad_plugin.h"
#include "rad_encoding.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The interface version these rows implement (include/exl3_abi.h:73). */
#define EXL3B_IFACE_VERSION 7

/* Ops (include/exl3_abi.h:292-296): a four-class form is its op | EXL3B_MOD4. */
enum {
    EXL3B_DOWN = 0, EXL3B_GATE_UP = 1, EXL3B_PREP_GU = 2, EXL3B_GU_DN = 3, EXL3B_MOD4 = 4,
    EXL3B_DOWN4 = 4, EXL3B_GATE_UP4 = 5, EXL3B_PREP_GU4 = 6, EXL3B_GU_DN4 = 7
};
static inline int exl3b_op_base(int op) { return op & ~EXL3B_MOD4; }

/* Planes of a class (include/exl3_abi.h:303-305). */
enum {
    EXL3B_P_CODES = 0, EXL3B_P_SUH = 1, EXL3B_P_SUH1 = 2, EXL3B_P_SVH = 3, EXL3B_P_DN_SUH = 4,
    EXL3B_P_DN_CODES = 5, EXL3B_P_DN_SVH = 6, EXL3B_N_P = 7
};
enum { EXL3B_MAX_CLASS = 4 };

/* Codebooks, numbered as exllamav3 numbers them (common/exl3_decode.h:68). */
enum { EXL3B_CB_3INST = 0, EXL3B_CB_MCG = 1, EXL3B_CB_MUL1 = 2 };

/* Operand positions of an op (include/exl3_abi.h:307-346): x, sorted, offset, y, operand count, class
 * count; plane[c][p] the operand of class c's table of plane p (-1: the op has no such table); ids the
 * optional router ids (prep_gu_mod4 only, else -1). */
typedef struct Exl3bPositions {
    int x, sorted, offset, y, n_opd, n_cls;
    int plane[EXL3B_MAX_CLASS][EXL3B_N_P];
    int ids;
} Exl3bPositions;

const Exl3bPositions* exl3b_positions(int op);
/* The op of a name ("moe_exl3_gate_up", ...), or -1 (include/exl3_abi.h:348-364). */
int         exl3b_op_of(const char* name);
const char* exl3b_op_name(int op);

/* The eight schemas in the reference's order (include/exl3_abi.h:366-627). */
int                exl3b_schema_count(void);
const RadOpSchema* exl3b_schema_at(int i);

/* Encoding names (include/exl3_encoding.h:45-80; common/exl3_decode.h:78-95). */
uint32_t    exl3b_codes_dtype(int bits);            /* RAD_U1..RAD_U8, RAD_DT_INVALID outside 1..8 */
int         exl3b_bits_of_dtype(uint32_t dtype);
int         exl3b_gemm_bits(const char* dtype);     /* "exl3k2".."exl3k8" -> 2..8, else -1 */
const char* exl3b_codebook_name(int cb);
int         exl3b_codebook_from_name(const char* name);
int         exl3b_encoding_make(int bits, int codebook, int stacked, RadEncoding* out);

/* The parsed geometry (include/exl3_abi.h:672-685). */
typedef struct Exl3bGeom {
    int     op;              /* the two-class op (a _mod4 op's base) */
    int     gate_up;         /* gate_up, prep_gu and gate_up_down: the stacked weight */
    int64_t M, n_expert, top_k;
    int     bits, codebook;
    int     n_class;
    int     h_rot, a_rot;
    int64_t rows[EXL3B_MAX_CLASS], cols[EXL3B_MAX_CLASS];
    int64_t x_cols, y_cols;
} Exl3bGeom;

int exl3b_geom_two_classes(const RadParam* p, int n_p);
/* RAD_OK or the reference's refusal (include/exl3_abi.h:693-749). */
int exl3b_geom_parse(const RadParam* p, int n_p, int op, int two_classes, Exl3bGeom* g);

static inline int     exl3b_class_of(const Exl3bGeom* g, int64_t e) { return (int)(e % g->n_class); }
static inline int64_t exl3b_entry_of(const Exl3bGeom* g, int64_t e) { return e / g->n_class; }
static inline int64_t exl3b_class_entries(const Exl3bGeom* g, int c) {
    return (g->n_expert - c + g->n_class - 1) / g->n_class;
}
/* Extents of plane p of a class's [rows, cols] weight (include/exl3_abi.h:654-664). */
void exl3b_plane_extents(int64_t rows, int64_t cols, int p, int64_t* r, int64_t* c);

/* gate_up_down as its halves (include/exl3_abi.h:751-845): the gate_up view (a_rot 0, h_rot 1) and the
 * down view (h_rot 1, class c at [K_c, N_c / 2]); `h` the caller's [T, max N_c / 2] f16 buffer. Parameter
 * arrays: gate_up up to 15, down up to 14. Operand arrays: gate_up 24, down 16. */
void exl3b_gd_params(const RadParam* p, int n_p, int mod4, RadParam* pg, int* n_pg, RadParam* pd, int* n_pd);
void exl3b_gd_operands(const RadTensor* t, const RadTensor* h, int mod4, RadTensor* tg, RadTensor* td);

#ifdef __cplusplus
}
#endif

#endif /* EXL3B200_ABI_H */
