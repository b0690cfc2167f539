/* exl3_oracle.h -- TEST INFRASTRUCTURE: this repository's CPU restatement of the EXL3 routed-expert
 * path, the checker the CUDA kernels are compared with. Never linked into the product library.
 *
 * Restates, in code of its own, the published algorithm of radiance-exl3's oracle:
 *   the trellis decode            common/exl3_decode.c:47-144, 193-221
 *   the tile-stream record        common/exl3_layout.c:14-56
 *   the 128-point rotation        common/exl3_decode.c:172-189
 *   the four routed-expert ops    kernels/exl3ref/ref.c:27-331 and docs/OPS-exl3.md:84-200
 * It is pinned against the vllm-exl3 golden decode and against the reference library itself built from
 * the reference sources (oracle/_ref): see tests/test_oracle.py.
 *
 * All fp16 / bf16 values travel as their bit patterns (uint16_t). */
#ifndef EXL3_ORACLE_H
#define EXL3_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_CB_3INST = 0, ORC_CB_MCG = 1, ORC_CB_MUL1 = 2 };
enum { ORC_DOWN = 0, ORC_GATE_UP = 1, ORC_PREP_GU = 2 };
enum { ORC_X_F16 = 0, ORC_X_BF16 = 1 };

/* State (low 16 bits) -> fp16 bits of its codebook value; 0x7E00 for an unknown codebook. */
uint16_t orc_codebook_value(uint32_t state, int codebook);

/* The decode of a whole exllamav3 trellis tensor int16 [kt][nt][16K] to W_hat [16 kt][16 nt] fp16 bits,
 * exllamav3's [k][n] order. 0, or -1 for bits / codebook out of range. */
int orc_trellis_decode(const uint16_t* trellis, int64_t kt, int64_t nt, int bits, int codebook,
                       uint16_t* w_hat);

/* The same decode read in radiance's [rows = n][cols = k] view: w_hat_nk[n * cols + k]. `record` is the
 * rectangle's tile-stream record (tile (tk, tn) at (tk * rows/16 + tn) * 16K). */
int orc_record_decode(const uint16_t* record, int64_t rows, int64_t cols, int bits, int codebook,
                      uint16_t* w_hat_nk);

/* Canonical uK codes plane [rows][cols] (LSB-first rows, `row_bytes` apart) <-> tile-stream record. */
int orc_codes_to_record(const uint8_t* codes, int64_t row_bytes, int64_t rows, int64_t cols, int bits,
                        uint16_t* record);
int orc_record_to_codes(const uint16_t* record, int64_t rows, int64_t cols, int bits, uint8_t* codes,
                        int64_t row_bytes);

/* In-place normalised 128-point Hadamard over each block of 128 of v[0..n). -1 unless n % 128 == 0. */
int orc_had128(float* v, int64_t n);

/* One op of the routed-expert family over canonical planes (the reference's input form).
 * Experts are tabled by class: expert e is class e % n_class, entry e / n_class, and its planes are
 * codes[e], suh[e], suh1[e], svh[e], dn_suh[e] (indexed by EXPERT here, not by entry). */
typedef struct OrcOp {
    int            op;                 /* ORC_DOWN / ORC_GATE_UP / ORC_PREP_GU */
    int            bits, codebook, h_rot, a_rot;
    int64_t        T, n_expert, top_k, n_class;
    int64_t        rows[4], cols[4];   /* class c's [rows, cols] */
    int64_t        x_cols, y_cols;
    const void*    x;                  /* token rows (gate_up a_rot 0, prep) or sorted rows */
    int            x_dtype;            /* ORC_X_F16 / ORC_X_BF16 */
    int64_t        x_rows, x_pitch;    /* elements */
    uint16_t*      y;                  /* f16 (gate_up, prep) or bf16 (down) */
    int64_t        y_pitch;
    const int32_t* sorted_tok;
    const int32_t* expert_offset;
    const uint8_t* const* codes;       /* [n_expert] canonical planes, rows dense */
    const uint16_t* const* suh;
    const uint16_t* const* suh1;
    const uint16_t* const* svh;
    const uint16_t* const* dn_suh;
    int            n_threads;          /* experts decoded and run in parallel; 1 = the reference's order */
    int            out_f16;            /* down only: round the output to f16 instead of bf16 (this library's
                                          f16-output linear; the reference's down writes bf16, ref.c:97-102) */
} OrcOp;

/* 0 ok; -1 bad arguments; -7 out of memory. Writes exactly what the op defines (zero rows, prep's
 * not-written rows left alone). */
int orc_moe_op(const OrcOp* o);

/* The routing producers around the path: a stable counting sort of (token, slot) pairs by expert
 * (the engine's moe_scatter contract as include/exl3_abi.h:96-158 states it), and the gather that
 * weights a token's slots and sums them in ascending slot order. */
int orc_moe_scatter(const int32_t* expert_ids, int64_t n_pairs, int64_t n_expert, int64_t expert_base,
                    int32_t* sorted_tok, int32_t* expert_offset);
/* y[t][n] = sum over slots s ascending of w[t][s] * bf16 value of rows[pos[t*top_k+s]][n], f32, written
 * as f32. pos = the inverse of sorted_tok (-1: slot dropped). */
int orc_moe_gather(const uint16_t* rows_bf16, int64_t row_pitch, const int32_t* sorted_tok, int64_t n_rows,
                   const float* w, int64_t n_tok, int64_t top_k, int64_t width, float* y);

#ifdef __cplusplus
}
#endif

#endif /* EXL3_ORACLE_H */
