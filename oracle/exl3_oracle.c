/* exl3_oracle.c -- TEST INFRASTRUCTURE: the CPU restatement of the EXL3 routed-expert path.
 *
 * This file is a checker. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it;
 * the product library never does. Built with -ffp-contract=off so every product and sum rounds
 * separately, as the reference contract requires (kernels/exl3ref/CMakeLists.txt:39-42).
 *
 * Written from the reference's published algorithm, each block citing the reference lines it restates.
 * Where the reference is scalar per bit, this reads whole symbols; the numbers are the same. */
#include "exl3_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#include "rad_types.h"   /* rad_f16_to_f32 / rad_f32_to_f16 / rad_f32_to_bf16 / rad_bf16_to_f32 */

/* ------------------------------------------------------------------ fp16 from an exact double
 * One round-to-nearest-even of an exact value (common/exl3_decode.c:25-39): every codebook value is one
 * such rounding of a sum that is exact in double. */
static uint16_t half_rne(double x) {
    const uint16_t sign = signbit(x) ? 0x8000u : 0u;
    double a = fabs(x);
    if (isnan(x)) return 0x7E00u;
    if (a >= 65520.0) return sign | 0x7C00u;
    if (a < 0x1p-14) return (uint16_t)(sign | (uint16_t)nearbyint(a * 0x1p24));
    int e;
    double m = nearbyint(ldexp(frexp(a, &e), 11));
    if (m == 2048.0) { m = 1024.0; ++e; }
    if (e + 14 >= 31) return sign | 0x7C00u;
    return (uint16_t)(sign | (uint16_t)((e + 14) << 10) | (uint16_t)(m - 1024.0));
}

/* ------------------------------------------------------------------ the codebooks
 * common/exl3_decode.c:43-67. mul1: h = state * 0x83DCD12D, value = fp16(1024 + bytesum(h)) * K_INV +
 * K_BIAS with one rounding (fp16 K_INV 0x1EEE, K_BIAS 0xC931). mcg: h = state * 0xCBAC1FED; 3inst:
 * h = state * 89226354 + 64248484; both then (h & 0x8FFF8FFF) ^ 0x3B603B60 and the two fp16 halves added
 * with one rounding. */
uint16_t orc_codebook_value(uint32_t state, int codebook) {
    uint32_t x = state & 0xFFFFu;
    if (codebook == ORC_CB_MUL1) {
        x *= 0x83DCD12Du;
        const uint32_t s = (x & 0xFFu) + ((x >> 8) & 0xFFu) + ((x >> 16) & 0xFFu) + (x >> 24);
        const double k_inv = (double)rad_f16_to_f32(0x1EEEu), k_bias = (double)rad_f16_to_f32(0xC931u);
        return half_rne((1024.0 + (double)s) * k_inv + k_bias);
    }
    if (codebook == ORC_CB_MCG) x *= 0xCBAC1FEDu;
    else if (codebook == ORC_CB_3INST) x = x * 89226354u + 64248484u;
    else return 0x7E00u;
    x = (x & 0x8FFF8FFFu) ^ 0x3B603B60u;
    return half_rne((double)rad_f16_to_f32((uint16_t)(x & 0xFFFFu)) + (double)rad_f16_to_f32((uint16_t)(x >> 16)));
}

/* ------------------------------------------------------------------ one tile
 * Position p = 8L + j sits at tile row (k axis) 2(L%4) + {0,1,8,9}[j%4], column (n axis) L/4 + 8(j/4)
 * (common/exl3_decode.c:71-76). */
static void pos_rc(int p, int* r, int* c) {
    const int L = p >> 3, j = p & 7;
    static const int roff[4] = { 0, 1, 8, 9 };
    *r = 2 * (L & 3) + roff[j & 3];
    *c = (L >> 2) + 8 * (j >> 2);
}

/* Symbol p of a tile: stream bits [pK, pK+K), the stream being 8K little-endian u32 words read MSB first
 * (common/exl3_decode.c:84-97). */
static void tile_syms(const uint16_t* tile, int bits, uint8_t* sym) {
    const int nw = 8 * bits;
    for (int p = 0; p < 256; ++p) {
        const int b = p * bits;
        const int w = b >> 5, o = b & 31;
        const uint64_t hi = (uint64_t)tile[2 * w] | ((uint64_t)tile[2 * w + 1] << 16);
        const int w2 = (w + 1) % nw;
        const uint64_t lo = (uint64_t)tile[2 * w2] | ((uint64_t)tile[2 * w2 + 1] << 16);
        const uint64_t v = (hi << 32) | lo;            /* 64 stream bits from word w, MSB first */
        sym[p] = (uint8_t)((v >> (64 - o - bits)) & ((1u << bits) - 1u));
    }
}

/* The inverse: symbols -> stream words (common/exl3_decode.c:99-109). */
static void tile_pack(const uint8_t* sym, int bits, uint16_t* tile) {
    uint32_t words[64];
    const int nw = 8 * bits;
    memset(words, 0, sizeof words);
    for (int p = 0; p < 256; ++p) {
        const uint32_t s = sym[p] & ((1u << bits) - 1u);
        for (int i = 0; i < bits; ++i) {
            const int b = p * bits + i;
            if ((s >> (bits - 1 - i)) & 1u) words[b >> 5] |= 1u << (31 - (b & 31));
        }
    }
    for (int w = 0; w < nw; ++w) {
        tile[2 * w] = (uint16_t)(words[w] & 0xFFFFu);
        tile[2 * w + 1] = (uint16_t)(words[w] >> 16);
    }
}

/* State of position p: the 16-bit window of the symbol stream ending at p's last bit, circular in the
 * tile (common/exl3_decode.c:111-121). */
static void tile_states(const uint8_t* sym, int bits, uint16_t* st) {
    const int back = (16 + bits - 1) / bits;
    for (int p = 0; p < 256; ++p) {
        uint32_t acc = 0;
        for (int i = back - 1; i >= 0; --i) acc = (acc << bits) | sym[(p - i + 256) & 255];
        st[p] = (uint16_t)(acc & 0xFFFFu);
    }
}

static int args_ok(int bits, int codebook) {
    return bits >= 1 && bits <= 8 && codebook >= ORC_CB_3INST && codebook <= ORC_CB_MUL1;
}

/* A 65536-entry value table per codebook, built once (the value depends on the state alone). */
static uint16_t* cb_table(int codebook) {
    static uint16_t* tab[3];
    static pthread_mutex_t mu = PTHREAD_MUTEX_INITIALIZER;
    pthread_mutex_lock(&mu);
    if (!tab[codebook]) {
        uint16_t* t = (uint16_t*)malloc(65536 * sizeof *t);
        if (t)
            for (uint32_t s = 0; s < 65536; ++s) t[s] = orc_codebook_value(s, codebook);
        tab[codebook] = t;
    }
    pthread_mutex_unlock(&mu);
    return tab[codebook];
}

int orc_trellis_decode(const uint16_t* trellis, int64_t kt, int64_t nt, int bits, int codebook,
                       uint16_t* w_hat) {
    uint8_t sym[256];
    uint16_t st[256];
    if (!trellis || !w_hat || kt < 0 || nt < 0 || !args_ok(bits, codebook)) return -1;
    const uint16_t* tab = cb_table(codebook);
    if (!tab) return -7;
    for (int64_t tk = 0; tk < kt; ++tk)
        for (int64_t tn = 0; tn < nt; ++tn) {
            tile_syms(trellis + (tk * nt + tn) * 16 * bits, bits, sym);
            tile_states(sym, bits, st);
            for (int p = 0; p < 256; ++p) {
                int r, c;
                pos_rc(p, &r, &c);
                w_hat[(tk * 16 + r) * (nt * 16) + tn * 16 + c] = tab[st[p]];
            }
        }
    return 0;
}

int orc_record_decode(const uint16_t* record, int64_t rows, int64_t cols, int bits, int codebook,
                      uint16_t* w_hat_nk) {
    uint8_t sym[256];
    uint16_t st[256];
    if (!record || !w_hat_nk || rows % 16 || cols % 16 || !args_ok(bits, codebook)) return -1;
    const uint16_t* tab = cb_table(codebook);
    if (!tab) return -7;
    const int64_t nt = rows / 16, kt = cols / 16;
    for (int64_t tk = 0; tk < kt; ++tk)
        for (int64_t tn = 0; tn < nt; ++tn) {
            tile_syms(record + (tk * nt + tn) * 16 * bits, bits, sym);
            tile_states(sym, bits, st);
            for (int p = 0; p < 256; ++p) {
                int r, c;
                pos_rc(p, &r, &c);
                w_hat_nk[(tn * 16 + c) * cols + tk * 16 + r] = tab[st[p]];
            }
        }
    return 0;
}

/* ------------------------------------------------------------------ the canonical plane
 * Element (i, j) of a uK plane is bits [jK, jK+K) of row i, LSB first (common/exl3_decode.c:148-168). */
static uint32_t plane_get(const uint8_t* row, int bits, int64_t j) {
    const int64_t b = j * bits;
    const uint32_t v = (uint32_t)row[b >> 3] | ((uint32_t)row[(b >> 3) + 1] << 8);
    return (v >> (b & 7)) & ((1u << bits) - 1u);
}
static uint32_t plane_get_safe(const uint8_t* row, int64_t row_bytes, int bits, int64_t j) {
    const int64_t b = j * bits;
    uint32_t v = row[b >> 3];
    if ((b >> 3) + 1 < row_bytes) v |= (uint32_t)row[(b >> 3) + 1] << 8;
    return (v >> (b & 7)) & ((1u << bits) - 1u);
}
static void plane_set(uint8_t* row, int bits, int64_t j, uint32_t value) {
    for (int i = 0; i < bits; ++i) {
        const int64_t b = j * bits + i;
        const uint8_t m = (uint8_t)(1u << (b & 7));
        if ((value >> i) & 1u) row[b >> 3] |= m;
        else row[b >> 3] &= (uint8_t)~m;
    }
}

/* Tile (tk, tn) of a rectangle keeps W_hat[k = 16tk + r][n = 16tn + c] at position (r, c); the canonical
 * plane keeps that symbol at element (n, k) (common/exl3_layout.c:66-104). */
int orc_codes_to_record(const uint8_t* codes, int64_t row_bytes, int64_t rows, int64_t cols, int bits,
                        uint16_t* record) {
    uint8_t sym[256];
    if (!codes || !record || bits < 1 || bits > 8 || rows % 16 || cols % 16 || rows < 0 || cols < 0) return -1;
    if (row_bytes < (cols * bits + 7) / 8) return -1;
    const int64_t nt = rows / 16, kt = cols / 16;
    for (int64_t tk = 0; tk < kt; ++tk)
        for (int64_t tn = 0; tn < nt; ++tn) {
            for (int p = 0; p < 256; ++p) {
                int r, c;
                pos_rc(p, &r, &c);
                sym[p] = (uint8_t)plane_get_safe(codes + (tn * 16 + c) * row_bytes, row_bytes, bits, tk * 16 + r);
            }
            tile_pack(sym, bits, record + (tk * nt + tn) * 16 * bits);
        }
    return 0;
}

int orc_record_to_codes(const uint16_t* record, int64_t rows, int64_t cols, int bits, uint8_t* codes,
                        int64_t row_bytes) {
    uint8_t sym[256];
    if (!codes || !record || bits < 1 || bits > 8 || rows % 16 || cols % 16 || rows < 0 || cols < 0) return -1;
    if (row_bytes < (cols * bits + 7) / 8) return -1;
    const int64_t nt = rows / 16, kt = cols / 16;
    for (int64_t tk = 0; tk < kt; ++tk)
        for (int64_t tn = 0; tn < nt; ++tn) {
            tile_syms(record + (tk * nt + tn) * 16 * bits, bits, sym);
            for (int p = 0; p < 256; ++p) {
                int r, c;
                pos_rc(p, &r, &c);
                plane_set(codes + (tn * 16 + c) * row_bytes, bits, tk * 16 + r, sym[p]);
            }
        }
    return 0;
}

/* W_hat of a canonical plane as exact fp16 values held in f32, [rows][cols]
 * (common/exl3_decode.c:193-221). */
static int plane_what(const uint8_t* codes, int64_t rows, int64_t cols, int bits, int codebook, float* out) {
    uint8_t sym[256];
    uint16_t st[256];
    const uint16_t* tab = cb_table(codebook);
    if (!tab) return -7;
    const int64_t rb = (cols * bits + 7) / 8, nt = rows / 16, kt = cols / 16;
    int pr[256], pc[256];
    for (int p = 0; p < 256; ++p) pos_rc(p, &pr[p], &pc[p]);
    for (int64_t tn = 0; tn < nt; ++tn)
        for (int64_t tk = 0; tk < kt; ++tk) {
            for (int p = 0; p < 256; ++p)
                sym[p] = (uint8_t)plane_get_safe(codes + (tn * 16 + pc[p]) * rb, rb, bits, tk * 16 + pr[p]);
            tile_states(sym, bits, st);
            for (int p = 0; p < 256; ++p)
                out[(tn * 16 + pc[p]) * cols + tk * 16 + pr[p]] = rad_f16_to_f32(tab[st[p]]);
        }
    (void)plane_get;
    return 0;
}

/* ------------------------------------------------------------------ the rotation
 * Butterfly stages h = 1, 2, ..., 64 in f32 (a+b low, a-b high), then one multiply by (float)(1/sqrt(128))
 * (common/exl3_decode.c:172-189). */
int orc_had128(float* v, int64_t n) {
    const float scale = 0.08838834764831844055f;
    if (!v || n < 0 || n % 128) return -1;
    for (int64_t base = 0; base < n; base += 128) {
        float* x = v + base;
        for (int h = 1; h < 128; h <<= 1)
            for (int i = 0; i < 128; i += 2 * h)
                for (int j = i; j < i + h; ++j) {
                    const float a = x[j], b = x[j + h];
                    x[j] = a + b;
                    x[j + h] = a - b;
                }
        for (int i = 0; i < 128; ++i) x[i] *= scale;
    }
    return 0;
}

/* ------------------------------------------------------------------ the ops (kernels/exl3ref/ref.c) */

static float h2f(uint16_t h) { return rad_f16_to_f32(h); }
static uint16_t f2h(float f) { return rad_f32_to_f16(f); }

/* xr = f16(had(f16(x * s))) (ref.c:27-32). */
static void prologue(const float* x, const uint16_t* s, int64_t cols, float* xr) {
    for (int64_t k = 0; k < cols; ++k) xr[k] = h2f(f2h(x[k] * h2f(s[k])));
    orc_had128(xr, cols);
    for (int64_t k = 0; k < cols; ++k) xr[k] = h2f(f2h(xr[k]));
}

/* acc[n] = sum over k ascending of xr[k] * what[n][k], f32, two roundings a step (ref.c:35-42). */
static void gemv(const float* xr, const float* what, int64_t rows, int64_t cols, float* acc) {
    for (int64_t n = 0; n < rows; ++n) {
        const float* w = what + n * cols;
        float s = 0.0f;
        for (int64_t k = 0; k < cols; ++k) s = s + xr[k] * w[k];
        acc[n] = s;
    }
}

static float silu(float g) { return g * (1.0f / (1.0f + expf(-g))); }   /* ref.c:44 */

static void load_row(const OrcOp* o, int64_t r, int64_t col0, int64_t cols, float* out) {
    const uint16_t* p = (const uint16_t*)o->x + r * o->x_pitch + col0;
    for (int64_t k = 0; k < cols; ++k) out[k] = o->x_dtype == ORC_X_BF16 ? rad_bf16_to_f32(p[k]) : h2f(p[k]);
}

typedef struct Work { float *what, *x, *xr, *acc; } Work;

/* prep_gu (ref.c:154-169; OPS-exl3.md:128-142): every row of the run, both halves side by side; a
 * negative sorted_tok gives a zero row of 2C; nothing outside the runs is written. */
static void prep_rows(const OrcOp* o, int64_t e, Work* wk) {
    const int c = (int)(e % o->n_class);
    const int64_t C = o->cols[c];
    const uint16_t* s[2] = { o->suh[e], o->suh1[e] };
    for (int64_t i = o->expert_offset[e]; i < o->expert_offset[e + 1]; ++i) {
        uint16_t* xr = o->y + i * o->y_pitch;
        if (o->sorted_tok[i] < 0) { memset(xr, 0, (size_t)(2 * C) * 2); continue; }
        load_row(o, o->sorted_tok[i] / o->top_k, 0, C, wk->x);
        for (int p = 0; p < 2; ++p) {
            prologue(wk->x, s[p], C, wk->xr);
            for (int64_t k = 0; k < C; ++k) xr[p * C + k] = f2h(wk->xr[k]);
        }
    }
}

/* gate_up and down for one expert's rows (ref.c:171-228; OPS-exl3.md:104-153). */
static int expert_rows(const OrcOp* o, int64_t e, Work* wk) {
    const int c = (int)(e % o->n_class);
    const int64_t R = o->rows[c], C = o->cols[c];
    const int gate_up = o->op == ORC_GATE_UP;
    const uint16_t* suh = o->suh[e];
    const uint16_t* suh1 = gate_up ? o->suh1[e] : 0;
    const uint16_t* svh = o->svh[e];
    int rc = plane_what(o->codes[e], R, C, o->bits, o->codebook, wk->what);
    if (rc) return rc;
    for (int64_t i = o->expert_offset[e]; i < o->expert_offset[e + 1]; ++i) {
        if (o->sorted_tok[i] < 0) continue;
        if (gate_up) {
            const int64_t W = R / 2;
            if (!o->a_rot) load_row(o, o->sorted_tok[i] / o->top_k, 0, C, wk->x);
            for (int p = 0; p < 2; ++p) {
                if (o->a_rot) load_row(o, i, p * C, C, wk->xr);
                else prologue(wk->x, p ? suh1 : suh, C, wk->xr);
                gemv(wk->xr, wk->what + p * W * C, W, C, wk->acc + p * W);
                orc_had128(wk->acc + p * W, W);
                for (int64_t n = 0; n < W; ++n) wk->acc[p * W + n] = wk->acc[p * W + n] * h2f(svh[p * W + n]);
            }
            uint16_t* h = o->y + i * o->y_pitch;
            if (!o->h_rot) {
                for (int64_t n = 0; n < W; ++n) h[n] = f2h(silu(wk->acc[n]) * wk->acc[W + n]);
                continue;
            }
            for (int64_t n = 0; n < W; ++n) wk->x[n] = h2f(f2h(silu(wk->acc[n]) * wk->acc[W + n]));
            prologue(wk->x, o->dn_suh[e], W, wk->xr);
            for (int64_t n = 0; n < W; ++n) h[n] = f2h(wk->xr[n]);
        } else {
            if (o->h_rot) {
                load_row(o, i, 0, C, wk->xr);
            } else {
                load_row(o, i, 0, C, wk->x);
                prologue(wk->x, suh, C, wk->xr);
            }
            gemv(wk->xr, wk->what, R, C, wk->acc);
            orc_had128(wk->acc, R);
            uint16_t* y = o->y + i * o->y_pitch;
            if (o->out_f16)   /* the f16-output linear (config 1): the same value rounded to f16 instead */
                for (int64_t n = 0; n < R; ++n) y[n] = f2h(wk->acc[n] * h2f(svh[n]));
            else
                for (int64_t n = 0; n < R; ++n) y[n] = rad_f32_to_bf16(wk->acc[n] * h2f(svh[n]));
        }
    }
    return 0;
}

typedef struct Job {
    const OrcOp* o;
    int64_t e0, e_step;
    int rc;
} Job;

static void* run_job(void* arg) {
    Job* j = (Job*)arg;
    const OrcOp* o = j->o;
    int64_t most = 0, widest = 0;
    for (int c = 0; c < o->n_class; ++c) {
        if (o->rows[c] * o->cols[c] > most) most = o->rows[c] * o->cols[c];
        if (o->rows[c] > widest) widest = o->rows[c];
    }
    const int64_t row = o->x_cols > widest ? o->x_cols : widest;
    Work wk = { malloc((size_t)(most + 1) * sizeof(float)), malloc((size_t)(row + 1) * sizeof(float)),
                malloc((size_t)(row + 1) * sizeof(float)), malloc((size_t)(widest + 1) * sizeof(float)) };
    j->rc = wk.what && wk.x && wk.xr && wk.acc ? 0 : -7;
    for (int64_t e = j->e0; e < o->n_expert && !j->rc; e += j->e_step) {
        int live = 0;
        for (int64_t i = o->expert_offset[e]; i < o->expert_offset[e + 1] && !live; ++i) live = o->sorted_tok[i] >= 0;
        if (o->op == ORC_PREP_GU) {
            if (o->expert_offset[e + 1] > o->expert_offset[e]) prep_rows(o, e, &wk);
        } else if (live) {
            j->rc = expert_rows(o, e, &wk);
        }
    }
    free(wk.what); free(wk.x); free(wk.xr); free(wk.acc);
    return 0;
}

int orc_moe_op(const OrcOp* o) {
    if (!o || !o->x || !o->y || !o->sorted_tok || !o->expert_offset || o->n_class < 1 || o->n_class > 4) return -1;
    if (o->op != ORC_PREP_GU && !args_ok(o->bits, o->codebook)) return -1;
    if (o->expert_offset[0] < 0 || o->expert_offset[o->n_expert] > o->T) return -1;
    for (int64_t e = 0; e < o->n_expert; ++e)
        if (o->expert_offset[e + 1] < o->expert_offset[e]) return -1;
    /* every output row zero first, except prep_gu (ref.c:307-311) */
    if (o->op != ORC_PREP_GU)
        for (int64_t i = 0; i < o->T; ++i) memset(o->y + i * o->y_pitch, 0, (size_t)o->y_cols * 2);
    int nt = o->n_threads > 1 ? o->n_threads : 1;
    if (nt > 256) nt = 256;
    Job jobs[256];
    pthread_t th[256];
    for (int t = 0; t < nt; ++t) {
        jobs[t].o = o;
        jobs[t].e0 = t;
        jobs[t].e_step = nt;
        jobs[t].rc = 0;
    }
    if (nt == 1) {
        run_job(&jobs[0]);
        return jobs[0].rc;
    }
    for (int t = 0; t < nt; ++t) pthread_create(&th[t], 0, run_job, &jobs[t]);
    int rc = 0;
    for (int t = 0; t < nt; ++t) {
        pthread_join(th[t], 0);
        if (jobs[t].rc) rc = jobs[t].rc;
    }
    return rc;
}

/* ------------------------------------------------------------------ routing around the path */

/* Stable counting sort of the flattened pairs token*top_k + slot by local expert id - expert_base; ids
 * outside [0, n_expert) are dropped and the tail is -1 (include/exl3_abi.h:109-124). */
int orc_moe_scatter(const int32_t* expert_ids, int64_t n_pairs, int64_t n_expert, int64_t expert_base,
                    int32_t* sorted_tok, int32_t* expert_offset) {
    if (!expert_ids || !sorted_tok || !expert_offset || n_expert < 1) return -1;
    int64_t* cnt = (int64_t*)calloc((size_t)n_expert + 1, sizeof *cnt);
    if (!cnt) return -7;
    for (int64_t i = 0; i < n_pairs; ++i) {
        const int64_t e = (int64_t)expert_ids[i] - expert_base;
        if (e >= 0 && e < n_expert) ++cnt[e + 1];
    }
    for (int64_t e = 0; e < n_expert; ++e) cnt[e + 1] += cnt[e];
    for (int64_t e = 0; e <= n_expert; ++e) expert_offset[e] = (int32_t)cnt[e];
    for (int64_t i = 0; i < n_pairs; ++i) sorted_tok[i] = -1;
    for (int64_t i = 0; i < n_pairs; ++i) {
        const int64_t e = (int64_t)expert_ids[i] - expert_base;
        if (e >= 0 && e < n_expert) sorted_tok[cnt[e]++] = (int32_t)i;
    }
    free(cnt);
    return 0;
}

int orc_moe_gather(const uint16_t* rows_bf16, int64_t row_pitch, const int32_t* sorted_tok, int64_t n_rows,
                   const float* w, int64_t n_tok, int64_t top_k, int64_t width, float* y) {
    if (!rows_bf16 || !sorted_tok || !w || !y) return -1;
    int64_t* pos = (int64_t*)malloc((size_t)(n_tok * top_k + 1) * sizeof *pos);
    if (!pos) return -7;
    for (int64_t f = 0; f < n_tok * top_k; ++f) pos[f] = -1;
    for (int64_t i = 0; i < n_rows; ++i)
        if (sorted_tok[i] >= 0 && sorted_tok[i] < n_tok * top_k) pos[sorted_tok[i]] = i;
    for (int64_t t = 0; t < n_tok; ++t)
        for (int64_t n = 0; n < width; ++n) {
            float acc = 0.0f;
            for (int64_t s = 0; s < top_k; ++s) {
                const int64_t i = pos[t * top_k + s];
                if (i < 0) continue;
                acc = acc + w[t * top_k + s] * rad_bf16_to_f32(rows_bf16[i * row_pitch + n]);
            }
            y[t * width + n] = acc;
        }
    free(pos);
    return 0;
}
