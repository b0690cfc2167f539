/* exl3b200_layer.c -- one routed-MoE layer as the engine's MoE block issues it, driven from C: router_topk then
 * moe_scatter (one fused launch for a few tokens), moe_exl3_gate_up (h_rot 1), moe_exl3_down (h_rot 1), moe_gather.
 * The two expert ops go through this library's own plugin rows with RadArgs built here, exactly as the engine calls
 * them (architectures/qwen4exp_exl3/rad_block_moe_exl3.h:1763-1900 issues the same sequence for a pass).
 *
 * Nothing here allocates: exl3b200_moe_layer_work_bytes() sizes one device block that the caller allocates once,
 * and exl3b200_moe_layer_carve() cuts it into the layer's buffers (routing, h, the down rows, the ops' scratch, the
 * gather's map). A forward then only enqueues kernels on the caller's stream. */
#include "exl3b200.h"
#include "exl3b200_abi.h"
#include "exl3b200_dev.h"

#include <stdio.h>
#include <string.h>

int exl3b_cuda_mark(void* event, void* stream);   /* exl3b200_p2p.cu: cudaEventRecord */

/* The stored dtype of a codes table (the layout hook's RadLayout.dtype; exl3b200_host.c). */
enum { LAYER_DT_RECORD = RAD_DT_PLUGIN_BASE + 0x3B2 };

static const RadKernelInfo* row_of(const char* op) {
    for (int i = 0; i < rad_kernel_count(); ++i) {
        const RadKernelInfo* k = rad_kernel_at(i);
        if (k && strcmp(k->op, op) == 0) return k;
    }
    return 0;
}

static int64_t up256(int64_t b) { return (b + 255) / 256 * 256; }

static void tens(RadTensor* t, const void* data, uint32_t dt, int rank, const int64_t* shape) {
    memset(t, 0, sizeof *t);
    t->data = (void*)data;
    t->dtype = dt;
    t->rank = (uint32_t)rank;
    for (int r = 0; r < rank; ++r) t->shape[r] = shape[r];
    rad_tensor_pack(t);
}

/* A table of per-expert stored records: [n][rows][cols], entry pointers in a device table (stride 0). */
static void table(RadTensor* t, const void* ptrs, int64_t n, int64_t rows, int64_t cols) {
    const int64_t sh[3] = { n, rows, cols };
    tens(t, ptrs, LAYER_DT_RECORD, 3, sh);
    t->stride[0] = 0;
}

static const char* dtype_name(int bits) {
    static const char* const names[9] = { "", "", "exl3k2", "exl3k3", "exl3k4", "exl3k5", "exl3k6", "exl3k7", "exl3k8" };
    return bits >= 2 && bits <= 8 ? names[bits] : "";
}

static const char* codebook_name(int cb) {
    return cb == 0 ? "3inst" : cb == 1 ? "mcg" : cb == 2 ? "mul1" : "";
}

/* The two ops' RadArgs for a pass of T tokens (T * top_k sorted rows). */
typedef struct LayerArgs {
    RadTensor gu_t[14], dn_t[10];
    RadParam gu_p[10], dn_p[10];
    RadArgs gu, dn;
} LayerArgs;

static int check_desc(const Exl3bLayerDesc* d) {
    if (!d) return RAD_E_INVAL;
    if (d->n_expert < 1 || d->n_local < 1 || d->expert_base < 0 || d->top_k < 1 || d->top_k > 32 ||
        d->hidden < 128 || d->width < 128 || d->hidden % 128 || d->width % 128)
        return RAD_E_SHAPE;
    if (d->bits_gu < 2 || d->bits_gu > 8 || d->bits_dn < 2 || d->bits_dn > 8 || d->codebook < 0 || d->codebook > 2)
        return RAD_E_INVAL;
    if (!d->gu_codes || !d->dn_codes || !d->suh || !d->suh1 || !d->svh_gu || !d->dn_suh || !d->svh_dn)
        return RAD_E_INVAL;
    return RAD_OK;
}

/* One pass of the two ops: gate_up reads x [x_rows][hidden] through sorted_tok (rows sorted rows, top_k slots a
 * token row), h [rows][width] between them, down writes y [rows][hidden] bf16. */
typedef struct Pass {
    const void*    x;
    int64_t        x_rows, top_k, rows;
    const int32_t* sorted_tok;
    const int32_t* expert_offset;
    void*          h;
    void*          y;
} Pass;

static void build_args(const Exl3bLayerDesc* d, const Pass* s, LayerArgs* a) {
    const int64_t E = d->n_local, H = d->hidden, W = d->width, R = s->rows, T = s->x_rows;
    memset(a, 0, sizeof *a);
    int np = 0;
    RadParam* p = a->gu_p;
    p[np++] = (RadParam)RAD_INT("M", T);
    p[np++] = (RadParam)RAD_INT("N", 2 * W);
    p[np++] = (RadParam)RAD_INT("K", H);
    p[np++] = (RadParam)RAD_INT("n_expert", E);
    p[np++] = (RadParam)RAD_INT("top_k", s->top_k);
    p[np++] = (RadParam)RAD_STR("dtype", dtype_name(d->bits_gu));
    p[np++] = (RadParam)RAD_STR("codebook", codebook_name(d->codebook));
    p[np++] = (RadParam)RAD_INT("h_rot", 1);
    p[np++] = (RadParam)RAD_INT("a_rot", 0);
    const int n_gu = np;
    np = 0;
    p = a->dn_p;
    p[np++] = (RadParam)RAD_INT("M", T);
    p[np++] = (RadParam)RAD_INT("N", H);
    p[np++] = (RadParam)RAD_INT("K", W);
    p[np++] = (RadParam)RAD_INT("n_expert", E);
    p[np++] = (RadParam)RAD_INT("top_k", s->top_k);
    p[np++] = (RadParam)RAD_STR("dtype", dtype_name(d->bits_dn));
    p[np++] = (RadParam)RAD_STR("codebook", codebook_name(d->codebook));
    p[np++] = (RadParam)RAD_INT("h_rot", 1);
    const int n_dn = np;
    /* gate_up: a, codes, suh, suh1, svh, dn_suh, sorted_tok, expert_offset, <odd class x5>, h */
    RadTensor* t = a->gu_t;
    tens(&t[0], s->x, RAD_F16, 2, (int64_t[]){ T, H });
    table(&t[1], d->gu_codes, E, 2 * W, H);
    tens(&t[2], d->suh, RAD_F16, 3, (int64_t[]){ E, 1, H });
    tens(&t[3], d->suh1, RAD_F16, 3, (int64_t[]){ E, 1, H });
    tens(&t[4], d->svh_gu, RAD_F16, 3, (int64_t[]){ E, 2 * W, 1 });
    tens(&t[5], d->dn_suh, RAD_F16, 3, (int64_t[]){ E, 1, W });
    tens(&t[6], s->sorted_tok, RAD_I32, 1, (int64_t[]){ R });
    tens(&t[7], s->expert_offset, RAD_I32, 1, (int64_t[]){ E + 1 });
    tens(&t[13], s->h, RAD_F16, 2, (int64_t[]){ R, W });
    /* down: h, codes, suh, svh, sorted_tok, expert_offset, <odd class x3>, y */
    t = a->dn_t;
    tens(&t[0], s->h, RAD_F16, 2, (int64_t[]){ R, W });
    table(&t[1], d->dn_codes, E, H, W);
    tens(&t[2], d->dn_suh, RAD_F16, 3, (int64_t[]){ E, 1, W });
    tens(&t[3], d->svh_dn, RAD_F16, 3, (int64_t[]){ E, H, 1 });
    tens(&t[4], s->sorted_tok, RAD_I32, 1, (int64_t[]){ R });
    tens(&t[5], s->expert_offset, RAD_I32, 1, (int64_t[]){ E + 1 });
    tens(&t[9], s->y, RAD_BF16, 2, (int64_t[]){ R, H });
    a->gu.t = a->gu_t;
    a->gu.n_t = 14;
    a->gu.p = a->gu_p;
    a->gu.n_p = n_gu;
    a->gu.world_size = 1;
    a->dn.t = a->dn_t;
    a->dn.n_t = 10;
    a->dn.p = a->dn_p;
    a->dn.n_p = n_dn;
    a->dn.world_size = 1;
}

static Pass layer_pass(const Exl3bLayerDesc* d, const Exl3bLayerBufs* b, const void* x, int64_t T) {
    const Pass s = { x, T, d->top_k, T * d->top_k, b->sorted_tok, b->expert_offset, b->h, b->y_rows };
    return s;
}

/* The scratch the two rows ask for over a pass of this shape (the tensor-core band's rotated input rows). */
static int64_t ops_scratch(const Exl3bLayerDesc* d, int64_t x_rows, int64_t top_k, int64_t rows, int64_t* gu_need,
                           int64_t* dn_need) {
    static uint8_t placeholder[256] __attribute__((aligned(256)));
    const Pass s = { placeholder, x_rows, top_k, rows, (const int32_t*)placeholder, (const int32_t*)placeholder,
                     placeholder, placeholder };
    LayerArgs a;
    build_args(d, &s, &a);
    const RadKernelInfo* gu = row_of("moe_exl3_gate_up");
    const RadKernelInfo* dn = row_of("moe_exl3_down");
    *gu_need = gu && gu->scratch ? gu->scratch(&a.gu) : 0;
    *dn_need = dn && dn->scratch ? dn->scratch(&a.dn) : 0;
    return up256(*gu_need) + up256(*dn_need);
}

static void mark(void* const* marks, int i, void* stream) {
    if (marks && marks[i]) exl3b_cuda_mark(marks[i], stream);
}

/* gate_up then down over one pass, with the scratch the rows ask for at this size (within what a carve set aside).
 * live: the ops over the live rows only (exl3b200_moe_op_live; a capacity-sized pass), down writing through
 * row_dst when given. ev: NULL or 3 marks (before gate_up, between, after down). */
static int run_ops(const Exl3bLayerDesc* d, const Pass* s, void* gu_scratch, int64_t gu_bytes, void* dn_scratch,
                   int64_t dn_bytes, int live, const uint64_t* row_dst, void* const* ev, void* stream) {
    LayerArgs a;
    build_args(d, s, &a);
    const RadKernelInfo* gu = row_of("moe_exl3_gate_up");
    const RadKernelInfo* dn = row_of("moe_exl3_down");
    if (!gu || !dn) return RAD_E_SCHEMA;
    const int64_t gu_need = gu->scratch ? gu->scratch(&a.gu) : 0;
    const int64_t dn_need = dn->scratch ? dn->scratch(&a.dn) : 0;
    if (gu_need > gu_bytes || dn_need > dn_bytes) return RAD_E_SCRATCH;
    a.gu.scratch = gu_need > 0 ? gu_scratch : 0;
    a.gu.scratch_bytes = gu_need > 0 ? gu_bytes : 0;
    a.dn.scratch = dn_need > 0 ? dn_scratch : 0;
    a.dn.scratch_bytes = dn_need > 0 ? dn_bytes : 0;
    mark(ev, 0, stream);
    int rc = live ? exl3b200_moe_op_live(&a.gu, 0, 0, stream) : gu->launch(&a.gu, stream);
    if (rc != RAD_OK) return rc;
    mark(ev, 1, stream);
    rc = live ? exl3b200_moe_op_live(&a.dn, 1, row_dst, stream)
              : row_dst ? exl3b200_moe_down_rows(&a.dn, row_dst, stream) : dn->launch(&a.dn, stream);
    if (rc != RAD_OK) return rc;
    mark(ev, 2, stream);
    return RAD_OK;
}

int64_t exl3b200_moe_layer_work_bytes(const Exl3bLayerDesc* d, int64_t max_tokens) {
    if (check_desc(d) != RAD_OK || max_tokens < 1) return -1;
    const int64_t P = max_tokens * d->top_k, E = d->n_local;
    int64_t gu = 0, dn = 0;
    const int64_t ops = ops_scratch(d, max_tokens, d->top_k, P, &gu, &dn);
    return up256(P * 4) + up256(P * 4) + up256(P * 4) + up256((E + 1) * 4) +
           up256(exl3b200_moe_scatter_work_bytes(P, E)) + up256(P * d->width * 2) + up256(P * d->hidden * 2) +
           ops + up256(exl3b200_moe_gather_work_bytes(max_tokens, d->top_k)) + 256;
}

int exl3b200_moe_layer_carve(const Exl3bLayerDesc* d, int64_t max_tokens, void* work, int64_t work_bytes,
                             Exl3bLayerBufs* b) {
    if (!b || !work || check_desc(d) != RAD_OK || max_tokens < 1) return RAD_E_INVAL;
    const int64_t need = exl3b200_moe_layer_work_bytes(d, max_tokens);
    if (need < 0 || work_bytes < need) return RAD_E_SCRATCH;
    const int64_t P = max_tokens * d->top_k, E = d->n_local;
    int64_t gu = 0, dn = 0;
    ops_scratch(d, max_tokens, d->top_k, P, &gu, &dn);
    uint8_t* p = (uint8_t*)(((uintptr_t)work + 255) / 256 * 256);
    memset(b, 0, sizeof *b);
    b->max_tokens = max_tokens;
    b->ids = (int32_t*)p;               p += up256(P * 4);
    b->w = (float*)p;                   p += up256(P * 4);
    b->sorted_tok = (int32_t*)p;        p += up256(P * 4);
    b->expert_offset = (int32_t*)p;     p += up256((E + 1) * 4);
    b->scatter_work = p;                p += up256(exl3b200_moe_scatter_work_bytes(P, E));
    b->h = (uint16_t*)p;                p += up256(P * d->width * 2);
    b->y_rows = (uint16_t*)p;           p += up256(P * d->hidden * 2);
    b->gu_scratch = gu > 0 ? p : 0;     b->gu_scratch_bytes = gu;  p += up256(gu);
    b->dn_scratch = dn > 0 ? p : 0;     b->dn_scratch_bytes = dn;  p += up256(dn);
    b->gather_work = p;
    return RAD_OK;
}

/* router + scatter, then the two ops (ev: NULL or 3 marks around them). */
static int layer_experts(const Exl3bLayerDesc* d, const Exl3bLayerBufs* b, const uint16_t* x, const float* logits,
                         int64_t T, void* const* ev, void* stream) {
    const int rc = exl3b200_router_scatter(logits, T, d->n_expert, d->top_k, b->ids, b->w, d->n_local,
                                           d->expert_base, b->sorted_tok, b->expert_offset, b->scatter_work, stream);
    if (rc != 0) return rc;
    const Pass s = layer_pass(d, b, x, T);
    return run_ops(d, &s, b->gu_scratch, b->gu_scratch_bytes, b->dn_scratch, b->dn_scratch_bytes, 0, 0, ev, stream);
}

int exl3b200_moe_layer_forward(const Exl3bLayerDesc* d, const Exl3bLayerBufs* b, const uint16_t* x,
                               const float* logits, int64_t T, void* out, int out_dtype, void* stream) {
    int rc = check_desc(d);
    if (rc != RAD_OK) return rc;
    if (!b || !x || !logits || !out || T < 0 || T > b->max_tokens) return RAD_E_INVAL;
    if (out_dtype != RAD_F32 && out_dtype != RAD_BF16) return RAD_E_DTYPE;
    if (T == 0) return RAD_OK;
    const int64_t P = T * d->top_k;
    rc = layer_experts(d, b, x, logits, T, 0, stream);
    if (rc != RAD_OK) return rc;
    if (out_dtype == RAD_F32)
        return exl3b200_moe_gather(b->y_rows, d->hidden, b->sorted_tok, P, b->w, T, d->top_k, d->hidden, (float*)out,
                                   b->gather_work, stream);
    return exl3b200_moe_gather_bf16(b->y_rows, d->hidden, b->sorted_tok, P, b->w, T, d->top_k, d->hidden,
                                    (uint16_t*)out, b->gather_work, stream);
}

/* ------------------------------------------------------------------------------------------------------------------
 * The MoE block: the routed layer, the shared expert over every token, the gather folding the shared arm in. */

static int check_block(const Exl3bBlockDesc* d) {
    if (!d) return RAD_E_INVAL;
    int rc = check_desc(&d->routed);
    if (rc == RAD_OK) rc = check_desc(&d->shared);
    if (rc != RAD_OK) return rc;
    const Exl3bLayerDesc* s = &d->shared;
    if (s->n_expert != 1 || s->n_local != 1 || s->expert_base != 0 || s->top_k != 1 || s->hidden != d->routed.hidden)
        return RAD_E_SHAPE;
    if (!d->sgate_w || ((uintptr_t)d->sgate_w & 15)) return RAD_E_INVAL;
    return RAD_OK;
}

int64_t exl3b200_moe_block_work_bytes(const Exl3bBlockDesc* d, int64_t max_tokens) {
    if (check_block(d) != RAD_OK || max_tokens < 1) return -1;
    const int64_t r = exl3b200_moe_layer_work_bytes(&d->routed, max_tokens);
    const int64_t s = exl3b200_moe_layer_work_bytes(&d->shared, max_tokens);
    return r < 0 || s < 0 ? -1 : up256(r) + s + 256;
}

int exl3b200_moe_block_carve(const Exl3bBlockDesc* d, int64_t max_tokens, void* work, int64_t work_bytes,
                             Exl3bBlockBufs* b) {
    if (!b || !work || check_block(d) != RAD_OK || max_tokens < 1) return RAD_E_INVAL;
    const int64_t need = exl3b200_moe_block_work_bytes(d, max_tokens);
    if (need < 0 || work_bytes < need) return RAD_E_SCRATCH;
    const int64_t r = exl3b200_moe_layer_work_bytes(&d->routed, max_tokens);
    uint8_t* p = (uint8_t*)(((uintptr_t)work + 255) / 256 * 256);
    int rc = exl3b200_moe_layer_carve(&d->routed, max_tokens, p, r, &b->routed);
    if (rc != RAD_OK) return rc;
    p += up256(r);
    return exl3b200_moe_layer_carve(&d->shared, max_tokens, p, need - (p - (uint8_t*)work),
                                    &b->shared);
}

int exl3b200_moe_block_forward(const Exl3bBlockDesc* d, const Exl3bBlockBufs* b, const uint16_t* x,
                               const float* logits, int64_t T, void* out, int out_dtype, void* stream) {
    int rc = check_block(d);
    if (rc != RAD_OK) return rc;
    if (!b || !x || !logits || !out || T < 0 || T > b->routed.max_tokens || T > b->shared.max_tokens)
        return RAD_E_INVAL;
    if (out_dtype != RAD_F32 && out_dtype != RAD_BF16) return RAD_E_DTYPE;
    if (T == 0) return RAD_OK;
    const Exl3bLayerDesc* r = &d->routed;
    /* the routed chain, then the shared arm over the same input (every token one row of its one expert) */
    rc = layer_experts(r, &b->routed, x, logits, T, 0, stream);
    if (rc != RAD_OK) return rc;
    rc = exl3b200_identity_routing(T, b->shared.sorted_tok, b->shared.expert_offset, stream);
    if (rc != 0) return rc;
    const Pass s = layer_pass(&d->shared, &b->shared, x, T);
    rc = run_ops(&d->shared, &s, b->shared.gu_scratch, b->shared.gu_scratch_bytes, b->shared.dn_scratch,
                 b->shared.dn_scratch_bytes, 0, 0, 0, stream);
    if (rc != RAD_OK) return rc;
    return exl3b200_moe_gather_fold(b->routed.y_rows, r->hidden, b->routed.sorted_tok, T * r->top_k, b->routed.w, T,
                                    r->top_k, r->hidden, b->shared.y_rows, x, r->hidden, d->sgate_w, out, out_dtype,
                                    b->routed.gather_work, stream);
}

/* ------------------------------------------------------------------------------------------------------------------
 * Expert parallelism over peer memory: the whole step of one rank. Rank r serves experts [r n_local, (r+1) n_local)
 * and routes its own tokens; the window layout and the exchange kernels are exl3b200_p2p.cu's. */

int64_t exl3b200_ep_window_layout(int64_t world, int64_t t_cap, int64_t top_k, int64_t hidden, int64_t* offs) {
    if (!offs || world < 1 || world > 32 || t_cap < 1 || top_k < 1 || top_k > 32 || hidden < 8 || hidden % 8)
        return -1;
    const int64_t p_cap = t_cap * top_k;
    offs[0] = 0;                                                  /* rows  [world][t_cap][hidden] f16 */
    offs[1] = up256(world * t_cap * hidden * 2);                  /* meta  [world][p_cap] u32 */
    offs[2] = offs[1] + up256(world * p_cap * 4);                 /* yback [p_cap][hidden] bf16 */
    offs[3] = offs[2] + up256(p_cap * hidden * 2);                /* ctl   [world][8] u32 */
    offs[4] = offs[3] + up256(world * 32);                        /* done  [2] u32 */
    offs[5] = offs[4] + 256;                                      /* sink  [hidden] bf16 */
    return offs[5] + up256(hidden * 2);
}

static int check_ep(const Exl3bEpDesc* e) {
    if (!e) return RAD_E_INVAL;
    const int rc = check_desc(&e->layer);
    if (rc != RAD_OK) return rc;
    const Exl3bLayerDesc* d = &e->layer;
    if (e->world < 1 || e->world > 32 || e->rank < 0 || e->rank >= e->world || e->max_tokens < 1 ||
        d->n_expert != e->world * d->n_local || d->expert_base != e->rank * d->n_local || d->n_local > 4096 ||
        e->max_tokens >= (1 << 20))
        return RAD_E_SHAPE;
    if (!e->window || !e->peers || !e->epoch || !e->status) return RAD_E_INVAL;
    return RAD_OK;
}

/* The local pass at capacity: every received pair (cap of them) in window rows [world * max_tokens][hidden]. */
static Pass ep_pass(const Exl3bEpDesc* e, const Exl3bEpBufs* b) {
    const Pass s = { (const uint8_t*)e->window + e->offs[0], e->world * e->max_tokens, 1, b->cap, b->sorted_row,
                     b->expert_offset, b->h, b->y_rows ? (void*)b->y_rows : (void*)b->h };
    return s;
}

int64_t exl3b200_ep_step_work_bytes(const Exl3bEpDesc* e) {
    if (check_ep(e) != RAD_OK) return -1;
    const Exl3bLayerDesc* d = &e->layer;
    const int64_t P = e->max_tokens * d->top_k, Q = e->world * P, G = e->world, E = d->n_local;
    int64_t gu = 0, dn = 0;
    const int64_t ops = ops_scratch(d, G * e->max_tokens, 1, Q, &gu, &dn);
    return 6 * up256(P * 4) + up256((G + 1) * 4) + up256(2 * G * 4) + up256((3 * G + 1) * 4) + 6 * up256(Q * 4) +
           up256((E + 1) * 4) + up256(Q * 8) + up256(Q * d->width * 2) +
           (e->fuse_combine ? 0 : up256(Q * d->hidden * 2)) + up256(exl3b200_moe_scatter_work_bytes(P, G)) +
           up256(exl3b200_moe_scatter_work_bytes(Q, E)) + ops +
           up256(exl3b200_moe_gather_work_bytes(e->max_tokens, d->top_k)) + 256;
}

int exl3b200_ep_step_carve(const Exl3bEpDesc* e, void* work, int64_t work_bytes, Exl3bEpBufs* b) {
    if (!b || !work || check_ep(e) != RAD_OK) return RAD_E_INVAL;
    const int64_t need = exl3b200_ep_step_work_bytes(e);
    if (need < 0 || work_bytes < need) return RAD_E_SCRATCH;
    const Exl3bLayerDesc* d = &e->layer;
    const int64_t P = e->max_tokens * d->top_k, Q = e->world * P, G = e->world, E = d->n_local;
    int64_t gu = 0, dn = 0;
    ops_scratch(d, G * e->max_tokens, 1, Q, &gu, &dn);
    uint8_t* p = (uint8_t*)(((uintptr_t)work + 255) / 256 * 256);
    memset(b, 0, sizeof *b);
    b->max_tokens = e->max_tokens;
    b->cap = Q;
    b->ids = (int32_t*)p;               p += up256(P * 4);
    b->w = (float*)p;                   p += up256(P * 4);
    b->dest = (int32_t*)p;              p += up256(P * 4);
    b->sorted_pairs = (int32_t*)p;      p += up256(P * 4);
    b->row_tok = (int32_t*)p;           p += up256(P * 4);
    b->send_meta = (uint32_t*)p;        p += up256(P * 4);
    b->dest_off = (int32_t*)p;          p += up256((G + 1) * 4);
    b->counts = (int32_t*)p;            p += up256(2 * G * 4);
    b->hdr = (int32_t*)p;               p += up256((3 * G + 1) * 4);
    b->pair_e = (int32_t*)p;            p += up256(Q * 4);
    b->pair_row = (int32_t*)p;          p += up256(Q * 4);
    b->dst_rank = (int32_t*)p;          p += up256(Q * 4);
    b->dst_pos = (int32_t*)p;           p += up256(Q * 4);
    b->sorted_pair = (int32_t*)p;       p += up256(Q * 4);
    b->sorted_row = (int32_t*)p;        p += up256(Q * 4);
    b->expert_offset = (int32_t*)p;     p += up256((E + 1) * 4);
    b->row_dst = (uint64_t*)p;          p += up256(Q * 8);
    b->h = (uint16_t*)p;                p += up256(Q * d->width * 2);
    if (!e->fuse_combine) { b->y_rows = (uint16_t*)p;  p += up256(Q * d->hidden * 2); }
    b->scatter_rank = p;                p += up256(exl3b200_moe_scatter_work_bytes(P, G));
    b->scatter_local = p;               p += up256(exl3b200_moe_scatter_work_bytes(Q, E));
    b->gu_scratch = gu > 0 ? p : 0;     b->gu_scratch_bytes = gu;  p += up256(gu);
    b->dn_scratch = dn > 0 ? p : 0;     b->dn_scratch_bytes = dn;  p += up256(dn);
    b->gather_work = p;
    return RAD_OK;
}

int exl3b200_ep_step_forward(const Exl3bEpDesc* e, const Exl3bEpBufs* b, const uint16_t* x, const float* logits,
                             int64_t T, void* out, int out_dtype, void* stream, void* const* marks) {
    int rc = check_ep(e);
    if (rc != RAD_OK) return rc;
    if (!b || !x || !logits || !out || T < 0 || T > b->max_tokens || b->cap != e->world * e->max_tokens *
        e->layer.top_k || (!e->fuse_combine && !b->y_rows))
        return RAD_E_INVAL;
    if (out_dtype != RAD_F32 && out_dtype != RAD_BF16) return RAD_E_DTYPE;
    const Exl3bLayerDesc* d = &e->layer;
    const int64_t k = d->top_k, P = T * k, G = e->world, H = d->hidden, nl = d->n_local, Q = b->cap;
    const int64_t Tc = e->max_tokens, Pc = Tc * k;
    void* const st = stream;
#define EP_TRY(call) do { rc = (call); if (rc != 0) return rc; } while (0)
    mark(marks, 0, st);
    /* every rank advances its epoch once a step, whatever its token count */
    EP_TRY(exl3b200_p2p_begin(e->epoch, st));
    EP_TRY(exl3b200_router_topk(logits, T, d->n_expert, k, b->ids, b->w, st));
    EP_TRY(exl3b200_ep_dest(b->ids, P, nl, G, b->dest, st));
    EP_TRY(exl3b200_moe_scatter(b->dest, P, G, 0, b->sorted_pairs, b->dest_off, b->scatter_rank, st));
    EP_TRY(exl3b200_ep_dedup_scan(b->ids, k, b->sorted_pairs, b->dest_off, P, nl, G, b->send_meta, b->row_tok,
                                  b->counts, st));
    mark(marks, 1, st);
    EP_TRY(exl3b200_p2p_dispatch(x, H, b->row_tok, b->send_meta, b->dest_off, b->counts, P, e->peers, e->offs,
                                 e->rank, G, Tc, Pc, H, e->epoch, st));
    EP_TRY(exl3b200_p2p_wait_dispatch(e->window, e->offs, G, e->epoch, b->hdr, st));
    mark(marks, 2, st);
    EP_TRY(exl3b200_p2p_unpack(e->window, e->offs, b->hdr, G, Tc, Pc, Q, b->pair_e, b->pair_row, b->dst_rank,
                               b->dst_pos, st));
    EP_TRY(exl3b200_moe_scatter(b->pair_e, Q, nl, 0, b->sorted_pair, b->expert_offset, b->scatter_local, st));
    EP_TRY(exl3b200_ep_map(b->sorted_pair, Q, b->pair_row, Q, b->sorted_row, st));
    if (e->fuse_combine)
        EP_TRY(exl3b200_p2p_row_dst(b->sorted_pair, Q, b->dst_rank, b->dst_pos, e->peers, e->offs, e->rank, G, Pc, H,
                                    b->row_dst, st));
    mark(marks, 3, st);
    const Pass s = ep_pass(e, b);
    /* down with the row table names its rows' dtype and width through y but stores every row at row_dst */
    EP_TRY(run_ops(d, &s, b->gu_scratch, b->gu_scratch_bytes, b->dn_scratch, b->dn_scratch_bytes, 1,
                   e->fuse_combine ? b->row_dst : 0, marks ? marks + 7 : 0, st));
    mark(marks, 4, st);
    if (e->fuse_combine)
        EP_TRY(exl3b200_p2p_signal_combine(e->peers, e->offs, e->rank, G, e->epoch, st));
    else
        EP_TRY(exl3b200_p2p_combine(b->y_rows, H, b->sorted_pair, Q, b->dst_rank, b->dst_pos, e->peers, e->offs,
                                    e->rank, G, Pc, H, e->epoch, st));
    EP_TRY(exl3b200_p2p_wait_combine(e->window, e->offs, G, e->epoch, e->status, st));
    mark(marks, 5, st);
    const uint16_t* yback = (const uint16_t*)((const uint8_t*)e->window + e->offs[2]);
    if (out_dtype == RAD_F32)
        EP_TRY(exl3b200_moe_gather(yback, H, b->sorted_pairs, P, b->w, T, k, H, (float*)out, b->gather_work, st));
    else
        EP_TRY(exl3b200_moe_gather_bf16(yback, H, b->sorted_pairs, P, b->w, T, k, H, (uint16_t*)out, b->gather_work,
                                        st));
    mark(marks, 6, st);
#undef EP_TRY
    return RAD_OK;
}

/* ------------------------------------------------------------------------------------------------------------------
 * The width split over peer memory: this rank's slice of every expert, then the partials summed through the
 * windows (exl3b200_tp.cu). */

int64_t exl3b200_tp_window_layout(int64_t world, int64_t max_tokens, int64_t hidden, int64_t* offs) {
    if (!offs || world < 1 || world > 32 || max_tokens < 1 || hidden < 4) return -1;
    const int64_t s_cap = (max_tokens + world - 1) / world;
    offs[0] = 0;                                                  /* part [world][s_cap][hidden] f32 */
    offs[1] = up256(world * s_cap * hidden * 4);                  /* red  [s_cap][hidden] f32 */
    offs[2] = offs[1] + up256(s_cap * hidden * 4);                /* ctl  [world][8] u32 */
    offs[3] = offs[2] + up256(world * 32);                        /* done [4] u32 */
    return offs[3] + 256;
}

int exl3b200_tp_step_forward(const Exl3bTpDesc* t, const Exl3bLayerBufs* b, const uint16_t* x, const float* logits,
                             int64_t T, float* out, int64_t out_pitch, void* stream, void* const* marks) {
    if (!t) return RAD_E_INVAL;
    int rc = check_desc(&t->layer);
    if (rc != RAD_OK) return rc;
    const Exl3bLayerDesc* d = &t->layer;
    if (t->world < 1 || t->world > 32 || t->rank < 0 || t->rank >= t->world || t->max_tokens < 1 ||
        d->n_local != d->n_expert || d->expert_base != 0)
        return RAD_E_SHAPE;
    if (!b || !x || !logits || !out || !t->window || !t->peers || !t->epoch || !t->status || T < 0 ||
        T > t->max_tokens || T > b->max_tokens || out_pitch < d->hidden)
        return RAD_E_INVAL;
    const int64_t k = d->top_k, H = d->hidden, s_cap = (t->max_tokens + t->world - 1) / t->world;
    mark(marks, 0, stream);
    rc = exl3b200_p2p_begin(t->epoch, stream);
    if (rc != 0) return rc;
    if (T > 0) {
        rc = exl3b200_router_scatter(logits, T, d->n_expert, k, b->ids, b->w, d->n_local, 0, b->sorted_tok,
                                     b->expert_offset, b->scatter_work, stream);
        if (rc != 0) return rc;
        mark(marks, 1, stream);
        const Pass s = layer_pass(d, b, x, T);
        rc = run_ops(d, &s, b->gu_scratch, b->gu_scratch_bytes, b->dn_scratch, b->dn_scratch_bytes, 0, 0,
                     marks ? marks + 4 : 0, stream);
        if (rc != RAD_OK) return rc;
    } else {
        mark(marks, 1, stream);
    }
    mark(marks, 2, stream);
    rc = exl3b200_tp_gather_rs(b->y_rows, H, b->sorted_tok, T * k, b->w, T, k, H, b->gather_work, t->peers, t->offs,
                               t->rank, t->world, s_cap, t->epoch, t->status, stream);
    if (rc != 0) return rc;
    rc = exl3b200_tp_reduce(t->peers, t->offs, t->rank, t->world, T, H, s_cap, t->epoch, stream);
    if (rc != 0) return rc;
    rc = exl3b200_tp_pull(t->peers, t->offs, t->rank, t->world, T, H, s_cap, out, out_pitch, t->epoch, t->status,
                          stream);
    if (rc != 0) return rc;
    mark(marks, 3, stream);
    return RAD_OK;
}
