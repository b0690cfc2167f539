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

static void build_args(const Exl3bLayerDesc* d, const Exl3bLayerBufs* b, const void* x, int64_t T, LayerArgs* a) {
    const int64_t E = d->n_local, H = d->hidden, W = d->width, R = T * d->top_k;
    memset(a, 0, sizeof *a);
    int np = 0;
    RadParam* p = a->gu_p;
    p[np++] = (RadParam)RAD_INT("M", T);
    p[np++] = (RadParam)RAD_INT("N", 2 * W);
    p[np++] = (RadParam)RAD_INT("K", H);
    p[np++] = (RadParam)RAD_INT("n_expert", E);
    p[np++] = (RadParam)RAD_INT("top_k", d->top_k);
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
    p[np++] = (RadParam)RAD_INT("top_k", d->top_k);
    p[np++] = (RadParam)RAD_STR("dtype", dtype_name(d->bits_dn));
    p[np++] = (RadParam)RAD_STR("codebook", codebook_name(d->codebook));
    p[np++] = (RadParam)RAD_INT("h_rot", 1);
    const int n_dn = np;
    /* gate_up: a, codes, suh, suh1, svh, dn_suh, sorted_tok, expert_offset, <odd class x5>, h */
    RadTensor* t = a->gu_t;
    tens(&t[0], x, RAD_F16, 2, (int64_t[]){ T, H });
    table(&t[1], d->gu_codes, E, 2 * W, H);
    tens(&t[2], d->suh, RAD_F16, 3, (int64_t[]){ E, 1, H });
    tens(&t[3], d->suh1, RAD_F16, 3, (int64_t[]){ E, 1, H });
    tens(&t[4], d->svh_gu, RAD_F16, 3, (int64_t[]){ E, 2 * W, 1 });
    tens(&t[5], d->dn_suh, RAD_F16, 3, (int64_t[]){ E, 1, W });
    tens(&t[6], b->sorted_tok, RAD_I32, 1, (int64_t[]){ R });
    tens(&t[7], b->expert_offset, RAD_I32, 1, (int64_t[]){ E + 1 });
    tens(&t[13], b->h, RAD_F16, 2, (int64_t[]){ R, W });
    /* down: h, codes, suh, svh, sorted_tok, expert_offset, <odd class x3>, y */
    t = a->dn_t;
    tens(&t[0], b->h, RAD_F16, 2, (int64_t[]){ R, W });
    table(&t[1], d->dn_codes, E, H, W);
    tens(&t[2], d->dn_suh, RAD_F16, 3, (int64_t[]){ E, 1, W });
    tens(&t[3], d->svh_dn, RAD_F16, 3, (int64_t[]){ E, H, 1 });
    tens(&t[4], b->sorted_tok, RAD_I32, 1, (int64_t[]){ R });
    tens(&t[5], b->expert_offset, RAD_I32, 1, (int64_t[]){ E + 1 });
    tens(&t[9], b->y_rows, RAD_BF16, 2, (int64_t[]){ R, H });
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

/* The scratch the two rows ask for at the largest pass (the tensor-core band's rotated input rows). */
static int64_t ops_scratch(const Exl3bLayerDesc* d, int64_t max_tokens, int64_t* gu_need, int64_t* dn_need) {
    static uint8_t placeholder[256] __attribute__((aligned(256)));
    Exl3bLayerBufs b;
    memset(&b, 0, sizeof b);
    b.sorted_tok = (int32_t*)placeholder;
    b.expert_offset = (int32_t*)placeholder;
    b.h = (uint16_t*)placeholder;
    b.y_rows = (uint16_t*)placeholder;
    LayerArgs a;
    build_args(d, &b, placeholder, max_tokens, &a);
    const RadKernelInfo* gu = row_of("moe_exl3_gate_up");
    const RadKernelInfo* dn = row_of("moe_exl3_down");
    *gu_need = gu && gu->scratch ? gu->scratch(&a.gu) : 0;
    *dn_need = dn && dn->scratch ? dn->scratch(&a.dn) : 0;
    return up256(*gu_need) + up256(*dn_need);
}

int64_t exl3b200_moe_layer_work_bytes(const Exl3bLayerDesc* d, int64_t max_tokens) {
    if (check_desc(d) != RAD_OK || max_tokens < 1) return -1;
    const int64_t P = max_tokens * d->top_k, E = d->n_local;
    int64_t gu = 0, dn = 0;
    const int64_t ops = ops_scratch(d, max_tokens, &gu, &dn);
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
    ops_scratch(d, max_tokens, &gu, &dn);
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

int exl3b200_moe_layer_forward(const Exl3bLayerDesc* d, const Exl3bLayerBufs* b, const uint16_t* x,
                               const float* logits, int64_t T, void* out, int out_dtype, void* stream) {
    int rc = check_desc(d);
    if (rc != RAD_OK) return rc;
    if (!b || !x || !logits || !out || T < 0 || T > b->max_tokens) return RAD_E_INVAL;
    if (out_dtype != RAD_F32 && out_dtype != RAD_BF16) return RAD_E_DTYPE;
    if (T == 0) return RAD_OK;
    const int64_t P = T * d->top_k;
    rc = exl3b200_router_scatter(logits, T, d->n_expert, d->top_k, b->ids, b->w, d->n_local, d->expert_base,
                                 b->sorted_tok, b->expert_offset, b->scatter_work, stream);
    if (rc != 0) return rc;
    LayerArgs a;
    build_args(d, b, x, T, &a);
    const RadKernelInfo* gu = row_of("moe_exl3_gate_up");
    const RadKernelInfo* dn = row_of("moe_exl3_down");
    if (!gu || !dn) return RAD_E_SCHEMA;
    /* the scratch each row asks for at this pass size: within what carve set aside for the largest */
    const int64_t gu_need = gu->scratch ? gu->scratch(&a.gu) : 0;
    const int64_t dn_need = dn->scratch ? dn->scratch(&a.dn) : 0;
    if (gu_need > b->gu_scratch_bytes || dn_need > b->dn_scratch_bytes) return RAD_E_SCRATCH;
    a.gu.scratch = gu_need > 0 ? b->gu_scratch : 0;
    a.gu.scratch_bytes = gu_need > 0 ? b->gu_scratch_bytes : 0;
    a.dn.scratch = dn_need > 0 ? b->dn_scratch : 0;
    a.dn.scratch_bytes = dn_need > 0 ? b->dn_scratch_bytes : 0;
    rc = gu->launch(&a.gu, stream);
    if (rc != RAD_OK) return rc;
    rc = dn->launch(&a.dn, stream);
    if (rc != RAD_OK) return rc;
    if (out_dtype == RAD_F32)
        return exl3b200_moe_gather(b->y_rows, d->hidden, b->sorted_tok, P, b->w, T, d->top_k, d->hidden, (float*)out,
                                   b->gather_work, stream);
    return exl3b200_moe_gather_bf16(b->y_rows, d->hidden, b->sorted_tok, P, b->w, T, d->top_k, d->hidden,
                                    (uint16_t*)out, b->gather_work, stream);
}
