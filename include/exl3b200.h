/* exl3b200.h -- the C ABI of libexl3b200.so, the B200 (sm_100a) library of the EXL3 routed-expert ops.
 *
 * 1. THE PLUGIN BOUNDARY. The library is a radiance kernel plugin (ABI 17), exporting exactly what the
 *    reference's device library exports (kernels/exl3r4d/rows.c:524-550) and the reference library's
 *    schemas (kernels/exl3ref/rows.c:249-258): the engine dlopens it, reads the schemas and the rows, and
 *    calls a row's `launch(const RadArgs*, RadStream)` with device pointers and a cudaStream_t. The rows
 *    serve moe_exl3_gate_up, moe_exl3_down, moe_exl3_prep_gu, moe_exl3_gate_up_down and their _mod4 forms
 *    (include/exl3_abi.h:160-288), every K 2..8 and every codebook.
 *
 * 2. DIRECT ENTRY POINTS (plain pointers and sizes) for a caller that holds its operands itself: the
 *    decode, the relayout, and the routing steps either side of the ops (router, scatter, gather).
 *
 * Every entry returns 0 (RAD_OK) or a negative status; nothing is written on a refusal. Device work is
 * enqueued on `stream` (a cudaStream_t; null = the legacy default stream) and is asynchronous: no entry
 * point on a launch path allocates, synchronises or reads the environment. */
#ifndef EXL3B200_H
#define EXL3B200_H

#include <stdint.h>

#include "rad_abi.h"
#include "rad_plugin.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ 1. the plugin exports */

/* == RAD_ABI_VERSION (kernels/exl3ref/rows.c:249). */
uint32_t             rad_plugin_abi_version(void);
/* {RAD_PLUGIN_KERNEL, "exl3b200", version, description, "sm_100a"} (kernels/exl3r4d/rows.c:528-534). */
const RadPluginInfo* rad_plugin_info(void);
/* The eight EXL3 schemas, identical to the reference's (include/exl3_abi.h:366-627;
 * kernels/exl3ref/rows.c:253-254). */
int                  rad_kernel_schema_count(void);
const RadOpSchema*   rad_kernel_schema_at(int i);
/* The device rows (kernels/exl3r4d/rows.c:369-520 are the rows these replace). */
int                  rad_kernel_count(void);
const RadKernelInfo* rad_kernel_at(int i);
/* Every row may run concurrently with itself: no state survives a launch (kernels/exl3r4d/rows.c:550). */
int                  rad_kernel_concurrent(int i);

/* ------------------------------------------------------------------ 2. direct entry points */

/* The stored form of a codes plane: the tile-stream record. Replaces the relayout / unrelayout hooks'
 * conversions (kernels/exl3r4d/layout.c:33-140; common/exl3_layout.h:31-42). Host memory. */
int exl3b200_codes_to_record(const uint8_t* codes, int64_t row_bytes, int64_t rows, int64_t cols, int bits,
                             uint16_t* record);
int exl3b200_record_to_codes(const uint16_t* record, int64_t rows, int64_t cols, int bits, uint8_t* codes,
                             int64_t row_bytes);

/* W_hat of one [rows, cols] record as fp16 bits, [rows][cols] (radiance's [n][k] view), on the device:
 * the decode every kernel runs, bit-exact with common/exl3_decode.c exl3_decode_what_rows
 * (common/exl3_decode.h:157-160). bits 1..8, codebook 0 3inst / 1 mcg / 2 mul1. */
int exl3b200_decode_what(const void* record, int64_t rows, int64_t cols, int bits, int codebook, void* w_hat,
                         void* stream);

/* Routing, the steps either side of the ops (the engine's router_topk / moe_scatter / moe_gather, whose
 * contract include/exl3_abi.h:90-158 states; docs/OPS-exl3.md:195-196 for the gather):
 *   router_topk:  logits f32 [n_tok, n_expert] -> softmax over all experts, the top_k largest (ties to the
 *                 lower id) as ids i32 [n_tok, top_k] and their probabilities w f32 [n_tok, top_k], in
 *                 descending order. n_expert <= 4096, top_k <= 32.
 *   moe_scatter:  a stable counting sort of the flattened pairs t*top_k + s by expert id - expert_base;
 *                 ids outside [0, n_expert) dropped; sorted_tok i32 [n_pairs] (-1 past the live count),
 *                 expert_offset i32 [n_expert + 1]. `work` is caller-provided device memory of
 *                 exl3b200_moe_scatter_work_bytes() bytes.
 *   moe_gather:   y f32 [n_tok][width] = sum over slots ascending of w * bf16 row of that slot's sorted row
 *                 (a dropped slot adds nothing); `rows` bf16 with row pitch `row_pitch` elements. `work` is
 *                 caller-provided device memory of exl3b200_moe_gather_work_bytes() bytes. Sizes whose pair
 *                 count n_tok * top_k would pass INT32_MAX are refused (RAD_E_SHAPE) before anything is enqueued. */
int     exl3b200_router_topk(const float* logits, int64_t n_tok, int64_t n_expert, int64_t top_k, int32_t* ids,
                             float* w, void* stream);
int64_t exl3b200_moe_scatter_work_bytes(int64_t n_pairs, int64_t n_expert);
int     exl3b200_moe_scatter(const int32_t* ids, int64_t n_pairs, int64_t n_expert, int64_t expert_base,
                             int32_t* sorted_tok, int32_t* expert_offset, void* work, void* stream);
/* router_topk over n_route experts then moe_scatter of its ids over [expert_base, expert_base + n_expert), as the
 * two calls above (the same results to the bit), in ONE launch when the tokens are few (n_tok <= 32, n_route <=
 * 512, n_expert <= 1024): the decode-size step's router and sort in one block. `work` as moe_scatter's. No
 * counterpart in the reference (the engine issues the two ops). */
int     exl3b200_router_scatter(const float* logits, int64_t n_tok, int64_t n_route, int64_t top_k, int32_t* ids,
                                float* w, int64_t n_expert, int64_t expert_base, int32_t* sorted_tok,
                                int32_t* expert_offset, void* work, void* stream);
int64_t exl3b200_moe_gather_work_bytes(int64_t n_tok, int64_t top_k);
int     exl3b200_moe_gather(const uint16_t* rows, int64_t row_pitch, const int32_t* sorted_tok, int64_t n_rows,
                            const float* w, int64_t n_tok, int64_t top_k, int64_t width, float* y, void* work,
                            void* stream);

/* moe_gather writing y as bf16 (the f32 sum of each element rounded to nearest even): the layer's output in the
 * engine's hidden-state type (the MoE block adds it to a bf16 stream, rad_block_moe_exl3.h:1660-1667). Same
 * arguments and refusals as exl3b200_moe_gather, y uint16 bf16 bits [n_tok][width]. */
int     exl3b200_moe_gather_bf16(const uint16_t* rows, int64_t row_pitch, const int32_t* sorted_tok, int64_t n_rows,
                                 const float* w, int64_t n_tok, int64_t top_k, int64_t width, uint16_t* y, void* work,
                                 void* stream);

/* moe_gather for a caller that cannot allocate device memory -- one whose memory is fixed up front (a serving
 * engine that owns a preallocated pool and forbids cudaMalloc on its launch path, a process running under a
 * strict device-memory budget, code that must not grow the CUDA allocator's footprint). No counterpart in the
 * reference: it is this library's own addition. Same arguments and result as exl3b200_moe_gather without `work`:
 * the inverse pair -> row map lives in a fixed 1 MiB device array inside this library, so n_tok * top_k must be at
 * most 262,144 (RAD_E_SHAPE beyond, nothing enqueued; the limit is tested factor by factor, so huge arguments
 * whose product would wrap around are refused too). The first call on each device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current; make that first call before any stream capture. The
 * call allocates nothing (no cudaMalloc, no cudaFree, no allocating library routine). Every call shares the one
 * array per device: calls that overlap on the GPU (two streams, or two threads) race and must be serialised by
 * the caller. */
int     exl3b200_moe_gather_noalloc(const uint16_t* rows, int64_t row_pitch, const int32_t* sorted_tok,
                                    int64_t n_rows, const float* w, int64_t n_tok, int64_t top_k, int64_t width,
                                    float* y, void* stream);

/* One routed-MoE layer, the sequence the engine's MoE block issues for a pass (rad_block_moe_exl3.h:1763-1900):
 * router_topk + moe_scatter -> moe_exl3_gate_up (h_rot 1) -> moe_exl3_down (h_rot 1) -> moe_gather, the two
 * expert ops through this library's plugin rows with RadArgs built in C. The caller holds the weights:
 *   gu_codes, dn_codes  device tables of n_local u64 addresses, each an expert's STORED record (the layout hook's
 *                       form: exl3b200_codes_to_record of gate's rows then up's for gate_up)
 *   suh, suh1 f16 [n_local][hidden]; svh_gu f16 [n_local][2 width]; dn_suh f16 [n_local][width];
 *   svh_dn f16 [n_local][hidden]   (stacked, dense)
 * Tokens route over n_expert experts; this caller serves [expert_base, expert_base + n_local) (the rest dropped).
 * exl3b200_moe_layer_work_bytes sizes ONE device block for up to max_tokens tokens a pass; the caller allocates it
 * once and exl3b200_moe_layer_carve cuts it into the buffers (ids, w, sorted_tok, expert_offset, h, the bf16 down
 * rows, the rows' scratch, the gather's map). exl3b200_moe_layer_forward then allocates, synchronises and reads
 * nothing on the host: it enqueues the kernels on `stream` and writes out [T][hidden] as f32 (out_dtype RAD_F32) or
 * bf16 (RAD_BF16). No counterpart in the reference (the engine drives the ops); the ops' results are the rows'. */
typedef struct Exl3bLayerDesc {
    int64_t     n_expert, n_local, expert_base;
    int64_t     hidden, width, top_k;
    int32_t     bits_gu, bits_dn, codebook;   /* codebook 0 3inst, 1 mcg, 2 mul1 */
    int32_t     pad0;
    const void* gu_codes;
    const void* dn_codes;
    const void* suh;
    const void* suh1;
    const void* svh_gu;
    const void* dn_suh;
    const void* svh_dn;
} Exl3bLayerDesc;
typedef struct Exl3bLayerBufs {
    int64_t   max_tokens;
    int32_t*  ids;            /* [max_tokens][top_k] */
    float*    w;              /* [max_tokens][top_k] */
    int32_t*  sorted_tok;     /* [max_tokens * top_k] */
    int32_t*  expert_offset;  /* [n_local + 1] */
    void*     scatter_work;
    uint16_t* h;              /* f16 [max_tokens * top_k][width] */
    uint16_t* y_rows;         /* bf16 [max_tokens * top_k][hidden] */
    void*     gu_scratch;
    int64_t   gu_scratch_bytes;
    void*     dn_scratch;
    int64_t   dn_scratch_bytes;
    void*     gather_work;
} Exl3bLayerBufs;
int64_t exl3b200_moe_layer_work_bytes(const Exl3bLayerDesc* desc, int64_t max_tokens);
int     exl3b200_moe_layer_carve(const Exl3bLayerDesc* desc, int64_t max_tokens, void* work, int64_t work_bytes,
                                 Exl3bLayerBufs* bufs);
int     exl3b200_moe_layer_forward(const Exl3bLayerDesc* desc, const Exl3bLayerBufs* bufs, const uint16_t* x,
                                   const float* logits, int64_t n_tok, void* out, int out_dtype, void* stream);

/* The MoE block pass without the engine (architectures/qwen4exp_exl3/rad_block_moe_exl3.h:1763-1967): the routed
 * layer beside the shared expert, the gather folding the shared arm in through its one-column sigmoid gate, as the
 * engine's moe_gather with act "sigmoid" does (rad_block_moe_exl3.h:1535-1548, 1961-1965):
 *   out[t] = sum over t's routed slots, ascending, of w * down row  +  sigmoid(g[t]) * shared(x[t]),
 *   g[t] = sum over h of x[t][h] * sgate_w[h] (f32),
 * the shared term added as one more weighted row (product, then sum, each rounded in f32). shared = the shared
 * expert's gate_up (h_rot 1) then down (h_rot 1) through the same plugin rows (n_expert 1, every token its own sorted
 * row). desc->shared: n_expert = n_local = 1, expert_base 0, top_k 1, hidden = desc->routed.hidden, its own width and
 * bitrates; sgate_w f16 [hidden], 16-byte aligned. Buffers: one device block (exl3b200_moe_block_work_bytes), cut by
 * exl3b200_moe_block_carve into the routed layer's and the shared expert's Exl3bLayerBufs (shared.y_rows is the
 * shared arm's bf16 output). The forward enqueues only. Not built here: the protected experts (the reference serves
 * them with FP8 grouped GEMMs over the trailing run of the offsets) and the norm and residual add around the block.
 *   exl3b200_moe_gather_fold: the fold alone (rows, sout, x, gate_w, y 16-byte aligned; row_pitch, width, x_cols
 *     multiples of 8; y_dtype RAD_F32 or RAD_BF16; work as exl3b200_moe_gather's).
 *   exl3b200_identity_routing: sorted_tok[i] = i for i < n_tok, expert_offset = {0, n_tok} (the shared expert's). */
typedef struct Exl3bBlockDesc {
    Exl3bLayerDesc  routed;
    Exl3bLayerDesc  shared;
    const void*     sgate_w;
} Exl3bBlockDesc;
typedef struct Exl3bBlockBufs {
    Exl3bLayerBufs  routed;
    Exl3bLayerBufs  shared;
} Exl3bBlockBufs;
int64_t exl3b200_moe_block_work_bytes(const Exl3bBlockDesc* desc, int64_t max_tokens);
int     exl3b200_moe_block_carve(const Exl3bBlockDesc* desc, int64_t max_tokens, void* work, int64_t work_bytes,
                                 Exl3bBlockBufs* bufs);
int     exl3b200_moe_block_forward(const Exl3bBlockDesc* desc, const Exl3bBlockBufs* bufs, const uint16_t* x,
                                   const float* logits, int64_t n_tok, void* out, int out_dtype, void* stream);
int     exl3b200_moe_gather_fold(const uint16_t* rows, int64_t row_pitch, const int32_t* sorted_tok, int64_t n_rows,
                                 const float* w, int64_t n_tok, int64_t top_k, int64_t width, const uint16_t* sout,
                                 const uint16_t* x, int64_t x_cols, const uint16_t* gate_w, void* y, int y_dtype,
                                 void* work, void* stream);
int     exl3b200_identity_routing(int64_t n_tok, int32_t* sorted_tok, int32_t* expert_offset, void* stream);

/* Expert parallelism (one process a GPU; expert e held by rank e / n_local; no counterpart in the reference,
 * which runs on one device -- the engine's EP plumbing would call these around its all-to-alls):
 *   ep_pack:      after moe_scatter over ALL n_local * world experts (sorted_pairs, expert_offset), for sorted
 *                 row j with pair p = sorted_pairs[j] >= 0: send_x[j] = x row p / top_k (hidden f16, row pitch
 *                 x_pitch elements), send_e[j] = ids[p] % n_local; send_counts[r] = the pairs bound for rank r
 *                 (expert_offset[(r+1)*n_local] - expert_offset[r*n_local]). hidden and x_pitch multiples of 8,
 *                 x and send_x 16-byte aligned.
 *   rows_scatter: dst row idx[j] = src row j for j < n_rows (rows of row_bytes, pitches in bytes, all multiples
 *                 of 16); idx outside [0, n_dst) skipped. Puts the down rows of the received pairs back into
 *                 arrival order before the all-to-all that returns them. */
int     exl3b200_ep_pack(const uint16_t* x, int64_t x_pitch, const int32_t* ids, int64_t top_k,
                         const int32_t* sorted_pairs, int64_t n_pairs, const int32_t* expert_offset, int64_t n_local,
                         int64_t world, int64_t hidden, uint16_t* send_x, int32_t* send_e, int32_t* send_counts,
                         void* stream);
int     exl3b200_rows_scatter(const void* src, int64_t src_pitch, const int32_t* idx, int64_t n_rows,
                              int64_t row_bytes, void* dst, int64_t dst_pitch, int64_t n_dst, void* stream);
/* The deduplicated dispatch (one row a distinct (token, rank), every pair still its own combine row):
 *   ep_dest:       dest[p] = ids[p] / n_local, -1 for a dropped slot (sort the pairs by it with moe_scatter over
 *                  `world` "experts": stable, so each rank's pairs come out in token order).
 *   ep_pack_dedup: for rank d's pairs sorted_pairs[dest_off[d] .. dest_off[d+1]) (n_pairs in all): the first
 *                  pair of each token makes row r of rank d (r = the rank's rows so far); row r's token goes to
 *                  row_tok[dest_off[d] + r] (scratch, n_pairs ints) and its x row to send_x[(rows of ranks before
 *                  d) + r]; pair j's meta is (r << 12) | (ids % n_local); counts[2d] = rows, counts[2d+1] = pairs.
 *                  n_local <= 4096, fewer than 2^20 tokens.
 *   ep_unpack:     received pairs (concatenated by source, recv_counts as counts above): pair q's local expert and
 *                  its row among the received rows (rows before its source + its r).
 *   ep_map:        out[i] = table[idx[i]] (-1 outside the table): the token row of each sorted pair. */
int     exl3b200_ep_dest(const int32_t* ids, int64_t n_pairs, int64_t n_local, int64_t world, int32_t* dest,
                         void* stream);
int     exl3b200_ep_pack_dedup(const uint16_t* x, int64_t x_pitch, const int32_t* ids, int64_t top_k,
                               const int32_t* sorted_pairs, const int32_t* dest_off, int64_t n_pairs, int64_t n_local,
                               int64_t world, int64_t hidden, uint16_t* send_x, uint32_t* send_meta,
                               int32_t* row_tok, int32_t* counts, void* stream);
int     exl3b200_ep_unpack(const uint32_t* meta, int64_t n_pairs, const int32_t* recv_counts, int64_t world,
                           int32_t* expert, int32_t* row, void* stream);
/* ep_pack_dedup's first step alone (send_meta, row_tok, counts; no rows copied): for the peer-memory dispatch. */
int     exl3b200_ep_dedup_scan(const int32_t* ids, int64_t top_k, const int32_t* sorted_pairs, const int32_t* dest_off,
                               int64_t n_pairs, int64_t n_local, int64_t world, uint32_t* send_meta, int32_t* row_tok,
                               int32_t* counts, void* stream);

/* Expert parallelism over peer memory (no collective library on the data path). Each rank owns a "window",
 * allocated here (device memory, zeroed) and exported by a 64-byte CUDA IPC handle that every other rank maps.
 * Every window has the same layout, byte offsets offs[6] = {rows, meta, yback, ctl, done, sink}:
 *   rows  [world][t_cap][hidden] f16, meta [world][p_cap] u32   what each source sent here (its own segment)
 *   yback [p_cap][hidden] bf16                                    the down row of each pair this rank sent
 *   ctl   [world][8] u32, done [2] u32                            epoch flags and counts; last-block counters
 *   sink  [H] bf16                                                where a row that would fall outside goes
 * peers[world] = every rank's window base as this rank maps it (its own for itself).
 *   p2p_dispatch:      after ep_dedup_scan: pair metas and the deduplicated token rows straight into the owners'
 *                      windows, then each owner's dispatch flag (epoch) with the counts.
 *   p2p_wait_dispatch: waits (bounded: exl3b200_set_peer_wait_ns) for every source's flag; hdr[3s .. 3s+2] =
 *                      rows, pairs, base of source s; hdr[3 world] = 0, or -1 if a wait gave up (the error word
 *                      is set too).
 *   p2p_unpack:        the received pairs (source-major): local expert, row in the window's rows, and where the
 *                      pair's down row returns (source rank, position).
 *   p2p_combine:       each sorted down row straight into its source's yback, then each source's combine flag.
 *   p2p_wait_combine:  waits (bounded) for every owner's combine flag; status[0] = 0 or -1.
 *   The combine fused into down instead of p2p_combine: p2p_row_dst (each sorted row's destination address in
 *   its source's window), exl3b200_moe_down_rows with that table (down's epilogue stores each row straight into
 *   the source over NVLink, fenced at system scope), then p2p_signal_combine (the flags).
 * Ranks call the same steps in the same order (the epoch advances once a step on every rank). No counterpart in the
 * reference (one device). */
int     exl3b200_ep_window_alloc(int64_t bytes, void** ptr);
int     exl3b200_ep_window_free(void* ptr);
int     exl3b200_ep_window_handle(void* ptr, void* handle64);
int     exl3b200_ep_window_open(const void* handle64, void** ptr);
int     exl3b200_ep_window_close(void* ptr);
int     exl3b200_p2p_dispatch(const uint16_t* x, int64_t x_pitch, const int32_t* row_tok, const uint32_t* meta,
                              const int32_t* dest_off, const int32_t* counts, int64_t n_slots, const uint64_t* peers,
                              const int64_t* offs, int64_t self, int64_t world, int64_t t_cap, int64_t p_cap,
                              int64_t hidden, const uint32_t* epoch, void* stream);
int     exl3b200_p2p_wait_dispatch(void* own, const int64_t* offs, int64_t world, const uint32_t* epoch,
                                   int32_t* hdr, void* stream);
int     exl3b200_p2p_unpack(const void* own, const int64_t* offs, const int32_t* hdr, int64_t world, int64_t t_cap,
                            int64_t p_cap, int64_t n_pairs, int32_t* expert, int32_t* row, int32_t* dst_rank,
                            int32_t* dst_pos, void* stream);
int     exl3b200_p2p_combine(const uint16_t* y_rows, int64_t y_pitch, const int32_t* sorted_pair, int64_t n_rows,
                             const int32_t* dst_rank, const int32_t* dst_pos, const uint64_t* peers,
                             const int64_t* offs, int64_t self, int64_t world, int64_t p_cap, int64_t hidden,
                             const uint32_t* epoch, void* stream);
int     exl3b200_p2p_wait_combine(const void* own, const int64_t* offs, int64_t world, const uint32_t* epoch,
                                  int32_t* status, void* stream);
int     exl3b200_p2p_row_dst(const int32_t* sorted_pair, int64_t n_rows, const int32_t* dst_rank,
                             const int32_t* dst_pos, const uint64_t* peers, const int64_t* offs, int64_t self,
                             int64_t world, int64_t p_cap, int64_t hidden, uint64_t* row_dst, void* stream);
int     exl3b200_p2p_signal_combine(const uint64_t* peers, const int64_t* offs, int64_t self, int64_t world,
                                    const uint32_t* epoch, void* stream);
/* The step's epoch lives in device memory (epoch[0], zero at set-up): p2p_begin bumps it first thing a step, and
 * every p2p step reads it there -- so a step captured in a CUDA graph replays with a fresh epoch each time. */
int     exl3b200_p2p_begin(uint32_t* epoch, void* stream);
/* moe_exl3_gate_up (down = 0) / moe_exl3_down (down = 1) over the live rows only: rows outside
 * [expert_offset[0], expert_offset[n_expert]) are left untouched instead of zeroed, so a caller may pass a
 * capacity-sized pass whose live count is known only on the device; down may write through row_dst. */
int     exl3b200_moe_op_live(const RadArgs* args, int down, const uint64_t* row_dst, void* stream);
/* moe_exl3_down with f16 output rows: the same operands (y f16 instead of bf16), checks and arithmetic as the
 * moe_exl3_down row, the f32 result times svh rounded once to f16. The single EXL3 linear of [M, K] f16 rows to
 * [M, N] f16 (n_expert 1, top_k 1, every row routed to the one expert). Its scratch (args->scratch) is sized by
 * exl3b200_moe_down_f16_scratch: the down row's own hook refuses an f16 y. Without it the launch runs the decode
 * band whatever the row count (the two bands agree within the ops' tolerance, not bit for bit). No counterpart in
 * the reference, whose down writes bf16 (kernels/exl3ref/ref.c:97-102). */
int     exl3b200_moe_down_f16(const RadArgs* args, void* stream);
int64_t exl3b200_moe_down_f16_scratch(const RadArgs* args);
/* moe_exl3_down (same RadArgs and checks as the row's launch) writing output row i at row_dst[i] (a device table
 * of row addresses, possibly in a peer's memory) instead of y + i * pitch. No counterpart in the reference. */
int     exl3b200_moe_down_rows(const RadArgs* args, const uint64_t* row_dst, void* stream);
int     exl3b200_ep_map(const int32_t* idx, int64_t n, const int32_t* table, int64_t n_table, int32_t* out,
                        void* stream);

/* The width ("column-block") tensor split over peer memory: the engine's all_reduce after the layer's partial
 * gather (architectures/qwen4exp_exl3/rad_block_moe_exl3.h:438-470, every rank holding whole 128-column blocks of
 * every expert's width and gathering a PARTIAL of the output), fused into the gather as a reduce-scatter then an
 * all-gather over NVLink. Windows come from exl3b200_ep_window_* as above; layout offs[4] = {part, red, ctl, done}:
 *   part [world][s_cap][H] f32   each source's partials of this rank's token slice
 *   red  [s_cap][H] f32          this rank's slice, reduced
 *   ctl  [world][8] u32, done [4] u32
 * Tokens are cut into world slices of s = ceil(n_tok / world) rows (s <= s_cap); rank o reduces slice o.
 *   tp_gather_rs: the gather (exl3b200_moe_gather's arithmetic over this rank's y rows), each token's partial
 *                 stored into its owner's part segment; then every owner's partials flag. status[0] = 0.
 *   tp_reduce:    waits (bounded) for every source's flag; sums this rank's slice over the sources in
 *                 ascending order into red; then every rank's reduced flag (held back if a wait gave up).
 *   tp_pull:      waits (bounded) for every owner's reduced flag; out[t] = the owner's red row (f32, row pitch
 *                 out_pitch floats); status[0] = -1 if a wait gave up (the error word is set too).
 * Every rank ends with the same bits; at world 1 they are exl3b200_moe_gather's. Ranks pass the same n_tok and call
 * the steps in the same order, after exl3b200_p2p_begin on their own epoch word. */
int     exl3b200_tp_gather_rs(const uint16_t* rows, int64_t row_pitch, const int32_t* sorted_tok, int64_t n_rows,
                              const float* w, int64_t n_tok, int64_t top_k, int64_t width, void* work,
                              const uint64_t* peers, const int64_t* offs, int64_t self, int64_t world, int64_t s_cap,
                              const uint32_t* epoch, int32_t* status, void* stream);
int     exl3b200_tp_reduce(const uint64_t* peers, const int64_t* offs, int64_t self, int64_t world, int64_t n_tok,
                           int64_t width, int64_t s_cap, const uint32_t* epoch, void* stream);
int     exl3b200_tp_pull(const uint64_t* peers, const int64_t* offs, int64_t self, int64_t world, int64_t n_tok,
                         int64_t width, int64_t s_cap, float* out, int64_t out_pitch, const uint32_t* epoch,
                         int32_t* status, void* stream);

/* Whole multi-GPU steps driven from C (one process a GPU; every rank calls the same entries in the same order). The
 * windows' layouts:
 *   exl3b200_ep_window_layout: the expert-parallel window for up to t_cap tokens a rank of top_k slots (p_cap =
 *     t_cap * top_k); offs[6] = {rows, meta, yback, ctl, done, sink}; returns the bytes to allocate (-1: refused).
 *   exl3b200_tp_window_layout: the width split's window for up to max_tokens tokens a step (s_cap =
 *     ceil(max_tokens / world) rows a slice); offs[4] = {part, red, ctl, done}; returns the bytes (-1: refused).
 * The expert-parallel step: exl3b200_ep_step_work_bytes sizes ONE device block (the routing, the received pairs at
 * capacity world * max_tokens * top_k, h, the row table, the ops' scratch, the gather's map) and
 * exl3b200_ep_step_carve cuts it; exl3b200_ep_step_forward then enqueues the whole step on `stream` and reads nothing
 * on the host -- p2p_begin, router_topk, ep_dest, the scatter over ranks, ep_dedup_scan, p2p_dispatch,
 * p2p_wait_dispatch, p2p_unpack, the local scatter, ep_map, then gate_up and down over the live rows through
 * exl3b200_moe_op_live (down writing each row into its source's window when fuse_combine, else p2p_combine),
 * p2p_wait_combine and the gather of the returned rows into out [n_tok][hidden] (RAD_F32 or RAD_BF16) -- so the
 * step can be captured in a CUDA graph. desc->layer describes this rank's experts: n_expert every rank's together
 * (world * n_local), expert_base = rank * n_local, the weight tables this rank's n_local experts. `epoch` (a device
 * u32, zero at set-up, advanced once a step) and `status` (a device i32: 0, or -1 once a combine wait gave up) are
 * the caller's; bufs->hdr[3 world] is the dispatch wait's status. `marks`: NULL, or 10 cudaEvent_t (NULL entries
 * skipped) recorded on the stream at the step's boundaries: 0 start, 1 after the dedup scan, 2 after the dispatch
 * wait, 3 after the local sort, 4 after down, 5 after the combine wait, 6 after the gather; 7, 8, 9 before gate_up,
 * between the ops, after down.
 * The width-split step: exl3b200_tp_step_forward runs this rank's slice of every expert (desc->layer: width = the
 * slice's columns, n_local = n_expert) over the layer buffers of exl3b200_moe_layer_carve, then sums the ranks'
 * partials over peer memory (tp_gather_rs, tp_reduce, tp_pull) into out (f32, row pitch out_pitch floats); every
 * rank passes the same x, logits and n_tok. marks: NULL or 7 events -- 0 start, 1 routed, 2 after down, 3 summed;
 * 4, 5, 6 before gate_up, between the ops, after down.
 * No counterpart in the reference (one device; the engine drives the ops and its all_reduce). */
typedef struct Exl3bEpDesc {
    Exl3bLayerDesc  layer;
    int64_t         rank, world;
    int64_t         max_tokens;     /* tokens a rank routes a step, at most (the window's t_cap) */
    int32_t         fuse_combine;   /* 1: down stores each row straight into its source's window */
    int32_t         pad0;
    void*           window;         /* this rank's window (exl3b200_ep_window_alloc) */
    const uint64_t* peers;          /* device [world]: every rank's window as this rank maps it */
    int64_t         offs[6];        /* exl3b200_ep_window_layout */
    uint32_t*       epoch;
    int32_t*        status;
} Exl3bEpDesc;
typedef struct Exl3bEpBufs {
    int64_t   max_tokens, cap;      /* cap = world * max_tokens * top_k: the received pairs at most */
    int32_t*  ids;                  /* [max_tokens][top_k] */
    float*    w;                    /* [max_tokens][top_k] */
    int32_t*  dest;                 /* [max_tokens * top_k] owner rank of each slot */
    int32_t*  sorted_pairs;         /* [max_tokens * top_k] slots by owner rank, token order inside */
    int32_t*  row_tok;              /* [max_tokens * top_k] */
    uint32_t* send_meta;            /* [max_tokens * top_k] */
    int32_t*  dest_off;             /* [world + 1] */
    int32_t*  counts;               /* [2 world]: rows, pairs sent to each rank */
    int32_t*  hdr;                  /* [3 world + 1]: rows, pairs, base from each source; [3 world] wait status */
    int32_t*  pair_e;               /* [cap] each received pair's local expert (-1 past the live count) */
    int32_t*  pair_row;             /* [cap] its row in the window's rows */
    int32_t*  dst_rank;             /* [cap] */
    int32_t*  dst_pos;              /* [cap] */
    int32_t*  sorted_pair;          /* [cap] received pairs by local expert */
    int32_t*  sorted_row;           /* [cap] their token rows (the ops' sorted_tok) */
    int32_t*  expert_offset;        /* [n_local + 1] */
    uint64_t* row_dst;              /* [cap] */
    uint16_t* h;                    /* f16 [cap][width] */
    uint16_t* y_rows;               /* bf16 [cap][hidden] when !fuse_combine, else NULL */
    void*     scatter_rank;
    void*     scatter_local;
    void*     gu_scratch;
    int64_t   gu_scratch_bytes;
    void*     dn_scratch;
    int64_t   dn_scratch_bytes;
    void*     gather_work;
} Exl3bEpBufs;
typedef struct Exl3bTpDesc {
    Exl3bLayerDesc  layer;
    int64_t         rank, world;
    int64_t         max_tokens;     /* tokens a step, at most */
    void*           window;
    const uint64_t* peers;
    int64_t         offs[4];        /* exl3b200_tp_window_layout */
    uint32_t*       epoch;
    int32_t*        status;         /* 0, or -1 once a wait gave up */
} Exl3bTpDesc;
int64_t exl3b200_ep_window_layout(int64_t world, int64_t t_cap, int64_t top_k, int64_t hidden, int64_t* offs);
int64_t exl3b200_tp_window_layout(int64_t world, int64_t max_tokens, int64_t hidden, int64_t* offs);
int64_t exl3b200_ep_step_work_bytes(const Exl3bEpDesc* desc);
int     exl3b200_ep_step_carve(const Exl3bEpDesc* desc, void* work, int64_t work_bytes, Exl3bEpBufs* bufs);
int     exl3b200_ep_step_forward(const Exl3bEpDesc* desc, const Exl3bEpBufs* bufs, const uint16_t* x,
                                 const float* logits, int64_t n_tok, void* out, int out_dtype, void* stream,
                                 void* const* marks);
int     exl3b200_tp_step_forward(const Exl3bTpDesc* desc, const Exl3bLayerBufs* bufs, const uint16_t* x,
                                 const float* logits, int64_t n_tok, float* out, int64_t out_pitch, void* stream,
                                 void* const* marks);

/* How long a kernel that waits on another rank's flag (p2p_wait_dispatch, p2p_wait_combine, tp_reduce, tp_pull)
 * waits before it gives up, sets its status and the error word, and returns: `ns` nanoseconds, or the default 5 s
 * for ns <= 0 (more than 600 s is refused, RAD_E_INVAL). Process-wide; each launch reads it when it is enqueued
 * (a CUDA graph keeps the value it was captured with). A short limit lets a caller -- or a test, with a flag that
 * nothing raises -- see the failure path without hanging a GPU. No counterpart in the reference (whose one wait,
 * the fused kernel's, has a fixed bound). */
int exl3b200_set_peer_wait_ns(int64_t ns);

/* The device error word of the current device: nonzero once a bounded wait inside a kernel gave up (the
 * launch then finished without a valid result). Reading it synchronises the device; `clear` resets it. Not
 * for a launch path. */
int exl3b200_read_error(int clear, int32_t* value);

#ifdef __cplusplus
}
#endif

#endif /* EXL3B200_H */
