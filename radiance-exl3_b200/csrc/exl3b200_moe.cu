// exl3b200_moe.cu -- the routing steps on either side of the routed-expert ops, and the device bookkeeping the
// host side needs (SM count, the error word). sm_100a CUDA, extern "C" shim.
//
//   k_router_topk     softmax over all experts, top-k (ties to the lower id), one warp a token
//   k_scatter_*       a STABLE counting sort of the flattened (token, slot) pairs by expert: the routing
//                     contract of include/exl3_abi.h:96-158 (sorted_tok, expert_offset, -1 past the live count)
//   k_gather          y[t] = sum over slots ascending of w[t,s] * row of (t,s), f32 (docs/OPS-exl3.md:195-196)
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "exl3b200_dev.h"
#include "exl3b200_gather.cuh"

namespace {

__device__ int32_t g_err_word;   // set by a kernel whose bounded wait gave up

constexpr int kScatterChunk = 1024;   // pairs a block of the large-sort path
constexpr int kSmallPairs = 2048;     // at most this many pairs: one block does the whole sort

// ------------------------------------------------------------------------------------------ router
// One warp a token: softmax over n_expert logits (max, then sum of exp in lane-strided order reduced by a
// butterfly), then top_k rounds of a warp argmax (larger logit first, lower id on a tie).
__global__ void k_router_topk(const float* __restrict__ logits, int64_t n_tok, int n_expert, int top_k,
                              int32_t* __restrict__ ids, float* __restrict__ w) {
    const int lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (t >= n_tok) return;
    const float* l = logits + t * n_expert;
    float mx = -INFINITY;
    for (int e = lane; e < n_expert; e += 32) mx = fmaxf(mx, l[e]);
    for (int m = 16; m; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, m));
    float s = 0.f;
    for (int e = lane; e < n_expert; e += 32) s += expf(l[e] - mx);
    for (int m = 16; m; m >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, m);
    uint32_t taken[4] = { 0u, 0u, 0u, 0u };   // lane's experts e = lane + 32 * q, q < 128 (n_expert <= 4096)
    for (int r = 0; r < top_k; ++r) {
        float best = -INFINITY;
        int bid = 0x7FFFFFFF;
        for (int q = 0, e = lane; e < n_expert; ++q, e += 32) {
            if ((taken[q >> 5] >> (q & 31)) & 1u) continue;
            const float v = l[e];
            if (v > best || (v == best && e < bid)) { best = v; bid = e; }
        }
        for (int m = 16; m; m >>= 1) {
            const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, m);
            const int oid = __shfl_xor_sync(0xFFFFFFFFu, bid, m);
            if (ov > best || (ov == best && oid < bid)) { best = ov; bid = oid; }
        }
        if (bid != 0x7FFFFFFF && (bid & 31) == lane) {
            const int q = bid >> 5;
            taken[q >> 5] |= 1u << (q & 31);
        }
        if (lane == 0) {
            ids[t * top_k + r] = bid == 0x7FFFFFFF ? -1 : bid;
            w[t * top_k + r] = bid == 0x7FFFFFFF ? 0.f : expf(best - mx) / s;
        }
    }
}

// An order-preserving 32-bit key of a logit: larger value, larger key; -0 keyed as +0 (they compare equal); NaN 0,
// never chosen (a NaN compares false, as in k_router_topk). fkey_inv gives the value back.
__device__ __forceinline__ uint32_t fkey(float f) {
    if (f != f) return 0u;
    const uint32_t b = __float_as_uint(f == 0.f ? 0.f : f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// The same router with the token's logits held in registers (RPL a lane, n_expert <= 32 * RPL): one read of the
// row, the softmax's max and sum in k_router_topk's order, then top_k rounds of a warp-wide redux over the lanes'
// current bests -- the largest key, then the lowest expert id holding it (the same choice as k_router_topk's
// argmax: larger logit first, lower id on a tie). Only the lane that gave up its best looks for its next one; lane r
// keeps round r's pick and the lanes write the ids and weights together at the end.
template <int RPL>
__device__ __forceinline__ void route_warp(const float* __restrict__ l, int n_expert, int top_k, int lane,
                                           int32_t* __restrict__ ids_t, float* __restrict__ w_t) {
    float v[RPL];
#pragma unroll
    for (int q = 0; q < RPL; ++q) {
        const int e = lane + 32 * q;
        v[q] = e < n_expert ? l[e] : 0.f;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int q = 0; q < RPL; ++q)
        if (lane + 32 * q < n_expert) mx = fmaxf(mx, v[q]);
    for (int m = 16; m; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, m));
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < RPL; ++q)
        if (lane + 32 * q < n_expert) s += expf(v[q] - mx);
    for (int m = 16; m; m >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, m);
    uint32_t key[RPL];
#pragma unroll
    for (int q = 0; q < RPL; ++q) key[q] = lane + 32 * q < n_expert ? fkey(v[q]) : 0u;
    // this lane's best: the largest key (a pairwise tree), then the lowest q holding it
    uint32_t bk;
    int bq;
    auto local_best = [&]() {
        uint32_t m[RPL];
#pragma unroll
        for (int q = 0; q < RPL; ++q) m[q] = key[q];
#pragma unroll
        for (int h = RPL / 2; h > 0; h >>= 1)
#pragma unroll
            for (int q = 0; q < h; ++q) m[q] = max(m[q], m[q + h]);
        bk = m[0];
        bq = 0;
#pragma unroll
        for (int q = RPL - 1; q >= 0; --q)
            if (key[q] == bk) bq = q;
    };
    local_best();
    int my_id = -1;
    float my_val = 0.f;
    for (int r = 0; r < top_k; ++r) {
        const uint32_t gk = __reduce_max_sync(0xFFFFFFFFu, bk);
        const uint32_t cand = (bk == gk && gk != 0u) ? (uint32_t)(lane + 32 * bq) : 0xFFFFFFFFu;
        const uint32_t gid = __reduce_min_sync(0xFFFFFFFFu, cand);
        if (lane == r) {
            my_id = gid == 0xFFFFFFFFu ? -1 : (int)gid;
            my_val = fkey_inv(gk);
        }
        if (gid != 0xFFFFFFFFu && (int)(gid & 31u) == lane) {
#pragma unroll
            for (int q = 0; q < RPL; ++q)
                if (q == (int)(gid >> 5)) key[q] = 0u;
            local_best();
        }
    }
    if (lane < top_k) {
        ids_t[lane] = my_id;
        w_t[lane] = my_id < 0 ? 0.f : expf(my_val - mx) / s;
    }
}

template <int RPL>
__global__ void k_router_topk_reg(const float* __restrict__ logits, int64_t n_tok, int n_expert, int top_k,
                                  int32_t* __restrict__ ids, float* __restrict__ w) {
    const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (t >= n_tok) return;
    route_warp<RPL>(logits + t * n_expert, n_expert, top_k, threadIdx.x & 31, ids + t * top_k, w + t * top_k);
}

// Exclusive scan of cnt[0 .. n) in place (block-wide: each thread a run, warp shuffles, warp totals); returns the
// total to every thread. `wtot` holds blockDim.x / 32 ints.
__device__ int block_scan_excl(int* cnt, int n, int* wtot) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int per = (n + blockDim.x - 1) / blockDim.x;
    const int e0 = tid * per, e1 = e0 + per < n ? e0 + per : n;
    int sum = 0;
    for (int e = e0; e < e1; ++e) sum += cnt[e];
    int incl = sum;
    for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xFFFFFFFFu, incl, d);
        if (lane >= d) incl += v;
    }
    if (lane == 31) wtot[warp] = incl;
    __syncthreads();
    int base = 0, total = 0;
    for (int w = 0; w < nw; ++w) {
        const int v = wtot[w];
        if (w < warp) base += v;
        total += v;
    }
    int acc = base + incl - sum;
    for (int e = e0; e < e1; ++e) {
        const int v = cnt[e];
        cnt[e] = acc;
        acc += v;
    }
    __syncthreads();
    return total;
}

// ------------------------------------------------------------------------------------------ scatter
__device__ __forceinline__ int local_expert(int32_t id, int64_t base, int n_expert) {
    const int64_t e = (int64_t)id - base;
    return e >= 0 && e < n_expert ? (int)e : -1;
}

// Stable placement of one chunk of up to 1024 pairs (one a thread, in order), the running per-expert
// positions in `run` (shared). Warps go one after another, so pairs of one expert land in flat order.
__device__ __forceinline__ void place_chunk(const int32_t* ids, int64_t c0, int64_t n_pairs, int64_t base, int n_expert,
                                            int* run, int32_t* sorted_tok) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int64_t f = c0 + tid;
    const int e = f < n_pairs ? local_expert(ids[f], base, n_expert) : -1;
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const int leader = __ffs(peers) - 1;
    for (int w = 0; w < nw; ++w) {
        if (warp == w && e >= 0) {
            sorted_tok[run[e] + rank] = (int32_t)f;
            __syncwarp(peers);
            if (lane == leader) run[e] += __popc(peers);
        }
        __syncthreads();
    }
}

// The same placement without the warp-by-warp walk: each warp's leader lanes record their expert's count in the
// warp's row of `wcnt` ([32 warps][n_expert], shared, all zero on entry), one pass turns every expert's column into
// the warps' first positions (and advances `run`), and every pair is then stored at once. Leaves `wcnt` zero.
__device__ __forceinline__ void place_chunk_fast(const int32_t* ids, int64_t c0, int64_t n_pairs, int64_t base,
                                                 int n_expert, int* run, int* wcnt, int32_t* sorted_tok) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int64_t f = c0 + tid;
    const int e = f < n_pairs ? local_expert(ids[f], base, n_expert) : -1;
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const bool leader = lane == __ffs(peers) - 1;
    if (e >= 0 && leader) wcnt[warp * n_expert + e] = __popc(peers);
    __syncthreads();
    for (int x = tid; x < n_expert; x += blockDim.x) {
        int acc = run[x];
        for (int w = 0; w < nw; ++w) {
            const int c = wcnt[w * n_expert + x];
            if (c) {
                wcnt[w * n_expert + x] = acc;
                acc += c;
            }
        }
        run[x] = acc;
    }
    __syncthreads();
    if (e >= 0) sorted_tok[wcnt[warp * n_expert + e] + rank] = (int32_t)f;
    __syncthreads();
    if (e >= 0 && leader) wcnt[warp * n_expert + e] = 0;
    __syncthreads();
}

// The fast placement's table fits shared memory up to this many experts ([32][n_expert] ints).
constexpr int kPlaceFastExperts = 1024;

// The whole sort in one block (few pairs): histogram, scan, stable placement, tail of -1.
// `ids` carries no __restrict__: the fused router below writes the ids earlier in the same kernel, so they must not be
// read through the read-only (non-coherent) path.
__device__ __forceinline__ void scatter_block(const int32_t* ids, int64_t n_pairs, int n_expert,
                                              int64_t base, int32_t* __restrict__ sorted_tok,
                                              int32_t* __restrict__ off, int* sm) {
    int* cnt = sm;                 // [n_expert + 1]
    const int tid = threadIdx.x;
    for (int e = tid; e <= n_expert; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int64_t f = tid; f < n_pairs; f += blockDim.x) {
        const int e = local_expert(ids[f], base, n_expert);
        if (e >= 0) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    __shared__ int wtot[32];
    const int live = block_scan_excl(cnt, n_expert, wtot);
    for (int e = tid; e < n_expert; e += blockDim.x) off[e] = cnt[e];
    if (tid == 0) off[n_expert] = live;
    for (int64_t f = live + tid; f < n_pairs; f += blockDim.x) sorted_tok[f] = -1;
    if (n_expert <= kPlaceFastExperts) {
        int* wcnt = sm + n_expert + 1;   // [32][n_expert]
        for (int x = tid; x < 32 * n_expert; x += blockDim.x) wcnt[x] = 0;
        __syncthreads();
        for (int64_t c0 = 0; c0 < n_pairs; c0 += blockDim.x)
            place_chunk_fast(ids, c0, n_pairs, base, n_expert, cnt, wcnt, sorted_tok);
    } else {
        for (int64_t c0 = 0; c0 < n_pairs; c0 += blockDim.x)
            place_chunk(ids, c0, n_pairs, base, n_expert, cnt, sorted_tok);
    }
}

__global__ void k_scatter_small(const int32_t* __restrict__ ids, int64_t n_pairs, int n_expert, int64_t base,
                                int32_t* __restrict__ sorted_tok, int32_t* __restrict__ off) {
    extern __shared__ int sm[];
    scatter_block(ids, n_pairs, n_expert, base, sorted_tok, off, sm);
}

// A few tokens (at most one a warp): the router and the whole sort in one block -- the tokens routed by the warps,
// then (their ids visible to the block after the barrier) the small sort. The same results as k_router_topk_reg
// followed by k_scatter_small, one launch instead of two.
constexpr int kFusedTokens = 32;
template <int RPL>
__global__ void __launch_bounds__(1024, 1) k_route_scatter_small(const float* __restrict__ logits, int64_t n_tok, int n_route, int top_k,
                                      int32_t* ids, float* __restrict__ w, int n_expert, int64_t base,
                                      int32_t* __restrict__ sorted_tok, int32_t* __restrict__ off) {
    extern __shared__ int sm[];
    const int warp = threadIdx.x >> 5;
    if (warp < n_tok)
        route_warp<RPL>(logits + (int64_t)warp * n_route, n_route, top_k, threadIdx.x & 31, ids + warp * top_k,
                        w + warp * top_k);
    __syncthreads();
    scatter_block(ids, n_tok * top_k, n_expert, base, sorted_tok, off, sm);
}

// Large path, step 1: per-chunk histograms hist[b][e].
__global__ void k_scatter_hist(const int32_t* __restrict__ ids, int64_t n_pairs, int n_expert, int64_t base,
                               int32_t* __restrict__ hist) {
    extern __shared__ int sm[];
    const int tid = threadIdx.x;
    for (int e = tid; e < n_expert; e += blockDim.x) sm[e] = 0;
    __syncthreads();
    const int64_t f = (int64_t)blockIdx.x * kScatterChunk + tid;
    if (f < n_pairs) {
        const int e = local_expert(ids[f], base, n_expert);
        if (e >= 0) atomicAdd(&sm[e], 1);
    }
    __syncthreads();
    for (int e = tid; e < n_expert; e += blockDim.x) hist[(int64_t)blockIdx.x * n_expert + e] = sm[e];
}

// Step 2 (one block): expert_offset, and hist[b][e] turned into chunk b's first position for expert e.
__global__ void k_scatter_scan(int32_t* __restrict__ hist, int nb, int n_expert, int32_t* __restrict__ off) {
    extern __shared__ int sm[];   // [n_expert] totals
    const int tid = threadIdx.x;
    constexpr int kB = 8;         // chunks a thread loads before it stores any (the loads overlap)
    for (int e = tid; e < n_expert; e += blockDim.x) {
        int acc = 0;
        for (int b0 = 0; b0 < nb; b0 += kB) {
            int v[kB];
#pragma unroll
            for (int q = 0; q < kB; ++q) v[q] = b0 + q < nb ? hist[(int64_t)(b0 + q) * n_expert + e] : 0;
#pragma unroll
            for (int q = 0; q < kB; ++q)
                if (b0 + q < nb) {
                    hist[(int64_t)(b0 + q) * n_expert + e] = acc;
                    acc += v[q];
                }
        }
        sm[e] = acc;
    }
    __syncthreads();
    __shared__ int wtot[32];
    const int live = block_scan_excl(sm, n_expert, wtot);
    for (int e = tid; e < n_expert; e += blockDim.x) off[e] = sm[e];
    if (tid == 0) off[n_expert] = live;
    for (int e = tid; e < n_expert; e += blockDim.x) {
        const int add = sm[e];
        for (int b0 = 0; b0 < nb; b0 += kB) {
            int v[kB];
#pragma unroll
            for (int q = 0; q < kB; ++q) v[q] = b0 + q < nb ? hist[(int64_t)(b0 + q) * n_expert + e] : 0;
#pragma unroll
            for (int q = 0; q < kB; ++q)
                if (b0 + q < nb) hist[(int64_t)(b0 + q) * n_expert + e] = v[q] + add;
        }
    }
}

// Step 3: stable placement of each chunk from its first positions; the tail of -1.
__global__ void k_scatter_place(const int32_t* __restrict__ ids, int64_t n_pairs, int n_expert, int64_t base,
                                const int32_t* __restrict__ hist, const int32_t* __restrict__ off,
                                int32_t* __restrict__ sorted_tok) {
    extern __shared__ int sm[];
    const int tid = threadIdx.x;
    for (int e = tid; e < n_expert; e += blockDim.x) sm[e] = hist[(int64_t)blockIdx.x * n_expert + e];
    if (n_expert <= kPlaceFastExperts) {
        int* wcnt = sm + n_expert + 1;   // [32][n_expert]
        for (int x = tid; x < 32 * n_expert; x += blockDim.x) wcnt[x] = 0;
        __syncthreads();
        place_chunk_fast(ids, (int64_t)blockIdx.x * kScatterChunk, n_pairs, base, n_expert, sm, wcnt, sorted_tok);
    } else {
        __syncthreads();
        place_chunk(ids, (int64_t)blockIdx.x * kScatterChunk, n_pairs, base, n_expert, sm, sorted_tok);
    }
    const int64_t live = off[n_expert];
    const int64_t f = (int64_t)blockIdx.x * kScatterChunk + tid;
    if (f >= live && f < n_pairs) sorted_tok[f] = -1;
}

// ------------------------------------------------------------------------------------------ gather
// One block a token; thread columns 4 at a time; slots in ascending order.
// The gather's output: f32, or bf16 (the f32 sum rounded to nearest even: the engine's hidden-state type).
__device__ __forceinline__ void gst(float* y, float v) { *y = v; }
__device__ __forceinline__ void gst(__nv_bfloat16* y, float v) { *y = __float2bfloat16_rn(v); }
__device__ __forceinline__ void gst8(float* y, const float a[8]) {
    float4* o = reinterpret_cast<float4*>(y);
    o[0] = make_float4(a[0], a[1], a[2], a[3]);
    o[1] = make_float4(a[4], a[5], a[6], a[7]);
}
__device__ __forceinline__ void gst8(__nv_bfloat16* y, const float a[8]) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(a[2 * q], a[2 * q + 1]);
        w[q] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(y) = u;
}

template <typename OutT>
__global__ void k_gather(const uint16_t* __restrict__ rows, int64_t pitch, const int32_t* __restrict__ pos,
                         const float* __restrict__ w, int top_k, int64_t width, OutT* __restrict__ y) {
    const int64_t t = blockIdx.x;
    for (int64_t n = 4 * (int64_t)threadIdx.x; n < width; n += 4 * (int64_t)blockDim.x) {
        float acc[4] = { 0.f, 0.f, 0.f, 0.f };
        for (int s = 0; s < top_k; ++s) {
            const int32_t i = pos[t * top_k + s];
            if (i < 0) continue;
            const float ws = w[t * top_k + s];
            const uint16_t* r = rows + (int64_t)i * pitch + n;
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (n + q < width) acc[q] = __fadd_rn(acc[q], __fmul_rn(ws, __bfloat162float(__ushort_as_bfloat16(r[q]))));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
            if (n + q < width) gst(y + t * width + n + q, acc[q]);
    }
}

// One block a token, a thread 8 columns (16-byte loads of bf16 rows): exl3b::gather_row8, the slots summed in
// ascending order exactly as k_gather does. rows 16-byte aligned with a pitch of a multiple of 8 elements, width a
// multiple of 8, y 16-byte aligned (the host checks).
template <typename OutT>
__global__ void k_gather_v8(const uint16_t* __restrict__ rows, int64_t pitch, const int32_t* __restrict__ pos,
                            const float* __restrict__ w, int top_k, int64_t width, OutT* __restrict__ y) {
    const int64_t t = blockIdx.x;
    for (int64_t n = 8 * (int64_t)threadIdx.x; n < width; n += 8 * (int64_t)blockDim.x) {
        float acc[8];
        exl3b::gather_row8(rows, pitch, pos + t * top_k, w + t * top_k, top_k, n, acc);
        gst8(y + t * width + n, acc);
    }
}

// A few tokens: one block a token finds its own slots' rows in sorted_tok (no inverse map, so no memset and no
// k_invert launch), then sums them exactly as k_gather_v8 does. At most kGatherSmallSlots slots a token.
constexpr int kGatherSmallSlots = 32;
constexpr int64_t kGatherSmallRows = 4096;
template <typename OutT>
__global__ void k_gather_small(const uint16_t* __restrict__ rows, int64_t pitch, const int32_t* __restrict__ sorted_tok,
                               int64_t n_rows, const float* __restrict__ w, int top_k, int64_t width,
                               OutT* __restrict__ y) {
    __shared__ int32_t pos[kGatherSmallSlots];
    const int64_t t = blockIdx.x;
    for (int s = threadIdx.x; s < top_k; s += blockDim.x) pos[s] = -1;
    __syncthreads();
    const int64_t f0 = t * top_k;
    for (int64_t i = threadIdx.x; i < n_rows; i += blockDim.x) {
        const int32_t f = sorted_tok[i];
        if (f >= f0 && f < f0 + top_k) pos[f - f0] = (int32_t)i;
    }
    __syncthreads();
    for (int64_t n = 8 * (int64_t)threadIdx.x; n < width; n += 8 * (int64_t)blockDim.x) {
        float acc[8];
        exl3b::gather_row8(rows, pitch, pos, w + t * top_k, top_k, n, acc);
        gst8(y + t * width + n, acc);
    }
}

// The gather with the shared expert folded in (the engine's moe_gather with act "sigmoid" over the routed rows, the
// shared arm's output and its one-column gate: architectures/qwen4exp_exl3/rad_block_moe_exl3.h:1535-1548, 1961-1965):
// y[t] = (the routed sum of k_gather_v8, slots in ascending order) + sigmoid(g[t]) * sout[t], the shared term added
// as one more weighted row (product then sum, each rounded in f32), g[t] = sum over h of x[t][h] * gate_w[h] (f16
// operands, f32 products and sums), sigmoid(g) = 1 / (1 + exp(-g)) in f32. One block a token; SMALL: the token's
// slots found in sorted_tok (k_gather_small's way), else through the inverse map pos.
template <typename OutT, bool SMALL>
__global__ void __launch_bounds__(256) k_gather_fold(const uint16_t* __restrict__ rows, int64_t pitch,
                                                     const int32_t* __restrict__ map, int64_t n_rows,
                                                     const float* __restrict__ w, int top_k, int64_t width,
                                                     const uint16_t* __restrict__ sout, const uint16_t* __restrict__ x,
                                                     int64_t x_cols, const uint16_t* __restrict__ gate_w,
                                                     OutT* __restrict__ y) {
    __shared__ int32_t spos[kGatherSmallSlots];
    __shared__ float part[8];
    const int64_t t = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    // the shared gate: each thread 8 columns at a time, then the warps' sums, then the block's (fixed order)
    float g = 0.f;
    for (int64_t h = 8 * (int64_t)tid; h < x_cols; h += 8 * (int64_t)blockDim.x) {
        const uint4 xv = *reinterpret_cast<const uint4*>(x + t * x_cols + h);
        const uint4 gv = *reinterpret_cast<const uint4*>(gate_w + h);
        const uint32_t xa[4] = { xv.x, xv.y, xv.z, xv.w }, ga[4] = { gv.x, gv.y, gv.z, gv.w };
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float xf = __half2float(__ushort_as_half((uint16_t)(xa[j >> 1] >> (16 * (j & 1)))));
            const float gf = __half2float(__ushort_as_half((uint16_t)(ga[j >> 1] >> (16 * (j & 1)))));
            g = __fadd_rn(g, __fmul_rn(xf, gf));
        }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) g = __fadd_rn(g, __shfl_xor_sync(0xFFFFFFFFu, g, d));
    if (lane == 0) part[wid] = g;
    if (SMALL) {
        for (int s = tid; s < top_k; s += blockDim.x) spos[s] = -1;
    }
    __syncthreads();
    g = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) g = __fadd_rn(g, part[i]);
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    const int32_t* pos_t = map + t * top_k;
    if (SMALL) {
        const int64_t f0 = t * top_k;
        for (int64_t i = tid; i < n_rows; i += blockDim.x) {
            const int32_t f = map[i];
            if (f >= f0 && f < f0 + top_k) spos[f - f0] = (int32_t)i;
        }
        __syncthreads();
        pos_t = spos;
    }
    for (int64_t n = 8 * (int64_t)tid; n < width; n += 8 * (int64_t)blockDim.x) {
        float acc[8];
        exl3b::gather_row8(rows, pitch, pos_t, w + t * top_k, top_k, n, acc);
        const uint4 sv = *reinterpret_cast<const uint4*>(sout + t * width + n);
        const uint32_t su[4] = { sv.x, sv.y, sv.z, sv.w };
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float b = __bfloat162float(__ushort_as_bfloat16((uint16_t)(su[j >> 1] >> (16 * (j & 1)))));
            acc[j] = __fadd_rn(acc[j], __fmul_rn(sig, b));
        }
        gst8(y + t * width + n, acc);
    }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

static inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// SM count and the error word of the current device, cached per device (no synchronisation).
int exl3b_cuda_device_info(int* sm_count, int32_t** err_word) {
    static int s_sm[64];
    static int32_t* s_err[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
    if (!s_sm[dev]) {
        int sm = 0;
        void* p = nullptr;
        if (cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
        if (cudaGetSymbolAddress(&p, g_err_word) != cudaSuccess) return -1;
        s_err[dev] = static_cast<int32_t*>(p);
        s_sm[dev] = sm;
    }
    *sm_count = s_sm[dev];
    *err_word = s_err[dev];
    return 0;
}

int exl3b_cuda_read_error(int clear, int32_t* value) {
    int32_t v = 0;
    if (cudaMemcpyFromSymbol(&v, g_err_word, sizeof v) != cudaSuccess) return -1;
    if (value) *value = v;
    if (clear) {
        const int32_t z = 0;
        if (cudaMemcpyToSymbol(g_err_word, &z, sizeof z) != cudaSuccess) return -1;
    }
    return 0;
}

int exl3b200_router_topk(const float* logits, int64_t n_tok, int64_t n_expert, int64_t top_k, int32_t* ids, float* w,
                         void* stream) {
    if (!logits || !ids || !w || n_tok < 0 || n_expert < 1 || n_expert > 4096 || top_k < 1 || top_k > 32 ||
        top_k > n_expert)
        return -12;
    if (n_tok == 0) return 0;
    const int wpb = 8;
    const unsigned grid = (unsigned)((n_tok + wpb - 1) / wpb);
    cudaStream_t st = as_stream(stream);
    if (n_expert <= 256)
        k_router_topk_reg<8><<<grid, wpb * 32, 0, st>>>(logits, n_tok, (int)n_expert, (int)top_k, ids, w);
    else if (n_expert <= 512)
        k_router_topk_reg<16><<<grid, wpb * 32, 0, st>>>(logits, n_tok, (int)n_expert, (int)top_k, ids, w);
    else if (n_expert <= 1024)
        k_router_topk_reg<32><<<grid, wpb * 32, 0, st>>>(logits, n_tok, (int)n_expert, (int)top_k, ids, w);
    else
        k_router_topk<<<grid, wpb * 32, 0, st>>>(logits, n_tok, (int)n_expert, (int)top_k, ids, w);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int64_t exl3b200_moe_scatter_work_bytes(int64_t n_pairs, int64_t n_expert) {
    const int64_t nb = (n_pairs + kScatterChunk - 1) / kScatterChunk;
    return (nb > 0 ? nb : 1) * n_expert * 4;
}

int exl3b200_moe_scatter(const int32_t* ids, int64_t n_pairs, int64_t n_expert, int64_t expert_base,
                         int32_t* sorted_tok, int32_t* expert_offset, void* work, void* stream) {
    if (!ids || !sorted_tok || !expert_offset || n_pairs < 0 || n_expert < 1 || n_expert > 16384) return -12;
    cudaStream_t st = as_stream(stream);
    const size_t smem = (size_t)(n_expert + 1) * 4;
    // the small sort and the placement also hold the fast placement's [32][n_expert] table when it fits
    const size_t smem_place = smem + (n_expert <= kPlaceFastExperts ? (size_t)32 * n_expert * 4 : 0);
    if (smem_place > 48 * 1024 &&
        (cudaFuncSetAttribute(k_scatter_small, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_place) !=
             cudaSuccess ||
         cudaFuncSetAttribute(k_scatter_place, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_place) !=
             cudaSuccess))
        return -6;
    if (n_pairs <= kSmallPairs) {
        k_scatter_small<<<1, 1024, smem_place, st>>>(ids, n_pairs, (int)n_expert, expert_base, sorted_tok,
                                                     expert_offset);
        return cudaGetLastError() == cudaSuccess ? 0 : -6;
    }
    if (!work) return -5;
    const int nb = (int)((n_pairs + kScatterChunk - 1) / kScatterChunk);
    int32_t* hist = static_cast<int32_t*>(work);
    k_scatter_hist<<<nb, kScatterChunk, smem, st>>>(ids, n_pairs, (int)n_expert, expert_base, hist);
    k_scatter_scan<<<1, 1024, smem, st>>>(hist, nb, (int)n_expert, expert_offset);
    k_scatter_place<<<nb, kScatterChunk, smem_place, st>>>(ids, n_pairs, (int)n_expert, expert_base, hist,
                                                           expert_offset, sorted_tok);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_router_scatter(const float* logits, int64_t n_tok, int64_t n_route, int64_t top_k, int32_t* ids,
                            float* w, int64_t n_expert, int64_t expert_base, int32_t* sorted_tok,
                            int32_t* expert_offset, void* work, void* stream) {
    if (!logits || !ids || !w || !sorted_tok || !expert_offset || n_tok < 0 || n_route < 1 || n_route > 4096 ||
        top_k < 1 || top_k > 32 || top_k > n_route || n_expert < 1 || n_expert > 16384)
        return -12;
    if (n_tok == 0) return exl3b200_moe_scatter(ids, 0, n_expert, expert_base, sorted_tok, expert_offset, work, stream);
    // fused for up to 32 tokens over at most 512 experts (a 1024-thread block holds 16 logits a lane in registers)
    if (n_tok <= kFusedTokens && n_route <= 512 && n_tok * top_k <= kSmallPairs && n_expert <= kPlaceFastExperts) {
        const size_t smem = (size_t)(n_expert + 1) * 4 + (size_t)32 * n_expert * 4;
        cudaStream_t st = as_stream(stream);
#define EXL3B_RS(R)                                                                                                  \
    do {                                                                                                             \
        auto kern = k_route_scatter_small<R>;                                                                        \
        if (smem > 48 * 1024 &&                                                                                      \
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)       \
            return -6;                                                                                               \
        kern<<<1, 1024, smem, st>>>(logits, n_tok, (int)n_route, (int)top_k, ids, w, (int)n_expert, expert_base,     \
                                    sorted_tok, expert_offset);                                                      \
    } while (0)
        if (n_route <= 256) EXL3B_RS(8);
        else EXL3B_RS(16);
#undef EXL3B_RS
        return cudaGetLastError() == cudaSuccess ? 0 : -6;
    }
    const int rc = exl3b200_router_topk(logits, n_tok, n_route, top_k, ids, w, stream);
    if (rc != 0) return rc;
    return exl3b200_moe_scatter(ids, n_tok * top_k, n_expert, expert_base, sorted_tok, expert_offset, work, stream);
}

int64_t exl3b200_moe_gather_work_bytes(int64_t n_tok, int64_t top_k) { return (n_tok * top_k > 0 ? n_tok * top_k : 1) * 4; }

extern "C++" {
template <typename OutT>
static int gather_impl(const uint16_t* rows, int64_t row_pitch, const int32_t* sorted_tok, int64_t n_rows,
                       const float* w, int64_t n_tok, int64_t top_k, int64_t width, OutT* y, void* work,
                       void* stream) {
    if (!rows || !sorted_tok || !w || !y || !work || n_tok < 0 || top_k < 1 || width < 1) return -12;
    // the pair count n_tok * top_k indexes int32 maps and the kernels take top_k as an int: sizes whose product
    // would not fit are refused before it is formed
    if (top_k > INT32_MAX || n_tok > INT32_MAX / top_k || width > INT32_MAX) return -1;
    if (n_tok == 0) return 0;
    cudaStream_t st = as_stream(stream);
    const bool v8 = aligned16(rows) && row_pitch % 8 == 0 && width % 8 == 0 && aligned16(y);
    if (v8 && n_rows <= kGatherSmallRows && top_k <= kGatherSmallSlots) {
        // few rows: each token finds its own rows, one launch
        k_gather_small<OutT><<<(unsigned)n_tok, 256, 0, st>>>(rows, row_pitch, sorted_tok, n_rows, w, (int)top_k, width, y);
        return cudaGetLastError() == cudaSuccess ? 0 : -6;
    }
    int32_t* pos = static_cast<int32_t*>(work);
    if (cudaMemsetAsync(pos, 0xFF, (size_t)(n_tok * top_k) * 4, st) != cudaSuccess) return -6;
    if (n_rows > 0)
        exl3b::k_invert<<<(unsigned)((n_rows + 255) / 256), 256, 0, st>>>(sorted_tok, n_rows, n_tok * top_k, pos);
    if (v8)
        k_gather_v8<OutT><<<(unsigned)n_tok, 256, 0, st>>>(rows, row_pitch, pos, w, (int)top_k, width, y);
    else
        k_gather<OutT><<<(unsigned)n_tok, 256, 0, st>>>(rows, row_pitch, pos, w, (int)top_k, width, y);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

}  // extern "C++"

int exl3b200_moe_gather(const uint16_t* rows, int64_t row_pitch, const int32_t* sorted_tok, int64_t n_rows,
                        const float* w, int64_t n_tok, int64_t top_k, int64_t width, float* y, void* work,
                        void* stream) {
    return gather_impl(rows, row_pitch, sorted_tok, n_rows, w, n_tok, top_k, width, y, work, stream);
}

int exl3b200_moe_gather_bf16(const uint16_t* rows, int64_t row_pitch, const int32_t* sorted_tok, int64_t n_rows,
                             const float* w, int64_t n_tok, int64_t top_k, int64_t width, uint16_t* y, void* work,
                             void* stream) {
    return gather_impl(rows, row_pitch, sorted_tok, n_rows, w, n_tok, top_k, width,
                       reinterpret_cast<__nv_bfloat16*>(y), work, stream);
}

// The gather with the shared arm folded in (k_gather_fold). rows, sout, x, gate_w and y 16-byte aligned; row_pitch,
// width and x_cols multiples of 8; y f32 (y_dtype RAD_F32 = 1) or bf16 (RAD_BF16 = 3); work as exl3b200_moe_gather's.
int exl3b200_moe_gather_fold(const uint16_t* rows, int64_t row_pitch, const int32_t* sorted_tok, int64_t n_rows,
                             const float* w, int64_t n_tok, int64_t top_k, int64_t width, const uint16_t* sout,
                             const uint16_t* x, int64_t x_cols, const uint16_t* gate_w, void* y, int y_dtype,
                             void* work, void* stream) {
    if (!rows || !sorted_tok || !w || !sout || !x || !gate_w || !y || !work || n_tok < 0 || n_rows < 0 || top_k < 1 ||
        width < 8 || x_cols < 8)
        return -12;
    if (top_k > INT32_MAX || n_tok > INT32_MAX / top_k || width > INT32_MAX) return -1;
    if (y_dtype != 1 && y_dtype != 3) return -2;
    if (!aligned16(rows) || !aligned16(sout) || !aligned16(x) || !aligned16(gate_w) || !aligned16(y) ||
        row_pitch % 8 || width % 8 || x_cols % 8)
        return -3;
    if (n_tok == 0) return 0;
    cudaStream_t st = as_stream(stream);
#define EXL3B_FOLD(OUT, SMALL, MAP)                                                                                   \
    k_gather_fold<OUT, SMALL><<<(unsigned)n_tok, 256, 0, st>>>(rows, row_pitch, MAP, n_rows, w, (int)top_k, width,     \
                                                              sout, x, x_cols, gate_w, static_cast<OUT*>(y))
    if (n_rows <= kGatherSmallRows && top_k <= kGatherSmallSlots) {
        if (y_dtype == 1) EXL3B_FOLD(float, true, sorted_tok);
        else EXL3B_FOLD(__nv_bfloat16, true, sorted_tok);
        return cudaGetLastError() == cudaSuccess ? 0 : -6;
    }
    int32_t* pos = static_cast<int32_t*>(work);
    if (cudaMemsetAsync(pos, 0xFF, (size_t)(n_tok * top_k) * 4, st) != cudaSuccess) return -6;
    if (n_rows > 0)
        exl3b::k_invert<<<(unsigned)((n_rows + 255) / 256), 256, 0, st>>>(sorted_tok, n_rows, n_tok * top_k, pos);
    if (y_dtype == 1) EXL3B_FOLD(float, false, pos);
    else EXL3B_FOLD(__nv_bfloat16, false, pos);
#undef EXL3B_FOLD
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

// The shared expert's routing: every token its own sorted row (sorted_tok[i] = i), one expert holding all n_tok.
__global__ void k_identity_routing(int64_t n_tok, int32_t* __restrict__ sorted_tok, int32_t* __restrict__ offset) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n_tok) sorted_tok[i] = (int32_t)i;
    if (i == 0) {
        offset[0] = 0;
        offset[1] = (int32_t)n_tok;
    }
}
int exl3b200_identity_routing(int64_t n_tok, int32_t* sorted_tok, int32_t* expert_offset, void* stream) {
    if (!sorted_tok || !expert_offset || n_tok < 0 || n_tok > INT32_MAX) return -12;
    k_identity_routing<<<(unsigned)((n_tok + 255) / 256 > 0 ? (n_tok + 255) / 256 : 1), 256, 0, as_stream(stream)>>>(
        n_tok, sorted_tok, expert_offset);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

// ------------------------------------------------------------------------------------------ the gather, allocating nothing
// The gather's one piece of scratch -- the inverse map from a (token, slot) pair to its sorted row -- lives in this
// fixed device array instead of memory the caller provides, for callers that cannot allocate device memory at all.
// At most kNoAllocMaxPairs pairs a call (1 MiB of int32). Every GPU that loads this library holds the array until
// the process exits.
constexpr int64_t kNoAllocMaxPairs = 1 << 18;
static __device__ __align__(256) int32_t g_noalloc_pos[kNoAllocMaxPairs];

int exl3b200_moe_gather_noalloc(const uint16_t* rows, int64_t row_pitch, const int32_t* sorted_tok, int64_t n_rows,
                                const float* w, int64_t n_tok, int64_t top_k, int64_t width, float* y, void* stream) {
    if (!rows || !sorted_tok || !w || !y || n_tok < 0 || top_k < 1 || width < 1 || n_rows < 0) return -12;
    // past the fixed array: refused before anything is enqueued (tested factor by factor, so that no product of
    // huge arguments can wrap around into the allowed range)
    if (top_k > kNoAllocMaxPairs || n_tok > kNoAllocMaxPairs / top_k || width > INT32_MAX) return -1;
    if (n_tok == 0) return 0;
    // Set-up, once per device, with that device current: the array's device address. The host-side name of a
    // __device__ array is not a device address; only cudaGetSymbolAddress gives one.
    static int32_t* s_pos[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -6;
    if (!s_pos[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_pos) != cudaSuccess || !p) return -6;
        s_pos[dev] = static_cast<int32_t*>(p);
    }
    int32_t* pos = s_pos[dev];
    cudaStream_t st = as_stream(stream);
    // the map starts as "no row" (-1) for every pair of this call; the array keeps the last call's contents
    if (cudaMemsetAsync(pos, 0xFF, (size_t)(n_tok * top_k) * 4, st) != cudaSuccess) return -6;
    if (n_rows > 0)
        exl3b::k_invert<<<(unsigned)((n_rows + 255) / 256), 256, 0, st>>>(sorted_tok, n_rows, n_tok * top_k, pos);
    if (aligned16(rows) && row_pitch % 8 == 0 && width % 8 == 0 && aligned16(y))
        k_gather_v8<float><<<(unsigned)n_tok, 256, 0, st>>>(rows, row_pitch, pos, w, (int)top_k, width, y);
    else
        k_gather<float><<<(unsigned)n_tok, 256, 0, st>>>(rows, row_pitch, pos, w, (int)top_k, width, y);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

}  // extern "C"
