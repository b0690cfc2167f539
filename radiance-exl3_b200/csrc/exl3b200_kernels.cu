// exl3b200_kernels.cu -- the sm_100a kernels of the EXL3 routed-expert path and the extern "C" shim the C
// host side calls. Hand-written CUDA; no library kernel is on this path.
//
//   k_decode_what    record -> W_hat fp16, one warp a 16x16 tile (the bit-exact decode, test vehicle)
//   k_prep           moe_exl3_prep_gu: xr = f16(had(f16(a[tok] * suh))) | ... suh.1, per sorted row
//   k_gemm_skinny    the decode band: trellis decode in registers straight into mma.sync B fragments,
//                    the packed record streamed by a producer warp with cp.async.bulk (TMA) into a
//                    shared-memory ring, split-K over a thread-block cluster reduced through distributed
//                    shared memory, and the output rotation / svh / SiLU*up / h_rot epilogue.
//
// Semantics are the reference's (docs/OPS-exl3.md:84-153; kernels/exl3ref/ref.c:27-228). The decode is
// bit-exact against common/exl3_decode.c:47-144: every codebook value is produced by the same single
// fp16 rounding (HFMA2 / HADD2, round to nearest even) of the same exact operands. The rotations run the
// butterfly stages h = 1, 2, ..., 64 in f32 in exactly the order of common/exl3_decode.c:172-189, so the
// prologue's xr matches the reference bit for bit.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "exl3b200_dev.h"
#include "exl3b200_decode.cuh"

namespace {

__device__ __forceinline__ void ldmatrix_x4(uint32_t r[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------------------------------------ the decode (test vehicle)
template <int BITS, int CB>
__global__ void k_decode_what(const uint32_t* __restrict__ record, int64_t rows, int64_t cols,
                              uint16_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t nt = rows / 16, kt = cols / 16;
    const int64_t tile = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (tile >= nt * kt) return;
    const int64_t tk = tile / nt, tn = tile % nt;
    uint32_t b[4];
    decode_lane<BITS, CB>(record + tile * 8 * BITS, lane, b);
    const int g = lane >> 2, t = lane & 3;
    // b[0]: (n = g, k = 2t, 2t+1); b[1]: (n = g, k = 2t+8, +9); b[2], b[3]: n + 8
    const int64_t n0 = tn * 16 + g, k0 = tk * 16 + 2 * t;
    uint32_t* o = reinterpret_cast<uint32_t*>(out);
    o[(n0 * cols + k0) / 2] = b[0];
    o[(n0 * cols + k0 + 8) / 2] = b[1];
    o[((n0 + 8) * cols + k0) / 2] = b[2];
    o[((n0 + 8) * cols + k0 + 8) / 2] = b[3];
}

// ------------------------------------------------------------------------------------------ prep
// A pass over (sorted row, group of four 128-blocks) tasks, one warp a task and eight lanes a block, each warp a
// contiguous run of tasks; the expert offsets staged once a CTA in shared memory (the owner of a row is a binary
// search there, once a row). gate_up
// (moe_exl3_prep_gu, and the tensor-core path's xr): the token row a[sorted_tok / top_k] rotated with suh into
// [0, C) and with suh.1 into [C, 2C) of row i; rows outside the runs are not written; a row whose sorted_tok is
// negative is zero across 2C (docs/OPS-exl3.md:128-142). down (h_rot 0 on the tensor-core path): row i of h rotated
// with suh into [0, C).
//
// A lane holds 16 consecutive values of its block (two 16-byte loads), so the butterfly stages h = 1 .. 8 run
// in its registers and only h = 16, 32, 64 cross lanes (a shuffle within the block's 8 lanes); 32 values a lane
// (two cross-lane stages) was measured slower: 80 registers, fewer warps to cover the loads. Every stage pairs
// the same elements with the same f32 operations as the reference's loop (common/exl3_decode.c:172-189), so xr is
// bit for bit the reference's.
constexpr int kPrepWarps = 8;
constexpr int kPrepV = 16;                      // values a lane
constexpr int kPrepLpb = 128 / kPrepV;          // lanes a 128-block
constexpr int kPrepBpw = 32 / kPrepLpb;         // blocks a warp task

// The 16-value form on packed pairs (v[q], v[q + 8]): stages h = 1, 2, 4 pair two packed registers element by
// element, h = 8 the two halves of one, the cross-lane stages one f32x2 FMA a pair -- every element through the same
// operations in the same order as the scalar form below, so the same bits.
__device__ __forceinline__ void had128_x16_pk(float v[16], int lb) {
    uint64_t P[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) P[q] = f2pk(v[q], v[q + 8]);
#pragma unroll
    for (int h = 1; h < 8; h <<= 1)
#pragma unroll
        for (int q = 0; q < 8; ++q)
            if (!(q & h)) {
                const uint64_t a = P[q], b = P[q + h];
                P[q] = add2(a, b);
                P[q + h] = sub2(a, b);
            }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        float a, b;
        f2upk(P[q], a, b);
        P[q] = f2pk(__fadd_rn(a, b), __fsub_rn(a, b));
    }
#pragma unroll
    for (int m = 1; m < 8; m <<= 1) {
        const float sg = (lb & m) ? -1.0f : 1.0f;       // p + (+-1) v: exact product, one rounding
        const uint64_t sg2 = f2pk(sg, sg);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            float lo, hi;
            f2upk(P[q], lo, hi);
            const float pl = __shfl_xor_sync(0xFFFFFFFFu, lo, m), ph = __shfl_xor_sync(0xFFFFFFFFu, hi, m);
            P[q] = fma2(sg2, P[q], f2pk(pl, ph));
        }
    }
    const uint64_t rs2 = f2pk(kRs, kRs);
#pragma unroll
    for (int q = 0; q < 8; ++q) f2upk(mul2(P[q], rs2), v[q], v[q + 8]);
}

template <int V>
__device__ __forceinline__ void had128_xv(float v[V], int lb) {
    if constexpr (V == 16) {
        had128_x16_pk(v, lb);
    } else {
#pragma unroll
        for (int h = 1; h < V; h <<= 1)
#pragma unroll
            for (int i = 0; i < V; ++i)
                if (!(i & h)) {
                    const float a = v[i], b = v[i + h];
                    v[i] = __fadd_rn(a, b);
                    v[i + h] = __fsub_rn(a, b);
                }
#pragma unroll
        for (int m = 1; m < 128 / V; m <<= 1) {
            const float sg = (lb & m) ? -1.0f : 1.0f;       // p + (+-1) v: exact product, one rounding
#pragma unroll
            for (int i = 0; i < V; ++i) {
                const float p = __shfl_xor_sync(0xFFFFFFFFu, v[i], m);
                v[i] = __fmaf_rn(sg, v[i], p);
            }
        }
#pragma unroll
        for (int i = 0; i < V; ++i) v[i] = __fmul_rn(v[i], kRs);
    }
}

// V consecutive 16-bit values as V/2 packed pairs (low half = the lower index)
template <int V>
__device__ __forceinline__ void ldv(const uint16_t* p, bool vec, uint32_t u[V / 2]) {
    if (vec) {
#pragma unroll
        for (int q = 0; q < V / 8; ++q) {
            const uint4 a = *reinterpret_cast<const uint4*>(p + 8 * q);
            u[4 * q] = a.x; u[4 * q + 1] = a.y; u[4 * q + 2] = a.z; u[4 * q + 3] = a.w;
        }
    } else {
#pragma unroll
        for (int q = 0; q < V / 2; ++q) u[q] = (uint32_t)p[2 * q] | ((uint32_t)p[2 * q + 1] << 16);
    }
}
// v = f32(f16(x * s)) for V values: the product rounded once to f16, as the reference's f16(f32 x * f32 s) (the
// product of two f16 values is exact in f32). f16 x: one HMUL2 a pair; bf16 x: in f32, then rounded.
template <int V>
__device__ __forceinline__ void scalev(const uint32_t x[V / 2], const uint32_t s[V / 2], bool bf, float v[V]) {
#pragma unroll
    for (int q = 0; q < V / 2; ++q) {
        if (!bf) {
            const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&x[q]), *reinterpret_cast<const __half2*>(&s[q]));
            const float2 f = __half22float2(r);
            v[2 * q] = f.x;
            v[2 * q + 1] = f.y;
        } else {
            v[2 * q] = h2f(f2h(__fmul_rn(bf2f((uint16_t)x[q]), h2f((uint16_t)s[q]))));
            v[2 * q + 1] = h2f(f2h(__fmul_rn(bf2f((uint16_t)(x[q] >> 16)), h2f((uint16_t)(s[q] >> 16)))));
        }
    }
}
// V f32 values rounded to f16 and stored (V/2 packed pairs)
template <int V>
__device__ __forceinline__ void stvf(uint16_t* p, bool vec, const float v[V]) {
    uint32_t u[V / 2];
#pragma unroll
    for (int q = 0; q < V / 2; ++q) {
        const __half2 h = __floats2half2_rn(v[2 * q], v[2 * q + 1]);
        u[q] = *reinterpret_cast<const uint32_t*>(&h);
    }
    if (vec) {
#pragma unroll
        for (int q = 0; q < V / 8; ++q)
            *reinterpret_cast<uint4*>(p + 8 * q) = make_uint4(u[4 * q], u[4 * q + 1], u[4 * q + 2], u[4 * q + 3]);
    } else {
#pragma unroll
        for (int q = 0; q < V / 2; ++q) { p[2 * q] = (uint16_t)u[q]; p[2 * q + 1] = (uint16_t)(u[q] >> 16); }
    }
}
__device__ __forceinline__ bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

__global__ void __launch_bounds__(kPrepWarps * 32) k_prep(const Exl3bOp op, uint16_t* __restrict__ dst_base,
                                                           int64_t dst_pitch, int ngrp) {
    extern __shared__ int32_t s_off[];                 // expert_offset [n_expert + 1]
    for (int64_t e = threadIdx.x; e <= op.n_expert; e += blockDim.x) s_off[e] = op.expert_offset[e];
    __syncthreads();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int lb = lane % kPrepLpb, bq = lane / kPrepLpb;   // the lane's V values: block Bpw g + bq, elements V lb ..
    const bool gu = op.op != EXL3B_OP_DOWN;
    const int64_t lo = s_off[0], hi = s_off[op.n_expert] < op.T ? s_off[op.n_expert] : op.T;
    const bool bf = gu && op.x_bf16;
    const bool xvec = al16(op.x) && (op.x_pitch % 8) == 0;
    const bool yvec = al16(dst_base) && (dst_pitch % 8) == 0;
    const uint32_t n_task = (uint32_t)((hi - lo) * ngrp);      // < 2^31 (the host checks)
    // each warp a contiguous run of tasks (group fastest), so consecutive tasks share their row and the row's set-up
    // (owner search, pointers, token) is done once a row; the runs differ by at most one task
    const uint64_t n_warps = (uint64_t)gridDim.x * kPrepWarps, gw = (uint64_t)blockIdx.x * kPrepWarps + w;
    const uint32_t t_begin = (uint32_t)(gw * n_task / n_warps), t_end = (uint32_t)((gw + 1) * n_task / n_warps);
    int64_t row = -1;
    ExpertView ev{};
    const uint16_t *src = nullptr, *s0 = nullptr, *s1 = nullptr;
    uint16_t* y = nullptr;
    int32_t tok = -1;
    bool svec = false;
    // the task's row and its group within the row, advanced with the task (no division a task)
    uint32_t rr = t_begin / (uint32_t)ngrp, gi = t_begin - rr * (uint32_t)ngrp;
    for (uint32_t task = t_begin; task < t_end; ++task, (++gi == (uint32_t)ngrp ? (gi = 0, ++rr) : 0)) {
        const int64_t i = lo + rr;
        if (i != row) {
            row = i;
            int a = 0, b = (int)op.n_expert;           // the owner: largest e with off[e] <= i
            while (b - a > 1) {
                const int mid = (a + b) >> 1;
                if (s_off[mid] <= i) a = mid; else b = mid;
            }
            ev = expert_view(op, a);
            y = dst_base + i * dst_pitch;
            tok = op.sorted_tok[i];
            const int64_t src_row = gu ? (int64_t)(tok / op.top_k) : i;
            src = static_cast<const uint16_t*>(op.x) + src_row * op.x_pitch;
            s0 = static_cast<const uint16_t*>(tab_entry(op.cls[ev.c].suh, ev.j));
            s1 = gu ? static_cast<const uint16_t*>(tab_entry(op.cls[ev.c].suh1, ev.j)) : s0;
            svec = al16(s0) && al16(s1);
        }
        const int64_t blk = (int64_t)gi * kPrepBpw + bq;
        const bool mine = blk * 128 < ev.C;            // lanes past the class's width idle (shuffles stay whole)
        const int64_t c = (mine ? blk : 0) * 128 + kPrepV * lb;
        if (tok < 0) {
            float z[kPrepV];
#pragma unroll
            for (int q = 0; q < kPrepV; ++q) z[q] = 0.f;
            if (mine) {
                stvf<kPrepV>(y + c, yvec, z);
                if (gu) stvf<kPrepV>(y + ev.C + c, yvec, z);
            }
            continue;
        }
        // the two halves one after the other
        uint32_t hx[kPrepV / 2], hs[kPrepV / 2];
        float va[kPrepV];
        ldv<kPrepV>(src + c, xvec, hx);
        ldv<kPrepV>(s0 + c, svec, hs);
        scalev<kPrepV>(hx, hs, bf, va);
        had128_xv<kPrepV>(va, lb);
        if (mine) stvf<kPrepV>(y + c, yvec, va);
        if (gu) {
            ldv<kPrepV>(s1 + c, svec, hs);
            scalev<kPrepV>(hx, hs, bf, va);
            had128_xv<kPrepV>(va, lb);
            if (mine) stvf<kPrepV>(y + ev.C + c, yvec, va);
        }
    }
}

// ------------------------------------------------------------------------------------------ the decode-band GEMM
//
// Unit = (expert e, row group g of up to 16*MCH of its rows, output block b of 128 columns). A cluster of
// `ksplit` CTAs runs one unit, CTA r taking 128-column chunks [r*nch/S, (r+1)*nch/S) of the class's input
// width; the partial sums meet in the cluster leader's shared memory (in rank order: deterministic).
// Persistent: the clusters walk the unit list, which every CTA derives from expert_offset the same way.
//
// Warps 0..7 decode and multiply; warp 8 is the producer (cp.async.bulk of each k-tile row of the block's
// eight tiles, per matrix, into an NST-stage ring). For gate_up, warp w owns the gate tile w and the up tile
// w of the block (matrices 0 and 1); for down, tile w.
constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kNst = 8;      // ring stages
constexpr int kTks = 4;      // k-tile rows a stage

template <int BITS, bool GU>
struct SkinnyCfg {
    static constexpr int MATS = GU ? 2 : 1;
    static constexpr int TILE_WORDS = 8 * BITS;
    static constexpr int COPY_BYTES = 8 * TILE_WORDS * 4;          // the block's 8 tiles of one k row
    static constexpr int STAGE_BYTES = kTks * MATS * COPY_BYTES;
    static constexpr int RED_COLS = MATS * 128 + 4;                 // f32 partial sums a row (padded)
};

// Shared-memory layout (bytes): [bars 256][unit prefix (n_expert+1) u32, 16-aligned][ring][xr / red]
__host__ __device__ inline int64_t skinny_prefix_bytes(int64_t n_expert) { return ((n_expert + 1) * 4 + 15) / 16 * 16; }

template <int BITS, int CB, bool GU, int MCH>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_skinny(const Exl3bOp op, int ksplit, int kc_max, int n_blocks) {
    using Cfg = SkinnyCfg<BITS, GU>;
    constexpr int MMAX = 16 * MCH;
    constexpr int MATS = Cfg::MATS;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kNst;
    int* s_misc = reinterpret_cast<int*>(smem + 2 * kNst * 8);           // [0] n_units
    uint32_t* prefix = reinterpret_cast<uint32_t*>(smem + 256);
    uint8_t* ring = smem + 256 + skinny_prefix_bytes(op.n_expert);
    uint8_t* xr_raw = ring + kNst * Cfg::STAGE_BYTES;
    const int xr_stride = kc_max + 8;                                     // halves a row (+16 B: no ldmatrix conflicts)
    uint16_t* xr = reinterpret_cast<uint16_t*>(xr_raw);                   // [MATS][MMAX][xr_stride]
    float* red = reinterpret_cast<float*>(xr_raw);                        // [MMAX][RED_COLS] (aliases xr)

    const int tid = threadIdx.x, warp = __shfl_sync(0xFFFFFFFFu, tid >> 5, 0), lane = tid & 31;
    const int S = ksplit;
    const uint32_t rank = S > 1 ? cluster_rank() : 0;
    const int64_t cluster_id = blockIdx.y, n_clusters = gridDim.y;
    const int64_t n_exp = op.n_expert;

    if (tid == 0) {
        for (int s = 0; s < kNst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // ---- the unit list: units of expert e = ceil(rows_e / MMAX) * n_blocks (block-scan of the counts)
    {
        // a block-wide exclusive scan: each thread a run of experts, warp shuffles, then the warp totals
        __shared__ uint32_t wsum[kThreads / 32];
        const int64_t per = (n_exp + kThreads - 1) / kThreads;
        const int64_t e0 = tid * per, e1 = e0 + per < n_exp ? e0 + per : n_exp;
        uint32_t sum = 0;
        for (int64_t e = e0; e < e1; ++e) {
            const int64_t r = op.expert_offset[e + 1] - op.expert_offset[e];
            sum += r > 0 ? (uint32_t)(((r + MMAX - 1) / MMAX) * n_blocks) : 0u;
        }
        uint32_t incl = sum;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, d);
            if (lane >= d) incl += v;
        }
        if (lane == 31) wsum[warp] = incl;
        __syncthreads();
        uint32_t base = 0;
        for (int w = 0; w < warp; ++w) base += wsum[w];
        uint32_t acc = base + incl - sum;
        for (int64_t e = e0; e < e1; ++e) {
            prefix[e] = acc;
            const int64_t r = op.expert_offset[e + 1] - op.expert_offset[e];
            acc += r > 0 ? (uint32_t)(((r + MMAX - 1) / MMAX) * n_blocks) : 0u;
        }
        if (tid == kThreads - 1) {
            prefix[n_exp] = acc;
            s_misc[0] = (int)acc;
        }
    }
    __syncthreads();
    if (S > 1) cluster_sync_all();
    const int64_t n_units = s_misc[0];

    // ---- rows no unit writes: zero (outside the runs, or a dropped slot), across the whole width (unless the
    // caller asked for the live rows only)
    if (!op.live_only) {
        const int64_t gcta = cluster_id * S + rank, ncta = n_clusters * S;
        for (int64_t i = gcta; i < op.T; i += ncta) {
            if (row_live(op, i)) continue;
            if (GU) {
                uint16_t* y = out_row(op, i);
                for (int64_t c = tid; c < op.y_cols; c += kThreads) y[c] = 0;
            } else {
                uint16_t* y = out_row(op, i);
                for (int64_t c = tid; c < op.y_cols; c += kThreads) y[c] = 0;
            }
        }
    }

    uint32_t it = 0;   // ring position, advanced identically by producer and consumers
    for (int64_t unit = cluster_id; unit < n_units; unit += n_clusters) {
        // which expert: the last e with prefix[e] <= unit
        int64_t lo = 0, hi = n_exp;
        while (hi - lo > 1) {
            const int64_t mid = (lo + hi) / 2;
            if ((int64_t)prefix[mid] <= unit) lo = mid; else hi = mid;
        }
        const int64_t e = lo;
        const int64_t local = unit - prefix[e];
        const int64_t grp = local / n_blocks, blk = local % n_blocks;
        const ExpertView ev = expert_view(op, e);
        const Exl3bClass& cl = op.cls[ev.c];
        const int64_t r0 = op.expert_offset[e] + grp * MMAX;
        const int64_t rend = op.expert_offset[e + 1];
        const int nr = (int)(rend - r0 < MMAX ? rend - r0 : MMAX);
        const int64_t width = GU ? ev.R / 2 : ev.R;                       // output columns of this class
        if (blk * 128 >= width) {
            // a narrower class: its rows are zero past its own width
            if (rank == 0 && warp < kConsumerWarps)
                for (int m = warp; m < nr; m += kConsumerWarps) {
                    const int64_t i = r0 + m;
                    if (!row_live(op, i)) continue;
                    uint16_t* y = out_row(op, i) + blk * 128;
                    for (int q = lane; q < 128; q += 32) y[q] = 0;
                }
            continue;
        }
        const int64_t nch = ev.C / 128;
        const int64_t ch0 = nch * rank / S, ch1 = nch * (rank + 1) / S;
        const int64_t k0 = ch0 * 128;
        const int ntk = (int)((ch1 - ch0) * 8);
        const int nstages = (ntk + kTks - 1) / kTks;

        if (warp == kConsumerWarps) {
            // ------------------------------------------------ producer (the whole warp runs the loop; the
            // elected lane issues the copies)
            const uint16_t* rec = static_cast<const uint16_t*>(tab_entry(cl.codes, ev.j));
            const int64_t wrows = GU ? ev.R / 2 : ev.R;                  // rows of one record
            const int64_t mat_elems = (ev.C / 16) * (wrows / 16) * 16 * BITS;
            for (int sidx = 0; sidx < nstages; ++sidx, ++it) {
                const uint32_t s = it % kNst, ph = (it / kNst) & 1;
                mbar_wait_warp(&empty[s], ph ^ 1, op.err);
                const int tk_first = sidx * kTks;
                const int n_in = ntk - tk_first < kTks ? ntk - tk_first : kTks;
                mbar_expect_tx_el(&full[s], (uint32_t)(n_in * MATS * Cfg::COPY_BYTES));
                for (int q = 0; q < n_in; ++q) {
                    const int64_t tk = ch0 * 8 + tk_first + q;
#pragma unroll
                    for (int mat = 0; mat < MATS; ++mat) {
                        const uint16_t* src = rec + mat * mat_elems + (tk * (wrows / 16) + blk * 8) * 16 * BITS;
                        tma_bulk_g2s_el(ring + s * Cfg::STAGE_BYTES + (q * MATS + mat) * Cfg::COPY_BYTES, src,
                                        Cfg::COPY_BYTES, &full[s]);
                    }
                }
            }
        } else {
            // ------------------------------------------------ consumers: the rotated input rows into xr
            const int nchl = (int)(ch1 - ch0);
            for (int task = warp; task < MATS * MMAX * nchl; task += kConsumerWarps) {
                const int mat = task / (MMAX * nchl);
                const int m = (task / nchl) % MMAX;
                const int chl = task % nchl;
                uint16_t* dst = xr + ((int64_t)mat * MMAX + m) * xr_stride + chl * 128 + 4 * lane;
                const int64_t i = r0 + m;
                const int32_t tok = m < nr ? op.sorted_tok[i] : -1;
                float v[4] = { 0.f, 0.f, 0.f, 0.f };
                if (tok >= 0) {
                    const int64_t kk = k0 + chl * 128 + 4 * lane;
                    const uint16_t* xs;
                    bool rotate;
                    const uint16_t* s = nullptr;
                    if (GU) {
                        if (op.a_rot) {
                            xs = static_cast<const uint16_t*>(op.x) + i * op.x_pitch + mat * ev.C + kk;
                            rotate = false;
                        } else {
                            xs = static_cast<const uint16_t*>(op.x) + (int64_t)(tok / op.top_k) * op.x_pitch + kk;
                            rotate = true;
                            s = static_cast<const uint16_t*>(tab_entry(mat ? cl.suh1 : cl.suh, ev.j)) + k0 + chl * 128;
                        }
                    } else {
                        xs = static_cast<const uint16_t*>(op.x) + i * op.x_pitch + kk;
                        rotate = !op.h_rot;
                        if (rotate) s = static_cast<const uint16_t*>(tab_entry(cl.suh, ev.j)) + k0 + chl * 128;
                    }
                    const bool bf = GU && !op.a_rot && op.x_bf16;
#pragma unroll
                    for (int q = 0; q < 4; ++q) v[q] = bf ? bf2f(xs[q]) : h2f(xs[q]);
                    if (rotate) {
                        prologue_warp(v, s, lane);
                    }
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) dst[q] = f2h(v[q]);
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");

            // ------------------------------------------------ main loop
            float acc[MATS][MCH][2][4];
#pragma unroll
            for (int mt = 0; mt < MATS; ++mt)
#pragma unroll
                for (int mc = 0; mc < MCH; ++mc)
#pragma unroll
                    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
                        for (int q = 0; q < 4; ++q) acc[mt][mc][nb][q] = 0.f;
            const int arow = (lane & 7) + 8 * ((lane >> 3) & 1), acol = 8 * (lane >> 4);
            const LaneDec<BITS> ldec = lane_dec<BITS>(lane);
            for (int sidx = 0; sidx < nstages; ++sidx, ++it) {
                const uint32_t s = it % kNst, ph = (it / kNst) & 1;
                mbar_wait_warp(&full[s], ph, op.err);
                const int tk_first = sidx * kTks;
                const int n_in = ntk - tk_first < kTks ? ntk - tk_first : kTks;
                for (int q = 0; q < n_in; ++q) {
                    const int tkl = tk_first + q;                       // k-tile index inside this CTA's range
#pragma unroll
                    for (int mat = 0; mat < MATS; ++mat) {
                        const uint32_t words = smem_u32(ring) + s * Cfg::STAGE_BYTES +
                                               (q * MATS + mat) * Cfg::COPY_BYTES + warp * Cfg::TILE_WORDS * 4;
                        uint32_t b[4];
                        decode_tile_s<BITS, CB>(words, ldec, b);
#pragma unroll
                        for (int mc = 0; mc < MCH; ++mc) {
                            uint32_t a[4];
                            ldmatrix_x4(a, xr + ((int64_t)mat * MMAX + mc * 16 + arow) * xr_stride + tkl * 16 + acol);
                            mma16816(acc[mat][mc][0], a, b[0], b[1]);
                            mma16816(acc[mat][mc][1], a, b[2], b[3]);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
            // partial sums -> red (aliases xr: every consumer warp must be done reading it)
            asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
            const int g = lane >> 2, t = lane & 3;
#pragma unroll
            for (int mat = 0; mat < MATS; ++mat)
#pragma unroll
                for (int mc = 0; mc < MCH; ++mc)
#pragma unroll
                    for (int nb = 0; nb < 2; ++nb) {
                        const int col = mat * 128 + warp * 16 + nb * 8 + 2 * t;
                        float* r0p = red + (mc * 16 + g) * Cfg::RED_COLS + col;
                        float* r1p = red + (mc * 16 + g + 8) * Cfg::RED_COLS + col;
                        r0p[0] = acc[mat][mc][nb][0];
                        r0p[1] = acc[mat][mc][nb][1];
                        r1p[0] = acc[mat][mc][nb][2];
                        r1p[1] = acc[mat][mc][nb][3];
                    }
        }
        if (S > 1) cluster_sync_all(); else __syncthreads();

        // ---------------------------------------------------- epilogue in the leader
        if (rank == 0 && warp < kConsumerWarps) {
            for (int m = warp; m < nr; m += kConsumerWarps) {
                const int64_t i = r0 + m;
                if (op.sorted_tok[i] < 0) continue;
                float v[MATS][4];
#pragma unroll
                for (int mat = 0; mat < MATS; ++mat) {
                    const float* src = red + m * Cfg::RED_COLS + mat * 128 + 4 * lane;
                    float4 sum = *reinterpret_cast<const float4*>(src);
                    for (int r = 1; r < S; ++r) {
                        const float4 p = ld_dsmem_f4(src, (uint32_t)r);
                        sum.x = __fadd_rn(sum.x, p.x);
                        sum.y = __fadd_rn(sum.y, p.y);
                        sum.z = __fadd_rn(sum.z, p.z);
                        sum.w = __fadd_rn(sum.w, p.w);
                    }
                    v[mat][0] = sum.x; v[mat][1] = sum.y; v[mat][2] = sum.z; v[mat][3] = sum.w;
                    had128_warp(v[mat], lane);
                }
                const uint16_t* svh = static_cast<const uint16_t*>(tab_entry(cl.svh, ev.j));
                if (GU) {
                    const int64_t W = ev.R / 2;
                    const int64_t n0 = blk * 128 + 4 * lane;
                    float h[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        h[q] = silu_mul(__fmul_rn(v[0][q], h2f(svh[n0 + q])), __fmul_rn(v[MATS - 1][q], h2f(svh[W + n0 + q])));
                    }
                    uint16_t* y = out_row(op, i) + n0;
                    if (op.h_rot) {
                        const uint16_t* dn = static_cast<const uint16_t*>(tab_entry(cl.dn_suh, ev.j)) + blk * 128;
#pragma unroll
                        for (int q = 0; q < 4; ++q) h[q] = h2f(f2h(h[q]));
                        prologue_warp(h, dn, lane);
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q) y[q] = f2h(h[q]);
                } else {
                    const int64_t n0 = blk * 128 + 4 * lane;
                    uint16_t* y = out_row(op, i) + n0;
                    float o[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) o[q] = __fmul_rn(v[0][q], h2f(svh[n0 + q]));
                    st4_out(op, y, o);
                }
            }
            if (op.row_dst) __threadfence_system();   // rows in another GPU's memory: visible before the kernel ends
        }
        if (S > 1) cluster_sync_all(); else __syncthreads();
    }
}

// Shared memory a skinny launch needs.
int64_t skinny_smem(int bits, int gu, int mch, int64_t kc_max, int64_t n_expert) {
    const int mats = gu ? 2 : 1, mmax = 16 * mch;
    const int64_t stage = (int64_t)kTks * mats * 8 * 8 * bits * 4;
    const int64_t xr = (int64_t)mats * mmax * (kc_max + 8) * 2;
    const int64_t red = (int64_t)mmax * (mats * 128 + 4) * 4;
    return 256 + skinny_prefix_bytes(n_expert) + kNst * stage + (xr > red ? xr : red);
}

template <int BITS, int CB, bool GU, int MCH>
int launch_skinny_t(const Exl3bOp* op, const Exl3bPlan* p, int kc_max, int n_blocks, cudaStream_t st) {
    auto kern = k_gemm_skinny<BITS, CB, GU, MCH>;
    const int smem = p->smem_bytes;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -6;
    if (p->ksplit > 1 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
        return -6;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)p->ksplit, (unsigned)p->clusters, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)p->ksplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, *op, p->ksplit, kc_max, n_blocks);
    return e == cudaSuccess ? 0 : -6;
}

template <int BITS, bool GU, int MCH>
int launch_skinny_cb(const Exl3bOp* op, const Exl3bPlan* p, int kc_max, int n_blocks, cudaStream_t st) {
    switch (op->codebook) {
    case 0: return launch_skinny_t<BITS, 0, GU, MCH>(op, p, kc_max, n_blocks, st);
    case 1: return launch_skinny_t<BITS, 1, GU, MCH>(op, p, kc_max, n_blocks, st);
    case 2: return launch_skinny_t<BITS, 2, GU, MCH>(op, p, kc_max, n_blocks, st);
    default: return -1;
    }
}

template <int BITS, bool GU>
int launch_skinny_m(const Exl3bOp* op, const Exl3bPlan* p, int kc_max, int n_blocks, cudaStream_t st) {
    switch (p->mch) {
    case 1: return launch_skinny_cb<BITS, GU, 1>(op, p, kc_max, n_blocks, st);
    case 2: return launch_skinny_cb<BITS, GU, 2>(op, p, kc_max, n_blocks, st);
    case 4: return launch_skinny_cb<BITS, GU, 4>(op, p, kc_max, n_blocks, st);
    default: return -1;
    }
}

template <bool GU>
int launch_skinny_b(const Exl3bOp* op, const Exl3bPlan* p, int kc_max, int n_blocks, cudaStream_t st) {
    switch (op->bits) {
    case 2: return launch_skinny_m<2, GU>(op, p, kc_max, n_blocks, st);
    case 3: return launch_skinny_m<3, GU>(op, p, kc_max, n_blocks, st);
    case 4: return launch_skinny_m<4, GU>(op, p, kc_max, n_blocks, st);
    case 5: return launch_skinny_m<5, GU>(op, p, kc_max, n_blocks, st);
    case 6: return launch_skinny_m<6, GU>(op, p, kc_max, n_blocks, st);
    case 7: return launch_skinny_m<7, GU>(op, p, kc_max, n_blocks, st);
    case 8: return launch_skinny_m<8, GU>(op, p, kc_max, n_blocks, st);
    default: return -1;
    }
}

}  // namespace

// ============================================================================================ the C shim
extern "C" {

static inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

int exl3b_cuda_decode_what(const void* record, int64_t rows, int64_t cols, int bits, int codebook, void* out,
                           void* stream) {
    if (!record || !out || rows <= 0 || cols <= 0 || rows % 16 || cols % 16) return -1;
    const int64_t tiles = (rows / 16) * (cols / 16);
    const int wpb = 8;
    const dim3 grid((unsigned)((tiles + wpb - 1) / wpb)), block(wpb * 32);
    const uint32_t* r = static_cast<const uint32_t*>(record);
    uint16_t* o = static_cast<uint16_t*>(out);
    cudaStream_t st = as_stream(stream);
#define EXL3B_DW(B, C) k_decode_what<B, C><<<grid, block, 0, st>>>(r, rows, cols, o)
#define EXL3B_DW_CB(B)                    \
    switch (codebook) {                   \
    case 0: EXL3B_DW(B, 0); break;        \
    case 1: EXL3B_DW(B, 1); break;        \
    case 2: EXL3B_DW(B, 2); break;        \
    default: return -1;                   \
    }
    switch (bits) {
    case 1: EXL3B_DW_CB(1); break;
    case 2: EXL3B_DW_CB(2); break;
    case 3: EXL3B_DW_CB(3); break;
    case 4: EXL3B_DW_CB(4); break;
    case 5: EXL3B_DW_CB(5); break;
    case 6: EXL3B_DW_CB(6); break;
    case 7: EXL3B_DW_CB(7); break;
    case 8: EXL3B_DW_CB(8); break;
    default: return -1;
    }
#undef EXL3B_DW_CB
#undef EXL3B_DW
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

// The rotation pass into `dst` (row pitch `dst_pitch` elements): prep_gu's xr (gate_up ops) or down's rotated h.
int exl3b_cuda_device_info(int* sm_count, int32_t** err_word);   // exl3b200_moe.cu

int exl3b_cuda_prep(const Exl3bOp* op, void* dst, int64_t dst_pitch, void* stream) {
    if (op->T <= 0) return 0;
    int sm = 0;
    int32_t* err = nullptr;
    if (exl3b_cuda_device_info(&sm, &err) != 0) return -6;
    int64_t cmax = 0;
    for (int c = 0; c < op->n_class; ++c)
        if (op->cls[c].cols > cmax) cmax = op->cls[c].cols;
    const int ngrp = (int)((cmax / 128 + kPrepBpw - 1) / kPrepBpw);   // tasks a row: groups of kPrepBpw 128-blocks
    if (op->T * ngrp >= ((int64_t)1 << 31)) return -1;
    // enough warps to keep every SM's memory pipeline full (8 CTAs of 8 warps an SM), no more than the tasks
    const int64_t want = (op->T * ngrp + kPrepWarps - 1) / kPrepWarps;
    const int64_t cap = (int64_t)sm * 8;
    const unsigned grid = (unsigned)(want < cap ? (want > 0 ? want : 1) : cap);
    const size_t smem = (size_t)(op->n_expert + 1) * 4;
    k_prep<<<grid, kPrepWarps * 32, smem, as_stream(stream)>>>(*op, static_cast<uint16_t*>(dst), dst_pitch, ngrp);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

// Plan a decode-band launch: the rows a unit holds, the K split and the persistent grid. `sm_count` and the
// occupancy come from the device the caller queried once (no query on the launch path).
int exl3b_plan_skinny(const Exl3bOp* op, int sm_count, Exl3bPlan* p) {
    const int gu = op->op == EXL3B_OP_GATE_UP;
    int64_t cmin = op->cls[0].cols, wmax = 0;
    for (int c = 0; c < op->n_class; ++c) {
        if (op->cls[c].cols < cmin) cmin = op->cls[c].cols;
        const int64_t w = gu ? op->cls[c].rows / 2 : op->cls[c].rows;
        if (w > wmax) wmax = w;
    }
    const int64_t n_blocks = wmax / 128;
    const int64_t live = op->n_expert < op->T ? op->n_expert : op->T;
    const int64_t rows_per = live > 0 ? (op->T + live - 1) / live : 1;
    int mch = rows_per <= 16 ? 1 : rows_per <= 32 ? 2 : 4;
    const int64_t mmax = 16 * mch;
    const int64_t units = (live + op->T / mmax + 1) * n_blocks;
    // split K until the units fill the machine twice over (a power of two, at most 8, at most the chunks)
    int S = 1;
    const int64_t nch_min = cmin / 128;
    while (S < 8 && units * S < 2 * sm_count && 2 * S <= nch_min) S *= 2;
    int64_t kc_max = 0;
    for (int c = 0; c < op->n_class; ++c) {
        const int64_t nch = op->cls[c].cols / 128;
        const int64_t per = (nch + S - 1) / S * 128;
        if (per > kc_max) kc_max = per;
    }
    int64_t smem = skinny_smem(op->bits, gu, mch, kc_max, op->n_expert);
    // too much shared memory: split K further first (the rows a unit holds decide how often a weight is decoded),
    // and only then hold fewer rows
    while (smem > 220 * 1024 && S < 8 && 2 * S <= nch_min) {
        S *= 2;
        kc_max = 0;
        for (int c = 0; c < op->n_class; ++c) {
            const int64_t nch = op->cls[c].cols / 128;
            const int64_t per = (nch + S - 1) / S * 128;
            if (per > kc_max) kc_max = per;
        }
        smem = skinny_smem(op->bits, gu, mch, kc_max, op->n_expert);
    }
    while (smem > 220 * 1024 && mch > 1) {
        mch /= 2;
        smem = skinny_smem(op->bits, gu, mch, kc_max, op->n_expert);
    }
    if (smem > 227 * 1024) return -1;
    const int64_t per_sm = smem <= 56 * 1024 ? 4 : smem <= 75 * 1024 ? 3 : smem <= 113 * 1024 ? 2 : 1;
    int64_t clusters = sm_count * per_sm / S;
    const int64_t units_max = (live + op->T / (16 * mch) + 1) * n_blocks;
    if (clusters > units_max) clusters = units_max;
    if (clusters < 1) clusters = 1;
    p->ksplit = S;
    p->mch = mch;
    p->clusters = (int)clusters;
    p->smem_bytes = (int)smem;
    return 0;
}

int exl3b_cuda_gemm_skinny(const Exl3bOp* op, const Exl3bPlan* p, void* stream) {
    const int gu = op->op == EXL3B_OP_GATE_UP;
    int64_t wmax = 0, kc_max = 0;
    for (int c = 0; c < op->n_class; ++c) {
        const int64_t w = gu ? op->cls[c].rows / 2 : op->cls[c].rows;
        if (w > wmax) wmax = w;
        const int64_t nch = op->cls[c].cols / 128;
        const int64_t per = (nch + p->ksplit - 1) / p->ksplit * 128;
        if (per > kc_max) kc_max = per;
    }
    cudaStream_t st = as_stream(stream);
    return gu ? launch_skinny_b<true>(op, p, (int)kc_max, (int)(wmax / 128), st)
              : launch_skinny_b<false>(op, p, (int)kc_max, (int)(wmax / 128), st);
}

}  // extern "C"
