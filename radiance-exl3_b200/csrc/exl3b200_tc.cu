// exl3b200_tc.cu -- the prefill band on the 5th-generation tensor cores: trellis decode fused into a tcgen05 grouped
// GEMM with its accumulators in tensor memory. sm_100a only.
//
// One persistent CTA an SM walks the unit list -- unit = (expert, up to 64 of its sorted rows, two 128-row output
// blocks: gate block b with up block b for gate_up, blocks 2q and 2q+1 for down) -- with warp-specialised roles:
//
//   warps 0..7   epilogue: tcgen05.ld of a finished unit's accumulators (lane quadrant = warp % 4, block = warp / 4),
//                the rotation over n (transposed through shared memory), svh, SiLU(gate)*up and h_rot / bf16, stores
//   warp 8       producer: cp.async.bulk (TMA) of the unit's record rows, and cp.async.bulk.tensor of the input rows
//                (xr / h, sorted order) through a 128-byte-swizzled tensor map
//   warp 9       TMEM allocator and MMA issuer: tcgen05.mma.cta_group::1.kind::f16, M=128 (weight rows), N=64
//                (sorted rows), K=16, A and B from shared memory, D in TMEM; tcgen05.commit frees stages
//   warps 10..25 decoders: each lane decodes 8 trellis positions of a tile (the same bit-exact decode as the
//                decode-band kernel) and stores them into the A tile in the canonical K-major SWIZZLE_128B layout
//
// Accumulators are double-buffered (two units x 2 blocks x 64 columns = 256 TMEM columns), so the epilogue of one
// unit runs while the next is decoded. Every wait is bounded (then the error word is set); TMEM is freed by the
// allocating warp before the CTA exits on every path.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "exl3b200_dev.h"
#include "exl3b200_decode.cuh"

namespace {

constexpr int kEpiWarps = 8;                         // two a TMEM lane quadrant (warp % 4)
constexpr int kProdWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kDecWarp0 = 10;
constexpr int kDecWarps = 16;
constexpr int kTcWarps = kDecWarp0 + kDecWarps;      // 26
constexpr int kTcThreads = kTcWarps * 32;           // 832
constexpr int kNT = 64;                              // sorted rows a unit (the MMA's N)
constexpr int kKC = 64;                              // k a pipeline chunk (one SWIZZLE_128B atom wide)
constexpr int kStA = 3, kStB = 3;                    // stages of the A and B rings
constexpr int kATile = 128 * kKC * 2;                // one block's A chunk: 16 KB
constexpr int kBTile = kNT * kKC * 2;                // one half's B chunk: 8 KB
constexpr int kEpiCols = 128 + 4;                    // staging row (f32), padded
constexpr int kTmemCols = 256;

template <int BITS>
struct TcCfg {
    static constexpr int TILE_BYTES = 32 * BITS;                 // one 16x16 tile of the record
    static constexpr int REC_ROW = 8 * TILE_BYTES;               // one block's 8 tiles of one k row
    static constexpr int REC_STAGE = 4 * 2 * REC_ROW;            // [tk 4][blk 2][8 tiles]
    // the record ring runs deep (the rows are small, latency-bound reads): 3..8 stages within 48 KB
    static constexpr int ST_R = (48 * 1024 / REC_STAGE) < 3 ? 3 : (48 * 1024 / REC_STAGE) > 8 ? 8 : (48 * 1024 / REC_STAGE);
};

// ------------------------------------------------------------------------------------------ smem descriptors
// K-major, SWIZZLE_128B: rows 128 B apart inside 8-row atoms of 1024 B (SBO), the 16-byte chunks of a row XOR-ed
// with the row's index in its atom; LBO unused (1). Version 1 (tcgen05), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);          // start address
    d |= (uint64_t)1 << 16;                                  // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;                        // SBO: 8-row atom stride
    d |= (uint64_t)1 << 46;                                  // version
    d |= (uint64_t)2 << 61;                                  // SWIZZLE_128B
    return d;
}
// kind::f16, A = B = f16, D = f32, both K-major, M = 128, N = kNT.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kNT >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float v[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 2-D tensor copy global -> shared (no multicast), completing on `bar`.
__device__ __forceinline__ void tma_tile_g2s(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// ------------------------------------------------------------------------------------------ units
// Unit u -> (expert, row group, block pair). Units of expert e: ceil(rows_e / 64) * n_pairs.
struct TcUnit {
    int64_t e, r0;
    int nr, pair;
};

__device__ __forceinline__ TcUnit tc_unit(const Exl3bOp& op, const uint32_t* prefix, int64_t unit, int n_pairs) {
    int64_t lo = 0, hi = op.n_expert;
    while (hi - lo > 1) {
        const int64_t mid = (lo + hi) / 2;
        if ((int64_t)prefix[mid] <= unit) lo = mid; else hi = mid;
    }
    TcUnit u;
    u.e = lo;
    const int64_t local = unit - prefix[lo];
    const int64_t grp = local / n_pairs;
    u.pair = (int)(local % n_pairs);
    u.r0 = op.expert_offset[lo] + grp * kNT;
    const int64_t rend = op.expert_offset[lo + 1];
    u.nr = (int)(rend - u.r0 < kNT ? rend - u.r0 : kNT);
    return u;
}

// ------------------------------------------------------------------------------------------ the kernel
template <int BITS, int CB, bool GU>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmap, const Exl3bOp op, int n_pairs) {
    using Cfg = TcCfg<BITS>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment of every swizzled tile
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a_ring = smem;                                        // [kStA][2][16 KB]
    uint8_t* b_ring = a_ring + kStA * 2 * kATile;                  // [kStB][2][8 KB]
    uint8_t* r_ring = b_ring + kStB * 2 * kBTile;                  // [ST_R][REC_STAGE]
    float* epi = reinterpret_cast<float*>(r_ring + Cfg::ST_R * Cfg::REC_STAGE);   // [2][16][kEpiCols]
    uint64_t* bars = reinterpret_cast<uint64_t*>(epi + 2 * 16 * kEpiCols);
    uint64_t* a_full = bars;                 // decoders -> MMA (count kDecWarps)
    uint64_t* a_empty = a_full + kStA;       // MMA commit -> decoders
    uint64_t* b_full = a_empty + kStA;       // producer tx -> MMA
    uint64_t* b_empty = b_full + kStB;       // MMA commit -> producer
    uint64_t* r_full = b_empty + kStB;       // producer tx -> decoders
    uint64_t* r_empty = r_full + Cfg::ST_R;  // decoders -> producer (count kDecWarps)
    uint64_t* acc_full = r_empty + Cfg::ST_R;  // MMA commit -> epilogue [2]
    uint64_t* acc_empty = acc_full + 2;      // epilogue -> MMA [2] (count kEpiWarps)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    uint32_t* prefix = tmem_slot + 4;        // [n_expert + 1]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t n_exp = op.n_expert;

    if (tid == 0) {
        for (int s = 0; s < kStA; ++s) { mbar_init(&a_full[s], kDecWarps); mbar_init(&a_empty[s], 1); }
        for (int s = 0; s < kStB; ++s) { mbar_init(&b_full[s], 1); mbar_init(&b_empty[s], 1); }
        for (int s = 0; s < Cfg::ST_R; ++s) { mbar_init(&r_full[s], 1); mbar_init(&r_empty[s], kDecWarps); }
        for (int s = 0; s < 2; ++s) { mbar_init(&acc_full[s], 1); mbar_init(&acc_empty[s], kEpiWarps); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // the unit list: ceil(rows_e / 64) * n_pairs units an expert, expert-major
    {
        __shared__ uint32_t part[kTcThreads];
        const int64_t per = (n_exp + kTcThreads - 1) / kTcThreads;
        const int64_t e0 = tid * per, e1 = e0 + per < n_exp ? e0 + per : n_exp;
        uint32_t sum = 0;
        for (int64_t e = e0; e < e1; ++e) {
            const int64_t r = op.expert_offset[e + 1] - op.expert_offset[e];
            sum += r > 0 ? (uint32_t)(((r + kNT - 1) / kNT) * n_pairs) : 0u;
        }
        part[tid] = sum;
        __syncthreads();
        if (tid == 0) {
            uint32_t acc = 0;
            for (int t = 0; t < kTcThreads; ++t) {
                const uint32_t v = part[t];
                part[t] = acc;
                acc += v;
            }
            prefix[n_exp] = acc;
        }
        __syncthreads();
        uint32_t acc = part[tid];
        for (int64_t e = e0; e < e1; ++e) {
            prefix[e] = acc;
            const int64_t r = op.expert_offset[e + 1] - op.expert_offset[e];
            acc += r > 0 ? (uint32_t)(((r + kNT - 1) / kNT) * n_pairs) : 0u;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int64_t n_units = prefix[n_exp];

    // rows no unit writes are zeroed (outside the runs, dropped slots), by every CTA over a slice of the rows
    if (warp < kEpiWarps || warp >= kDecWarp0) {
        const int64_t lt = warp < kEpiWarps ? tid : tid - (kDecWarp0 - kEpiWarps) * 32;   // 0 .. nthr-1
        const int64_t nthr = (kEpiWarps + kDecWarps) * 32;
        for (int64_t i = blockIdx.x; i < op.T; i += gridDim.x) {
            const bool live = i >= op.expert_offset[0] && i < op.expert_offset[n_exp] && op.sorted_tok[i] >= 0;
            if (live) continue;
            uint16_t* y = static_cast<uint16_t*>(op.y) + i * op.y_pitch;
            for (int64_t c = lt; c < op.y_cols; c += nthr) y[c] = 0;
        }
    }

    if (warp == kProdWarp) {
        // ---------------------------------------------------------------- producer
        // lane 0 streams the record rows, lane 1 the input-row tiles: two independent rings, so neither waits on
        // the other's consumer
        if (lane < 2) {
            uint32_t ri = 0, bi = 0;
            for (int64_t unit = blockIdx.x; unit < n_units; unit += gridDim.x) {
                const TcUnit u = tc_unit(op, prefix, unit, n_pairs);
                const ExpertView ev = expert_view(op, u.e);
                const Exl3bClass& cl = op.cls[ev.c];
                const int64_t wrows = GU ? ev.R / 2 : ev.R;          // rows of one record
                if ((int64_t)u.pair * 256 >= (GU ? 2 * wrows : wrows)) continue;   // a narrower class
                const int nck = (int)(ev.C / kKC);
                if (lane == 0) {
                    const uint16_t* rec = static_cast<const uint16_t*>(tab_entry(cl.codes, ev.j));
                    const int64_t mat_elems = (ev.C / 16) * (wrows / 16) * 16 * BITS;
                    for (int ck = 0; ck < nck; ++ck, ++ri) {
                        const uint32_t s = ri % Cfg::ST_R, ph = (ri / Cfg::ST_R) & 1;
                        mbar_wait(&r_empty[s], ph ^ 1, op.err);
                        mbar_expect_tx(&r_full[s], (uint32_t)Cfg::REC_STAGE);
                        for (int q = 0; q < 4; ++q) {
                            const int64_t tk = (int64_t)ck * 4 + q;
                            uint8_t* dst = r_ring + s * Cfg::REC_STAGE + q * 2 * Cfg::REC_ROW;
                            if (GU) {
                                for (int m = 0; m < 2; ++m) {
                                    const uint16_t* src = rec + m * mat_elems + (tk * (wrows / 16) + u.pair * 8) * 16 * BITS;
                                    tma_bulk_g2s(dst + m * Cfg::REC_ROW, src, Cfg::REC_ROW, &r_full[s]);
                                }
                            } else {
                                const uint16_t* src = rec + (tk * (wrows / 16) + u.pair * 16) * 16 * BITS;
                                tma_bulk_g2s(dst, src, 2 * Cfg::REC_ROW, &r_full[s]);
                            }
                        }
                    }
                } else {
                    // input rows of each chunk (sorted rows r0 .. r0+63; zero fill past T)
                    for (int ck = 0; ck < nck; ++ck, ++bi) {
                        const uint32_t s = bi % kStB, ph = (bi / kStB) & 1;
                        mbar_wait(&b_empty[s], ph ^ 1, op.err);
                        mbar_expect_tx(&b_full[s], (uint32_t)((GU ? 2 : 1) * kBTile));
                        for (int m = 0; m < (GU ? 2 : 1); ++m)
                            tma_tile_g2s(b_ring + (s * 2 + m) * kBTile, &tmap, (int)(m * ev.C + ck * kKC), (int)u.r0,
                                         &b_full[s]);
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            // the ring bases' descriptors; a stage, block and k step only add to the start-address field (the
            // shared-memory window is below 256 KB, so the 14-bit field never carries)
            const uint64_t a_desc0 = sw128_desc(smem_u32(a_ring)), b_desc0 = sw128_desc(smem_u32(b_ring));
            uint32_t ai = 0, bi = 0, ui = 0;
            for (int64_t unit = blockIdx.x; unit < n_units; unit += gridDim.x) {
                const TcUnit u = tc_unit(op, prefix, unit, n_pairs);
                const ExpertView ev = expert_view(op, u.e);
                const int64_t wrows = GU ? ev.R / 2 : ev.R;
                if ((int64_t)u.pair * 256 >= (GU ? 2 * wrows : wrows)) continue;
                const uint32_t buf = ui & 1, uph = (ui >> 1) & 1;
                mbar_wait(&acc_empty[buf], uph ^ 1, op.err);
                tc_fence_after();
                const int nck = (int)(ev.C / kKC);
                for (int ck = 0; ck < nck; ++ck) {
                    const uint32_t sa = ai % kStA, pa = (ai / kStA) & 1;
                    const uint32_t sb = bi % kStB, pb = (bi / kStB) & 1;
                    mbar_wait(&a_full[sa], pa, op.err);
                    mbar_wait(&b_full[sb], pb, op.err);
                    tc_fence_after();
                    const uint64_t da = a_desc0 + (uint64_t)((sa * 2 * kATile) >> 4);
                    const uint64_t db = b_desc0 + (uint64_t)((sb * 2 * kBTile) >> 4);
                    const uint32_t d = tmem + buf * (2 * kNT);
#pragma unroll
                    for (int blk = 0; blk < 2; ++blk)
#pragma unroll
                        for (int ks = 0; ks < kKC / 16; ++ks)
                            umma_f16(d + blk * kNT, da + (uint64_t)((blk * kATile + ks * 32) >> 4),
                                     db + (uint64_t)(((GU ? blk : 0) * kBTile + ks * 32) >> 4), (ck | ks) ? 1u : 0u);
                    umma_commit(&a_empty[sa]);
                    umma_commit(&b_empty[sb]);
                    ++ai;
                    ++bi;
                }
                umma_commit(&acc_full[buf]);
                ++ui;
            }
        }
        __syncwarp();
    } else if (warp >= kDecWarp0) {
        // ---------------------------------------------------------------- decoders
        const int dw = warp - kDecWarp0;           // 0..15: block dw / 8, tile column dw % 8
        const int blk = dw >> 3, tn = dw & 7;
        const int g = lane >> 2, t = lane & 3;
        const LaneDec<BITS> ld = lane_dec<BITS>(lane);
        // this lane's places in the SW128 K-major A tile: row n = 16 tn + g (+8) at (n/8)*1024 + (n%8)*128, the
        // 16-byte chunk c = k/8 at (c ^ (n%8)) * 16, k = 16 q + 2t (+8)
        const uint32_t row_lo = (uint32_t)((2 * tn) * 1024 + g * 128 + 4 * t);
        const uint32_t xg = (uint32_t)g << 4;
        const uint32_t tile_off = (uint32_t)(blk * Cfg::REC_ROW + tn * Cfg::TILE_BYTES);
        uint32_t ai = 0, ri = 0;
        for (int64_t unit = blockIdx.x; unit < n_units; unit += gridDim.x) {
            const TcUnit u = tc_unit(op, prefix, unit, n_pairs);
            const ExpertView ev = expert_view(op, u.e);
            const int64_t wrows = GU ? ev.R / 2 : ev.R;
            if ((int64_t)u.pair * 256 >= (GU ? 2 * wrows : wrows)) continue;
            const int nck = (int)(ev.C / kKC);
            for (int ck = 0; ck < nck; ++ck) {
                const uint32_t sr = ri % Cfg::ST_R, pr = (ri / Cfg::ST_R) & 1;
                const uint32_t sa = ai % kStA, pa = (ai / kStA) & 1;
                mbar_wait(&r_full[sr], pr, op.err);
                mbar_wait(&a_empty[sa], pa ^ 1, op.err);
                uint8_t* arow = a_ring + (sa * 2 + blk) * kATile + row_lo;
                const uint8_t* rst = r_ring + sr * Cfg::REC_STAGE + tile_off;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint32_t b[4];
                    decode_tile<BITS, CB>(rst + q * 2 * Cfg::REC_ROW, ld, b);
                    const uint32_t c0 = ((uint32_t)(2 * q) << 4) ^ xg, c1 = ((uint32_t)(2 * q + 1) << 4) ^ xg;
                    *reinterpret_cast<uint32_t*>(arow + c0) = b[0];
                    *reinterpret_cast<uint32_t*>(arow + c1) = b[1];
                    *reinterpret_cast<uint32_t*>(arow + 1024 + c0) = b[2];
                    *reinterpret_cast<uint32_t*>(arow + 1024 + c1) = b[3];
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&a_full[sa]);
                    mbar_arrive(&r_empty[sr]);
                }
                ++ai;
                ++ri;
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue (warps 0..7)
        const int q = warp & 3;                      // TMEM lanes 32q .. 32q+31 = weight rows of a block
        const int eb = warp >> 2;                    // the block this warp moves out of TMEM
        uint32_t ui = 0;
        for (int64_t unit = blockIdx.x; unit < n_units; unit += gridDim.x) {
            const TcUnit u = tc_unit(op, prefix, unit, n_pairs);
            const ExpertView ev = expert_view(op, u.e);
            const Exl3bClass& cl = op.cls[ev.c];
            const int64_t wrows = GU ? ev.R / 2 : ev.R;
            if ((int64_t)u.pair * 256 >= (GU ? 2 * wrows : wrows)) {
                // a narrower class: its live rows are zero across this pair's columns
                const int64_t c0 = (int64_t)u.pair * (GU ? 128 : 256), nc = GU ? 128 : 256;
                for (int m = 0; m < u.nr; ++m) {
                    const int64_t i = u.r0 + m;
                    if (op.sorted_tok[i] < 0) continue;
                    uint16_t* y = static_cast<uint16_t*>(op.y) + i * op.y_pitch + c0;
                    for (int64_t c = tid; c < nc; c += kEpiWarps * 32) y[c] = 0;
                }
                continue;
            }
            // the unit's output scales, held for all its rows: lane l owns columns 4l .. 4l+3 of each block
            const uint16_t* svh = static_cast<const uint16_t*>(tab_entry(cl.svh, ev.j));
            float s0[4], s1[4], sd[4];
            const int64_t n0 = (int64_t)u.pair * (GU ? 128 : 256) + 4 * lane;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                s0[e] = h2f(svh[n0 + e]);
                s1[e] = GU ? h2f(svh[ev.R / 2 + n0 + e]) : h2f(svh[n0 + 128 + e]);
                sd[e] = 0.f;
            }
            const uint16_t* dn = GU && op.h_rot ? static_cast<const uint16_t*>(tab_entry(cl.dn_suh, ev.j)) : nullptr;
            uint16_t dsuh[4] = { 0, 0, 0, 0 };
            if (dn) {
#pragma unroll
                for (int e = 0; e < 4; ++e) dsuh[e] = dn[(int64_t)u.pair * 128 + 4 * lane + e];
            }
            (void)sd;
            const uint32_t buf = ui & 1, uph = (ui >> 1) & 1;
            mbar_wait(&acc_full[buf], uph, op.err);
            tc_fence_after();
            for (int sl = 0; sl < kNT / 16; ++sl) {
                if (sl * 16 >= u.nr) break;
                // TMEM -> staging [blk][16 rows][n]: this warp's block, its 32 weight rows
                {
                    float v[16];
                    tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + buf * (2 * kNT) + eb * kNT + sl * 16, v);
#pragma unroll
                    for (int j = 0; j < 16; ++j) epi[(eb * 16 + j) * kEpiCols + 32 * q + lane] = v[j];
                }
                asm volatile("bar.sync 2, %0;" ::"n"(kEpiWarps * 32) : "memory");
                // rows: warp w takes rows w and w + 8 of the slice
                for (int j = warp; j < 16; j += kEpiWarps) {
                    const int m = sl * 16 + j;
                    if (m >= u.nr) continue;
                    const int64_t i = u.r0 + m;
                    if (op.sorted_tok[i] < 0) continue;
                    const float4 av = *reinterpret_cast<const float4*>(&epi[(0 * 16 + j) * kEpiCols + 4 * lane]);
                    const float4 bv = *reinterpret_cast<const float4*>(&epi[(1 * 16 + j) * kEpiCols + 4 * lane]);
                    float a[4] = { av.x, av.y, av.z, av.w }, b[4] = { bv.x, bv.y, bv.z, bv.w };
                    had128_warp(a, lane);
                    had128_warp(b, lane);
                    uint16_t* y = static_cast<uint16_t*>(op.y) + i * op.y_pitch + n0;
                    if (GU) {
                        float h[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float gte = __fmul_rn(a[e], s0[e]);
                            const float up = __fmul_rn(b[e], s1[e]);
                            const float sg = __fmul_rn(gte, __frcp_rn(__fadd_rn(1.0f, expf(-gte))));
                            h[e] = __fmul_rn(sg, up);
                        }
                        if (dn) {
#pragma unroll
                            for (int e = 0; e < 4; ++e) h[e] = h2f(f2h(__fmul_rn(h2f(f2h(h[e])), h2f(dsuh[e]))));
                            had128_warp(h, lane);
                        }
                        uint2 pk;
                        pk.x = (uint32_t)f2h(h[0]) | ((uint32_t)f2h(h[1]) << 16);
                        pk.y = (uint32_t)f2h(h[2]) | ((uint32_t)f2h(h[3]) << 16);
                        if ((reinterpret_cast<uintptr_t>(y) & 7) == 0) {
                            *reinterpret_cast<uint2*>(y) = pk;
                        } else {
#pragma unroll
                            for (int e = 0; e < 4; ++e) y[e] = f2h(h[e]);
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            y[e] = f2bf(__fmul_rn(a[e], s0[e]));
                            y[128 + e] = f2bf(__fmul_rn(b[e], s1[e]));
                        }
                    }
                }
                asm volatile("bar.sync 2, %0;" ::"n"(kEpiWarps * 32) : "memory");
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
            ++ui;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

template <int BITS, int CB, bool GU>
int launch_tc_t(const CUtensorMap& map, const Exl3bOp* op, int n_pairs, int grid, int smem, cudaStream_t st) {
    auto kern = k_gemm_tc<BITS, CB, GU>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -6;
    kern<<<grid, kTcThreads, smem, st>>>(map, *op, n_pairs);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

template <bool GU>
int launch_tc_b(const CUtensorMap& map, const Exl3bOp* op, int n_pairs, int grid, int smem, cudaStream_t st) {
#define EXL3B_TC_CB(B)                                                          \
    switch (op->codebook) {                                                     \
    case 0: return launch_tc_t<B, 0, GU>(map, op, n_pairs, grid, smem, st);     \
    case 1: return launch_tc_t<B, 1, GU>(map, op, n_pairs, grid, smem, st);     \
    case 2: return launch_tc_t<B, 2, GU>(map, op, n_pairs, grid, smem, st);     \
    default: return -1;                                                         \
    }
    switch (op->bits) {
    case 2: EXL3B_TC_CB(2)
    case 3: EXL3B_TC_CB(3)
    case 4: EXL3B_TC_CB(4)
    case 5: EXL3B_TC_CB(5)
    case 6: EXL3B_TC_CB(6)
    case 7: EXL3B_TC_CB(7)
    case 8: EXL3B_TC_CB(8)
    default: return -1;
    }
#undef EXL3B_TC_CB
}

}  // namespace

// ============================================================================================ the C shim
extern "C" {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

int64_t exl3b_tc_smem_bytes(int bits) {
    const int64_t rec_stage = 4 * 2 * 8 * 32 * bits;
    int64_t st_r = 48 * 1024 / rec_stage;
    st_r = st_r < 3 ? 3 : st_r > 8 ? 8 : st_r;
    const int64_t b = (int64_t)kStA * 2 * kATile + (int64_t)kStB * 2 * kBTile + st_r * rec_stage +
                      2 * 16 * kEpiCols * 4 + 256;
    return 1024 + b;   // the alignment slack; the unit prefix follows (added by the caller)
}

// The B operand of the tensor-core path: rows [T] x `cols` f16 with row pitch `pitch` elements, read in
// 64 x 64 boxes, 128-byte swizzled.
static int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t pitch) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return -6;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (pitch * 2) % 16) return -3;
    const cuuint64_t dims[2] = { (cuuint64_t)cols, (cuuint64_t)rows };
    const cuuint64_t strides[1] = { (cuuint64_t)(pitch * 2) };
    const cuuint32_t box[2] = { (cuuint32_t)kKC, (cuuint32_t)kNT };
    const cuuint32_t estr[2] = { 1, 1 };
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -6;
}

// gate_up (xr = the rotated input, [T][2 * x_cols] f16 in sorted order, gate half then up half per row) or down
// (h_rot 1: h itself, [T][x_cols]). Every class's input width must be a multiple of 64 and its output a multiple of
// 256 rows (gate_up: 2 x 128, down: 256) -- the host checks.
int exl3b_cuda_gemm_tc(const Exl3bOp* op, const void* xin, int64_t xin_pitch, int sm_count, void* stream) {
    const bool gu = op->op == EXL3B_OP_GATE_UP;
    int64_t wmax = 0;
    for (int c = 0; c < op->n_class; ++c) {
        const int64_t w = gu ? op->cls[c].rows : op->cls[c].rows;
        if (w > wmax) wmax = w;
    }
    const int n_pairs = (int)(wmax / 256);
    CUtensorMap map;
    const int64_t cols = gu ? 2 * op->x_cols : op->x_cols;
    int rc = make_map(&map, xin, op->T, cols, xin_pitch);
    if (rc) return rc;
    const int64_t smem = exl3b_tc_smem_bytes(op->bits) + ((op->n_expert + 1) * 4 + 15) / 16 * 16 + 16;
    if (smem > 227 * 1024) return -1;
    int grid = sm_count;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return gu ? launch_tc_b<true>(map, op, n_pairs, grid, (int)smem, st)
              : launch_tc_b<false>(map, op, n_pairs, grid, (int)smem, st);
}

}  // extern "C"
