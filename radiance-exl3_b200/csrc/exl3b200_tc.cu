// exl3b200_tc.cu -- the prefill band on the 5th-generation tensor cores: trellis decode fused into a tcgen05 grouped
// GEMM with its accumulators in tensor memory. sm_100a only.
//
// One persistent CTA an SM walks the unit list -- unit = (expert, up to 64 of its sorted rows, two 128-row output
// blocks: gate block b with up block b for gate_up, blocks 2q and 2q+1 for down) -- with warp-specialised roles.
// The WIDE form takes up to 128 rows a unit: a unit of more than 64 rows decodes its weights once and multiplies
// both 64-row halves, each half into its own accumulator buffer (two MMA sets a chunk), so an expert's weights are
// decoded once a 128 rows (the host picks it for passes of many rows an expert and many units).
//
//   warps 0..7   epilogue: tcgen05.ld of a finished unit's accumulators (lane quadrant = warp % 4, block = warp / 4),
//                the rotation over n (transposed through shared memory), svh, SiLU(gate)*up and h_rot / bf16, stores
//   warp 8       record producer: cp.async.bulk (TMA) of the unit's record rows into a deep ring
//   warp 9       input producer: cp.async.bulk.tensor of the input rows (xr / h, sorted order) through a
//                128-byte-swizzled tensor map
//   warps 10, 11 MMA issuers (warp 10 also allocates TMEM): tcgen05.mma.cta_group::1.kind::f16, M=128 (weight rows),
//                N=64 (sorted rows), K=16, one warp a block; A (the decoded weights) from TENSOR memory, B from
//                shared memory, D in tensor memory; tcgen05.commit frees stages
//   warps 12..27 decoders: each lane decodes 8 trellis positions of a tile (the same bit-exact decode as the
//                decode-band kernel) -- exactly the 16x128b.x2 tcgen05.st fragment of a 16-row x 16-k A tile
//                (lane g: rows g, g+8; 32-bit columns t, t+4 = k pairs 2t, 2t+8) -- and stores it into tensor
//                memory; a decoder warp writes only its own TMEM lane quadrant (warp % 4)
//
// Tensor memory (512 columns): two accumulator buffers (2 x 2 blocks x 64 columns, so the epilogue of one 64-row
// half runs while the next is computed; a wide unit takes both) and kStA A stages of 2 blocks x kKC / 2 columns (128 lanes x kKC k of f16).
// Shared memory holds only the input-row ring, the record ring and the epilogue's staging. Every wait is bounded
// (then the error word is set); TMEM is freed by the allocating warp before the CTA exits on every path.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "exl3b200_dev.h"
#include "exl3b200_decode.cuh"

namespace {

constexpr int kEpiWarps = 8;                         // two a TMEM lane quadrant (warp % 4)
constexpr int kRecWarp = 8;
constexpr int kBWarp = 9;
constexpr int kMmaWarp = 10;                         // block 0's MMAs (and the TMEM allocation); 11: block 1's
constexpr int kDecWarp0 = 12;
#ifndef EXL3B_TC_DEC_TN
#define EXL3B_TC_DEC_TN 1
#endif
constexpr int kDecTn = EXL3B_TC_DEC_TN;              // 16-row tile rows a decoder warp takes (1 or 2)
constexpr int kDecWarps = 16 / kDecTn;               // 16 / kDecTn: 4 / kDecTn a lane quadrant
constexpr int kTcWarps = kDecWarp0 + kDecWarps;      // 28
constexpr int kTcThreads = kTcWarps * 32;           // 896
constexpr int kNT = 64;                              // sorted rows a half unit (the MMA's N; one accumulator buffer)
constexpr int kUG = 2 * kNT;                         // sorted rows a wide unit at most (two halves)
constexpr int kWideUnitsPerSm = 4;                   // wide units are chosen only with at least this many an SM
constexpr int kWideMinCols = 1024;                   // ... and an input at least this wide (16+ chunks a unit)
constexpr int kBox = 64;                             // k of one TMA box = one SWIZZLE_128B atom row (128 B)
constexpr int kKC = 128;                             // k a pipeline chunk: one handoff between the roles
constexpr int kKT = kKC / 16;                        // k tiles a chunk
constexpr int kNBox = kKC / kBox;                    // boxes a half of a chunk
constexpr int kStA = 2;                              // A stages (tensor memory)
constexpr int kBTile = kNT * kBox * 2;               // one box of input rows: 8 KB
constexpr int kBHalf = kNBox * kBTile;               // one half's input rows of a chunk
constexpr int kEpiCols = 128 + 4;                    // staging row (f32), padded
constexpr int kAccCols = 2 * 2 * kNT;                // 256: two units x two blocks
constexpr int kAStageCols = 2 * kKC / 2;             // two blocks x kKC k of f16 (two a 32-bit column)
constexpr int kTmemCols = 512;
constexpr int kUnitTab = 160;                        // a CTA's units held in a shared table (more: looked up)
static_assert(kAccCols + kStA * kAStageCols <= kTmemCols, "tensor memory");

template <int BITS>
struct TcCfg {
    static constexpr int TILE_BYTES = 32 * BITS;                 // one 16x16 tile of the record
    static constexpr int REC_ROW = 8 * TILE_BYTES;               // one block's 8 tiles of one k row
    static constexpr int REC_STAGE = kKT * 2 * REC_ROW;          // [tk][blk 2][8 tiles]
    // the record ring runs deep (the rows are small, latency-bound reads): 3..12 stages within 64 KB
    static constexpr int ST_R = (64 * 1024 / REC_STAGE) < 3 ? 3 : (64 * 1024 / REC_STAGE) > 12 ? 12 : (64 * 1024 / REC_STAGE);
    // input-row stages: as many as shared memory leaves beside the record ring
    static constexpr int ST_B = BITS >= 6 ? 3 : 4;
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

// The 8 MMAs of one 128-row block over a 128-k chunk (K = 16 each): A from tensor memory at ta, ta + 8, ..., B from
// the two 64-k boxes of the input stage (descriptors db0, db1; a 16-k step adds 32 bytes = 2 to the start address).
// One elected lane issues all eight; the first accumulates only when `acc` is nonzero, the others always.
__device__ __forceinline__ void umma_block8_el(uint32_t d, uint32_t ta, uint64_t db0, uint64_t db1, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p, e, t;\n .reg .b32 a;\n .reg .b64 b;\n"
        " setp.ne.b32 p, %4, 0;\n setp.eq.b32 t, 0, 0;\n elect.sync _|e, 0xffffffff;\n"
        " @e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %5, p;\n"
        " add.u32 a, %1, 8;  add.u64 b, %2, 2;\n @e tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %5, t;\n"
        " add.u32 a, %1, 16; add.u64 b, %2, 4;\n @e tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %5, t;\n"
        " add.u32 a, %1, 24; add.u64 b, %2, 6;\n @e tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %5, t;\n"
        " add.u32 a, %1, 32;\n @e tcgen05.mma.cta_group::1.kind::f16 [%0], [a], %3, %5, t;\n"
        " add.u32 a, %1, 40; add.u64 b, %3, 2;\n @e tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %5, t;\n"
        " add.u32 a, %1, 48; add.u64 b, %3, 4;\n @e tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %5, t;\n"
        " add.u32 a, %1, 56; add.u64 b, %3, 6;\n @e tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %5, t;\n"
        "}\n" ::"r"(d), "r"(ta), "l"(db0), "l"(db1), "r"(acc), "r"(kIdesc));
}
__device__ __forceinline__ void tmem_st_16x128b_x2(uint32_t taddr, uint32_t r0, uint32_t r1, uint32_t r2,
                                                   uint32_t r3) {
    asm volatile("tcgen05.st.sync.aligned.16x128b.x2.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r0), "r"(r1),
                 "r"(r2), "r"(r3));
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void umma_commit_el(uint64_t* bar) {
    asm volatile("{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
                 " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::
                     "r"(smem_u32(bar))
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

// 2-D tensor copy global -> this CTA's shared memory, completing on `bar`; whole warp, elected lane issues.
__device__ __forceinline__ void tma_tile_g2s_el(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
        " @e cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n}\n" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// ------------------------------------------------------------------------------------------ units
// Unit u -> (expert, row group, block pair). Units of expert e: ceil(rows_e / 128) * n_pairs. The record also holds
// what every role derives from the expert (its class, its entry in the class's tables, whether the pair exists for
// that class's width), computed once when the CTA builds its unit table, so no role divides in its loop.
struct TcUnit {
    int64_t r0;        // first sorted row
    int32_t e, j;      // expert, entry in its class's tables
    int16_t nr, pair;  // rows (<= 128: more than 64 makes a wide unit), output block pair
    int16_t c, live;   // class; 0: the pair lies past the class's width (its rows are zero there)
};

template <int UG>
__device__ __forceinline__ TcUnit tc_unit(const Exl3bOp& op, const uint32_t* prefix, int64_t unit, int n_pairs) {
    int64_t lo = 0, hi = op.n_expert;
    while (hi - lo > 1) {
        const int64_t mid = (lo + hi) / 2;
        if ((int64_t)prefix[mid] <= unit) lo = mid; else hi = mid;
    }
    TcUnit u;
    u.e = (int32_t)lo;
    const int64_t local = unit - prefix[lo];
    const int64_t grp = local / n_pairs;
    u.pair = (int16_t)(local % n_pairs);
    u.r0 = op.expert_offset[lo] + grp * UG;
    const int64_t rend = op.expert_offset[lo + 1];
    u.nr = (int16_t)(rend - u.r0 < UG ? rend - u.r0 : UG);
    const ExpertView ev = expert_view(op, lo);
    u.c = (int16_t)ev.c;
    u.j = (int32_t)ev.j;
    u.live = (int64_t)u.pair * 256 < ev.R ? 1 : 0;   // gate_up: 128 gate + 128 up rows a pair; down: 256 rows
    return u;
}

// A ring position: stage and phase advanced together (no division a chunk).
struct Ring {
    uint32_t s = 0, ph = 0;
    __device__ __forceinline__ void next(uint32_t n) {
        if (++s == n) { s = 0; ph ^= 1u; }
    }
};

// ------------------------------------------------------------------------------------------ the kernel
template <int BITS, int CB, bool GU, bool WIDE>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmap, const Exl3bOp op, int n_pairs) {
    using Cfg = TcCfg<BITS>;
    constexpr int UG = WIDE ? kUG : kNT;                // sorted rows a unit at most
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment of every swizzled tile, as an offset from the shared array (the pointers stay visibly in
    // shared memory, so every access through them is a shared-memory instruction, not a generic one)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    constexpr int kStB = Cfg::ST_B;
    uint8_t* b_ring = smem;                                        // [kStB][half 2][box kNBox][8 KB]
    uint8_t* r_ring = b_ring + kStB * 2 * kBHalf;                  // [ST_R][REC_STAGE]
    float* epi = reinterpret_cast<float*>(r_ring + Cfg::ST_R * Cfg::REC_STAGE);   // [2][16][kEpiCols]
    uint64_t* bars = reinterpret_cast<uint64_t*>(epi + 2 * 16 * kEpiCols);
    uint64_t* a_full = bars;                 // decoders -> MMA (count kDecWarps): an A stage is in tensor memory
    uint64_t* a_empty = a_full + kStA;       // MMA commit -> decoders
    uint64_t* b_full = a_empty + kStA;       // producer tx -> MMA
    uint64_t* b_empty = b_full + kStB;       // MMA commit -> producer
    uint64_t* r_full = b_empty + kStB;       // producer tx -> decoders
    uint64_t* r_empty = r_full + Cfg::ST_R;  // MMA warp (once every decoder has finished the stage) -> producer
    uint64_t* acc_full = r_empty + Cfg::ST_R;  // MMA commit -> epilogue [2]
    uint64_t* acc_empty = acc_full + 2;      // epilogue -> MMA [2] (count kEpiWarps)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    uint32_t* prefix = tmem_slot + 4;        // [n_expert + 1]
    __shared__ TcUnit utab[kUnitTab];

    // the warp index through a shuffle: the compiler then knows it is warp-uniform, and so is everything a role
    // derives from it
    const int tid = threadIdx.x, warp = __shfl_sync(0xFFFFFFFFu, tid >> 5, 0), lane = tid & 31;
    const int64_t n_exp = op.n_expert;

    if (tid == 0) {
        // the stages and accumulators are released by both MMA warps' commits (two arrivals)
        for (int s = 0; s < kStA; ++s) { mbar_init(&a_full[s], kDecWarps); mbar_init(&a_empty[s], 2); }
        for (int s = 0; s < kStB; ++s) { mbar_init(&b_full[s], 1); mbar_init(&b_empty[s], 2); }
        for (int s = 0; s < Cfg::ST_R; ++s) { mbar_init(&r_full[s], 1); mbar_init(&r_empty[s], 1); }
        for (int s = 0; s < 2; ++s) { mbar_init(&acc_full[s], 2); mbar_init(&acc_empty[s], kEpiWarps); }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // the unit list: ceil(rows_e / 128) * n_pairs units an expert, expert-major. prefix[e] = the first unit of
    // expert e (a block-wide exclusive scan of the per-expert counts, each thread a run of experts)
    {
        __shared__ uint32_t wsum[kTcWarps];
        const int64_t per = (n_exp + kTcThreads - 1) / kTcThreads;
        const int64_t e0 = tid * per, e1 = e0 + per < n_exp ? e0 + per : n_exp;
        uint32_t sum = 0;
        for (int64_t e = e0; e < e1; ++e) {
            const int64_t r = op.expert_offset[e + 1] - op.expert_offset[e];
            sum += r > 0 ? (uint32_t)(((r + UG - 1) / UG) * n_pairs) : 0u;
        }
        uint32_t incl = sum;                                   // inclusive scan within the warp
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
            acc += r > 0 ? (uint32_t)(((r + UG - 1) / UG) * n_pairs) : 0u;
        }
        if (tid == kTcThreads - 1) prefix[n_exp] = acc;
    }
    __syncthreads();
    // this CTA's units (blockIdx.x + i * gridDim.x), looked up once into a shared table
    const int64_t n_units = prefix[n_exp];
    const int64_t n_mine = n_units > blockIdx.x ? (n_units - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    for (int64_t i = tid; i < n_mine && i < kUnitTab; i += kTcThreads)
        utab[i] = tc_unit<UG>(op, prefix, blockIdx.x + i * gridDim.x, n_pairs);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // the allocated base, read from shared memory and broadcast from lane 0: the compiler then knows it is the same in
    // every lane, and the tensor-memory addresses and MMA operands derived from it stay warp-uniform
    const uint32_t tmem = __shfl_sync(0xFFFFFFFFu, *tmem_slot, 0);
    auto unit_at = [&](int64_t i) -> TcUnit {
        return i < kUnitTab ? utab[i] : tc_unit<UG>(op, prefix, blockIdx.x + i * gridDim.x, n_pairs);
    };

    // rows no unit writes are zeroed (outside the runs, dropped slots): the grid's threads test the rows in
    // parallel; a thread clears the (rare) dead row it finds
    if (!op.live_only && (warp < kEpiWarps || warp >= kDecWarp0)) {
        const int64_t lt = warp < kEpiWarps ? tid : tid - (kDecWarp0 - kEpiWarps) * 32;   // 0 .. nthr-1
        const int64_t nthr = (kEpiWarps + kDecWarps) * 32;
        const int64_t lo = op.expert_offset[0], hi = op.expert_offset[n_exp];
        for (int64_t i = (int64_t)blockIdx.x * nthr + lt; i < op.T; i += (int64_t)gridDim.x * nthr) {
            if (i >= lo && i < hi && op.sorted_tok[i] >= 0) continue;
            uint16_t* y = out_row(op, i);
            for (int64_t c = 0; c < op.y_cols; ++c) y[c] = 0;
        }
        if (op.row_dst) __threadfence_system();
    }

    if (warp == kRecWarp || warp == kBWarp) {
        // ---------------------------------------------------------------- producers
        // warp 8 streams the record rows, warp 9 the input-row tiles: two rings, two warps, so neither producer's
        // wait holds up the other. Each warp runs its loop whole; one elected lane issues the copies.
        Ring rr, br;
        for (int64_t ui_ = 0; ui_ < n_mine; ++ui_) {
            const TcUnit u = unit_at(ui_);
            if (!u.live) continue;                                   // a narrower class: nothing to stream
            const Exl3bClass& cl = op.cls[u.c];
            const int64_t wrows = GU ? cl.rows / 2 : cl.rows;       // rows of one record
            const int nck = (int)(cl.cols / kKC);
            if (warp == kRecWarp) {
                const uint16_t* rec = static_cast<const uint16_t*>(tab_entry(cl.codes, u.j));
                const int64_t mat_elems = (cl.cols / 16) * (wrows / 16) * 16 * BITS;
                // the unit's first tile of k row 0 (per matrix); k row tk adds tk * the record's k-row stride
                const uint16_t* src0 = rec + (int64_t)u.pair * (GU ? 8 : 16) * 16 * BITS;
                const int64_t krow = (wrows / 16) * 16 * BITS;
                for (int ck = 0; ck < nck; ++ck, rr.next(Cfg::ST_R)) {
                    mbar_wait_warp(&r_empty[rr.s], rr.ph ^ 1, op.err);
                    mbar_expect_tx_el(&r_full[rr.s], (uint32_t)Cfg::REC_STAGE);
                    uint8_t* dst0 = r_ring + rr.s * Cfg::REC_STAGE;
                    const uint16_t* srck = src0 + (int64_t)ck * kKT * krow;
#pragma unroll
                    for (int q = 0; q < kKT; ++q) {
                        uint8_t* dst = dst0 + q * 2 * Cfg::REC_ROW;
                        if (GU) {
                            tma_bulk_g2s_el(dst, srck + q * krow, Cfg::REC_ROW, &r_full[rr.s]);
                            tma_bulk_g2s_el(dst + Cfg::REC_ROW, srck + mat_elems + q * krow, Cfg::REC_ROW,
                                            &r_full[rr.s]);
                        } else {
                            tma_bulk_g2s_el(dst, srck + q * krow, 2 * Cfg::REC_ROW, &r_full[rr.s]);
                        }
                    }
                }
            } else {
                // input rows of each chunk, a stage a 64-row half (rows r0 .. r0+63, then r0+64 .. for a wide unit;
                // zero fill past T)
                const int nh = WIDE && u.nr > kNT ? 2 : 1;
                for (int ck = 0; ck < nck; ++ck) {
                    for (int hh = 0; hh < nh; ++hh, br.next(kStB)) {
                        mbar_wait_warp(&b_empty[br.s], br.ph ^ 1, op.err);
                        mbar_expect_tx_el(&b_full[br.s], (uint32_t)((GU ? 2 : 1) * kBHalf));
#pragma unroll
                        for (int m = 0; m < (GU ? 2 : 1); ++m)
#pragma unroll
                            for (int bx = 0; bx < kNBox; ++bx)
                                tma_tile_g2s_el(b_ring + (br.s * 2 + m) * kBHalf + bx * kBTile, &tmap,
                                                (int)(m * cl.cols + ck * kKC + bx * kBox), (int)(u.r0 + hh * kNT),
                                                &b_full[br.s]);
                    }
                }
            }
        }
    } else if (warp == kMmaWarp || warp == kMmaWarp + 1) {
        // ---------------------------------------------------------------- MMA issuers (whole warp, elected lane)
        // warp 10 issues block 0's MMAs, warp 11 block 1's: the two blocks accumulate into their own TMEM columns, so
        // each block's k steps stay in one warp's issue order, and the issue -- which holds a warp at the tensor
        // cores' rate -- is spread over two SM sub-partitions. Each warp commits its own MMAs to the stage and
        // accumulator barriers (two arrivals each). The input ring's base descriptor; a stage, half and k step only
        // add to the start-address field (the shared-memory window is below 256 KB, so the 14-bit field never
        // carries). Once every decoder has filled a chunk's A stage it has also finished reading the chunk's record
        // stage, so warp 10 hands that stage back to the record producer (one arrive a chunk).
        // A wide unit multiplies each chunk's A stage by both of its input stages, half h into accumulator buffer
        // (ab + h) & 1: the buffers are taken in sequence (ab counts the halves so far), so the epilogue of one half
        // overlaps the next half's MMAs whatever the mix of wide and narrow units.
        const int blk = warp - kMmaWarp;
        const uint64_t b_desc0 = sw128_desc(smem_u32(b_ring));
        Ring ar, br, rr;
        uint32_t ab = 0;
        for (int64_t ui_ = 0; ui_ < n_mine; ++ui_) {
            const TcUnit u = unit_at(ui_);
            if (!u.live) continue;
            const int nck = (int)(op.cls[u.c].cols / kKC);
            const int nh = WIDE && u.nr > kNT ? 2 : 1;
            for (int hh = 0; hh < nh; ++hh)
                mbar_wait_warp(&acc_empty[(ab + hh) & 1], (((ab + hh) >> 1) & 1) ^ 1, op.err);
            tc_fence_after();
            for (int ck = 0; ck < nck; ++ck, ar.next(kStA), rr.next(Cfg::ST_R)) {
                mbar_wait2_warp(&a_full[ar.s], ar.ph, &b_full[br.s], br.ph, op.err);
                Ring b2 = br;
                if (nh == 2) {
                    b2.next(kStB);
                    mbar_wait_warp(&b_full[b2.s], b2.ph, op.err);
                }
                tc_fence_after();
                if (blk == 0 && lane == 0) mbar_arrive(&r_empty[rr.s]);
                __syncwarp();
                const uint32_t ta = tmem + kAccCols + ar.s * kAStageCols + blk * (kKC / 2);
                for (int hh = 0; hh < nh; ++hh, br.next(kStB)) {
                    const uint32_t d = tmem + ((ab + hh) & 1) * (2 * kNT) + blk * kNT;
                    const uint64_t dbb = b_desc0 + (uint64_t)((br.s * 2 * kBHalf + (GU ? blk : 0) * kBHalf) >> 4);
                    umma_block8_el(d, ta, dbb, dbb + (uint64_t)(kBTile >> 4), ck ? 1u : 0u);
                    umma_commit_el(&b_empty[br.s]);
                }
                umma_commit_el(&a_empty[ar.s]);
            }
            for (int hh = 0; hh < nh; ++hh) umma_commit_el(&acc_full[(ab + hh) & 1]);
            ab += nh;
        }
    } else if (warp >= kDecWarp0) {
        // ---------------------------------------------------------------- decoders
        // warp -> (lane quadrant q = warp % 4, j): block j / 2, tile row tn = 2q + j % 2 -- weight rows 16 tn ..
        // 16 tn + 15 of the block, TMEM lanes of quadrant q only; every k tile of the chunk
        const int q = warp & 3, j = (warp - kDecWarp0) >> 2;
        const int blk = kDecTn == 1 ? j >> 1 : j, tn = kDecTn == 1 ? 2 * q + (j & 1) : 2 * q;
        const LaneDec<BITS> ld = lane_dec<BITS>(lane);
        const uint32_t tile_off = (uint32_t)(blk * Cfg::REC_ROW + tn * Cfg::TILE_BYTES);
        const uint32_t a_t0 = tmem + ((uint32_t)(16 * tn) << 16) + kAccCols + blk * (kKC / 2);
        Ring ar, rr;
        for (int64_t ui_ = 0; ui_ < n_mine; ++ui_) {
            const TcUnit u = unit_at(ui_);
            if (!u.live) continue;
            const int nck = (int)(op.cls[u.c].cols / kKC);
            for (int ck = 0; ck < nck; ++ck, ar.next(kStA), rr.next(Cfg::ST_R)) {
                mbar_wait2_warp(&r_full[rr.s], rr.ph, &a_empty[ar.s], ar.ph ^ 1, op.err);
                tc_fence_after();
                const uint32_t rst = smem_u32(r_ring) + rr.s * Cfg::REC_STAGE + tile_off;
                const uint32_t ta = a_t0 + ar.s * kAStageCols;
#pragma unroll
                for (int tt = 0; tt < kDecTn; ++tt) {
                    // every tile's stream words of the chunk first, so no tile waits on its shared-memory loads
                    TileWords w[kKT];
#pragma unroll
                    for (int tk = 0; tk < kKT; ++tk)
                        w[tk] = tile_words_s<BITS>(rst + tk * 2 * Cfg::REC_ROW + tt * Cfg::TILE_BYTES, ld);
#pragma unroll
                    for (int tk = 0; tk < kKT; ++tk) {
                        uint32_t b[4];
                        decode_words<BITS, CB>(w[tk], ld, b);
                        tmem_st_16x128b_x2(ta + ((uint32_t)(16 * tt) << 16) + tk * 8, b[0], b[2], b[1], b[3]);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_full[ar.s]);
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue (warps 0..7)
        const int q = warp & 3;                      // TMEM lanes 32q .. 32q+31 = weight rows of a block
        const int eb = warp >> 2;                    // the block this warp moves out of TMEM
        uint32_t ab = 0;                             // accumulator halves taken so far (the MMA warps' sequence)
        for (int64_t ui_ = 0; ui_ < n_mine; ++ui_) {
            const TcUnit u = unit_at(ui_);
            const Exl3bClass& cl = op.cls[u.c];
            if (!u.live) {
                // a narrower class: its live rows are zero across this pair's columns
                const int64_t c0 = (int64_t)u.pair * (GU ? 128 : 256), nc = GU ? 128 : 256;
                for (int m = 0; m < u.nr; ++m) {
                    const int64_t i = u.r0 + m;
                    if (op.sorted_tok[i] < 0) continue;
                    uint16_t* y = out_row(op, i) + c0;
                    for (int64_t c = tid; c < nc; c += kEpiWarps * 32) y[c] = 0;
                }
                continue;
            }
            // the unit's output scales, held for all its rows: lane l owns columns 4l .. 4l+3 of each block
            const uint16_t* svh = static_cast<const uint16_t*>(tab_entry(cl.svh, u.j));
            float s0[4], s1[4], sd[4];
            const int64_t n0 = (int64_t)u.pair * (GU ? 128 : 256) + 4 * lane;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                s0[e] = h2f(svh[n0 + e]);
                s1[e] = GU ? h2f(svh[cl.rows / 2 + n0 + e]) : h2f(svh[n0 + 128 + e]);
                sd[e] = 0.f;
            }
            const uint16_t* dn = GU && op.h_rot ? static_cast<const uint16_t*>(tab_entry(cl.dn_suh, u.j)) : nullptr;
            uint16_t dsuh[4] = { 0, 0, 0, 0 };
            if (dn) {
#pragma unroll
                for (int e = 0; e < 4; ++e) dsuh[e] = dn[(int64_t)u.pair * 128 + 4 * lane + e];
            }
            (void)sd;
            // the unit's halves in turn (one for a narrow unit), each out of its accumulator buffer
            const int nh = WIDE && u.nr > kNT ? 2 : 1;
            for (int hh = 0; hh < nh; ++hh) {
                const int64_t r0 = u.r0 + hh * kNT;
                const int nr = hh ? u.nr - kNT : (u.nr < kNT ? u.nr : kNT);
                // the sorted_tok entries of this warp's rows (m = 8 l + warp, one a lane of the first eight), loaded
                // once a half while the accumulators are still being computed
                int32_t tokv = -1;
                if (lane < kNT / kEpiWarps && kEpiWarps * lane + warp < nr) tokv = op.sorted_tok[r0 + kEpiWarps * lane + warp];
                const uint32_t buf = ab & 1, uph = (ab >> 1) & 1;
                mbar_wait_warp(&acc_full[buf], uph, op.err);
                tc_fence_after();
                for (int sl = 0; sl < kNT / 16; ++sl) {
                    if (sl * 16 >= nr) break;
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
                        const int32_t tok = __shfl_sync(0xFFFFFFFFu, tokv, m / kEpiWarps);
                        if (m >= nr || tok < 0) continue;
                        const int64_t i = r0 + m;
                        const float4 av = *reinterpret_cast<const float4*>(&epi[(0 * 16 + j) * kEpiCols + 4 * lane]);
                        const float4 bv = *reinterpret_cast<const float4*>(&epi[(1 * 16 + j) * kEpiCols + 4 * lane]);
                        float a[4] = { av.x, av.y, av.z, av.w }, b[4] = { bv.x, bv.y, bv.z, bv.w };
                        had128_warp(a, lane);
                        had128_warp(b, lane);
                        uint16_t* y = out_row(op, i) + n0;
                        if (GU) {
                            float h[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) h[e] = silu_mul(__fmul_rn(a[e], s0[e]), __fmul_rn(b[e], s1[e]));
                            if (dn) {
                                hrot_scale4(h, dsuh);
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
                            float lo[4], hi[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                lo[e] = __fmul_rn(a[e], s0[e]);
                                hi[e] = __fmul_rn(b[e], s1[e]);
                            }
                            st4_out(op, y, lo);
                            st4_out(op, y + 128, hi);
                        }
                    }
                    asm volatile("bar.sync 2, %0;" ::"n"(kEpiWarps * 32) : "memory");
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[buf]);
                ++ab;
            }
        }
        // rows written through a row table may live in another GPU's memory: make them visible system-wide before
        // this thread (and so the kernel) completes, ahead of whatever flag the caller raises next
        if (op.row_dst) __threadfence_system();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

template <int BITS, int CB, bool GU>
int launch_tc_t(const CUtensorMap& map, const Exl3bOp* op, int n_pairs, int grid, int smem, bool wide, cudaStream_t st) {
    auto kern = wide ? k_gemm_tc<BITS, CB, GU, true> : k_gemm_tc<BITS, CB, GU, false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -6;
    kern<<<grid, kTcThreads, smem, st>>>(map, *op, n_pairs);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

template <bool GU>
int launch_tc_b(const CUtensorMap& map, const Exl3bOp* op, int n_pairs, int grid, int smem, bool wide, cudaStream_t st) {
#define EXL3B_TC_CB(B)                                                              \
    switch (op->codebook) {                                                         \
    case 0: return launch_tc_t<B, 0, GU>(map, op, n_pairs, grid, smem, wide, st);   \
    case 1: return launch_tc_t<B, 1, GU>(map, op, n_pairs, grid, smem, wide, st);   \
    case 2: return launch_tc_t<B, 2, GU>(map, op, n_pairs, grid, smem, wide, st);   \
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
    const int64_t rec_stage = (int64_t)kKT * 2 * 8 * 32 * bits;
    int64_t st_r = 64 * 1024 / rec_stage;
    st_r = st_r < 3 ? 3 : st_r > 12 ? 12 : st_r;
    const int64_t st_b = bits >= 6 ? 3 : 4;
    const int64_t b = st_b * 2 * kBHalf + st_r * rec_stage + 2 * 16 * kEpiCols * 4 + 512;
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
    const cuuint32_t box[2] = { (cuuint32_t)kBox, (cuuint32_t)kNT };
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
    // wide units (decode once a 128 rows) where experts hold many rows, the wide units still outnumber the SMs
    // several times over, and a unit's decode is long against its epilogue (an input of >= 1024 columns: gate_up's
    // 2048, not down's 512, where the doubled epilogue cost more than the decode saved): expert parallelism's
    // received passes, prefill over few experts. Elsewhere -- few rows an expert, or a pass whose units would leave
    // SMs idle (one large expert) -- the 64-row units, whose kernel carries no wide-unit code.
    const int64_t n_exp = op->n_expert > 0 ? op->n_expert : 1;
    const bool wide = op->x_cols >= kWideMinCols && op->T >= (int64_t)kUG * n_exp &&
                      (op->T / kUG) * n_pairs >= (int64_t)kWideUnitsPerSm * sm_count;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return gu ? launch_tc_b<true>(map, op, n_pairs, grid, (int)smem, wide, st)
              : launch_tc_b<false>(map, op, n_pairs, grid, (int)smem, wide, st);
}

}  // extern "C"
