// exl3b200_decode.cuh -- device code shared by the sm_100a kernels of libexl3b200.so: the bit-exact trellis decode
// of one lane's eight positions, the 128-point rotation in the reference's stage order, the mbarrier / TMA bulk-copy
// helpers with bounded waits, and the expert lookups of the routing contract. Included by each .cu file (every
// function is internal to the including translation unit).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "exl3b200_dev.h"

namespace {

constexpr float kRs = 0.08838834764831844055f;   // (float)(1 / sqrt(128))
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // a bounded mbarrier wait gives up after 2 s (error word set)
constexpr uint32_t kSuspendNs = 100000u;          // a waiting thread sleeps in hardware up to this long a try

// ------------------------------------------------------------------------------------------ small helpers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float bf2f(uint16_t h) { return __bfloat162float(__ushort_as_bfloat16(h)); }
__device__ __forceinline__ uint16_t f2bf(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }

// Entry j of a plane table (stacked or pointer table).
__device__ __forceinline__ const void* tab_entry(const Exl3bTab& t, int64_t j) {
    if (t.stride_bytes == 0) return reinterpret_cast<const void* const*>(t.base)[j];
    return static_cast<const uint8_t*>(t.base) + j * t.stride_bytes;
}

// ------------------------------------------------------------------------------------------ codebooks
// Two states -> one half2 (low = first). mul1: fp16(1024 + bytesum(s * 0x83DCD12D)) is built exactly as the
// bits 0x6400 + bytesum (dp4a with that addend), then ONE fp16 FMA by K_INV (0x1EEE) plus K_BIAS (0xC931).
// mcg / 3inst: (h & 0x8FFF8FFF) ^ 0x3B603B60, the two fp16 halves added once. common/exl3_decode.c:43-67.
template <int CB>
__device__ __forceinline__ uint32_t cb_pair(uint32_t s0, uint32_t s1) {
    if constexpr (CB == 2) {
        const uint32_t x0 = s0 * 0x83DCD12Du, x1 = s1 * 0x83DCD12Du;
        const uint32_t u0 = __dp4a(x0, 0x01010101u, 0x6400u);
        const uint32_t u1 = __dp4a(x1, 0x01010101u, 0x6400u);
        const uint32_t h = u1 * 65536u + u0;   // the pair packed by an IMAD (FMA pipe): u0, u1 < 2^16
        const __half2 kinv = __halves2half2(__ushort_as_half(0x1EEE), __ushort_as_half(0x1EEE));
        const __half2 kbias = __halves2half2(__ushort_as_half(0xC931), __ushort_as_half(0xC931));
        const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&h), kinv, kbias);
        return *reinterpret_cast<const uint32_t*>(&r);
    } else {
        uint32_t x0, x1;
        if constexpr (CB == 1) {
            x0 = s0 * 0xCBAC1FEDu;
            x1 = s1 * 0xCBAC1FEDu;
        } else {
            x0 = s0 * 89226354u + 64248484u;
            x1 = s1 * 89226354u + 64248484u;
        }
        x0 = (x0 & 0x8FFF8FFFu) ^ 0x3B603B60u;
        x1 = (x1 & 0x8FFF8FFFu) ^ 0x3B603B60u;
        const uint32_t lo = __byte_perm(x0, x1, 0x5410), hi = __byte_perm(x0, x1, 0x7632);
        const __half2 r = __hadd2(*reinterpret_cast<const __half2*>(&lo), *reinterpret_cast<const __half2*>(&hi));
        return *reinterpret_cast<const uint32_t*>(&r);
    }
}

// ------------------------------------------------------------------------------------------ one tile, one lane
// Lane L of a warp decodes trellis positions 8L .. 8L+7 of a 16x16 tile (8K u32 words, one MSB-first stream,
// circular). Position 8L+j's 16-bit state is the stream window ending at bit (8L+j+1)K. The eight positions
// are exactly the mma.m16n8k16 B fragments of the tile's two n8 halves (k = 2(L%4) + {0,1,8,9},
// n = L/4 and L/4 + 8), so the four returned half2 are: b[0], b[1] the first n8 block's fragment registers,
// b[2], b[3] the second's.
//
// The lane's eight windows span 16 + 7K bits starting at S = (8L+1)K - 16 (circular): inside two stream words from
// word S/32 for K <= 4, three for K >= 5. The words are realigned once (funnel shifts by S % 32) so the first window
// starts at the top bit; every window is then at a compile-time position: one shift and a mask, a single shift or
// PRMT where it lies at the top or on a byte boundary of one word. For K = 4 and K = 8 every lane's S % 32 is the
// same (20, 24), so no realignment is needed at all.
template <int BITS>
struct KDec {
    static constexpr int NWQ = BITS <= 4 ? 2 : 3;              // stream words a lane's windows span
    static constexpr bool FIXED = BITS == 4 || BITS == 8;      // every lane's first window at the same bit offset
    static constexpr int OFF = BITS == 4 ? 20 : BITS == 8 ? 24 : 0;
};

// What a lane needs to find its windows in any tile of a given K: the byte offsets of its two or three stream words
// and the first window's bit offset in the first. Computed once a kernel.
template <int BITS>
struct LaneDec {
    uint32_t o0, o1, o2;       // byte offsets of words a, a+1, a+2 (circular in the tile)
    uint32_t off;              // the first window's start bit in word a
};

template <int BITS>
__device__ __forceinline__ LaneDec<BITS> lane_dec(int lane) {
    constexpr int NW = 8 * BITS;
    constexpr int NB = 256 * BITS;
    LaneDec<BITS> d;
    const int base = ((8 * lane + 1) * BITS - 16 + NB) % NB;   // first window's start bit
    const int a = base >> 5;
    d.off = (uint32_t)(base & 31);
    d.o0 = (uint32_t)(a * 4);
    d.o1 = (uint32_t)(((a + 1) % NW) * 4);
    d.o2 = (uint32_t)(((a + 2) % NW) * 4);
    return d;
}

// The stream words a lane's windows span, read from a generic pointer or -- the kernels' record rings -- straight
// from a shared-memory address.
struct TileWords {
    uint32_t w0, w1, w2;
};
template <int BITS>
__device__ __forceinline__ TileWords tile_words(const uint8_t* __restrict__ tile, const LaneDec<BITS>& d) {
    TileWords w;
    w.w0 = *reinterpret_cast<const uint32_t*>(tile + d.o0);
    w.w1 = *reinterpret_cast<const uint32_t*>(tile + d.o1);
    w.w2 = KDec<BITS>::NWQ == 3 ? *reinterpret_cast<const uint32_t*>(tile + d.o2) : 0u;
    return w;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
template <int BITS>
__device__ __forceinline__ TileWords tile_words_s(uint32_t tile, const LaneDec<BITS>& d) {
    TileWords w;
    w.w0 = lds_u32(tile + d.o0);
    w.w1 = lds_u32(tile + d.o1);
    w.w2 = KDec<BITS>::NWQ == 3 ? lds_u32(tile + d.o2) : 0u;
    return w;
}

// Bits [S, S + 16) (counted from the least significant bit) of the 32*NWQ-bit value q2:q1:q0 (q2 the top word; q0
// unused for NWQ = 2), as a clean 16-bit value. S is a compile-time constant.
template <int S, int NWQ>
__device__ __forceinline__ uint32_t win16(uint32_t q2, uint32_t q1, uint32_t q0) {
    constexpr int TOP = 32 * NWQ;
    // the word the window's low bit falls in, and the one above it
    constexpr int LOWW = S / 32;                               // 0 = lowest word
    constexpr int SH = S % 32;
    const uint32_t lo = NWQ == 3 ? (LOWW == 2 ? q2 : LOWW == 1 ? q1 : q0) : (LOWW == 1 ? q2 : q1);
    static_assert(S + 16 <= TOP, "window inside the span");
    if constexpr (SH <= 16) {
        // inside one word
        if constexpr (SH == 16) return lo >> 16;
        else if constexpr (SH == 8) return __byte_perm(lo, 0u, 0x4421);
        else if constexpr (SH == 0) return __byte_perm(lo, 0u, 0x4410);
        else return (lo >> SH) & 0xFFFFu;
    } else {
        const uint32_t hi = NWQ == 3 ? (LOWW == 1 ? q2 : q1) : q2;
        return __funnelshift_r(lo, hi, SH) & 0xFFFFu;
    }
}

// The eight states of a lane's windows: window j starts (from the top of the span) at off + jK.
template <int BITS>
__device__ __forceinline__ void lane_states(const TileWords& w, const LaneDec<BITS>& d, uint32_t st[8]) {
    using K = KDec<BITS>;
    uint32_t q2, q1, q0 = 0;
    constexpr int SHIFT0 = 32 * K::NWQ - 16 - K::OFF;          // window 0's low bit, before realignment
    if constexpr (K::FIXED) {
        q2 = w.w0;
        q1 = w.w1;
        if constexpr (K::NWQ == 3) q0 = w.w2;
    } else if constexpr (K::NWQ == 2) {
        q2 = __funnelshift_l(w.w1, w.w0, d.off);               // the span's first bit at the top
        q1 = w.w1 << d.off;
    } else {
        q2 = __funnelshift_l(w.w1, w.w0, d.off);
        q1 = __funnelshift_l(w.w2, w.w1, d.off);
        q0 = w.w2 << d.off;
    }
    st[0] = win16<SHIFT0 - 0 * BITS, K::NWQ>(q2, q1, q0);
    st[1] = win16<SHIFT0 - 1 * BITS, K::NWQ>(q2, q1, q0);
    st[2] = win16<SHIFT0 - 2 * BITS, K::NWQ>(q2, q1, q0);
    st[3] = win16<SHIFT0 - 3 * BITS, K::NWQ>(q2, q1, q0);
    st[4] = win16<SHIFT0 - 4 * BITS, K::NWQ>(q2, q1, q0);
    st[5] = win16<SHIFT0 - 5 * BITS, K::NWQ>(q2, q1, q0);
    st[6] = win16<SHIFT0 - 6 * BITS, K::NWQ>(q2, q1, q0);
    st[7] = win16<SHIFT0 - 7 * BITS, K::NWQ>(q2, q1, q0);
}

template <int BITS, int CB>
__device__ __forceinline__ void decode_words(const TileWords& w, const LaneDec<BITS>& d, uint32_t b[4]) {
    uint32_t st[8];
    lane_states<BITS>(w, d, st);
    b[0] = cb_pair<CB>(st[0], st[1]);
    b[1] = cb_pair<CB>(st[2], st[3]);
    b[2] = cb_pair<CB>(st[4], st[5]);
    b[3] = cb_pair<CB>(st[6], st[7]);
}

template <int BITS, int CB>
__device__ __forceinline__ void decode_tile(const uint8_t* __restrict__ tile, const LaneDec<BITS>& d, uint32_t b[4]) {
    decode_words<BITS, CB>(tile_words<BITS>(tile, d), d, b);
}
// The same, the tile at a shared-memory address (explicit shared loads).
template <int BITS, int CB>
__device__ __forceinline__ void decode_tile_s(uint32_t tile, const LaneDec<BITS>& d, uint32_t b[4]) {
    decode_words<BITS, CB>(tile_words_s<BITS>(tile, d), d, b);
}

// One lane's eight positions of the tile at `w` (the per-lane setup done in place).
template <int BITS, int CB>
__device__ __forceinline__ void decode_lane(const uint32_t* __restrict__ w, int lane, uint32_t b[4]) {
    const LaneDec<BITS> d = lane_dec<BITS>(lane);
    decode_tile<BITS, CB>(reinterpret_cast<const uint8_t*>(w), d, b);
}

// ------------------------------------------------------------------------------------------ 128-point rotation
// Packed f32 pairs (sm_100's f32x2 arithmetic: two IEEE round-to-nearest operations an instruction), used by k_prep's
// 16-value rotation. (The 4-value rotation below stays scalar: packed, the epilogues measured 1-5 % slower.)
__device__ __forceinline__ uint64_t f2pk(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2upk(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// A warp holds one 128-vector, lane l the elements 4l .. 4l+3. Stages h = 1, 2 inside the lane, h = 4 .. 64
// across lanes; a+b stays low, a-b goes high, exactly as common/exl3_decode.c:179-185; then x (float)(1/sqrt(128)).
__device__ __forceinline__ void had128_warp(float v[4], int lane) {
    float a, b;
    a = v[0]; b = v[1]; v[0] = __fadd_rn(a, b); v[1] = __fsub_rn(a, b);
    a = v[2]; b = v[3]; v[2] = __fadd_rn(a, b); v[3] = __fsub_rn(a, b);
    a = v[0]; b = v[2]; v[0] = __fadd_rn(a, b); v[2] = __fsub_rn(a, b);
    a = v[1]; b = v[3]; v[1] = __fadd_rn(a, b); v[3] = __fsub_rn(a, b);
    // across lanes: the low lane of a pair keeps a + b, the high lane a - b, written as one FMA p + (+-1) v (the
    // product by +-1 is exact, so the FMA rounds exactly as the add or the subtract would)
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const float sg = (lane & m) ? -1.0f : 1.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float p = __shfl_xor_sync(0xFFFFFFFFu, v[i], m);
            v[i] = __fmaf_rn(sg, v[i], p);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __fmul_rn(v[i], kRs);
}

// SiLU(g) * u in f32 (kernels/exl3ref/ref.c:44, 209): g / (1 + e^-g) with the exponential and the reciprocal from the
// special-function unit (ex2.approx, rcp.approx: a few ulp of f32, far inside the ops' stated tolerance). g very
// negative: e^-g = inf and the quotient is -0, as the reference's g * (1 / (1 + inf)).
__device__ __forceinline__ float silu_mul(float g, float u) {
    return __fmul_rn(__fdividef(g, __fadd_rn(1.0f, __expf(-g))), u);
}
// down's input scale on gate_up's h (h_rot): v = f32(f16(f16(h) * s)) for four values, as the reference's
// f16(f32(f16 h) * f32 s) -- the product of two f16 values is exact in f32, so one HMUL2 (exact product, one
// round-to-nearest-even to f16) gives the same bits.
__device__ __forceinline__ void hrot_scale4(float h[4], const uint16_t s[4]) {
    const __half2 a = __floats2half2_rn(h[0], h[1]), b = __floats2half2_rn(h[2], h[3]);
    const __half2 sa = __halves2half2(__ushort_as_half(s[0]), __ushort_as_half(s[1]));
    const __half2 sb = __halves2half2(__ushort_as_half(s[2]), __ushort_as_half(s[3]));
    const float2 ra = __half22float2(__hmul2(a, sa)), rb = __half22float2(__hmul2(b, sb));
    h[0] = ra.x; h[1] = ra.y; h[2] = rb.x; h[3] = rb.y;
}

// f16(had(f16(x * s))) of one 128-block held as above (kernels/exl3ref/ref.c:27-32).
__device__ __forceinline__ void prologue_warp(float v[4], const uint16_t* __restrict__ s, int lane) {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = h2f(f2h(__fmul_rn(v[i], h2f(s[4 * lane + i]))));
    had128_warp(v, lane);
}

// ------------------------------------------------------------------------------------------ mbarrier / TMA
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Bounded wait for the phase of `parity`; false (and the error word set) when it never completed.
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait for the phase of `parity`: the thread is suspended by the hardware between tries (it takes no issue
// slots while it waits), and gives up after kWaitLimitNs with the error word set.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* err) {
    const uint32_t a = smem_u32(bar);
    uint64_t t0 = 0;
    for (;;) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(a), "r"(parity), "r"(kSuspendNs)
            : "memory");
        if (done) return true;
        const uint64_t now = globaltimer_ns();
        if (!t0) t0 = now;
        else if (now - t0 > kWaitLimitNs) break;
    }
    if (err) atomicOr(err, 1);
    return false;
}
// Two bounded waits at once: both try_waits are in flight together, so a chunk that needs two barriers pays one
// barrier round trip, not two (a try_wait on a completed phase still takes a shared-memory round trip).
__device__ __forceinline__ bool mbar_wait2(uint64_t* bar1, uint32_t par1, uint64_t* bar2, uint32_t par2,
                                           int32_t* err) {
    const uint32_t a1 = smem_u32(bar1), a2 = smem_u32(bar2);
    uint64_t t0 = 0;
    uint32_t d1 = 0, d2 = 0;
    for (;;) {
        uint32_t r1 = 1, r2 = 1;
        if (!d1)
            asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
                         " selp.u32 %0, 1, 0, p;\n}\n"
                         : "=r"(r1) : "r"(a1), "r"(par1), "r"(kSuspendNs) : "memory");
        if (!d2)
            asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
                         " selp.u32 %0, 1, 0, p;\n}\n"
                         : "=r"(r2) : "r"(a2), "r"(par2), "r"(kSuspendNs) : "memory");
        d1 |= r1;
        d2 |= r2;
        if (d1 && d2) return true;
        const uint64_t now = globaltimer_ns();
        if (!t0) t0 = now;
        else if (now - t0 > kWaitLimitNs) break;
    }
    if (err) atomicOr(err, 1);
    return false;
}
__device__ __forceinline__ bool mbar_wait2_warp(uint64_t* bar1, uint32_t par1, uint64_t* bar2, uint32_t par2,
                                                int32_t* err) {
    const bool ok = mbar_wait2(bar1, par1, bar2, par2, err);
    __syncwarp();
    return ok;
}
// mbar_wait by a whole warp, reconverged after it: every lane has seen the phase before the warp goes on to a
// .sync.aligned or elected instruction.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int32_t* err) {
    const bool ok = mbar_wait(bar, parity, err);
    __syncwarp();
    return ok;
}
// One bulk (non-tensor) TMA copy global -> this CTA's shared memory, completing on `bar`. 16-byte aligned
// addresses and a size that is a multiple of 16 (the host refuses weights that are not).
__device__ __forceinline__ void tma_bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// Elected-lane forms: the whole warp executes the statement, so its operands stay warp-uniform, and the one lane
// elect.sync picks issues it. (A single-lane branch around these asynchronous-unit instructions runs them several
// times slower than their issue rate.)
__device__ __forceinline__ void mbar_expect_tx_el(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
                 " @e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n}\n" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void tma_bulk_g2s_el(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
                 " @e cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n}\n" ::
                     "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ float4 ld_dsmem_f4(const float* local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(remote)
                 : "memory");
    return v;
}


// ------------------------------------------------------------------------------------------ expert lookups
struct ExpertView {
    int c;
    int64_t j, R, C;
};
__device__ __forceinline__ ExpertView expert_view(const Exl3bOp& op, int64_t e) {
    ExpertView v;
    v.c = (int)(e % op.n_class);
    v.j = e / op.n_class;
    v.R = op.cls[v.c].rows;
    v.C = op.cls[v.c].cols;
    return v;
}
// Four bf16 values stored as one 8-byte word where the address allows (a row written over NVLink then moves in
// full 256-byte warp stores), else one by one.
__device__ __forceinline__ void st4_bf16(uint16_t* y, const float v[4]) {
    const uint16_t b0 = f2bf(v[0]), b1 = f2bf(v[1]), b2 = f2bf(v[2]), b3 = f2bf(v[3]);
    if ((reinterpret_cast<uintptr_t>(y) & 7) == 0) {
        uint2 u;
        u.x = (uint32_t)b0 | ((uint32_t)b1 << 16);
        u.y = (uint32_t)b2 | ((uint32_t)b3 << 16);
        *reinterpret_cast<uint2*>(y) = u;
    } else {
        y[0] = b0; y[1] = b1; y[2] = b2; y[3] = b3;
    }
}
// Four f16 values, stored the same way (the f16-output linear).
__device__ __forceinline__ void st4_f16(uint16_t* y, const float v[4]) {
    const uint16_t b0 = f2h(v[0]), b1 = f2h(v[1]), b2 = f2h(v[2]), b3 = f2h(v[3]);
    if ((reinterpret_cast<uintptr_t>(y) & 7) == 0) {
        uint2 u;
        u.x = (uint32_t)b0 | ((uint32_t)b1 << 16);
        u.y = (uint32_t)b2 | ((uint32_t)b3 << 16);
        *reinterpret_cast<uint2*>(y) = u;
    } else {
        y[0] = b0; y[1] = b1; y[2] = b2; y[3] = b3;
    }
}
// down's output row: bf16 (the op's type), or f16 for the f16-output linear
__device__ __forceinline__ void st4_out(const Exl3bOp& op, uint16_t* y, const float v[4]) {
    if (op.out_f16) st4_f16(y, v);
    else st4_bf16(y, v);
}
// Where output row i goes: y + i * pitch, or -- when the caller gave a row table (the expert-parallel combine
// writing straight into the sources' memory) -- row_dst[i].
__device__ __forceinline__ uint16_t* out_row(const Exl3bOp& op, int64_t i) {
    return op.row_dst ? reinterpret_cast<uint16_t*>(op.row_dst[i]) : static_cast<uint16_t*>(op.y) + i * op.y_pitch;
}
__device__ __forceinline__ bool row_live(const Exl3bOp& op, int64_t i) {
    return i >= op.expert_offset[0] && i < op.expert_offset[op.n_expert] && op.sorted_tok[i] >= 0;
}

}  // namespace
