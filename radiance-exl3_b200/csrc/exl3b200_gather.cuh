// exl3b200_gather.cuh -- the gather's inverse map and one token's gather over 8 columns, shared by the one-GPU
// gather (exl3b200_moe.cu) and the tensor-split gather that writes each token's partial to the rank reducing it
// (exl3b200_tp.cu).
//
// y[t][n..n+8) = sum over slots s ascending of w[t,s] * rows[pos[t,s]][n..n+8) (bf16 rows, f32 products and sums,
// each rounded as the reference's gather does: docs/OPS-exl3.md:195-196). Every live slot's row is loaded before
// any is summed. rows 16-byte aligned with a pitch of a multiple of 8 elements (the host checks).
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace exl3b {

constexpr int kGatherSlots = 8;

// pos[f] = the sorted row of flat (token, slot) pair f (pos prefilled with -1: a pair no row holds stays -1).
static __global__ void k_invert(const int32_t* __restrict__ sorted_tok, int64_t n_rows, int64_t n_pairs,
                                int32_t* __restrict__ pos) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows) return;
    const int32_t f = sorted_tok[i];
    if (f >= 0 && f < n_pairs) pos[f] = (int32_t)i;
}

// pos_t, w_t: the token's top_k sorted rows (-1: no row) and weights.
__device__ __forceinline__ void gather_row8(const uint16_t* __restrict__ rows, int64_t pitch,
                                            const int32_t* __restrict__ pos_t, const float* __restrict__ w_t,
                                            int top_k, int64_t n, float acc[8]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int s0 = 0; s0 < top_k; s0 += kGatherSlots) {
        uint4 r[kGatherSlots];
        float ws[kGatherSlots];
        bool live[kGatherSlots];
#pragma unroll
        for (int q = 0; q < kGatherSlots; ++q) {
            live[q] = false;
            if (s0 + q >= top_k) continue;
            const int32_t i = pos_t[s0 + q];
            if (i < 0) continue;
            live[q] = true;
            ws[q] = w_t[s0 + q];
            r[q] = *reinterpret_cast<const uint4*>(rows + (int64_t)i * pitch + n);
        }
#pragma unroll
        for (int q = 0; q < kGatherSlots; ++q) {
            if (!live[q]) continue;
            const uint32_t u[4] = { r[q].x, r[q].y, r[q].z, r[q].w };
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint16_t b = (uint16_t)(u[j >> 1] >> (16 * (j & 1)));
                acc[j] = __fadd_rn(acc[j], __fmul_rn(ws[q], __bfloat162float(__ushort_as_bfloat16(b))));
            }
        }
    }
}

}  // namespace exl3b
