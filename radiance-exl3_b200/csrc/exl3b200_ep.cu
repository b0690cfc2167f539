// exl3b200_ep.cu -- the device steps of expert parallelism around the routed-expert ops, sm_100a CUDA, extern "C".
//
// Experts are held in contiguous blocks: expert e lives on rank e / n_local. A step on each rank:
//   router -> stable scatter of its (token, slot) pairs over ALL experts (so the sorted pairs are grouped by the
//   rank that holds their expert) -> k_ep_pack (the token row of every sorted pair, its local expert id, the
//   per-rank counts) -> all-to-all of the rows -> stable scatter of the received rows over the local experts ->
//   gate_up, down -> k_rows_scatter (the down rows back into arrival order) -> all-to-all back -> the gather over
//   the sorted pairs, which sums each token's slots in ascending order exactly as on one GPU.
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

// One warp a sorted pair: its token's row copied in 16-byte pieces, its local expert id; block 0 also writes the
// number of pairs bound for each rank from the expert offsets.
__global__ void k_ep_pack(const uint4* __restrict__ x, int64_t x_pitch16, const int32_t* __restrict__ ids, int top_k,
                          const int32_t* __restrict__ sorted_pairs, int64_t n_pairs,
                          const int32_t* __restrict__ expert_offset, int n_local, int world, int row16,
                          uint4* __restrict__ send_x, int32_t* __restrict__ send_e, int32_t* __restrict__ counts) {
    if (blockIdx.x == 0 && threadIdx.x < (unsigned)world) {
        const int r = threadIdx.x;
        counts[r] = expert_offset[(r + 1) * n_local] - expert_offset[r * n_local];
    }
    const int lane = threadIdx.x & 31;
    const int64_t j = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (j >= n_pairs) return;
    const int32_t p = sorted_pairs[j];
    if (p < 0) return;   // a row past the live count of the sort: nothing is sent for it
    const uint4* src = x + (int64_t)(p / top_k) * x_pitch16;
    uint4* dst = send_x + j * row16;
    for (int q = lane; q < row16; q += 32) dst[q] = src[q];
    if (lane == 0) send_e[j] = ids[p] % n_local;
}

// One warp a row: dst[idx[j]] = src[j], rows of row16 16-byte pieces; an index outside [0, n_dst) is skipped.
__global__ void k_rows_scatter(const uint4* __restrict__ src, int64_t src_pitch16, const int32_t* __restrict__ idx,
                               int64_t n_rows, int row16, uint4* __restrict__ dst, int64_t dst_pitch16,
                               int64_t n_dst) {
    const int lane = threadIdx.x & 31;
    const int64_t j = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (j >= n_rows) return;
    const int32_t d = idx[j];
    if (d < 0 || d >= n_dst) return;
    const uint4* s = src + j * src_pitch16;
    uint4* o = dst + (int64_t)d * dst_pitch16;
    for (int q = lane; q < row16; q += 32) o[q] = s[q];
}

constexpr int kWarpsPerBlock = 8;

inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace

extern "C" {

int exl3b200_ep_pack(const uint16_t* x, int64_t x_pitch, const int32_t* ids, int64_t top_k,
                     const int32_t* sorted_pairs, int64_t n_pairs, const int32_t* expert_offset, int64_t n_local,
                     int64_t world, int64_t hidden, uint16_t* send_x, int32_t* send_e, int32_t* send_counts,
                     void* stream) {
    if (!x || !ids || !sorted_pairs || !expert_offset || !send_x || !send_e || !send_counts) return -12;
    if (n_pairs < 0 || top_k < 1 || n_local < 1 || world < 1 || world > 1024 || hidden < 8 || x_pitch < hidden)
        return -12;
    if (hidden % 8 || x_pitch % 8 || !al16(x) || !al16(send_x)) return -3;
    const unsigned blocks = (unsigned)((n_pairs + kWarpsPerBlock - 1) / kWarpsPerBlock);
    k_ep_pack<<<blocks > 0 ? blocks : 1, kWarpsPerBlock * 32 > world ? kWarpsPerBlock * 32 : (unsigned)world, 0,
                static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint4*>(x), x_pitch / 8, ids, (int)top_k, sorted_pairs, n_pairs, expert_offset,
        (int)n_local, (int)world, (int)(hidden / 8), reinterpret_cast<uint4*>(send_x), send_e, send_counts);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_rows_scatter(const void* src, int64_t src_pitch, const int32_t* idx, int64_t n_rows, int64_t row_bytes,
                          void* dst, int64_t dst_pitch, int64_t n_dst, void* stream) {
    if (!src || !idx || !dst || n_rows < 0 || n_dst < 0 || row_bytes < 16 || src_pitch < row_bytes ||
        dst_pitch < row_bytes)
        return -12;
    if (row_bytes % 16 || src_pitch % 16 || dst_pitch % 16 || !al16(src) || !al16(dst)) return -3;
    if (n_rows == 0) return 0;
    const unsigned blocks = (unsigned)((n_rows + kWarpsPerBlock - 1) / kWarpsPerBlock);
    k_rows_scatter<<<blocks, kWarpsPerBlock * 32, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(src), src_pitch / 16, idx, n_rows, (int)(row_bytes / 16), static_cast<uint4*>(dst),
        dst_pitch / 16, n_dst);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

}  // extern "C"
