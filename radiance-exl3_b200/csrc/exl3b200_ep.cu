// exl3b200_ep.cu -- the device bookkeeping of expert parallelism around the routed-expert ops, sm_100a CUDA,
// extern "C". Experts are held in contiguous blocks: expert e lives on rank e / n_local.
//
//   k_ep_dest          the owning rank of each (token, slot) pair
//   k_ep_dedup_scan    per owner rank (its pairs sorted stably by rank, so in token order): one row a distinct
//                      token, a meta word a pair (the row within that rank's block, the local expert), the counts
//   k_ep_dedup_copy    those rows packed contiguously a rank (for a collective library's all-to-all)
//   k_ep_unpack        received pairs: local expert and row index (rows before its source + its row)
//   k_ep_map           sorted pair -> its token row (the sorted_tok the ops read, top_k 1)
//   k_ep_pack          the non-deduplicated pack (one row a pair), k_rows_scatter (rows into arrival order)
// The peer-memory exchange itself is exl3b200_p2p.cu.
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

// dest[p] = ids[p] / n_local (the rank that holds pair p's expert), -1 for a dropped slot.
__global__ void k_ep_dest(const int32_t* __restrict__ ids, int64_t n_pairs, int n_local, int world,
                          int32_t* __restrict__ dest) {
    const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= n_pairs) return;
    const int32_t e = ids[p];
    const int32_t d = e >= 0 ? e / n_local : -1;
    dest[p] = d < world ? d : -1;
}

// The deduplicated pack, step 1 -- one block a destination rank d: its pairs, sorted_pairs[o_d .. o_{d+1})
// (stable by rank, so in token order), make one row per distinct token (the first pair of each token carries it).
// Row r of rank d: row_tok[o_d + r] = its token; pair j's meta = (r << 12) | local expert; counts[2d] = rows,
// counts[2d + 1] = pairs.
constexpr int kDedupThreads = 1024;
__global__ void __launch_bounds__(kDedupThreads) k_ep_dedup_scan(
    const int32_t* __restrict__ ids, int top_k, const int32_t* __restrict__ sorted_pairs,
    const int32_t* __restrict__ dest_off, int n_local, uint32_t* __restrict__ send_meta, int32_t* __restrict__ row_tok,
    int32_t* __restrict__ counts) {
    __shared__ int wtot[kDedupThreads / 32];
    __shared__ int s_run;
    const int d = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t o0 = dest_off[d], o1 = dest_off[d + 1];
    if (tid == 0) s_run = 0;
    __syncthreads();
    for (int64_t c0 = o0; c0 < o1; c0 += kDedupThreads) {
        const int64_t j = c0 + tid;
        const bool in = j < o1;
        const int32_t p = in ? sorted_pairs[j] : -1;
        const int32_t t = p >= 0 ? p / top_k : -1;
        const int32_t tprev = in && j > o0 ? sorted_pairs[j - 1] / top_k : -2;
        const int flag = (in && p >= 0 && t != tprev) ? 1 : 0;
        int incl = flag;                               // inclusive block scan of the flags
#pragma unroll
        for (int dd = 1; dd < 32; dd <<= 1) {
            const int v = __shfl_up_sync(0xFFFFFFFFu, incl, dd);
            if (lane >= dd) incl += v;
        }
        if (lane == 31) wtot[warp] = incl;
        __syncthreads();
        int base = 0, total = 0;
        for (int w = 0; w < kDedupThreads / 32; ++w) {
            const int v = wtot[w];
            if (w < warp) base += v;
            total += v;
        }
        const int run = s_run;
        const int r = run + base + incl - 1;          // the row this pair's token is in (within rank d)
        if (in && p >= 0) send_meta[j] = ((uint32_t)r << 12) | (uint32_t)(ids[p] % n_local);
        if (flag) row_tok[o0 + r] = t;
        __syncthreads();
        if (tid == 0) s_run = run + total;
        __syncthreads();
    }
    if (tid == 0) {
        counts[2 * d] = s_run;
        counts[2 * d + 1] = (int32_t)(o1 - o0);
    }
}

// Step 2 -- one warp a slot j of the rank-ordered pair range: if j is row r < rows_d of its rank d, token row
// row_tok[j] goes to send_x[(rows of ranks before d) + r], so each rank's rows are contiguous and in rank order.
__global__ void k_ep_dedup_copy(const uint4* __restrict__ x, int64_t x_pitch16, const int32_t* __restrict__ dest_off,
                                const int32_t* __restrict__ counts, const int32_t* __restrict__ row_tok, int world,
                                int64_t n_slots, int row16, uint4* __restrict__ send_x) {
    const int lane = threadIdx.x & 31;
    const int64_t j = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (j >= n_slots) return;
    int64_t base = 0;
    int d = 0;
    for (; d < world; ++d) {
        if (j < dest_off[d + 1]) break;
        base += counts[2 * d];
    }
    if (d >= world) return;
    const int64_t r = j - dest_off[d];
    if (r >= counts[2 * d]) return;
    const uint4* src = x + (int64_t)row_tok[j] * x_pitch16;
    uint4* dst = send_x + (base + r) * row16;
    for (int u = lane; u < row16; u += 32) dst[u] = src[u];
}

// Received pairs, concatenated by source rank (pairs of source s: recv_counts[2s + 1], rows recv_counts[2s]):
// pair q's row in the received rows is (rows before source s) + (meta >> 12), its local expert meta & 0xFFF.
__global__ void k_ep_unpack(const uint32_t* __restrict__ meta, int64_t n_pairs, const int32_t* __restrict__ recv_counts,
                            int world, int32_t* __restrict__ expert, int32_t* __restrict__ row) {
    const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= n_pairs) return;
    int64_t pb = 0, rb = 0;
    for (int s = 0; s < world; ++s) {
        const int64_t np = recv_counts[2 * s + 1];
        if (q < pb + np) break;
        pb += np;
        rb += recv_counts[2 * s];
    }
    const uint32_t m = meta[q];
    expert[q] = (int32_t)(m & 0xFFFu);
    row[q] = (int32_t)(rb + (m >> 12));
}

// out[i] = table[idx[i]] (idx outside [0, n_table) gives -1).
__global__ void k_ep_map(const int32_t* __restrict__ idx, int64_t n, const int32_t* __restrict__ table, int64_t n_table,
                         int32_t* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int32_t j = idx[i];
    out[i] = j >= 0 && j < n_table ? table[j] : -1;
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

int exl3b200_ep_dest(const int32_t* ids, int64_t n_pairs, int64_t n_local, int64_t world, int32_t* dest,
                     void* stream) {
    if (!ids || !dest || n_pairs < 0 || n_local < 1 || world < 1) return -12;
    if (n_pairs == 0) return 0;
    k_ep_dest<<<(unsigned)((n_pairs + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        ids, n_pairs, (int)n_local, (int)world, dest);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_ep_pack_dedup(const uint16_t* x, int64_t x_pitch, const int32_t* ids, int64_t top_k,
                           const int32_t* sorted_pairs, const int32_t* dest_off, int64_t n_pairs, int64_t n_local,
                           int64_t world, int64_t hidden, uint16_t* send_x, uint32_t* send_meta, int32_t* row_tok,
                           int32_t* counts, void* stream) {
    if (!x || !ids || !sorted_pairs || !dest_off || !send_x || !send_meta || !row_tok || !counts) return -12;
    if (top_k < 1 || n_local < 1 || n_local > 4096 || world < 1 || world > 65535 || hidden < 8 || x_pitch < hidden ||
        n_pairs < 0 || n_pairs / top_k >= ((int64_t)1 << 20))
        return -12;
    if (hidden % 8 || x_pitch % 8 || !al16(x) || !al16(send_x)) return -3;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    k_ep_dedup_scan<<<(unsigned)world, kDedupThreads, 0, st>>>(ids, (int)top_k, sorted_pairs, dest_off, (int)n_local,
                                                               send_meta, row_tok, counts);
    if (n_pairs > 0)
        k_ep_dedup_copy<<<(unsigned)((n_pairs + kWarpsPerBlock - 1) / kWarpsPerBlock), kWarpsPerBlock * 32, 0, st>>>(
            reinterpret_cast<const uint4*>(x), x_pitch / 8, dest_off, counts, row_tok, (int)world, n_pairs,
            (int)(hidden / 8), reinterpret_cast<uint4*>(send_x));
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_ep_dedup_scan(const int32_t* ids, int64_t top_k, const int32_t* sorted_pairs, const int32_t* dest_off,
                           int64_t n_pairs, int64_t n_local, int64_t world, uint32_t* send_meta, int32_t* row_tok,
                           int32_t* counts, void* stream) {
    if (!ids || !sorted_pairs || !dest_off || !send_meta || !row_tok || !counts) return -12;
    if (top_k < 1 || n_local < 1 || n_local > 4096 || world < 1 || world > 65535 || n_pairs < 0 ||
        n_pairs / top_k >= ((int64_t)1 << 20))
        return -12;
    k_ep_dedup_scan<<<(unsigned)world, kDedupThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        ids, (int)top_k, sorted_pairs, dest_off, (int)n_local, send_meta, row_tok, counts);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_ep_unpack(const uint32_t* meta, int64_t n_pairs, const int32_t* recv_counts, int64_t world,
                       int32_t* expert, int32_t* row, void* stream) {
    if (!meta || !recv_counts || !expert || !row || n_pairs < 0 || world < 1) return -12;
    if (n_pairs == 0) return 0;
    k_ep_unpack<<<(unsigned)((n_pairs + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        meta, n_pairs, recv_counts, (int)world, expert, row);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_ep_map(const int32_t* idx, int64_t n, const int32_t* table, int64_t n_table, int32_t* out,
                    void* stream) {
    if (!idx || !table || !out || n < 0 || n_table < 0) return -12;
    if (n == 0) return 0;
    k_ep_map<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(idx, n, table, n_table, out);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

}  // extern "C"
