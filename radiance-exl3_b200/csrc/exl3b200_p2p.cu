// exl3b200_p2p.cu -- expert parallelism over peer memory: the dispatch and the combine write straight into the
// other ranks' memory over NVLink (plain stores to CUDA-IPC-mapped pointers, no TMA), and each rank
// learns that its peers' data has landed from per-(source, destination) epoch flags. sm_100a CUDA, extern "C".
//
// Every rank owns one "window" (cudaMalloc'ed here, exported by IPC handle, mapped by every peer), the same layout
// on every rank, offsets in bytes from its base:
//   rows   [world][t_cap][hidden] f16   token rows rank s sent here, segment s
//   meta   [world][p_cap] u32           pair metas rank s sent here: (row in segment << 12) | local expert
//   yback  [p_cap][hidden] bf16         the down row of each pair THIS rank sent, written by the pair's owner at
//                                       the pair's position in this rank's sorted-by-rank order
//   ctl    [world][8] u32               from rank s: [0] dispatch epoch, [1] rows, [2] pairs, [3] the pairs' base in
//                                       s's sorted order, [4] combine epoch
//   done   [2] u32                      last-block counters of the dispatch and the combine kernels
//   sink   [hidden] bf16                one spare row: where a row that would fall outside a window goes instead
// A step: k_p2p_dispatch (rows + metas + counts, then the flag) -> k_p2p_wait_dispatch (every source's flag, bounded)
// -> the local ops -> k_p2p_combine (each pair's down row to its source, then the flag) -> k_p2p_wait_combine.
//
// Reuse across steps is safe by construction: rank s writes step e + 1 into rank d's rows/meta only after it has
// seen d's combine flag for step e, which d raises after its gate_up (the last reader of rows) of step e; rank d
// writes step e + 1 into s's yback only after s's dispatch flag for e + 1, which s raises after its gather (the
// reader of yback) of step e. Every wait gives up after a bounded time and reports it (status word and error word).
#include <cuda_runtime.h>
#include <stdint.h>

#include "exl3b200_sys.cuh"

namespace {


struct Win {
    int64_t rows, meta, yback, ctl, done, sink;   // byte offsets in every window (sink: one spare row)
};

using exl3b::gtimer;
using exl3b::ld_acquire_sys;
using exl3b::st_release_sys;

__device__ __forceinline__ uint8_t* wbase(const uint64_t* peers, int r) {
    return reinterpret_cast<uint8_t*>(peers[r]);
}

// One warp a slot j of this rank's sorted-by-rank pairs: the pair's meta to its owner d's meta segment, and -- for
// the first r < rows_d slots of d -- token row row_tok[j] to d's rows segment. The last block to finish raises every
// owner's dispatch flag (after the counts).
__global__ void k_p2p_dispatch(const uint4* __restrict__ x, int64_t x_pitch16, const int32_t* __restrict__ row_tok,
                               const uint32_t* __restrict__ meta, const int32_t* __restrict__ dest_off,
                               const int32_t* __restrict__ counts, int64_t n_slots, const uint64_t* __restrict__ peers,
                               Win w, int self, int world, int64_t t_cap, int64_t p_cap, int row16,
                               const uint32_t* __restrict__ epoch_p, int32_t* err) {
    const int lane = threadIdx.x & 31;
    for (int64_t j = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; j < n_slots;
         j += (int64_t)gridDim.x * (blockDim.x / 32)) {
        int d = 0;
        while (d < world && j >= dest_off[d + 1]) ++d;
        if (d >= world) continue;
        const int64_t r = j - dest_off[d];
        if (r >= p_cap) {                     // past the segment: refused, reported
            if (lane == 0) atomicOr(err, 4);
            continue;
        }
        uint8_t* base = wbase(peers, d);
        if (lane == 0) reinterpret_cast<uint32_t*>(base + w.meta)[(int64_t)self * p_cap + r] = meta[j];
        if (r < counts[2 * d]) {
            if (r >= t_cap) {
                if (lane == 0) atomicOr(err, 4);
                continue;
            }
            const uint4* src = x + (int64_t)row_tok[j] * x_pitch16;
            uint4* dst = reinterpret_cast<uint4*>(base + w.rows) + ((int64_t)self * t_cap + r) * row16;
            for (int u = lane; u < row16; u += 32) dst[u] = src[u];
        }
    }
    __threadfence_system();                  // this thread's stores, visible system-wide before the count below
    __syncthreads();
    __shared__ bool last;
    if (threadIdx.x == 0) {
        uint32_t* done = reinterpret_cast<uint32_t*>(wbase(peers, self) + w.done);
        last = atomicAdd(&done[0], 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    if ((int)threadIdx.x < world) {
        const int d = threadIdx.x;
        uint32_t* ctl = reinterpret_cast<uint32_t*>(wbase(peers, d) + w.ctl) + self * 8;
        ctl[1] = (uint32_t)counts[2 * d];
        ctl[2] = (uint32_t)counts[2 * d + 1];
        ctl[3] = (uint32_t)dest_off[d];
        __threadfence_system();
        st_release_sys(&ctl[0], *epoch_p);
    }
    if (threadIdx.x == 0) reinterpret_cast<uint32_t*>(wbase(peers, self) + w.done)[0] = 0;
}

// Lane s waits (bounded) for source s's dispatch flag of this epoch, then hands its counts to the host:
// hdr[3s] = rows, hdr[3s + 1] = pairs, hdr[3s + 2] = base; hdr[3 world] = 0, or -1 when a wait gave up.
__global__ void k_p2p_wait_dispatch(uint8_t* own, Win w, int world, const uint32_t* epoch_p, int32_t* hdr,
                                    int32_t* err, uint64_t limit_ns) {
    const int s = threadIdx.x;
    const uint32_t epoch = *epoch_p;
    bool ok = true;
    if (s < world) {
        const uint32_t* ctl = reinterpret_cast<const uint32_t*>(own + w.ctl) + s * 8;
        const uint64_t t0 = gtimer();
        while ((int32_t)(ld_acquire_sys(&ctl[0]) - epoch) < 0) {
            if (gtimer() - t0 > limit_ns) { ok = false; break; }
            __nanosleep(256);
        }
        hdr[3 * s] = ok ? (int32_t)ld_acquire_sys(&ctl[1]) : 0;
        hdr[3 * s + 1] = ok ? (int32_t)ld_acquire_sys(&ctl[2]) : 0;
        hdr[3 * s + 2] = ok ? (int32_t)ld_acquire_sys(&ctl[3]) : 0;
    }
    const bool all = __all_sync(0xFFFFFFFFu, ok);
    if (s == 0) {
        hdr[3 * world] = all ? 0 : -1;
        if (!all) atomicOr(err, 8);
    }
}

// Received pair q (source-major, then the source's order): its local expert, its row in the window's rows
// (segment s, row meta >> 12), and where its down row goes back (source s, position base_s + j).
__global__ void k_p2p_unpack(const uint8_t* own, Win w, const int32_t* __restrict__ hdr, int world, int64_t t_cap,
                             int64_t p_cap, int64_t n_pairs, int32_t* __restrict__ expert, int32_t* __restrict__ row,
                             int32_t* __restrict__ dst_rank, int32_t* __restrict__ dst_pos) {
    const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= n_pairs) return;
    int64_t pb = 0;
    int s = 0;
    for (; s < world; ++s) {
        const int64_t np = hdr[3 * s + 1];
        if (q < pb + np) break;
        pb += np;
    }
    if (s >= world) {                   // past the received pairs (a capacity-sized pass): a dropped entry
        expert[q] = -1;
        row[q] = -1;
        dst_rank[q] = -1;
        dst_pos[q] = -1;
        return;
    }
    const int64_t j = q - pb;
    const uint32_t m = j < p_cap ? __ldcv(reinterpret_cast<const uint32_t*>(own + w.meta) + (int64_t)s * p_cap + j) : 0u;
    if (j >= p_cap || (int64_t)(m >> 12) >= t_cap) {   // outside the segments: the pair is dropped (expert -1)
        expert[q] = -1;
        row[q] = -1;
        dst_rank[q] = -1;
        dst_pos[q] = -1;
        return;
    }
    expert[q] = (int32_t)(m & 0xFFFu);
    row[q] = (int32_t)((int64_t)s * t_cap + (m >> 12));
    dst_rank[q] = s;
    dst_pos[q] = hdr[3 * s + 2] + (int32_t)j;
}

// One warp a sorted row i of the local pass: the down row y_rows[i] of pair q = sorted_pair[i] goes to its source's
// yback at its position. The last block raises every source's combine flag.
__global__ void k_p2p_combine(const uint4* __restrict__ y_rows, int64_t y_pitch16, const int32_t* __restrict__ sorted_pair,
                              int64_t n_rows, const int32_t* __restrict__ dst_rank, const int32_t* __restrict__ dst_pos,
                              const uint64_t* __restrict__ peers, Win w, int self, int world, int64_t p_cap, int row16,
                              const uint32_t* __restrict__ epoch_p, int32_t* err) {
    const int lane = threadIdx.x & 31;
    for (int64_t i = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; i < n_rows;
         i += (int64_t)gridDim.x * (blockDim.x / 32)) {
        const int32_t q = sorted_pair[i];
        if (q < 0 || q >= n_rows) continue;
        const int s = dst_rank[q];
        const int64_t pos = dst_pos[q];
        if (s < 0 || s >= world || pos < 0 || pos >= p_cap) {
            if (lane == 0) atomicOr(err, 4);
            continue;
        }
        const uint4* src = y_rows + i * y_pitch16;
        uint4* dst = reinterpret_cast<uint4*>(wbase(peers, s) + w.yback) + pos * row16;
        for (int u = lane; u < row16; u += 32) dst[u] = src[u];
    }
    __threadfence_system();
    __syncthreads();
    __shared__ bool last;
    if (threadIdx.x == 0) {
        uint32_t* done = reinterpret_cast<uint32_t*>(wbase(peers, self) + w.done);
        last = atomicAdd(&done[1], 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    if ((int)threadIdx.x < world) {
        uint32_t* ctl = reinterpret_cast<uint32_t*>(wbase(peers, threadIdx.x) + w.ctl) + self * 8;
        st_release_sys(&ctl[4], *epoch_p);
    }
    if (threadIdx.x == 0) reinterpret_cast<uint32_t*>(wbase(peers, self) + w.done)[1] = 0;
}

// Lane d waits (bounded) for owner d's combine flag of this epoch; status[0] = 0, or -1 when a wait gave up.
__global__ void k_p2p_wait_combine(const uint8_t* own, Win w, int world, const uint32_t* epoch_p, int32_t* status,
                                   int32_t* err, uint64_t limit_ns) {
    const int d = threadIdx.x;
    const uint32_t epoch = *epoch_p;
    bool ok = true;
    if (d < world) {
        const uint32_t* ctl = reinterpret_cast<const uint32_t*>(own + w.ctl) + d * 8;
        const uint64_t t0 = gtimer();
        while ((int32_t)(ld_acquire_sys(&ctl[4]) - epoch) < 0) {
            if (gtimer() - t0 > limit_ns) { ok = false; break; }
            __nanosleep(256);
        }
    }
    const bool all = __all_sync(0xFFFFFFFFu, ok);
    if (d == 0) {
        status[0] = all ? 0 : -1;
        if (!all) atomicOr(err, 8);
    }
}

// The combine fused into down: row_dst[i] = where sorted row i's down row goes -- source s's yback at the pair's
// position (an address in s's window as this rank maps it); a pair outside the windows goes to this rank's sink row
// (error word set).
__global__ void k_p2p_row_dst(const int32_t* __restrict__ sorted_pair, int64_t n_rows,
                              const int32_t* __restrict__ dst_rank, const int32_t* __restrict__ dst_pos,
                              const uint64_t* __restrict__ peers, Win w, int self, int world, int64_t p_cap,
                              int64_t hidden, uint64_t* __restrict__ row_dst, int32_t* err) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows) return;
    const int32_t q = sorted_pair[i];
    if (q < 0) {                        // past the live rows of a capacity-sized pass: never written
        row_dst[i] = peers[self] + (uint64_t)w.sink;
        return;
    }
    const int s = q < n_rows ? dst_rank[q] : -1;
    const int64_t pos = q < n_rows ? dst_pos[q] : -1;
    if (s < 0 || s >= world || pos < 0 || pos >= p_cap) {
        atomicOr(err, 4);
        row_dst[i] = peers[self] + (uint64_t)w.sink;
        return;
    }
    row_dst[i] = peers[s] + (uint64_t)w.yback + (uint64_t)(pos * hidden * 2);
}

// After the down launch that wrote through the row table (its threads fenced their stores at system scope before
// completing): every source's combine flag for this epoch.
__global__ void k_p2p_signal_combine(const uint64_t* __restrict__ peers, Win w, int self, int world,
                                     const uint32_t* __restrict__ epoch_p) {
    const int s = threadIdx.x;
    if (s >= world) return;
    __threadfence_system();
    uint32_t* ctl = reinterpret_cast<uint32_t*>(wbase(peers, s) + w.ctl) + self * 8;
    st_release_sys(&ctl[4], *epoch_p);
}

// A step's epoch lives in device memory (so a captured step replays with a new one): bumped first thing a step.
__global__ void k_p2p_begin(uint32_t* epoch_p) { epoch_p[0] += 1u; }

inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }
constexpr int kWarps = 8;

inline int grid_for(int64_t n_items, int sm) {
    int64_t g = (n_items + kWarps - 1) / kWarps;
    const int64_t cap = (int64_t)sm * 8;
    if (g > cap) g = cap;
    return (int)(g > 0 ? g : 1);
}

}  // namespace

extern "C" {

int exl3b_cuda_device_info(int* sm_count, int32_t** err_word);   // exl3b200_moe.cu

// A caller's CUDA event recorded on the stream (the step drivers' phase marks; C code has no runtime headers).
int exl3b_cuda_mark(void* event, void* stream) {
    return cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)) == cudaSuccess ? 0 : -6;
}

// How long a kernel that waits on another rank's flag (the dispatch and combine waits here, the width split's
// reduce and pull) waits before it gives up and reports: 5 s unless the caller set otherwise. Read at each launch
// and passed to the kernel as an argument.
static const int64_t kPeerWaitDefaultNs = 5000000000ll;
static int64_t g_peer_wait_ns = kPeerWaitDefaultNs;

uint64_t exl3b_peer_wait_ns(void) { return (uint64_t)__atomic_load_n(&g_peer_wait_ns, __ATOMIC_RELAXED); }

int exl3b200_set_peer_wait_ns(int64_t ns) {
    if (ns > 600ll * 1000000000ll) return -12;
    __atomic_store_n(&g_peer_wait_ns, ns <= 0 ? kPeerWaitDefaultNs : ns, __ATOMIC_RELAXED);
    return 0;
}

int exl3b200_ep_window_alloc(int64_t bytes, void** ptr) {
    if (!ptr || bytes <= 0) return -12;
    void* p = nullptr;
    if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return -7;
    if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess) { cudaFree(p); return -6; }
    *ptr = p;
    return 0;
}
int exl3b200_ep_window_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? 0 : -6; }
int exl3b200_ep_window_handle(void* ptr, void* handle64) {
    if (!ptr || !handle64) return -12;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return -6;
    static_assert(sizeof(h) == 64, "IPC handle size");
    for (int i = 0; i < 64; ++i) static_cast<char*>(handle64)[i] = h.reserved[i];
    return 0;
}
int exl3b200_ep_window_open(const void* handle64, void** ptr) {
    if (!handle64 || !ptr) return -12;
    cudaIpcMemHandle_t h;
    for (int i = 0; i < 64; ++i) h.reserved[i] = static_cast<const char*>(handle64)[i];
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return -6;
    *ptr = p;
    return 0;
}
int exl3b200_ep_window_close(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? 0 : -6; }

// offs[5] = {rows, meta, yback, ctl, done} byte offsets of the window layout (the same on every rank).
int exl3b200_p2p_dispatch(const uint16_t* x, int64_t x_pitch, const int32_t* row_tok, const uint32_t* meta,
                          const int32_t* dest_off, const int32_t* counts, int64_t n_slots, const uint64_t* peers,
                          const int64_t* offs, int64_t self, int64_t world, int64_t t_cap, int64_t p_cap,
                          int64_t hidden, const uint32_t* epoch, void* stream) {
    if (!x || !row_tok || !meta || !dest_off || !counts || !peers || !offs || world < 1 || world > 32 || self < 0 ||
        self >= world || n_slots < 0 || hidden < 8 || hidden % 8 || x_pitch % 8 || !al16(x))
        return -12;
    int sm = 0;
    int32_t* err = nullptr;
    if (exl3b_cuda_device_info(&sm, &err) != 0) return -6;
    const Win w = { offs[0], offs[1], offs[2], offs[3], offs[4], offs[5] };
    k_p2p_dispatch<<<grid_for(n_slots, sm), kWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint4*>(x), x_pitch / 8, row_tok, meta, dest_off, counts, n_slots, peers, w, (int)self,
        (int)world, t_cap, p_cap, (int)(hidden / 8), epoch, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_p2p_wait_dispatch(void* own, const int64_t* offs, int64_t world, const uint32_t* epoch, int32_t* hdr,
                               void* stream) {
    if (!own || !offs || !hdr || !epoch || world < 1 || world > 32) return -12;
    int sm = 0;
    int32_t* err = nullptr;
    if (exl3b_cuda_device_info(&sm, &err) != 0) return -6;
    const Win w = { offs[0], offs[1], offs[2], offs[3], offs[4], offs[5] };
    k_p2p_wait_dispatch<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint8_t*>(own), w, (int)world,
                                                                        epoch, hdr, err, exl3b_peer_wait_ns());
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_p2p_unpack(const void* own, const int64_t* offs, const int32_t* hdr, int64_t world, int64_t t_cap,
                        int64_t p_cap, int64_t n_pairs, int32_t* expert, int32_t* row, int32_t* dst_rank,
                        int32_t* dst_pos, void* stream) {
    if (!own || !offs || !hdr || !expert || !row || !dst_rank || !dst_pos || world < 1 || n_pairs < 0) return -12;
    if (n_pairs == 0) return 0;
    const Win w = { offs[0], offs[1], offs[2], offs[3], offs[4], offs[5] };
    k_p2p_unpack<<<(unsigned)((n_pairs + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(own), w, hdr, (int)world, t_cap, p_cap, n_pairs, expert, row, dst_rank, dst_pos);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_p2p_combine(const uint16_t* y_rows, int64_t y_pitch, const int32_t* sorted_pair, int64_t n_rows,
                         const int32_t* dst_rank, const int32_t* dst_pos, const uint64_t* peers, const int64_t* offs,
                         int64_t self, int64_t world, int64_t p_cap, int64_t hidden, const uint32_t* epoch,
                         void* stream) {
    if (!y_rows || !sorted_pair || !dst_rank || !dst_pos || !peers || !offs || world < 1 || world > 32 || self < 0 ||
        self >= world || n_rows < 0 || hidden < 8 || hidden % 8 || y_pitch % 8 || !al16(y_rows))
        return -12;
    int sm = 0;
    int32_t* err = nullptr;
    if (exl3b_cuda_device_info(&sm, &err) != 0) return -6;
    const Win w = { offs[0], offs[1], offs[2], offs[3], offs[4], offs[5] };
    k_p2p_combine<<<grid_for(n_rows, sm), kWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint4*>(y_rows), y_pitch / 8, sorted_pair, n_rows, dst_rank, dst_pos, peers, w,
        (int)self, (int)world, p_cap, (int)(hidden / 8), epoch, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_p2p_begin(uint32_t* epoch, void* stream) {
    if (!epoch) return -12;
    k_p2p_begin<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(epoch);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_p2p_row_dst(const int32_t* sorted_pair, int64_t n_rows, const int32_t* dst_rank, const int32_t* dst_pos,
                         const uint64_t* peers, const int64_t* offs, int64_t self, int64_t world, int64_t p_cap,
                         int64_t hidden, uint64_t* row_dst, void* stream) {
    if (!sorted_pair || !dst_rank || !dst_pos || !peers || !offs || !row_dst || world < 1 || world > 32 || self < 0 ||
        self >= world || n_rows < 0 || hidden < 8)
        return -12;
    if (n_rows == 0) return 0;
    int sm = 0;
    int32_t* err = nullptr;
    if (exl3b_cuda_device_info(&sm, &err) != 0) return -6;
    const Win w = { offs[0], offs[1], offs[2], offs[3], offs[4], offs[5] };
    k_p2p_row_dst<<<(unsigned)((n_rows + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        sorted_pair, n_rows, dst_rank, dst_pos, peers, w, (int)self, (int)world, p_cap, hidden, row_dst, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_p2p_signal_combine(const uint64_t* peers, const int64_t* offs, int64_t self, int64_t world,
                                const uint32_t* epoch, void* stream) {
    if (!peers || !offs || !epoch || world < 1 || world > 32 || self < 0 || self >= world) return -12;
    const Win w = { offs[0], offs[1], offs[2], offs[3], offs[4], offs[5] };
    k_p2p_signal_combine<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(peers, w, (int)self, (int)world, epoch);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_p2p_wait_combine(const void* own, const int64_t* offs, int64_t world, const uint32_t* epoch,
                              int32_t* status, void* stream) {
    if (!own || !offs || !status || !epoch || world < 1 || world > 32) return -12;
    int sm = 0;
    int32_t* err = nullptr;
    if (exl3b_cuda_device_info(&sm, &err) != 0) return -6;
    const Win w = { offs[0], offs[1], offs[2], offs[3], offs[4], offs[5] };
    k_p2p_wait_combine<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint8_t*>(own), w,
                                                                       (int)world, epoch, status, err,
                                                                       exl3b_peer_wait_ns());
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

}  // extern "C"
