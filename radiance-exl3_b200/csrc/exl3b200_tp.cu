// exl3b200_tp.cu -- the width ("column-block") tensor split over peer memory: every rank holds a slice of EVERY
// expert's intermediate width (whole 128-column blocks), runs gate_up and down over all routed rows on its slice and
// gathers a per-token PARTIAL of the layer's output; the partials summed over the ranks are the layer's output
// (architectures/qwen4exp_exl3/rad_block_moe_exl3.h:438-470: "each rank computes its gate/up rows and its K slice of
// down for every routed expert; the routing weight scales each partial and the all-reduce sums them"). The reference
// engine sums with its all_reduce op; here the sum is fused into the gather as a reduce-scatter over NVLink followed
// by an all-gather, all plain loads and stores to CUDA-IPC-mapped windows (no TMA). sm_100a CUDA,
// extern "C".
//
// Tokens are cut into `world` contiguous slices of s = ceil(T / world) rows; rank o reduces slice o. Every rank's
// window, the same layout everywhere (byte offsets from its base):
//   part [world][s_cap][H] f32   source s's partials of this rank's slice, segment s
//   red  [s_cap][H] f32          this rank's slice, reduced
//   ctl  [world][8] u32          from rank s: [0] partials epoch, [1] reduced epoch
//   done [4] u32                 [0] gather counter, [1] reduce counter, [2] reduce blocks that gave up
// A step (after exl3b200_p2p_begin bumped the device epoch):
//   k_tp_gather_rs  each token's partial (the one-GPU gather's sum, exl3b::gather_row8) stored straight into the
//                   owning rank's part segment; the last block raises every owner's partials flag
//   k_tp_reduce     waits (bounded) for every source's partials flag, sums slice o's segments in ascending source
//                   order into red; the last block raises every rank's reduced flag (none if a block gave up)
//   k_tp_pull       waits (bounded) for every owner's reduced flag and copies each slice into this rank's output
// Every rank so ends with the same bits (each token summed once, by its owner, in source order 0..world-1; at one
// rank the output is the one-GPU gather's, bit for bit).
//
// Reuse across steps is safe by construction: source s writes step e + 1 into owner o's part only after s's pull of
// step e saw o's reduced flag of e, which o raises after its reduce blocks have read part; o writes red of step e + 1
// only after every source's partials flag of e + 1, which each source raises after its pull of step e has read red.
// Ranks agree on T (the routed tokens are replicated under the width split). Every wait gives up after a bounded time
// and reports it (status word and the library's error word).
#include <cuda_runtime.h>
#include <stdint.h>

#include "exl3b200_gather.cuh"
#include "exl3b200_sys.cuh"

namespace {

using exl3b::gtimer;
using exl3b::ld_acquire_sys;
using exl3b::st_release_sys;


struct TpWin {
    int64_t part, red, ctl, done;   // byte offsets in every window
};

__device__ __forceinline__ uint8_t* wbase(const uint64_t* peers, int r) {
    return reinterpret_cast<uint8_t*>(peers[r]);
}

// Thread 0 of a block: every rank's flag `slot` at this epoch or later, waiting at most limit_ns in all.
__device__ bool wait_all(const uint8_t* own, TpWin win, int world, int slot, uint32_t epoch, uint64_t limit_ns) {
    const uint32_t* ctl = reinterpret_cast<const uint32_t*>(own + win.ctl);
    const uint64_t t0 = gtimer();
    for (int s = 0; s < world; ++s) {
        while ((int32_t)(ld_acquire_sys(&ctl[s * 8 + slot]) - epoch) < 0) {
            if (gtimer() - t0 > limit_ns) return false;
            __nanosleep(128);
        }
    }
    return true;
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// One block a token: the token's partial over this rank's slice of every expert, to its owner's part segment.
__global__ void k_tp_gather_rs(const uint16_t* __restrict__ rows, int64_t pitch, const int32_t* __restrict__ pos,
                               const float* __restrict__ w, int top_k, int64_t width, int64_t slice, int64_t s_cap,
                               const uint64_t* __restrict__ peers, TpWin win, int self, int world,
                               const uint32_t* __restrict__ epoch_p, int32_t* status) {
    const int64_t t = blockIdx.x;
    const int o = (int)(t / slice);
    const int64_t j = t - (int64_t)o * slice;
    float* dst = reinterpret_cast<float*>(wbase(peers, o) + win.part) + ((int64_t)self * s_cap + j) * width;
    for (int64_t n = 8 * (int64_t)threadIdx.x; n < width; n += 8 * (int64_t)blockDim.x) {
        float acc[8];
        exl3b::gather_row8(rows, pitch, pos + t * top_k, w + t * top_k, top_k, n, acc);
        float4* d = reinterpret_cast<float4*>(dst + n);
        d[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        d[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    if (t == 0 && threadIdx.x == 0) status[0] = 0;
    __threadfence_system();                  // this thread's stores, visible system-wide before the count below
    __syncthreads();
    __shared__ bool last;
    if (threadIdx.x == 0) {
        uint32_t* done = reinterpret_cast<uint32_t*>(wbase(peers, self) + win.done);
        last = atomicAdd(&done[0], 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    if ((int)threadIdx.x < world) {
        const int d = threadIdx.x;
        __threadfence_system();
        st_release_sys(reinterpret_cast<uint32_t*>(wbase(peers, d) + win.ctl) + self * 8 + 0, *epoch_p);
    }
    if (threadIdx.x == 0) reinterpret_cast<uint32_t*>(wbase(peers, self) + win.done)[0] = 0;
}

// This rank's slice, summed over the sources in ascending order (source 0's partial is the start, so one rank's
// sum is its partial exactly).
__global__ void k_tp_reduce(const uint64_t* __restrict__ peers, TpWin win, int self, int world, int64_t n_rows,
                            int64_t w4, int64_t s_cap, const uint32_t* __restrict__ epoch_p, int32_t* err,
                            uint64_t limit_ns) {
    uint8_t* own = wbase(peers, self);
    const uint32_t epoch = *epoch_p;
    __shared__ bool ok;
    if (threadIdx.x == 0) ok = wait_all(own, win, world, 0, epoch, limit_ns);
    __syncthreads();
    uint32_t* done = reinterpret_cast<uint32_t*>(own + win.done);
    if (ok) {
        const float4* part = reinterpret_cast<const float4*>(own + win.part);
        float4* red = reinterpret_cast<float4*>(own + win.red);
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_rows * w4;
             i += (int64_t)gridDim.x * blockDim.x) {
            float4 a = __ldcg(part + i);
            for (int s = 1; s < world; ++s) a = add4(a, __ldcg(part + (int64_t)s * s_cap * w4 + i));
            red[i] = a;
        }
    } else if (threadIdx.x == 0) {
        atomicOr(err, 8);
        atomicAdd(&done[2], 1u);
    }
    __threadfence_system();
    __syncthreads();
    __shared__ bool last;
    if (threadIdx.x == 0) last = atomicAdd(&done[1], 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __shared__ bool failed;
    if (threadIdx.x == 0) failed = atomicAdd(&done[2], 0u) != 0;
    __syncthreads();
    if (!failed && (int)threadIdx.x < world) {   // a block that gave up holds every rank's flag back: they report too
        __threadfence_system();
        st_release_sys(reinterpret_cast<uint32_t*>(wbase(peers, threadIdx.x) + win.ctl) + self * 8 + 1, epoch);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        done[1] = 0;
        done[2] = 0;
    }
}

// Every owner's reduced slice into this rank's output (f32 [T][H], row pitch out_pitch4 float4s).
__global__ void k_tp_pull(const uint64_t* __restrict__ peers, TpWin win, int self, int world, int64_t n_tok,
                          int64_t w4, int64_t slice, float4* __restrict__ out, int64_t out_pitch4,
                          const uint32_t* __restrict__ epoch_p, int32_t* status, int32_t* err, uint64_t limit_ns) {
    __shared__ bool ok;
    if (threadIdx.x == 0) ok = wait_all(wbase(peers, self), win, world, 1, *epoch_p, limit_ns);
    __syncthreads();
    if (!ok) {
        if (threadIdx.x == 0) {
            status[0] = -1;
            atomicOr(err, 8);
        }
        return;
    }
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_tok * w4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / w4, c = i - t * w4;
        const int o = (int)(t / slice);
        const float4* red = reinterpret_cast<const float4*>(wbase(peers, o) + win.red);
        out[t * out_pitch4 + c] = __ldcg(red + (t - (int64_t)o * slice) * w4 + c);
    }
}

inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

inline int grid_for(int64_t n, int sm) {
    int64_t g = (n + 255) / 256;
    const int64_t cap = (int64_t)sm * 8;
    if (g > cap) g = cap;
    return (int)(g > 0 ? g : 1);
}

inline TpWin tp_win(const int64_t* offs) { return TpWin{ offs[0], offs[1], offs[2], offs[3] }; }

}  // namespace

extern "C" {

int exl3b_cuda_device_info(int* sm_count, int32_t** err_word);   // exl3b200_moe.cu
uint64_t exl3b_peer_wait_ns(void);                                // exl3b200_p2p.cu

// The gather (exl3b200_moe_gather's arithmetic) writing each token's partial into its owner's window, then the
// owners' partials flags. offs[4] = {part, red, ctl, done}.
int exl3b200_tp_gather_rs(const uint16_t* rows, int64_t row_pitch, const int32_t* sorted_tok, int64_t n_rows,
                          const float* w, int64_t n_tok, int64_t top_k, int64_t width, void* work,
                          const uint64_t* peers, const int64_t* offs, int64_t self, int64_t world, int64_t s_cap,
                          const uint32_t* epoch, int32_t* status, void* stream) {
    if (!rows || !sorted_tok || !w || !work || !peers || !offs || !epoch || !status || n_tok < 0 || top_k < 1 ||
        width < 8 || width % 8 || row_pitch % 8 || !al16(rows) || world < 1 || world > 32 || self < 0 ||
        self >= world)
        return -12;
    if (n_tok == 0) return 0;
    const int64_t slice = (n_tok + world - 1) / world;
    if (slice > s_cap) return -12;
    int sm = 0;
    int32_t* err = nullptr;
    if (exl3b_cuda_device_info(&sm, &err) != 0) return -6;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t* pos = static_cast<int32_t*>(work);
    if (cudaMemsetAsync(pos, 0xFF, (size_t)(n_tok * top_k) * 4, st) != cudaSuccess) return -6;
    if (n_rows > 0)
        exl3b::k_invert<<<(unsigned)((n_rows + 255) / 256), 256, 0, st>>>(sorted_tok, n_rows, n_tok * top_k, pos);
    k_tp_gather_rs<<<(unsigned)n_tok, 256, 0, st>>>(rows, row_pitch, pos, w, (int)top_k, width, slice, s_cap, peers,
                                                    tp_win(offs), (int)self, (int)world, epoch, status);
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_tp_reduce(const uint64_t* peers, const int64_t* offs, int64_t self, int64_t world, int64_t n_tok,
                       int64_t width, int64_t s_cap, const uint32_t* epoch, void* stream) {
    if (!peers || !offs || !epoch || n_tok < 0 || width < 4 || width % 4 || world < 1 || world > 32 || self < 0 ||
        self >= world)
        return -12;
    if (n_tok == 0) return 0;
    const int64_t slice = (n_tok + world - 1) / world;
    if (slice > s_cap) return -12;
    int64_t n_rows = n_tok - self * slice;
    n_rows = n_rows < 0 ? 0 : (n_rows > slice ? slice : n_rows);
    int sm = 0;
    int32_t* err = nullptr;
    if (exl3b_cuda_device_info(&sm, &err) != 0) return -6;
    const int64_t w4 = width / 4;
    k_tp_reduce<<<grid_for(n_rows * w4, sm), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        peers, tp_win(offs), (int)self, (int)world, n_rows, w4, s_cap, epoch, err, exl3b_peer_wait_ns());
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

int exl3b200_tp_pull(const uint64_t* peers, const int64_t* offs, int64_t self, int64_t world, int64_t n_tok,
                     int64_t width, int64_t s_cap, float* out, int64_t out_pitch, const uint32_t* epoch,
                     int32_t* status, void* stream) {
    if (!peers || !offs || !epoch || !status || !out || n_tok < 0 || width < 4 || width % 4 || out_pitch % 4 ||
        out_pitch < width || !al16(out) || world < 1 || world > 32 || self < 0 || self >= world)
        return -12;
    if (n_tok == 0) return 0;
    const int64_t slice = (n_tok + world - 1) / world;
    if (slice > s_cap) return -12;
    int sm = 0;
    int32_t* err = nullptr;
    if (exl3b_cuda_device_info(&sm, &err) != 0) return -6;
    const int64_t w4 = width / 4;
    k_tp_pull<<<grid_for(n_tok * w4, sm), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        peers, tp_win(offs), (int)self, (int)world, n_tok, w4, slice, reinterpret_cast<float4*>(out),
        out_pitch / 4, epoch, status, err, exl3b_peer_wait_ns());
    return cudaGetLastError() == cudaSuccess ? 0 : -6;
}

}  // extern "C"
