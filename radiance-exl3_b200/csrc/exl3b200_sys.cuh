// exl3b200_sys.cuh -- the system-scope flag primitives the peer-memory kernels share (exl3b200_p2p.cu,
// exl3b200_tp.cu): a release store and an acquire load at system scope, and the global nanosecond timer every
// bounded wait measures itself against.
#pragma once
#include <stdint.h>

namespace exl3b {

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

}  // namespace exl3b
