// Shared device helpers for the sm_100a decode kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef __CUDACC__
#error "compile with nvcc"
#endif

namespace laic {

enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8 };
// GGML block types accepted at upload and held on the device as one of the above
enum : int { T_Q5_0 = 6 };

constexpr int kWarp = 32;

// Codes a bounded device wait writes into its launch's error word when it runs
// out (about one second of SM clocks); the host turns them into messages.
enum : int {
    kErrMbarrier = 1,     // a bulk copy into shared memory never completed (mbarrier wait)
    kErrTeamMerge = 2,    // a warp team's partial-sum slot was never released
    kErrGridBarrier = 3,  // a persistent kernel's grid barrier was not reached by every CTA
    kErrPeerFlag = 4,     // a tensor-parallel peer never published its allreduce slice
    kErrDepCounter = 5,   // a persistent kernel's dependency counter never reached its target
};

// Programmatic dependent launch: wait until the previous kernel in the stream
// has completed (and its writes are visible); let the next kernel start early.
// Both are no-ops when the launch did not use the PDL attribute.
__device__ __forceinline__ void pdl_wait() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
    asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}
__device__ __forceinline__ void pdl_launch_dependents() {
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ >= 900
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum; `red` must hold blockDim.x/32 floats. All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float s = 0.f;
    for (int i = 0; i < nw; ++i) s += red[i];
    return s;
}

// Streaming 16-byte load that skips L1 allocation (weights are read once per step).
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ unsigned short ldg_u16(const unsigned short* p) {
    unsigned short r;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ float h2f_bits(unsigned short b) { return __half2float(__ushort_as_half(b)); }

}  // namespace laic
