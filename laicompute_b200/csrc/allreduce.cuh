// One-shot allreduce of the residual over the tensor-parallel ranks through
// peer memory (NVLink), for the small messages of decode (nseq x hidden floats).
//
// Every rank owns a mailbox in its own HBM, mapped into the other ranks (CUDA
// IPC): two buffers (alternating calls) of [ranks][n] floats plus one flag per
// (buffer, source rank, CTA). CTA c of rank r owns the slice c of the vector:
//   1. it stores its slice into slot r of every rank's mailbox (plain stores
//      through NVLink), fences at system scope and sets its flag in every
//      rank's mailbox to the call's epoch;
//   2. it waits (bounded) until the flags of slice c from all ranks carry the
//      epoch in its own mailbox, then adds the slots in rank order (the same
//      order on every rank, so the ranks get bit-identical sums).
// A call's epoch comes from a per-rank device counter that the last CTA
// advances, so a captured graph replays correctly. Two buffers suffice: a rank
// can only start call k+2 after every rank finished writing call k+1, which
// they do after finishing call k.
#pragma once
#include "common.cuh"

namespace laic {

constexpr int kArMaxRanks = 8;
constexpr int kArCtas = 32;      // slices (CTAs) per call
constexpr int kArThreads = 256;

struct ArParams {
    float* x;                       // [n] in/out (the residual)
    int n;
    int rank, ranks;
    float* box[kArMaxRanks];        // every rank's mailbox data: [2][ranks][nmax]
    unsigned* flags[kArMaxRanks];   // every rank's mailbox flags: [2][ranks][kArCtas]
    int nmax;
    unsigned* epoch;                // this rank's call counter
    unsigned* done;                 // this rank's finished-CTA counter (zero between calls)
    int* err;                       // set when a wait runs out
    long long spin_limit;           // clock cycles a flag wait may take (0: about one second)
};

__global__ void __launch_bounds__(kArThreads) allreduce_oneshot_kernel(const ArParams p) {
    pdl_wait();
    __shared__ unsigned ep_s;
    if (threadIdx.x == 0) ep_s = *reinterpret_cast<volatile unsigned*>(p.epoch) + 1u;  // this call's epoch
    __syncthreads();
    const unsigned ep = ep_s;
    const int buf = ep & 1u;
    const int c = blockIdx.x;
    const int per = (p.n + gridDim.x - 1) / gridDim.x;
    const int lo = c * per, hi = min(p.n, lo + per);

    // 1. this rank's slice into slot `rank` of every mailbox
    for (int r = 0; r < p.ranks; ++r) {
        float* dst = p.box[r] + ((size_t)buf * p.ranks + p.rank) * p.nmax;
        for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = p.x[i];
    }
    __syncthreads();
    if (threadIdx.x < p.ranks) {
        __threadfence_system();
        unsigned* f = p.flags[threadIdx.x] + ((size_t)buf * p.ranks + p.rank) * kArCtas + c;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(ep) : "memory");
    }
    // 2. wait for every rank's slice in this mailbox, then add in rank order
    if (threadIdx.x < p.ranks) {
        const unsigned* f = p.flags[p.rank] + ((size_t)buf * p.ranks + threadIdx.x) * kArCtas + c;
        const long long t0 = clock64();
        const long long spin = p.spin_limit > 0 ? p.spin_limit : 2000000000LL;
        unsigned v;
        while (true) {
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
            if (v == ep) break;
            if (clock64() - t0 > spin) { atomicExch(p.err, kErrPeerFlag); break; }
        }
    }
    __syncthreads();
    const float* mine = p.box[p.rank] + (size_t)buf * p.ranks * p.nmax;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        float s = 0.f;
        for (int r = 0; r < p.ranks; ++r) s += __ldcv(mine + (size_t)r * p.nmax + i);
        p.x[i] = s;
    }
    pdl_launch_dependents();
    // the last CTA advances the epoch for the next call
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.done, 1u) == gridDim.x - 1) {
            *p.done = 0u;
            __threadfence();
            *reinterpret_cast<volatile unsigned*>(p.epoch) = ep;
        }
    }
}

}  // namespace laic
