// Instantiations and launch of the persistent one-sequence decode-step kernel
// (stream_step.cuh): Q4_0 or Q8_0 projections, head_dim 64 or 128, 1 to 8 query
// heads per KV head.
#include <algorithm>

#include "launch.cuh"
#include "stream_step.cuh"

namespace laic {

using LsFn = void (*)(LsParams);

template <int WT, int D>
static LsFn ls_pick_g(int G) {
    if (G <= 1) return ls_step_kernel<WT, D, 1>;
    if (G <= 2) return ls_step_kernel<WT, D, 2>;
    if (G <= 4) return ls_step_kernel<WT, D, 4>;
    return ls_step_kernel<WT, D, 8>;
}
template <int WT>
static LsFn ls_pick_d(int D, int G) {
    return D == 64 ? ls_pick_g<WT, 64>(G) : ls_pick_g<WT, 128>(G);
}
static LsFn ls_pick(int type, int D, int G) {
    if ((type != T_Q4_0 && type != T_Q8_0) || (D != 64 && D != 128) || G < 1 || G > 8) return nullptr;
    return type == T_Q4_0 ? ls_pick_d<T_Q4_0>(D, G) : ls_pick_d<T_Q8_0>(D, G);
}

static int pow2_at_least(int g) { return g <= 1 ? 1 : g <= 2 ? 2 : g <= 4 ? 4 : 8; }

size_t ls_smem(int type, int stages, int D, int G, int nb_max, int att_runs) {
    const int GM = pow2_at_least(G);
    size_t b = (size_t)stages * kLsStage;                                   // attention ring
    b += (size_t)kLsWarps * kLsWRing * (type == T_Q4_0 ? ls_wstage(T_Q4_0) : ls_wstage(T_Q8_0));  // weight rings
    b += (size_t)(2 * kLsMaxStages + kLsWarps * kLsWRing + 2 + 2 * kLsWarps * kLsPQ) * 8;  // mbarriers
    b += (size_t)kLsWarps * kLsPQ * 16 * 4;                                 // tile pieces queues
    b += (size_t)GM * D * 4;                                                // attention: merged output
    b += (size_t)att_runs * (GM + 1) * 4;                                   // attention: merge weights, run offsets
    b += 16 + 64 + kLsWarps * 5 * 4;                                        // alignment + broadcast words + trace counters
    // alignment + activation records, or the consumer warps' attention states and weights
    b += 128 + std::max(ls_rec_bytes(nb_max), (size_t)kLsWarps * GM * (D + 3) * 4);
    return b;
}

int ls_stage_bytes() { return kLsStage; }
int ls_trace_warp_words() { return kLsWarps * 5; }
int ls_trace_stamps() { return kLsStamps; }
int ls_max_stages() { return kLsMaxStages; }
int ls_positions_per_chunk(int D) { return ls_cp(D); }
size_t ls_record_bytes(int nb) { return ls_rec_bytes(nb); }

cudaError_t ls_prepare(int type, int D, int G, size_t smem, int* blocks_per_sm) {
    auto k = ls_pick(type, D, G);
    *blocks_per_sm = 0;
    if (!k) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, k, kLsThreads, smem);
}

cudaError_t ls_launch(int type, int D, int G, const LsParams& p, int grid, size_t smem, cudaStream_t st, bool pdl) {
    auto k = ls_pick(type, D, G);
    if (!k) return cudaErrorInvalidValue;
    return launch_k(k, dim3(grid), dim3(kLsThreads), smem, st, pdl, p);
}

}  // namespace laic
