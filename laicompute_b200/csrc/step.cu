// Instantiations and cooperative launch of the one-sequence decode-step kernel.
#include "launch.cuh"
#include "step_kernel.cuh"

namespace laic {

template <int WT, int D>
static void (*step_pick_g(int G))(StepParams) {
    if (G <= 1) return step_kernel<WT, D, 1>;
    if (G <= 2) return step_kernel<WT, D, 2>;
    if (G <= 4) return step_kernel<WT, D, 4>;
    return step_kernel<WT, D, 8>;
}
template <int WT>
static void (*step_pick_d(int D, int G))(StepParams) {
    return D == 64 ? step_pick_g<WT, 64>(G) : step_pick_g<WT, 128>(G);
}
static void (*step_pick(int type, int D, int G))(StepParams) {
    if ((type != T_Q4_0 && type != T_Q8_0) || (D != 64 && D != 128) || G < 1 || G > 8) return nullptr;
    return type == T_Q4_0 ? step_pick_d<T_Q4_0>(D, G) : step_pick_d<T_Q8_0>(D, G);
}

size_t step_smem(int type, int nb_max, int D) { return step_smem_bytes(type, nb_max, D); }

cudaError_t step_prepare(int type, int D, int G, size_t smem, int* blocks_per_sm) {
    auto k = step_pick(type, D, G);
    *blocks_per_sm = 0;
    if (!k) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, k, kSkWarps * 32, smem);
}

cudaError_t step_launch(int type, int D, int G, const StepParams& p, int grid, size_t smem, cudaStream_t st) {
    auto k = step_pick(type, D, G);
    if (!k) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kSkWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid barriers rely on it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, p);
}

}  // namespace laic
