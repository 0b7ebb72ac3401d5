// Dispatch of the fragment-tile matvec over weight type, n-tiles and epilogue.
#include "launch.cuh"
#include "mma_matvec.cuh"
#include "mv_streamk.cuh"

namespace laic {

void (*mv_kernel_q4_0(int nt, int epi, bool kv32))(MvParams);
void (*mv_kernel_q8_0(int nt, int epi, bool kv32))(MvParams);
void (*mv_kernel_f16(int nt, int epi, bool kv32))(MvParams);
void (*mv_sk_kernel_q4_0(int nt, int epi, bool kv32, int warps))(MvParams);
void (*mv_sk_kernel_q8_0(int nt, int epi, bool kv32, int warps))(MvParams);
void (*mv_sk_kernel_f16(int nt, int epi, bool kv32, int warps))(MvParams);
void (*mv_wide_kernel_q4_0(int nt))(MvParams);
void (*mv_wide_kernel_q8_0(int nt))(MvParams);
void (*mv_wide_kernel_f16(int nt))(MvParams);

static void (*mv_wide_kernel(int type, int nt))(MvParams) {
    if (type == T_Q4_0) return mv_wide_kernel_q4_0(nt);
    if (type == T_Q8_0) return mv_wide_kernel_q8_0(nt);
    return mv_wide_kernel_f16(nt);
}

cudaError_t mv_wide_launch(int type, int nt, const MvParams& p, int grid, int groups, size_t smem, cudaStream_t st,
                           bool pdl) {
    return launch_k(mv_wide_kernel(type, nt), dim3(grid, groups), dim3(kMvThreads), smem, st, pdl, p);
}

static void (*mv_sk_kernel(int type, int nt, int epi, bool kv32, int warps = kSkWarps))(MvParams) {
    if (type == T_Q4_0) return mv_sk_kernel_q4_0(nt, epi, kv32, warps);
    if (type == T_Q8_0) return mv_sk_kernel_q8_0(nt, epi, kv32, warps);
    return mv_sk_kernel_f16(nt, epi, kv32, warps);
}

int sk_warps_for(int type, int nt, int nb, int rows) {
    return nt == 0 && type != T_F16 && nb >= 128 && rows >= 4096 ? kSkWarpsWide : kSkWarps;
}

cudaError_t mv_sk_launch(int type, int nt, int epi, bool kv32, const MvParams& p, int grid, size_t smem,
                         cudaStream_t st, bool pdl, int warps) {
    return launch_k(mv_sk_kernel(type, nt, epi, kv32, warps), dim3(grid), dim3(warps * 32), smem, st, pdl, p);
}

static void (*mv_kernel(int type, int nt, int epi, bool kv32))(MvParams) {
    if (type == T_Q4_0) return mv_kernel_q4_0(nt, epi, kv32);
    if (type == T_Q8_0) return mv_kernel_q8_0(nt, epi, kv32);
    return mv_kernel_f16(nt, epi, kv32);
}

cudaError_t mv_launch(int type, int nt, int epi, bool kv32, const MvParams& p, int grid, int groups, size_t smem,
                      cudaStream_t st, bool pdl) {
    return launch_k(mv_kernel(type, nt, epi, kv32), dim3(grid, groups), dim3(kMvThreads), smem, st, pdl, p);
}

cudaError_t xprep_launch(const XPrepParams& p, int nk, cudaStream_t st, bool pdl) {
    return launch_k(xprep_kernel, dim3(nk, p.nseq), dim3(kXPrepThreads), 0, st, pdl, p);
}

cudaError_t mv_set_attributes() {
    for (int type : {T_Q4_0, T_Q8_0, T_F16})
        for (int nt : {1, 2, 4, 8}) {
            cudaError_t e = cudaFuncSetAttribute(mv_wide_kernel(type, nt), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 227 * 1024);
            if (e != cudaSuccess) return e;
        }
    for (int type : {T_Q4_0, T_Q8_0, T_F16})
        for (int nt : {1, 2, 4, 8})
            for (int epi : {EPI_STORE, EPI_ADD, EPI_SWIGLU, EPI_QKV})
                for (bool kv32 : {false, true}) {
                    cudaError_t e = cudaFuncSetAttribute(mv_kernel(type, nt, epi, kv32),
                                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
                    if (e != cudaSuccess) return e;
                    if (nt <= 4) {
                        e = cudaFuncSetAttribute(mv_sk_kernel(type, nt, epi, kv32),
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
                        if (e != cudaSuccess) return e;
                    }
                    if (nt == 1 && type != T_F16)  // the integer variant (nt 0), with either warp count
                        for (int w : {kSkWarps, kSkWarpsWide}) {
                            e = cudaFuncSetAttribute(mv_sk_kernel(type, 0, epi, kv32, w),
                                                     cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
                            if (e != cudaSuccess) return e;
                        }
                }
    return cudaSuccess;
}

}  // namespace laic
