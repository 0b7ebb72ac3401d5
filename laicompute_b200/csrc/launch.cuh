// Host-side launch helper: cudaLaunchKernelEx with optional programmatic
// dependent launch (the kernel may start while its predecessor drains; it
// orders itself with griddepcontrol.wait before touching dependent data).
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace laic {

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                     Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same with a thread-block cluster of (cluster_x, 1, 1) CTAs.
template <typename... KArgs, typename... Args>
cudaError_t launch_cluster_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                             int cluster_x, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cluster_x;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

struct MvParams;
struct XPrepParams;
// Launch the activation preparation of the tile kernel: grid (nk, nseq).
cudaError_t xprep_launch(const XPrepParams& p, int nk, cudaStream_t st, bool pdl);
// Launch the fragment-tile matvec for one weight type (defined in mv_<type>.cu).
cudaError_t mv_launch(int type, int nt, int epi, bool kv32, const MvParams& p, int grid, int groups, size_t smem,
                      cudaStream_t st, bool pdl);
// Launch the wide matvec (EPI_STORE; each warp owns whole row tiles), grid (grid, groups).
cudaError_t mv_wide_launch(int type, int nt, const MvParams& p, int grid, int groups, size_t smem, cudaStream_t st,
                           bool pdl);
// Launch the team matvec (defined in mv_<type>.cu), nt = 1, 2 or 4; nt = 0 is the one-sequence integer
// variant, which runs with `warps` = kSkWarps or kSkWarpsWide warps per CTA (sk_warps_for).
cudaError_t mv_sk_launch(int type, int nt, int epi, bool kv32, const MvParams& p, int grid, size_t smem,
                         cudaStream_t st, bool pdl, int warps);
// Warps per CTA of a team-matvec launch: kSkWarpsWide for one sequence of a Q4_0/Q8_0 matrix with at
// least 128 blocks per row and 4096 rows, else kSkWarps.
int sk_warps_for(int type, int nt, int nb, int rows);
// Raise the dynamic shared memory limit of every instantiation (call before any graph capture).
cudaError_t mv_set_attributes();

// Batched prefill GEMM (gemm_sm100.cu): C[M][N] fp32 = A[M][K] fp16 x W[N][K]^T fp16.
size_t gemm_f16_workspace(int M, int N, int K);
cudaError_t gemm_f16(int M, int N, int K, const void* A, const void* W, float* C, void* workspace, size_t ws_bytes,
                     cudaStream_t st);

struct LsParams;
// Persistent one-sequence decode-step kernel (stream_step.cu): shared memory for an attention
// ring of `stages` stages, the consumer warps' weight rings and activation records of nb_max blocks, its layout constants, attribute
// setup with the resulting CTAs per SM (call before capture), and its launch (one CTA per SM).
size_t ls_smem(int type, int stages, int D, int G, int nb_max, int att_runs);
int ls_stage_bytes();
int ls_trace_stamps();
int ls_trace_warp_words();  // trace words per CTA after the phase stamps
int ls_max_stages();
int ls_positions_per_chunk(int D);
size_t ls_record_bytes(int nb);  // activation records of a vector of nb blocks
cudaError_t ls_prepare(int type, int D, int G, size_t smem, int* blocks_per_sm);
cudaError_t ls_launch(int type, int D, int G, const LsParams& p, int grid, size_t smem, cudaStream_t st, bool pdl);

}  // namespace laic
