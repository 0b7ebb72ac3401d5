// Instantiations of the fragment-tile matvec for one weight type.
#include "launch.cuh"
#include "mma_matvec.cuh"
#include "mv_streamk.cuh"

namespace laic {

template <int NT>
static void (*pick_q4_0(int epi, bool kv32))(MvParams) {
    switch (epi) {
    case EPI_STORE: return mv_mma_kernel<T_Q4_0, NT, EPI_STORE, __half>;
    case EPI_ADD: return mv_mma_kernel<T_Q4_0, NT, EPI_ADD, __half>;
    case EPI_SWIGLU: return mv_mma_kernel<T_Q4_0, NT, EPI_SWIGLU, __half>;
    default: return kv32 ? mv_mma_kernel<T_Q4_0, NT, EPI_QKV, float> : mv_mma_kernel<T_Q4_0, NT, EPI_QKV, __half>;
    }
}

void (*mv_kernel_q4_0(int nt, int epi, bool kv32))(MvParams) {
    switch (nt) {
    case 1: return pick_q4_0<1>(epi, kv32);
    case 2: return pick_q4_0<2>(epi, kv32);
    case 4: return pick_q4_0<4>(epi, kv32);
    default: return pick_q4_0<8>(epi, kv32);
    }
}

template <int NT, int W = kSkWarps>
static void (*pick_sk_q4_0(int epi, bool kv32))(MvParams) {
    switch (epi) {
    case EPI_STORE: return mv_sk_kernel<T_Q4_0, NT, EPI_STORE, __half, W>;
    case EPI_ADD: return mv_sk_kernel<T_Q4_0, NT, EPI_ADD, __half, W>;
    case EPI_SWIGLU: return mv_sk_kernel<T_Q4_0, NT, EPI_SWIGLU, __half, W>;
    default: return kv32 ? mv_sk_kernel<T_Q4_0, NT, EPI_QKV, float, W> : mv_sk_kernel<T_Q4_0, NT, EPI_QKV, __half, W>;
    }
}

void (*mv_sk_kernel_q4_0(int nt, int epi, bool kv32, int warps))(MvParams) {
    // nt 0: the single-sequence integer variant (also with kSkWarpsWide warps)
    if (nt == 0 && warps == kSkWarpsWide) return pick_sk_q4_0<0, kSkWarpsWide>(epi, kv32);
    return nt == 0 ? pick_sk_q4_0<0>(epi, kv32) : nt == 1 ? pick_sk_q4_0<1>(epi, kv32)
         : nt == 2 ? pick_sk_q4_0<2>(epi, kv32) : pick_sk_q4_0<4>(epi, kv32);
}

void (*mv_wide_kernel_q4_0(int nt))(MvParams) {
    switch (nt) {
    case 1: return mv_wide_kernel<T_Q4_0, 1>;
    case 2: return mv_wide_kernel<T_Q4_0, 2>;
    case 4: return mv_wide_kernel<T_Q4_0, 4>;
    default: return mv_wide_kernel<T_Q4_0, 8>;
    }
}

}  // namespace laic
