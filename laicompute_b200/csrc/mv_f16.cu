// Instantiations of the fragment-tile matvec for one weight type.
#include "launch.cuh"
#include "mma_matvec.cuh"
#include "mv_streamk.cuh"

namespace laic {

template <int NT>
static void (*pick_f16(int epi, bool kv32))(MvParams) {
    switch (epi) {
    case EPI_STORE: return mv_mma_kernel<T_F16, NT, EPI_STORE, __half>;
    case EPI_ADD: return mv_mma_kernel<T_F16, NT, EPI_ADD, __half>;
    case EPI_SWIGLU: return mv_mma_kernel<T_F16, NT, EPI_SWIGLU, __half>;
    default: return kv32 ? mv_mma_kernel<T_F16, NT, EPI_QKV, float> : mv_mma_kernel<T_F16, NT, EPI_QKV, __half>;
    }
}

void (*mv_kernel_f16(int nt, int epi, bool kv32))(MvParams) {
    switch (nt) {
    case 1: return pick_f16<1>(epi, kv32);
    case 2: return pick_f16<2>(epi, kv32);
    case 4: return pick_f16<4>(epi, kv32);
    default: return pick_f16<8>(epi, kv32);
    }
}

template <int NT>
static void (*pick_sk_f16(int epi, bool kv32))(MvParams) {
    switch (epi) {
    case EPI_STORE: return mv_sk_kernel<T_F16, NT, EPI_STORE, __half>;
    case EPI_ADD: return mv_sk_kernel<T_F16, NT, EPI_ADD, __half>;
    case EPI_SWIGLU: return mv_sk_kernel<T_F16, NT, EPI_SWIGLU, __half>;
    default: return kv32 ? mv_sk_kernel<T_F16, NT, EPI_QKV, float> : mv_sk_kernel<T_F16, NT, EPI_QKV, __half>;
    }
}

void (*mv_sk_kernel_f16(int nt, int epi, bool kv32, int /*warps: F16 runs kSkWarps*/))(MvParams) {
    return nt == 1 ? pick_sk_f16<1>(epi, kv32) : nt == 2 ? pick_sk_f16<2>(epi, kv32) : pick_sk_f16<4>(epi, kv32);
}

void (*mv_wide_kernel_f16(int nt))(MvParams) {
    switch (nt) {
    case 1: return mv_wide_kernel<T_F16, 1>;
    case 2: return mv_wide_kernel<T_F16, 2>;
    case 4: return mv_wide_kernel<T_F16, 4>;
    default: return mv_wide_kernel<T_F16, 8>;
    }
}

}  // namespace laic
