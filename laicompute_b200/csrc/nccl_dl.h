// NCCL entry points resolved at run time (dlopen of libnccl.so.2).
//
// The engine needs NCCL only for tensor parallelism (tp_size > 1), so the
// library does not link against it: a process that already loaded NCCL (for
// example through torch.distributed) shares that copy, and a single-GPU
// process never loads it. The declarations mirror nccl.h for the handful of
// calls used here (types are ABI-stable across NCCL 2.x).
#pragma once
#include <string>

struct CUstream_st;  // cudaStream_t is CUstream_st*

namespace laic {

typedef struct ncclComm* ncclComm_t;
struct ncclUniqueId { char internal[128]; };
enum ncclResult_t : int { ncclSuccess = 0 };
enum ncclDataType_t : int { ncclFloat32 = 7 };
enum ncclRedOp_t : int { ncclSum = 0 };

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              CUstream_st*) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, CUstream_st*) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

// The resolved API, or nullptr with `why` set when NCCL cannot be loaded.
const NcclApi* nccl_api(std::string& why);

}  // namespace laic
