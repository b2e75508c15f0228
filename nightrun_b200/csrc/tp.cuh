// Tensor parallelism over NCCL: the library resolves NCCL at run time (the
// libnccl.so.2 already loaded by the process, e.g. by PyTorch, else the
// system one), so it links no NCCL and single-GPU use never needs it.
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>
#include <stdint.h>

namespace nrc {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  const char* (*error_string)(ncclResult_t);
};
// The resolved API, or null when no libnccl.so.2 can be loaded.
const NcclApi* nccl_api();

// After an all-gather of `chunk` values per token per rank (recv holds
// [rank][nt][chunk]): dst[t * ld + g * chunk + i] = recv[g][t][i] (resid == 0)
// or dst[...] += rs * recv[g][t][i] (resid != 0, vec::saxpy: the same two
// roundings as the single-GPU residual add).
cudaError_t tp_unpack_run(const float* recv, float* dst, int ld, int chunk, int nt, int nranks, int resid, float rs,
                          cudaStream_t s);

}  // namespace nrc
