// NCCL resolved at run time, and the unpack step of the tensor-parallel
// all-gathers.
#include <dlfcn.h>

#include <mutex>

#include "common.cuh"
#include "tp.cuh"

namespace nrc {

const NcclApi* nccl_api() {
  static NcclApi api{};
  static bool ok = false;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather && api.all_reduce &&
         api.error_string;
  });
  return ok ? &api : nullptr;
}

namespace {
__global__ void k_tp_unpack(const float* __restrict__ recv, float* dst, int ld, int chunk, int nt, int nranks,
                            int resid, float rs) {
  const size_t total = (size_t)nranks * nt * chunk;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % chunk);
    const int t = (int)((i / chunk) % nt);
    const int g = (int)(i / ((size_t)chunk * nt));
    float* d = dst + (size_t)t * ld + (size_t)g * chunk + c;
    *d = resid ? __fadd_rn(*d, __fmul_rn(rs, recv[i])) : recv[i];
  }
}
}  // namespace

cudaError_t tp_unpack_run(const float* recv, float* dst, int ld, int chunk, int nt, int nranks, int resid, float rs,
                          cudaStream_t s) {
  const size_t total = (size_t)nranks * nt * chunk;
  if (total == 0) return cudaSuccess;
  const int blocks = (int)((total + 255) / 256 < 1024 ? (total + 255) / 256 : 1024);
  k_tp_unpack<<<blocks, 256, 0, s>>>(recv, dst, ld, chunk, nt, nranks, resid, rs);
  return cudaGetLastError();
}

}  // namespace nrc
