// Decode kernels of the tolerance mode (one token): the north star allows
// 1e-5 relative L2 per matvec and 1e-3 max-abs on the final logits, so sums
// are tree-reduced instead of the reference's sequential chains.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemv.cuh"

namespace nrc {

// One decode GEMV over weights resident in a model's data section (every
// matrix 16-byte aligned; reads may run up to 15 bytes past a matrix's end,
// which the data section's slack covers). Uses GemvArgs with nt == 1 and f32
// activations (xf, optional norm_w); every epilogue of GemvArgs.
cudaError_t fast_gemv_run(const GemvArgs& a, cudaStream_t stream, bool pdl);

}  // namespace nrc
