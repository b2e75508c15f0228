// Device-side synthetic weight generation (synth.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

namespace nrc {

uint64_t synth_tensor_key(uint64_t seed, uint32_t kind, uint32_t layer);
// Fill one tensor (rows x cols of `dtype`: 0 F32, 1 Q8_0, 2 Q4_K, 3 Q6_K) at dst.
cudaError_t synth_fill(uint8_t* dst, int dtype, uint32_t kind, uint64_t rows, uint64_t cols, uint64_t key,
                       cudaStream_t s);

}  // namespace nrc
