// Token sampling on the device: Sampler::sample (crates/nr-model/src/sample.rs:32-96).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace nrc {

constexpr int SAMPLE_TOPK = 64;            // sample.rs:12 TOP_K
constexpr int SAMPLE_CHUNK = 1024;         // logits per CTA of the candidate pass
constexpr int SAMPLE_MAX_N = 1 << 18;      // largest vocabulary (candidates merged in one CTA)

struct SampleArgs {
  const float* logits;  // [n]
  int n;
  float temperature, top_p;
  unsigned long long* rng;      // xorshift64 state (Sampler::rng), advanced by one draw
  unsigned long long* cand;     // scratch: sample_scratch_bytes(n)
  uint32_t* out_idx;            // chosen token (or null)
  unsigned long long* out_key;  // or the chosen token as an argmax key (argmax_index(key) == token)
};

size_t sample_scratch_bytes(int n);
// temperature > 0 only (the greedy case is vec::argmax, fused elsewhere).
cudaError_t sample_run(const SampleArgs& a, cudaStream_t s, bool pdl);

}  // namespace nrc
