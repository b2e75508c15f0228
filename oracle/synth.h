// TEST INFRASTRUCTURE ONLY — synthetic model recipe (see synth.cpp).
#pragma once
#include <vector>

#include "oracle.h"

namespace oracle {

// Layout shared with the ctypes wrapper (oracle/oracle.py) and with the
// product's nrc_synth_cfg (include/nrcuda.h); 4-byte fields only.
struct SynthCfg {
  uint32_t arch, dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, ctx_train;
  float rope_theta, norm_eps, rope_factor, rope_low, rope_high, rope_orig_ctx;
  float embed_scale, attn_scale, residual_scale, logit_scale;
  uint32_t quant;              // 0: every linear weight Q8_0; 1: Q4_K_M-style Q4_K/Q6_K mix
  uint32_t tied;               // 1: output shares token_embd (FLAG_TIED_EMBEDDINGS)
  uint32_t rope_freqs_tensor;  // 1: write a rope_freqs factor tensor
  char name[48];
};

struct SynthTensor {
  uint16_t kind, layer, dtype;
  uint32_t rows, cols;
  uint64_t offset, size;
};

float synth_gauss(uint64_t key, uint64_t idx);
void synth_tensor_list(const SynthCfg& cfg, std::vector<SynthTensor>& out);
uint64_t synth_nrm_size(const SynthCfg& cfg);
int synth_nrm_write(const SynthCfg& cfg, uint64_t seed, uint8_t* out, uint64_t cap, int threads);

}  // namespace oracle
