// Streaming quantized GEMV / small-batch GEMM (host interface).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace nrc {

// Epilogues fused into the GEMV.
enum GemvEpi {
  EPI_STORE = 0,   // y[t*ld + r] = s * scale            (scale_inplace when scale != 1)
  EPI_RESID = 1,   // resid[t*ld + r] += rs * s          (vec::saxpy, vec.rs:68-72)
  EPI_SWIGLU = 2,  // seg0 = gate, seg1 = up: y = silu(gate) * up   (vec::swiglu, vec.rs:44-50)
  EPI_ARGMAX = 3,  // EPI_STORE + running argmax key of token 0 (vec::argmax, vec.rs:80-90)
};

struct GemvSegArg {
  const void* w;  // rows x K weight blocks of `fmt`
  float* y;       // output base (EPI_STORE / EPI_ARGMAX / EPI_SWIGLU on seg 0)
  int rows;
  int ld;  // output row stride between tokens
};

struct GemvArgs {
  int fmt;  // FMT_Q8_0 / FMT_Q4K / FMT_Q6K
  int K;    // columns
  int nt;   // tokens (1..8)
  GemvSegArg seg[3];
  int nseg;
  int pair;  // 1: seg0/seg1 are gate/up of the same rows (EPI_SWIGLU)
  // Activations: either pre-quantized blocks (Q8_0 for FMT_Q8_0, Q8_K otherwise),
  // [nt][K/blk], or f32 [nt][xf_ld] quantized in the prologue (after an
  // optional RMSNorm with norm_w/eps).
  const void* xq;
  const float* xf;
  int xf_ld;
  // With xf: CTA 0 also stores the quantized activations here as blocks
  // (Q8_0 34 B, or Q8_K 292 B whose bsums hold each 32-value sum in the even
  // slot), so a following launch over other weights of the same input takes
  // them as xq instead of normalizing and quantizing again.
  void* xq_out;
  // EPI_SWIGLU: also store silu(gate) * up as Q8_0 blocks [nt][rows / 32] (the
  // down projection's activations, quantized once) when one warp of the launch
  // forms each 32-row block; gemv_run sets *yq_done to 1 when it does, else 0.
  uint8_t* yq_out;
  int* yq_done;
  const float* norm_w;
  float eps;
  int fast_norm;  // tolerance mode: the RMSNorm sum of squares as a tree (not the reference's chain)
  int epi;
  float scale;
  float* resid;
  int resid_ld;
  float rs;
  unsigned long long* argmax_key;  // one key (token 0)
  int argmax_base;                 // index of row 0 in the argmax key (a vocabulary shard's first row)
  unsigned* err;                   // device error word
  // Optional L2 prefetch of the weights the next kernel will stream (a hint:
  // results do not depend on it). Every CTA prefetches its share once its
  // own first ring of stages is in flight.
  const void* pf;
  size_t pf_bytes;
};

// Launch on `stream`; `pdl` enables programmatic dependent launch.
cudaError_t gemv_run(const GemvArgs& a, cudaStream_t stream, bool pdl);

}  // namespace nrc
