// Batched Q8_0 GEMM on the 5th-generation tensor cores (mma.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace nrc {

// Activations for the tensor-core GEMM: nt rows of K f32 values (optionally
// RMS-normalised) quantized exactly as q8::quantize, laid out per token group
// (tg) and block (b) in the UMMA K-major canonical layout:
//   xq[((tg * bpr + b) * NS + n) ...]  -> 16-byte unit (n % 8)*16 + (n / 8)*256 + c*128
//   xd[(tg * bpr + b) * NS + n]         -> f32 block scale
// Tokens n >= nt are zero.
struct MmaActArgs {
  const float* x;
  int x_ld;
  const float* norm_w;  // nullable
  float eps;
  int nt, K, NS, ntg;
  uint8_t* xq;
  float* xd;
};
cudaError_t mma_quant_act_run(const MmaActArgs& a, cudaStream_t s, bool pdl);

struct MmaSeg {
  const void* w;  // rows x K Q8_0 blocks, 16-byte aligned
  float* y;       // output of EPI_STORE: y[tok * ld + row]
  int rows;
  int ld;
};

struct MmaArgs {
  MmaSeg seg[3];  // up to three weight matrices sharing the activations (one launch)
  int nseg;
  int K;          // K % 256 == 0
  const uint8_t* xq;
  const float* xd;
  int nt, NS, ntg;
  int epi;  // EPI_STORE or EPI_RESID (gemv.cuh)
  float scale;
  float* resid;
  int resid_ld;
  float rs;
  unsigned* err;
};
cudaError_t mma_q8_run(const MmaArgs& a, cudaStream_t s, bool pdl);
// Pre-quantized Q8_0 activation blocks [nt][K/32] -> the canonical tiles above.
cudaError_t mma_pack_q8_run(const uint8_t* x, int nt, int K, int NS, int ntg, uint8_t* xq, float* xd, cudaStream_t s);
// Bytes of the canonical activation tiles and scales for nt tokens.
// K-quant GEMM (mma_kq.cu): Q4_K or Q6_K weights x Q8_K activations. The
// activations are quantize_q8k'd per token into canonical tiles of 32-value
// chunks, xq[((tg * nsb + sb) * T + tile) * NS * 32 ...] with T = 8 tiles per
// super-block, or T = 16 for Q6_K weights (masked: each chunk as two tiles
// keeping one 16-value half, the other half zero), their block scales
// xd[(tg * nsb + sb) * NS + n] and chunk sums xb[((tg * nsb + sb) * NS + n) * 8
// + chunk] (nsb = K / 256). NS is mma_kq_ns(fmt) (32 tokens).
struct MmaKqActArgs {
  const float* x;
  int x_ld;
  const float* norm_w;  // nullable
  float eps;
  int nt, K, NS, ntg;
  uint8_t* xq;
  float* xd;
  int* xb;
  int masked;  // Q6_K layout
};
cudaError_t mma_kq_act_run(const MmaKqActArgs& a, cudaStream_t s, bool pdl);
cudaError_t mma_kq_pack_run(const uint8_t* x, int nt, int K, int NS, int ntg, int masked, uint8_t* xq, float* xd,
                            int* xb, cudaStream_t s);
struct MmaKqArgs {
  int fmt;        // FMT_Q4K or FMT_Q6K
  MmaSeg seg[3];  // weights: 16-byte aligned
  int nseg;
  int K;
  const uint8_t* xq;
  const float* xd;
  const int* xb;
  int nt, NS, ntg;
  int epi;  // EPI_STORE or EPI_RESID
  float scale;
  float* resid;
  int resid_ld;
  float rs;
  unsigned* err;
};
cudaError_t mma_kq_run(const MmaKqArgs& a, cudaStream_t s, bool pdl);
int mma_kq_ns(int fmt);

inline size_t mma_xq_bytes(int nt, int K) {
  const int NS = nt <= 16 ? 16 : (nt <= 32 ? 32 : 64);
  const int ntg = (nt + NS - 1) / NS;
  return (size_t)ntg * NS * K;
}

// Token-group width used for nt tokens.
inline int mma_ns(int nt) { return nt <= 16 ? 16 : (nt <= 32 ? 32 : 64); }

// Token-group width for `tiles` 128-row weight tiles and nt <= 64 tokens:
// the widest group (fewest weight re-reads) that still launches >= 120 CTAs,
// never wider than nt needs; the narrowest (16) when none does.
inline void mma_choose(int tiles, int nt, int* ns, int* ntg) {
  for (int cand : {64, 32}) {
    const int g = (nt + cand - 1) / cand;
    if (cand <= mma_ns(nt) && g * tiles >= 120) {
      *ns = cand;
      *ntg = g;
      return;
    }
  }
  *ns = 16;
  *ntg = (nt + 15) / 16;
}

}  // namespace nrc
