// Host launchers of the element kernels (ops.cu) and the attention kernels (attn.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace nrc {

cudaError_t op_quantize_q8_0(const float* x, void* out, size_t n, cudaStream_t s);
cudaError_t op_dequantize_q8_0(const void* b, float* out, size_t n, cudaStream_t s);
cudaError_t op_quantize_q8k(const float* x, void* out, size_t n, cudaStream_t s);
cudaError_t op_dequant_q4k(const void* b, float* out, size_t nblocks, cudaStream_t s);
cudaError_t op_dequant_q6k(const void* b, float* out, size_t nblocks, cudaStream_t s);
cudaError_t op_f32_to_f16(const float* x, uint16_t* o, size_t n, cudaStream_t s);
cudaError_t op_f16_to_f32(const uint16_t* x, float* o, size_t n, cudaStream_t s);
cudaError_t op_rmsnorm(float* out, const float* x, const float* w, size_t n, size_t rows, float eps,
                       cudaStream_t s);
cudaError_t op_softmax(float* x, size_t n, size_t rows, cudaStream_t s);
cudaError_t op_swiglu(float* g, const float* u, size_t n, cudaStream_t s);
cudaError_t op_argmax(const float* x, size_t n, unsigned long long* key_scratch, uint32_t* out, cudaStream_t s);
cudaError_t op_expf(const float* x, float* y, size_t n, cudaStream_t s);
cudaError_t op_wait_selftest(unsigned* err, unsigned long long limit_ns, int kind, cudaStream_t s);
cudaError_t op_expf_hash(unsigned long long* out, int chunk0, int nchunks, cudaStream_t s);

// Position-dependent kernels of the forward pass. Positions are read from
// device memory (pos_dev[0] + token index) so a captured CUDA graph replays
// unchanged for every decode step.
struct RopeArgs {
  float* q;        // [nt][att_dim], rotated in place
  const float* k;  // [nt][kv_dim]
  const float* v;  // [nt][kv_dim]
  const float* q_norm;  // per-head RMSNorm weights (Qwen3) or null
  const float* k_norm;
  float eps;
  const float* cos_tab;  // [ctx][head_dim/2]
  const float* sin_tab;
  int style;  // 0 Adjacent, 1 Neox
  uint16_t* kcache;  // this layer's [ctx][kv_dim] (sequence 0)
  uint16_t* vcache;
  int nt, n_heads, n_kv_heads, head_dim, ctx;
  const uint32_t* pos_dev;
  // Several sequences in one pass: token t sits at position pos_tok[t] of
  // sequence seq_tok[t], whose cache starts seq_stride elements after
  // sequence 0's. Null pos_tok: positions pos_dev[0] + t of sequence 0.
  const uint32_t* pos_tok;
  const uint32_t* seq_tok;
  size_t seq_stride;
  // Fused decode only: the output also as Q8_0 blocks (q8::quantize, q8.rs:
  // 27-44), the next projection's input, or null.
  uint8_t* xq_out;
};
cudaError_t rope_append_run(const RopeArgs& a, cudaStream_t s, bool pdl);

struct AttnArgs {
  float* q;           // [nt][att_dim]: rotated by rope_append, or raw when fused
  float* out;         // [nt][att_dim]
  uint16_t* kcache;   // this layer's [ctx][kv_dim]
  uint16_t* vcache;
  float scale;
  int nt, n_heads, n_kv_heads, head_dim, ctx;
  const uint32_t* pos_dev;
  // Decode (nt == 1) with the per-head norms, RoPE and the KV append fused in
  // (then q, k, v are the raw projections of the token).
  int fused;
  const float* k;
  const float* v;
  const float* q_norm;
  const float* k_norm;
  float eps;
  const float* cos_tab;
  const float* sin_tab;
  int style;
  // Several sequences (RopeArgs: pos_tok, seq_tok, seq_stride); null pos_tok
  // = positions pos_dev[0] + t of sequence 0. Not with `fused`.
  const uint32_t* pos_tok;
  const uint32_t* seq_tok;
  size_t seq_stride;
  // Fused decode only: the output also as Q8_0 blocks (q8::quantize, q8.rs:
  // 27-44), the next projection's input, or null.
  uint8_t* xq_out;
};
// Shared memory of one attention CTA (its score rows hold `ctx` positions);
// contexts needing more than ATTN_MAX_SMEM are rejected at context creation.
constexpr size_t ATTN_MAX_SMEM = 200 * 1024;
size_t attention_smem_bytes(int n_heads, int n_kv_heads, int head_dim, int ctx, int nt);
// fast: the tolerance mode's tree-reduced variant (same inputs and outputs).
cudaError_t attention_run(const AttnArgs& a, cudaStream_t s, bool pdl, bool fast = false);

// Embedding rows (QMat::dequant_row, infer.rs:37-56) times embed_scale for nt
// tokens read from tok_dev; also clears the greedy-argmax key.
struct EmbedArgs {
  const uint8_t* embed;
  int fmt, dim;
  float embed_scale;
  const uint32_t* tok_dev;
  int nt;
  float* x;  // [nt][dim]
  unsigned long long* argmax_key;
};
// Multi-sequence passes: gather the classifier rows of x; then each row's
// greedy argmax and its sequence's bookkeeping (next token, next input,
// position after the row's token, history [seq][ctx]).
cudaError_t gather_rows_run(const float* x, int dim, const uint32_t* rows, int nrows, float* out, cudaStream_t s,
                            bool pdl);
cudaError_t rows_argmax_run(const float* logits, int vocab, int nrows, const uint32_t* rows, const uint32_t* seq,
                            const uint32_t* pos, uint32_t* bpos, uint32_t* btok, uint32_t* bnext, uint32_t* bhist,
                            int ctx, cudaStream_t s, bool pdl);
cudaError_t embed_run(const EmbedArgs& a, cudaStream_t s, bool pdl);

// Decode the argmax key into next_tok (and tok_in[0], the next step's input),
// record it in hist[pos], then advance the device position by n.
cudaError_t step_finish_run(uint32_t* pos_dev, uint32_t n, const unsigned long long* key, uint32_t* next_tok,
                            uint32_t* tok_in, uint32_t* hist, cudaStream_t s, bool pdl);

}  // namespace nrc
