/*
 * nrcuda — B200 (sm_100a) implementation of NIGHTRUN's quantized transformer
 * forward path behind a C ABI.
 *
 * Every entry point returns 0 (NRC_OK) on success and a negative NRC_ERR_*
 * status otherwise; none aborts. Where the reference asserts (panics), the
 * matching entry point returns NRC_ERR_INVALID (or the code named below) and
 * leaves its outputs untouched; nrc_last_error() gives a one-line reason.
 *
 * Kernel-level entry points take DEVICE pointers and a cudaStream_t (passed as
 * void*, NULL = legacy default stream) and are asynchronous on that stream.
 * Block arrays use the reference's in-place byte layouts:
 *   Q8_0  34 B per 32 values   (crates/nr-tensor/src/q8.rs:11-14)
 *   Q4_K 144 B per 256 values  (crates/nr-tensor/src/kquant.rs:26-31)
 *   Q6_K 210 B per 256 values  (crates/nr-tensor/src/kquant.rs:37-42)
 *   Q8_K 292 B per 256 values  (crates/nr-tensor/src/kquant.rs:46-52)
 * Weight arrays of the matvec/matmul entry points need 2-byte alignment only.
 */
#ifndef NRCUDA_H
#define NRCUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NRC_OK 0
#define NRC_ERR_INVALID (-1)      /* shape/argument violation (reference: assert!) */
#define NRC_ERR_CUDA (-2)         /* a CUDA runtime call failed */
#define NRC_ERR_ALLOC (-3)        /* device memory exhausted (reference: "inference arena exhausted") */
#define NRC_ERR_DEVICE (-4)       /* a kernel reported an error (bounded wait expired) */
#define NRC_ERR_TOO_SHORT (-10)   /* ParseError::TooShort   (crates/nr-model/src/format.rs:219) */
#define NRC_ERR_BAD_MAGIC (-11)   /* ParseError::BadMagic   (format.rs:220) */
#define NRC_ERR_BAD_VERSION (-12) /* ParseError::BadVersion (format.rs:221) */
#define NRC_ERR_META_CRC (-13)    /* ParseError::MetaCrc    (format.rs:222) */
#define NRC_ERR_BAD_TABLE (-14)   /* ParseError::BadTable   (format.rs:223) */
#define NRC_ERR_MISSING (-15)     /* ParseError::MissingTensor (format.rs:224) */
#define NRC_ERR_DATA_CRC (-16)    /* Model::verify_data returned false (format.rs:410-422) */
#define NRC_ERR_UNSUPPORTED (-17) /* GGUF the converter rejects: architecture, SSM/MoE, tensor type (tools/nrconvert/src/main.rs:63-110, 246-252) */
#define NRC_ERR_CTX_FULL (-20)    /* "context window exhausted" (crates/nr-model/src/infer.rs:513, 605) */
#define NRC_ERR_BAD_BATCH (-21)   /* prefill batch outside 1..=MAX_BATCH (infer.rs:604, 754) */
#define NRC_ERR_BAD_TOKEN (-22)   /* token id >= vocab (the reference would panic on the slice) */

#define NRC_MAX_BATCH 64 /* infer.rs:101 */

/* Last error message of the calling thread ("" if none). */
const char* nrc_last_error(void);
/* Synchronize `stream` and report (then clear) any error a kernel-level entry point's kernel
 * recorded on the current device (NRC_ERR_DEVICE: a bounded wait expired). */
int nrc_sync_check(void* stream);
/* Diagnostic with no counterpart in the reference: runs one kernel whose bounded wait can never be
 * satisfied (kind 0: an mbarrier arrival withheld; kind 1: a shared-memory flag never raised) and
 * gives up after limit_ns (1 ns .. 10 s), exactly as the pipelined kernels' waits do. Returns
 * NRC_ERR_DEVICE (the expiry was recorded and reported, the error word cleared); the device and
 * every context stay usable. */
int nrc_wait_selftest(int kind, uint64_t limit_ns, void* stream);
/* Library version: major*10000 + minor*100 + patch. */
int nrc_version(void);

/* ---------------------------------------------------------------- nr-tensor */

/* q8::quantize (crates/nr-tensor/src/q8.rs:27-44): n f32 -> n/32 Q8_0 blocks. n % 32 == 0. */
int nrc_quantize_q8_0(const float* x, void* out_blocks, size_t n, void* stream);
/* q8::dequantize (q8.rs:47-55). */
int nrc_dequantize_q8_0(const void* blocks, float* out, size_t n, void* stream);
/* kquant::quantize_q8k (crates/nr-tensor/src/kquant.rs:157-187): n % 256 == 0. */
int nrc_quantize_q8k(const float* x, void* out_blocks, size_t n, void* stream);
/* kquant::dequant_q4k / dequant_q6k over nblocks blocks (kquant.rs:95-142). */
int nrc_dequant_q4k(const void* blocks, float* out, size_t nblocks, void* stream);
int nrc_dequant_q6k(const void* blocks, float* out, size_t nblocks, void* stream);

/* kernels::matvec_q8 (crates/nr-tensor/src/kernels.rs:36-47):
 * y[r] = dot(w[r,:], x), w = rows x cols Q8_0, x = cols/32 Q8_0 blocks.
 * Bit-identical to the reference's scalar dot (kernels.rs:72-82). */
int nrc_matvec_q8_0(float* y, const void* w, const void* x, size_t rows, size_t cols, void* stream);
/* kernels::matmul_q8 (kernels.rs:91-143): y is [batch][rows], xs is [batch][cols/32].
 * Like every kernel-level entry point it is asynchronous: an expired bounded wait inside its
 * kernels is reported by a later nrc_sync_check on the same stream. */
int nrc_matmul_q8_0(float* y, const void* w, const void* xs, size_t rows, size_t cols, size_t batch,
                    void* stream);
/* nrc_matmul_q8_0 that allocates nothing. No counterpart in the reference:
 * kernels::matmul_q8 (kernels.rs:91-143) needs no memory of its own on the CPU,
 * while the device version's tensor-core path stages activation tiles. This
 * variant keeps them in a static device array of NRC_NOALLOC_SCRATCH_BYTES
 * (error word, 64 tokens x NRC_NOALLOC_MAX_COLS int8 tiles, their f32
 * scales), so callers without an allocator can use it. Results are
 * bit-identical to nrc_matmul_q8_0.
 *  - cols > NRC_NOALLOC_MAX_COLS is rejected with NRC_ERR_INVALID.
 *  - Only the error word must start at zero; every call clears it itself.
 *  - The first call on a device resolves the array's address
 *    (cudaGetSymbolAddress) and sets kernel attributes.
 *  - Every call blocks the host until its kernels have finished (it reads the
 *    error word back and synchronizes `stream`), so it must never be made while
 *    `stream` is being captured into a CUDA graph.
 *  - Calls overlapping in time on one device (several streams or threads)
 *    race on the array: serialize them. */
#define NRC_NOALLOC_MAX_COLS 16384
#define NRC_NOALLOC_SCRATCH_BYTES (256 + 64 * NRC_NOALLOC_MAX_COLS + 64 * (NRC_NOALLOC_MAX_COLS / 32) * 4)
int nrc_matmul_q8_0_noalloc(float* y, const void* w, const void* xs, size_t rows, size_t cols, size_t batch,
                            void* stream);
/* kquant::matvec_q4k / matvec_q6k (kquant.rs:536-564), Q8_K activations;
 * bit-identical to dot_q4k_scalar / dot_q6k_scalar (kquant.rs:192-250). */
int nrc_matvec_q4k(float* y, const void* w, const void* x, size_t rows, size_t cols, void* stream);
int nrc_matvec_q6k(float* y, const void* w, const void* x, size_t rows, size_t cols, void* stream);
/* kquant::matmul_q4k / matmul_q6k (kquant.rs:566-639). */
int nrc_matmul_q4k(float* y, const void* w, const void* xs, size_t rows, size_t cols, size_t batch,
                   void* stream);
int nrc_matmul_q6k(float* y, const void* w, const void* xs, size_t rows, size_t cols, size_t batch,
                   void* stream);

/* f16::f32_to_f16 / f16_to_f32 (crates/nr-tensor/src/f16.rs:3-56), elementwise. */
int nrc_f32_to_f16(const float* x, uint16_t* out, size_t n, void* stream);
int nrc_f16_to_f32(const uint16_t* x, float* out, size_t n, void* stream);
/* vec::rmsnorm (crates/nr-tensor/src/vec.rs:4-14) over `rows` independent rows of n. */
int nrc_rmsnorm(float* out, const float* x, const float* w, size_t n, size_t rows, float eps, void* stream);
/* vec::softmax (vec.rs:30-41) over `rows` independent rows of n, in place. */
int nrc_softmax(float* x, size_t n, size_t rows, void* stream);
/* vec::swiglu (vec.rs:44-50): gate[i] = silu(gate[i]) * up[i]. */
int nrc_swiglu(float* gate, const float* up, size_t n, void* stream);
/* The expf of vec::softmax / vec::swiglu (vec.rs:34, 47; crate libm 0.2.16), elementwise. This
 * library evaluates a correctly rounded binary32 exp (the test oracle evaluates the same one). */
int nrc_expf(const float* x, float* y, size_t n, void* stream);
/* Test support: hash of nrc_expf's output bits over every binary32 input, one 64-bit value per
 * chunk of 2^20 consecutive bit patterns, chunks [chunk0, chunk0 + nchunks) of 4096. */
int nrc_expf_hash(uint64_t* out_dev, int chunk0, int nchunks, void* stream);
/* vec::argmax (vec.rs:80-90): first maximum; writes the index to *out_dev (uint32, device). */
int nrc_argmax(const float* x, size_t n, uint32_t* out_dev, void* stream);
/* Sampler::sample (crates/nr-model/src/sample.rs:32-96) over n device logits (n <= 262144):
 * temperature <= 0 is vec::argmax; otherwise the top-64 prefilter (the reference's min-heap,
 * replayed exactly when logits tie at its boundary), softmax with temperature in descending
 * order, the top_p nucleus cut and one xorshift64 draw from *rng_dev (device uint64, the
 * Sampler's state: seed | 1 at Sampler::new, advanced once per draw). Candidates with equal
 * logits are ordered by ascending index (the reference's sort_unstable_by leaves that order
 * unspecified). Writes the token id to *out_dev (uint32, device). */
int nrc_sample(const float* logits, size_t n, float temperature, float top_p, uint64_t* rng_dev, uint32_t* out_dev,
               void* stream);
/* rope::rope_freqs (crates/nr-tensor/src/rope.rs:14-34), computed on the host into out_host
 * (head_dim/2 values); factor <= 0 disables the Llama-3 scaling. */
int nrc_rope_freqs(float* out_host, size_t head_dim, float theta, float factor, float low_freq_factor,
                   float high_freq_factor, float original_context);
/* rope::apply (rope.rs:49-65) for one position: x holds len/head_dim heads; style 0 = Adjacent,
 * 1 = Neox. freqs_host are the head_dim/2 frequencies. */
int nrc_rope_apply(float* x, size_t len, size_t head_dim, const float* freqs_host, size_t pos, int style,
                   void* stream);

/* ----------------------------------------------------------------- nr-model */

typedef struct nrc_model nrc_model;
typedef struct nrc_ctx nrc_ctx;

/* Header metadata (crates/nr-model/src/format.rs:127-156). */
typedef struct nrc_meta {
  int32_t arch; /* 1 Llama3, 2 Qwen3, 3 Granite */
  uint32_t dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, ctx_train;
  float rope_theta, norm_eps, rope_factor, rope_low, rope_high, rope_orig_ctx;
  uint32_t flags;
  float embed_scale, attn_scale, residual_scale, logit_scale;
  char name[48];
} nrc_meta;

/* Synthetic-model recipe (deterministic; identical bytes to the CPU generator of the tests). */
typedef struct nrc_synth_cfg {
  uint32_t arch, dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, ctx_train;
  float rope_theta, norm_eps, rope_factor, rope_low, rope_high, rope_orig_ctx;
  float embed_scale, attn_scale, residual_scale, logit_scale;
  uint32_t quant; /* 0: all Q8_0; 1: Q4_K_M-style Q4_K/Q6_K mix */
  uint32_t tied;
  uint32_t rope_freqs_tensor;
  char name[48];
} nrc_synth_cfg;

/* Model::parse (format.rs:260-406) of a host .nrm blob, then one upload of its data section to
 * `device`. verify_crc != 0 also checks data_crc (Model::verify_data, format.rs:410-422). The blob
 * may be freed after the call. */
int nrc_model_load(const uint8_t* blob, size_t len, int device, int verify_crc, nrc_model** out);
/* GGUF ingestion (tools/nrconvert/src/gguf.rs; main.rs:180-453): a GGUF v2/v3 file of a dense
 * llama / qwen3 / granite model with F32 / Q8_0 / Q4_K / Q6_K tensors as a .nrm v3 blob: the
 * converter's tensor order, 64-byte alignment, header fields and CRCs, with the tokenizer section
 * left empty. out == NULL: only *out_len is set. Conditions the converter panics or exits on
 * return NRC_ERR_TOO_SHORT / BAD_MAGIC / BAD_VERSION / MISSING / UNSUPPORTED. */
int nrc_gguf_to_nrm(const uint8_t* gguf, size_t len, uint8_t* out, size_t out_cap, size_t* out_len);
/* nrc_gguf_to_nrm, then nrc_model_load (data CRC verified) of the result. */
int nrc_model_load_gguf(const uint8_t* gguf, size_t len, int device, nrc_model** out);
/* Build a seeded synthetic model directly in device memory (no host copy of the weights). */
int nrc_model_synth(const nrc_synth_cfg* cfg, uint64_t seed, int device, nrc_model** out);
int nrc_model_meta(const nrc_model* m, nrc_meta* out);
/* Size of, and export to, a complete .nrm blob (header, empty tokenizer, table, data). */
size_t nrc_model_nrm_size(const nrc_model* m);
int nrc_model_export(const nrc_model* m, uint8_t* out, size_t cap);
/* CRC-32 of the device-resident data section (checks an upload or a synthetic build). */
int nrc_model_data_crc(const nrc_model* m, uint32_t* out);
int nrc_model_free(nrc_model* m);

/* InferCtx::required_bytes (crates/nr-model/src/infer.rs:334-350): device bytes of KV cache and
 * scratch for a context of ctx positions. */
int nrc_ctx_required_bytes(const nrc_model* m, size_t ctx, size_t* out);
/* InferCtx::new (infer.rs:352-492): binds the weights (shape-checked), builds the RoPE tables and
 * allocates the device arena (KV cache f16 [layer][ctx][kv_dim], activations). The context owns
 * one CUDA stream. */
int nrc_ctx_new(const nrc_model* m, size_t ctx, nrc_ctx** out);
int nrc_ctx_free(nrc_ctx* c);
/* InferCtx::forward (infer.rs:510-595): one token at the current position; copies the logits to
 * logits_host (vocab floats) when it is not NULL, and the greedy choice (vec::argmax, i.e.
 * Sampler with temperature 0, crates/nr-model/src/sample.rs:33-35) to *next_host when not NULL. */
int nrc_ctx_forward(nrc_ctx* c, uint32_t token, float* logits_host, uint32_t* next_host);
/* InferCtx::prefill_chunk (infer.rs:601-750): 1..=64 tokens; last token's logits. */
int nrc_ctx_prefill_chunk(nrc_ctx* c, const uint32_t* tokens_host, size_t n, float* logits_host,
                          uint32_t* next_host);
/* InferCtx::prefill (infer.rs:753-759): any length, in chunks of 64. */
int nrc_ctx_prefill(nrc_ctx* c, const uint32_t* tokens_host, size_t n, float* logits_host,
                    uint32_t* next_host);
/* Greedy generation of n tokens after `first` entirely on the device (one CUDA-graph replay per
 * token); writes the n generated ids. Equivalent to n x (forward + argmax). */
int nrc_ctx_generate(nrc_ctx* c, uint32_t first, size_t n, uint32_t* out_host);
/* Enqueue n greedy decode steps on the context's stream without waiting: each step consumes the
 * token the previous step chose (on the device). Needs a prior forward/prefill. Pair with
 * nrc_ctx_sync, which waits, advances pos and returns the last chosen token. */
int nrc_ctx_decode_async(nrc_ctx* c, size_t n);
int nrc_ctx_sync(nrc_ctx* c, uint32_t* next_host);
/* Decode arithmetic of a context. NRC_MODE_EXACT (default): every sum in the reference's order,
 * logits and KV cache bit-identical to its scalar path. NRC_MODE_FAST: single-token decode steps
 * add the RMSNorm sum of squares and the attention softmax and V sums as trees (block dots, their
 * roundings, the activation quantization and the matvec row sums are unchanged). A reordered sum
 * can move an activation quant by one step, so logits drift from the scalar path about as far as
 * the reference's own AVX2 path drifts (its x86 kernels reorder sums too). Prefill chunks stay
 * exact. The reference's counterpart is the choice between its scalar and AVX2 kernels
 * (crates/nr-tensor/src/kernels.rs:227-286). */
#define NRC_MODE_EXACT 0
#define NRC_MODE_FAST 1
int nrc_ctx_set_mode(nrc_ctx* c, int mode);
/* Sampler::new(temperature, top_p, seed) (sample.rs:15-21) attached to the context: from now on
 * every step that chooses a next token draws once with it (each forward, each prefill_chunk, the
 * last chunk of a prefill, every generated / decode_async step), on the device. temperature <= 0
 * restores greedy argmax. The logits the steps return are unchanged. */
int nrc_ctx_set_sampler(nrc_ctx* c, float temperature, float top_p, uint64_t seed);
int nrc_ctx_reset(nrc_ctx* c);              /* infer.rs:494-496 */
size_t nrc_ctx_pos(const nrc_ctx* c);       /* InferCtx::pos */
size_t nrc_ctx_remaining(const nrc_ctx* c); /* infer.rs:504-506 */
/* Device pointer to the most recent logits (infer.rs:499-501). */
int nrc_ctx_logits_device(const nrc_ctx* c, const float** out);
/* The context's CUDA stream (cudaStream_t). */
void* nrc_ctx_stream(const nrc_ctx* c);
/* Copy the f16 K and V cache rows of (layer, pos) to the host (kv_dim values each). */
int nrc_ctx_kv(nrc_ctx* c, size_t layer, size_t pos, uint16_t* k_host, uint16_t* v_host);

/* ---------------------------------------------------- tensor parallelism over NCCL */
/* One sequence over nranks GPUs, one process (or thread) per GPU. Each rank computes whole output
 * rows with the full K: its KV-head groups of wq / wk / wv and attention, equal row ranges of wo,
 * ffn_gate / ffn_up, ffn_down and the classifier; the activations the next layer needs whole
 * (attention output, residual stream, SwiGLU output, logits) are all-gathered and the greedy key
 * all-reduced (max). No partial sums cross ranks, so logits and tokens are bit-identical to one
 * GPU (the reference's residual adds, crates/nr-model/src/infer.rs:574-575 and :582-583, stay
 * single roundings). The model must be loaded on each rank's device; NCCL is resolved at run time
 * (libnccl.so.2). n_kv_heads, dim, ffn_dim and vocab must divide by nranks.
 * nrc_tp_unique_id (on one rank) creates the NCCL id (128 bytes) every rank passes to
 * nrc_tp_ctx_new; the single-sequence entry points then drive the context on every rank in the
 * same order (they block until their collectives finish). nrc_ctx_kv returns this rank's KV heads. */
int nrc_tp_unique_id(uint8_t* id_out128);
int nrc_tp_ctx_new(const nrc_model* m, size_t ctx, int nranks, int rank, const uint8_t* id128, nrc_ctx** out);
/* This rank's shard: {nranks, rank, q head0, q heads, kv head0, kv heads, dim row0, dim rows,
 * ffn row0, ffn rows, vocab row0, vocab rows}. */
int nrc_tp_shard(const nrc_ctx* c, int32_t* out12);

/* ---------------------------------------------------- several sequences (batched streams) */
/* A context of n_seqs independent sequences decoded together: the reference runs one InferCtx
 * per stream (crates/nr-model/src/infer.rs:319-778); here each sequence has its own KV cache and
 * position and every linear layer runs once per pass over all sequences' tokens. Per sequence,
 * logits and tokens are bit-identical to a single-sequence context. Greedy choice only; the
 * single-sequence entry points (nrc_ctx_forward, ...) reject such a context, nrc_ctx_reset /
 * nrc_ctx_free / nrc_ctx_stream apply. */
int nrc_batch_new(const nrc_model* m, size_t ctx, size_t n_seqs, nrc_ctx** out);
/* InferCtx::prefill (infer.rs:753-759) of every sequence: prompts back to back in tokens_host,
 * lens_host[s] >= 1 tokens for sequence s; several sequences share each pass of up to
 * max(64, n_seqs) tokens. next_host (optional, n_seqs ids) receives each greedy choice. */
int nrc_batch_prefill(nrc_ctx* c, const uint32_t* tokens_host, const uint32_t* lens_host, uint32_t* next_host);
/* One decode step of every sequence (InferCtx::forward, infer.rs:510-595), each consuming the token
 * it chose last; logits_host (optional) receives [n_seqs][vocab], next_host (optional) [n_seqs]. */
int nrc_batch_step(nrc_ctx* c, float* logits_host, uint32_t* next_host);
/* n decode steps of every sequence on the device (graph replays); out_host[s * n + i] receives
 * sequence s's choice after step i. */
int nrc_batch_generate(nrc_ctx* c, size_t n, uint32_t* out_host);
/* Enqueue n decode steps without waiting; nrc_batch_sync waits and returns the last choices. */
int nrc_batch_decode_async(nrc_ctx* c, size_t n);
int nrc_batch_sync(nrc_ctx* c, uint32_t* next_host);
size_t nrc_batch_size(const nrc_ctx* c);
size_t nrc_batch_pos(const nrc_ctx* c, size_t seq);
/* Copy sequence seq's f16 K and V cache rows of (layer, pos) to the host. */
int nrc_batch_kv(nrc_ctx* c, size_t seq, size_t layer, size_t pos, uint16_t* k_host, uint16_t* v_host);

#ifdef __cplusplus
}
#endif
#endif /* NRCUDA_H */
