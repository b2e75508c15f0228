// TEST INFRASTRUCTURE ONLY — data types of the nr-model restatement
// (crates/nr-model/src/format.rs:14-234, infer.rs:18-320, sample.rs:5-21).
#pragma once
#include <vector>

#include "oracle.h"

namespace oracle {

constexpr size_t HEADER_SIZE = 192;  // format.rs:16
constexpr size_t NAME_LEN = 48;      // format.rs:17
constexpr size_t ENTRY_SIZE = 32;    // format.rs:18
constexpr size_t DATA_ALIGN = 64;    // format.rs:19
constexpr uint32_t FLAG_TIED_EMBEDDINGS = 1;
constexpr int MAX_BATCH = 64;  // infer.rs:101

enum { ARCH_LLAMA3 = 1, ARCH_QWEN3 = 2, ARCH_GRANITE = 3 };  // format.rs:25-29
enum { DT_F32 = 0, DT_Q8_0 = 1, DT_Q4K = 2, DT_Q6K = 3 };     // format.rs:97-102
enum {                                                        // format.rs:53-69
  TK_TOK_EMBED = 1,
  TK_OUTPUT_NORM = 2,
  TK_OUTPUT = 3,
  TK_ROPE_FREQS = 4,
  TK_ATTN_NORM = 10,
  TK_ATTN_Q = 11,
  TK_ATTN_K = 12,
  TK_ATTN_V = 13,
  TK_ATTN_O = 14,
  TK_FFN_NORM = 15,
  TK_FFN_GATE = 16,
  TK_FFN_UP = 17,
  TK_FFN_DOWN = 18,
  TK_ATTN_Q_NORM = 19,
  TK_ATTN_K_NORM = 20,
};
// ParseError (format.rs:218-225) plus the assert!s of infer.rs, as codes.
enum {
  PE_OK = 0,
  PE_TOO_SHORT = -1,
  PE_BAD_MAGIC = -2,
  PE_BAD_VERSION = -3,
  PE_META_CRC = -4,
  PE_BAD_TABLE = -5,
  PE_MISSING = -6,
  PE_CTX_FULL = -20,
  PE_BAD_BATCH = -21,
  PE_BAD_TOKEN = -22,
};

struct Meta {  // format.rs:127-156
  int arch;
  uint32_t dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, ctx_train;
  float rope_theta, norm_eps, rope_factor, rope_low, rope_high, rope_orig_ctx;
  uint32_t flags;
  float embed_scale, attn_scale, residual_scale, logit_scale;
  char name[NAME_LEN];
};

struct TensorEntry {  // format.rs:166-175
  uint16_t kind, layer, dtype;
  uint64_t offset, size;
  uint32_t rows, cols;
};

struct Model {  // format.rs:227-234
  Meta meta;
  std::vector<TensorEntry> entries;
  const uint8_t* blob = nullptr;
  size_t blob_len = 0;
  const uint8_t* data = nullptr;
  uint64_t data_size = 0;
  uint32_t data_crc = 0;
  uint64_t tok_off = 0, tok_size = 0;
};

bool dtype_byte_size(int dtype, uint64_t n, uint64_t* out);
int model_parse(const uint8_t* blob, size_t len, Model* m);
bool model_verify_data(const Model* m);
const TensorEntry* model_tensor(const Model* m, int kind, int layer);
bool model_has_tensor(const Model* m, int kind);

struct QMat {  // infer.rs:20-24
  int dtype;
  const void* p;
};

struct Dims {  // infer.rs:61-73
  size_t dim, att_dim, n_layers, n_heads, n_kv_heads, head_dim, kv_dim, ffn_dim, vocab, ctx;
};

struct LayerW {  // infer.rs:75-88
  const float* attn_norm;
  const float* q_norm;
  const float* k_norm;
  QMat wq, wk, wv, wo;
  const float* ffn_norm;
  QMat w_gate, w_up, w_down;
};

struct Ctx {  // infer.rs:264-301
  Dims dims;
  QMat embed, output;
  std::vector<LayerW> layers;
  const float* out_norm;
  float norm_eps;
  int rope_style;
  float embed_scale, att_score_scale, residual_scale, logit_recip;
  std::vector<float> freqs, x, xb, xb2, q, attn_out, k, v, att, gate, up, logits;
  std::vector<BlockQ8_0> q8;
  std::vector<BlockQ8K> q8k;
  std::vector<float> bx, bxb, bq, battn, bk, bv, bgate, bup;
  std::vector<uint16_t> key_cache, val_cache;
  size_t pos;
};

int ctx_new(const Model* m, size_t ctx, Ctx* c);
int ctx_forward(Ctx* c, uint32_t token);
int ctx_prefill_chunk(Ctx* c, const uint32_t* tokens, size_t b);
int ctx_prefill(Ctx* c, const uint32_t* tokens, size_t n);

struct Sampler {  // sample.rs:5-21
  float temperature, top_p;
  uint64_t rng;
};
uint32_t sampler_sample(Sampler* s, const float* logits, size_t n);

}  // namespace oracle
