// TEST INFRASTRUCTURE ONLY — restatement of crates/nr-model/src/{format,infer,sample}.rs.
// See oracle.h for the pinning status. Every function cites the reference
// lines it follows.
#include <math.h>

#include <vector>

#include "model.h"
#include "expf_cr.h"

namespace oracle {

// ----------------------------------------------------------- format.rs:236-257
namespace {
struct Cursor {
  const uint8_t* b;
  size_t p;
  uint16_t u16() { uint16_t v; memcpy(&v, b + p, 2); p += 2; return v; }
  uint32_t u32() { uint32_t v; memcpy(&v, b + p, 4); p += 4; return v; }
  uint64_t u64() { uint64_t v; memcpy(&v, b + p, 8); p += 8; return v; }
  float f32() { return bits_f32(u32()); }
};
}  // namespace

// ------------------------------------------------------------ format.rs:104-124
bool dtype_byte_size(int dtype, uint64_t n, uint64_t* out) {
  switch (dtype) {
    case DT_F32:
      if (n > UINT64_MAX / 4) return false;
      *out = n * 4;
      return true;
    case DT_Q8_0:
      if (n % 32) return false;
      if (n / 32 > UINT64_MAX / 34) return false;
      *out = n / 32 * 34;
      return true;
    case DT_Q4K:
      if (n % 256) return false;
      if (n / 256 > UINT64_MAX / 144) return false;
      *out = n / 256 * 144;
      return true;
    case DT_Q6K:
      if (n % 256) return false;
      if (n / 256 > UINT64_MAX / 210) return false;
      *out = n / 256 * 210;
      return true;
  }
  return false;
}

// ------------------------------------------------------------ format.rs:260-406
int model_parse(const uint8_t* blob, size_t len, Model* m) {
  if (len < HEADER_SIZE) return PE_TOO_SHORT;
  if (memcmp(blob, "NRUN", 4) != 0) return PE_BAD_MAGIC;
  Cursor c{blob, 4};
  uint32_t version = c.u32();
  if (version != 3) return PE_BAD_VERSION;
  uint32_t arch = c.u32();
  if (arch < 1 || arch > 3) return PE_BAD_TABLE;
  Meta& mt = m->meta;
  mt.arch = (int)arch;
  mt.dim = c.u32();
  mt.n_layers = c.u32();
  mt.n_heads = c.u32();
  mt.n_kv_heads = c.u32();
  mt.head_dim = c.u32();
  mt.ffn_dim = c.u32();
  mt.vocab = c.u32();
  mt.ctx_train = c.u32();
  mt.rope_theta = c.f32();
  mt.norm_eps = c.f32();
  mt.rope_factor = c.f32();
  mt.rope_low = c.f32();
  mt.rope_high = c.f32();
  mt.rope_orig_ctx = c.f32();
  mt.flags = c.u32();
  mt.embed_scale = c.f32();
  mt.attn_scale = c.f32();
  mt.residual_scale = c.f32();
  mt.logit_scale = c.f32();
  memcpy(mt.name, blob + c.p, NAME_LEN);
  c.p += NAME_LEN;
  uint64_t tok_off = c.u64(), tok_size = c.u64(), table_off = c.u64();
  uint64_t tensor_count = c.u32();
  (void)c.u32();
  uint64_t data_off = c.u64(), data_size = c.u64();
  uint32_t data_crc = c.u32();
  uint32_t meta_crc = c.u32();
  if (!isfinite(mt.embed_scale) || !isfinite(mt.attn_scale) || mt.attn_scale < 0.0f ||
      !isfinite(mt.residual_scale) || mt.residual_scale <= 0.0f || !isfinite(mt.logit_scale) ||
      mt.logit_scale <= 0.0f)
    return PE_BAD_TABLE;
  uint64_t table_len;
  if (__builtin_mul_overflow(tensor_count, (uint64_t)ENTRY_SIZE, &table_len)) return PE_BAD_TABLE;
  uint64_t table_end, data_end, tok_end;
  if (__builtin_add_overflow(table_off, table_len, &table_end)) return PE_TOO_SHORT;
  if (__builtin_add_overflow(data_off, data_size, &data_end)) return PE_TOO_SHORT;
  if (__builtin_add_overflow(tok_off, tok_size, &tok_end)) return PE_TOO_SHORT;
  if (len < table_end || len < data_end || len < tok_end) return PE_TOO_SHORT;
  uint32_t crc = 0xffffffffu;
  crc = crc32_update(crc, blob, HEADER_SIZE - 8);
  const uint8_t zeros[8] = {0};
  crc = crc32_update(crc, zeros, 8);
  crc = crc32_update(crc, blob + tok_off, tok_size);
  crc = crc32_update(crc, blob + table_off, table_len);
  if ((crc ^ 0xffffffffu) != meta_crc) return PE_META_CRC;
  m->entries.clear();
  Cursor tc{blob, table_off};
  for (uint64_t i = 0; i < tensor_count; i++) {
    TensorEntry e;
    e.kind = tc.u16();
    e.layer = tc.u16();
    uint16_t dt = tc.u16();
    if (dt > 3) return PE_BAD_TABLE;
    e.dtype = dt;
    (void)tc.u16();
    e.offset = tc.u64();
    e.size = tc.u64();
    e.rows = tc.u32();
    e.cols = tc.u32();
    uint64_t end;
    if (__builtin_add_overflow(e.offset, e.size, &end)) return PE_BAD_TABLE;
    if (end > data_size) return PE_BAD_TABLE;
    if (e.offset % DATA_ALIGN != 0) return PE_BAD_TABLE;
    uint64_t n = (uint64_t)e.rows * (uint64_t)e.cols;
    uint64_t bs;
    if (!dtype_byte_size(e.dtype, n, &bs) || bs != e.size) return PE_BAD_TABLE;
    m->entries.push_back(e);
  }
  m->blob = blob;
  m->blob_len = len;
  m->data = blob + data_off;
  m->data_size = data_size;
  m->data_crc = data_crc;
  m->tok_off = tok_off;
  m->tok_size = tok_size;
  return PE_OK;
}

// ------------------------------------------------------------ format.rs:410-422
bool model_verify_data(const Model* m) {
  return crc32(m->data, m->data_size) == m->data_crc;
}

// ------------------------------------------------------------ format.rs:424-439
const TensorEntry* model_tensor(const Model* m, int kind, int layer) {
  for (const auto& e : m->entries)
    if (e.kind == kind && e.layer == layer) return &e;
  return nullptr;
}
bool model_has_tensor(const Model* m, int kind) {
  for (const auto& e : m->entries)
    if (e.kind == kind) return true;
  return false;
}

// -------------------------------------------------- infer.rs:37-56 (QMat::dequant_row)
static void dequant_row(const QMat& w, size_t r, size_t cols, float* out) {
  if (w.dtype == DT_Q8_0) {
    size_t bpr = cols / QK8_0;
    q8_dequantize((const BlockQ8_0*)w.p + r * bpr, cols, out);
  } else if (w.dtype == DT_Q4K) {
    size_t bpr = cols / QK_K;
    for (size_t i = 0; i < bpr; i++) dequant_q4k((const BlockQ4K*)w.p + r * bpr + i, out + i * QK_K);
  } else {
    size_t bpr = cols / QK_K;
    for (size_t i = 0; i < bpr; i++) dequant_q6k((const BlockQ6K*)w.p + r * bpr + i, out + i * QK_K);
  }
}

// ------------------------------------------------------ infer.rs:110-262 (Acts)
static void acts_matvec(Ctx* c, float* y, size_t rows, QMat w, const float* x, size_t cols) {
  if (w.dtype == DT_Q8_0) {
    q8_quantize(x, cols, c->q8.data());
    matvec_q8(y, (const BlockQ8_0*)w.p, c->q8.data(), rows, cols);
  } else if (w.dtype == DT_Q4K) {
    quantize_q8k(x, cols, c->q8k.data());
    matvec_q4k(y, (const BlockQ4K*)w.p, c->q8k.data(), rows, cols);
  } else {
    quantize_q8k(x, cols, c->q8k.data());
    matvec_q6k(y, (const BlockQ6K*)w.p, c->q8k.data(), rows, cols);
  }
}

static void acts_matmul(Ctx* c, float* y, size_t rows, QMat w, const float* xs, size_t cols,
                        size_t batch) {
  if (w.dtype == DT_Q8_0) {
    size_t bpr = cols / QK8_0;
    for (size_t b = 0; b < batch; b++) q8_quantize(xs + b * cols, cols, c->q8.data() + b * bpr);
    matmul_q8(y, (const BlockQ8_0*)w.p, c->q8.data(), rows, cols, batch);
  } else {
    size_t bpr = cols / QK_K;
    for (size_t b = 0; b < batch; b++) quantize_q8k(xs + b * cols, cols, c->q8k.data() + b * bpr);
    if (w.dtype == DT_Q4K)
      matmul_q4k(y, (const BlockQ4K*)w.p, c->q8k.data(), rows, cols, batch);
    else
      matmul_q6k(y, (const BlockQ6K*)w.p, c->q8k.data(), rows, cols, batch);
  }
}

struct Job {
  float* y;
  size_t rows;
  QMat w;
};

static void acts_matmul_group(Ctx* c, Job* jobs, int n, const float* xs, size_t cols, size_t batch) {
  bool q8_ready = false, q8k_ready = false;
  for (int i = 0; i < n; i++) {
    QMat w = jobs[i].w;
    if (w.dtype == DT_Q8_0) {
      size_t bpr = cols / QK8_0;
      if (!q8_ready) {
        for (size_t b = 0; b < batch; b++) q8_quantize(xs + b * cols, cols, c->q8.data() + b * bpr);
        q8_ready = true;
      }
      matmul_q8(jobs[i].y, (const BlockQ8_0*)w.p, c->q8.data(), jobs[i].rows, cols, batch);
    } else {
      size_t bpr = cols / QK_K;
      if (!q8k_ready) {
        for (size_t b = 0; b < batch; b++) quantize_q8k(xs + b * cols, cols, c->q8k.data() + b * bpr);
        q8k_ready = true;
      }
      if (w.dtype == DT_Q4K)
        matmul_q4k(jobs[i].y, (const BlockQ4K*)w.p, c->q8k.data(), jobs[i].rows, cols, batch);
      else
        matmul_q6k(jobs[i].y, (const BlockQ6K*)w.p, c->q8k.data(), jobs[i].rows, cols, batch);
    }
  }
}

static void acts_matvec_group(Ctx* c, Job* jobs, int n, const float* x, size_t cols) {
  bool q8_ready = false, q8k_ready = false;
  for (int i = 0; i < n; i++) {
    QMat w = jobs[i].w;
    if (w.dtype == DT_Q8_0) {
      if (!q8_ready) {
        q8_quantize(x, cols, c->q8.data());
        q8_ready = true;
      }
      matvec_q8(jobs[i].y, (const BlockQ8_0*)w.p, c->q8.data(), jobs[i].rows, cols);
    } else {
      if (!q8k_ready) {
        quantize_q8k(x, cols, c->q8k.data());
        q8k_ready = true;
      }
      if (w.dtype == DT_Q4K)
        matvec_q4k(jobs[i].y, (const BlockQ4K*)w.p, c->q8k.data(), jobs[i].rows, cols);
      else
        matvec_q6k(jobs[i].y, (const BlockQ6K*)w.p, c->q8k.data(), jobs[i].rows, cols);
    }
  }
}

// ------------------------------------------------------------ infer.rs:352-492
int ctx_new(const Model* m, size_t ctx, Ctx* c) {
  const Meta& mt = m->meta;
  Dims& d = c->dims;
  d.dim = mt.dim;
  d.att_dim = (size_t)mt.n_heads * mt.head_dim;
  d.n_layers = mt.n_layers;
  d.n_heads = mt.n_heads;
  d.n_kv_heads = mt.n_kv_heads;
  d.head_dim = mt.head_dim;
  d.kv_dim = (size_t)mt.n_kv_heads * mt.head_dim;
  d.ffn_dim = mt.ffn_dim;
  d.vocab = mt.vocab;
  d.ctx = ctx;
  auto f32t = [&](int kind, int layer, size_t n, const float** out) -> int {
    const TensorEntry* e = model_tensor(m, kind, layer);
    if (!e) return PE_MISSING;
    if (e->dtype != DT_F32 || (size_t)e->rows * e->cols != n) return PE_MISSING;
    *out = (const float*)(m->data + e->offset);
    return PE_OK;
  };
  auto mat = [&](int kind, int layer, size_t rows, size_t cols, QMat* out) -> int {
    const TensorEntry* e = model_tensor(m, kind, layer);
    if (!e) return PE_MISSING;
    if (e->rows != rows || e->cols != cols) return PE_MISSING;
    if (e->dtype == DT_F32) return PE_BAD_TABLE;
    out->dtype = e->dtype;
    out->p = m->data + e->offset;
    return PE_OK;
  };
  int rc;
  if ((rc = mat(TK_TOK_EMBED, 0, d.vocab, d.dim, &c->embed))) return rc;
  bool is_qwen = mt.arch == ARCH_QWEN3;
  if (!is_qwen && model_has_tensor(m, TK_ATTN_Q_NORM)) return PE_MISSING;
  c->layers.resize(d.n_layers);
  for (size_t l = 0; l < d.n_layers; l++) {
    LayerW& w = c->layers[l];
    if ((rc = f32t(TK_ATTN_NORM, (int)l, d.dim, &w.attn_norm))) return rc;
    w.q_norm = w.k_norm = nullptr;
    if (is_qwen) {
      if ((rc = f32t(TK_ATTN_Q_NORM, (int)l, d.head_dim, &w.q_norm))) return rc;
      if ((rc = f32t(TK_ATTN_K_NORM, (int)l, d.head_dim, &w.k_norm))) return rc;
    }
    if ((rc = mat(TK_ATTN_Q, (int)l, d.att_dim, d.dim, &w.wq))) return rc;
    if ((rc = mat(TK_ATTN_K, (int)l, d.kv_dim, d.dim, &w.wk))) return rc;
    if ((rc = mat(TK_ATTN_V, (int)l, d.kv_dim, d.dim, &w.wv))) return rc;
    if ((rc = mat(TK_ATTN_O, (int)l, d.dim, d.att_dim, &w.wo))) return rc;
    if ((rc = f32t(TK_FFN_NORM, (int)l, d.dim, &w.ffn_norm))) return rc;
    if ((rc = mat(TK_FFN_GATE, (int)l, d.ffn_dim, d.dim, &w.w_gate))) return rc;
    if ((rc = mat(TK_FFN_UP, (int)l, d.ffn_dim, d.dim, &w.w_up))) return rc;
    if ((rc = mat(TK_FFN_DOWN, (int)l, d.dim, d.ffn_dim, &w.w_down))) return rc;
  }
  if ((rc = f32t(TK_OUTPUT_NORM, 0, d.dim, &c->out_norm))) return rc;
  if (mt.flags & FLAG_TIED_EMBEDDINGS)
    c->output = c->embed;
  else if ((rc = mat(TK_OUTPUT, 0, d.vocab, d.dim, &c->output)))
    return rc;
  // Rope frequencies (infer.rs:427-445).
  c->freqs.assign(d.head_dim / 2, 0.0f);
  Llama3Scaling sc{mt.rope_factor, mt.rope_low, mt.rope_high, mt.rope_orig_ctx};
  if (model_has_tensor(m, TK_ROPE_FREQS)) {
    rope_freqs(c->freqs.data(), d.head_dim, mt.rope_theta, nullptr);
    const TensorEntry* e = model_tensor(m, TK_ROPE_FREQS, 0);
    const float* factors = (const float*)(m->data + e->offset);
    size_t nf = (size_t)e->rows * e->cols;
    for (size_t i = 0; i < c->freqs.size() && i < nf; i++) c->freqs[i] /= factors[i];
  } else {
    rope_freqs(c->freqs.data(), d.head_dim, mt.rope_theta, mt.rope_factor > 0.0f ? &sc : nullptr);
  }
  c->norm_eps = mt.norm_eps;
  c->rope_style = (mt.arch == ARCH_QWEN3) ? ROPE_NEOX : ROPE_ADJACENT;
  c->embed_scale = mt.embed_scale;
  c->att_score_scale = mt.attn_scale != 0.0f ? mt.attn_scale : 1.0f / sqrtf((float)mt.head_dim);
  c->residual_scale = mt.residual_scale;
  c->logit_recip = 1.0f / mt.logit_scale;
  size_t maxd = d.dim;
  if (d.att_dim > maxd) maxd = d.att_dim;
  if (d.ffn_dim > maxd) maxd = d.ffn_dim;
  c->x.assign(d.dim, 0);
  c->xb.assign(d.dim, 0);
  c->xb2.assign(d.dim, 0);
  c->q.assign(d.att_dim, 0);
  c->attn_out.assign(d.att_dim, 0);
  c->k.assign(d.kv_dim, 0);
  c->v.assign(d.kv_dim, 0);
  c->att.assign(d.n_heads * ctx, 0);
  c->gate.assign(d.ffn_dim, 0);
  c->up.assign(d.ffn_dim, 0);
  c->logits.assign(d.vocab, 0);
  c->q8.assign(MAX_BATCH * (maxd / QK8_0), BlockQ8_0{});
  c->q8k.assign(MAX_BATCH * (maxd / QK_K) + 1, BlockQ8K{});
  size_t dmax = d.dim > d.att_dim ? d.dim : d.att_dim;
  c->bx.assign(MAX_BATCH * d.dim, 0);
  c->bxb.assign(MAX_BATCH * dmax, 0);
  c->bq.assign(MAX_BATCH * d.att_dim, 0);
  c->battn.assign(MAX_BATCH * d.att_dim, 0);
  c->bk.assign(MAX_BATCH * d.kv_dim, 0);
  c->bv.assign(MAX_BATCH * d.kv_dim, 0);
  c->bgate.assign(MAX_BATCH * d.ffn_dim, 0);
  c->bup.assign(MAX_BATCH * d.ffn_dim, 0);
  c->key_cache.assign(d.n_layers * ctx * d.kv_dim, 0);
  c->val_cache.assign(d.n_layers * ctx * d.kv_dim, 0);
  c->pos = 0;
  return PE_OK;
}

// GQA attention for one query vector at position `pos` (infer.rs:553-572 and 661-685).
static void attend(Ctx* c, size_t l, const float* q, float* out, size_t pos) {
  const Dims& d = c->dims;
  size_t gqa = d.n_heads / d.n_kv_heads;
  float scale = c->att_score_scale;
  for (size_t h = 0; h < d.n_heads; h++) {
    const float* qh = q + h * d.head_dim;
    size_t kvh = (h / gqa) * d.head_dim;
    float* att = c->att.data() + h * d.ctx;
    for (size_t t = 0; t <= pos; t++) {
      size_t krow = (l * d.ctx + t) * d.kv_dim + kvh;
      att[t] = dot_f16(c->key_cache.data() + krow, qh, d.head_dim) * scale;
    }
    softmax(att, pos + 1);
    float* o = out + h * d.head_dim;
    for (size_t i = 0; i < d.head_dim; i++) o[i] = 0.0f;
    for (size_t t = 0; t <= pos; t++) {
      size_t vrow = (l * d.ctx + t) * d.kv_dim + kvh;
      axpy_f16(o, att[t], c->val_cache.data() + vrow, d.head_dim);
    }
  }
}

// ------------------------------------------------------------ infer.rs:510-595
int ctx_forward(Ctx* c, uint32_t token) {
  const Dims& d = c->dims;
  size_t pos = c->pos;
  if (pos >= d.ctx) return PE_CTX_FULL;
  if (token >= d.vocab) return PE_BAD_TOKEN;
  dequant_row(c->embed, token, d.dim, c->x.data());
  if (c->embed_scale != 1.0f) scale_inplace(c->x.data(), d.dim, c->embed_scale);
  for (size_t l = 0; l < d.n_layers; l++) {
    const LayerW& w = c->layers[l];
    rmsnorm(c->xb.data(), c->x.data(), w.attn_norm, d.dim, c->norm_eps);
    Job qkv[3] = {{c->q.data(), d.att_dim, w.wq}, {c->k.data(), d.kv_dim, w.wk}, {c->v.data(), d.kv_dim, w.wv}};
    acts_matvec_group(c, qkv, 3, c->xb.data(), d.dim);
    if (w.q_norm && w.k_norm) {
      for (size_t h = 0; h < d.n_heads; h++) rmsnorm_inplace(c->q.data() + h * d.head_dim, w.q_norm, d.head_dim, c->norm_eps);
      for (size_t h = 0; h < d.n_kv_heads; h++) rmsnorm_inplace(c->k.data() + h * d.head_dim, w.k_norm, d.head_dim, c->norm_eps);
    }
    rope_apply(c->q.data(), d.att_dim, d.head_dim, c->freqs.data(), pos, c->rope_style);
    rope_apply(c->k.data(), d.kv_dim, d.head_dim, c->freqs.data(), pos, c->rope_style);
    size_t cache_row = (l * d.ctx + pos) * d.kv_dim;
    for (size_t i = 0; i < d.kv_dim; i++) {
      c->key_cache[cache_row + i] = f32_to_f16(c->k[i]);
      c->val_cache[cache_row + i] = f32_to_f16(c->v[i]);
    }
    attend(c, l, c->q.data(), c->attn_out.data(), pos);
    acts_matvec(c, c->xb2.data(), d.dim, w.wo, c->attn_out.data(), d.att_dim);
    saxpy(c->x.data(), c->residual_scale, c->xb2.data(), d.dim);
    rmsnorm(c->xb.data(), c->x.data(), w.ffn_norm, d.dim, c->norm_eps);
    Job gu[2] = {{c->gate.data(), d.ffn_dim, w.w_gate}, {c->up.data(), d.ffn_dim, w.w_up}};
    acts_matvec_group(c, gu, 2, c->xb.data(), d.dim);
    swiglu(c->gate.data(), c->up.data(), d.ffn_dim);
    acts_matvec(c, c->xb2.data(), d.dim, w.w_down, c->gate.data(), d.ffn_dim);
    saxpy(c->x.data(), c->residual_scale, c->xb2.data(), d.dim);
  }
  rmsnorm(c->xb.data(), c->x.data(), c->out_norm, d.dim, c->norm_eps);
  acts_matvec(c, c->logits.data(), d.vocab, c->output, c->xb.data(), d.dim);
  if (c->logit_recip != 1.0f) scale_inplace(c->logits.data(), d.vocab, c->logit_recip);
  c->pos += 1;
  return PE_OK;
}

// ------------------------------------------------------------ infer.rs:597-750
int ctx_prefill_chunk(Ctx* c, const uint32_t* tokens, size_t b) {
  const Dims& d = c->dims;
  if (b < 1 || b > MAX_BATCH) return PE_BAD_BATCH;
  if (c->pos + b > d.ctx) return PE_CTX_FULL;
  for (size_t i = 0; i < b; i++)
    if (tokens[i] >= d.vocab) return PE_BAD_TOKEN;
  size_t base = c->pos;
  for (size_t i = 0; i < b; i++) {
    float* row = c->bx.data() + i * d.dim;
    dequant_row(c->embed, tokens[i], d.dim, row);
    if (c->embed_scale != 1.0f) scale_inplace(row, d.dim, c->embed_scale);
  }
  for (size_t l = 0; l < d.n_layers; l++) {
    const LayerW& w = c->layers[l];
    for (size_t i = 0; i < b; i++)
      rmsnorm(c->bxb.data() + i * d.dim, c->bx.data() + i * d.dim, w.attn_norm, d.dim, c->norm_eps);
    Job qkv[3] = {{c->bq.data(), d.att_dim, w.wq}, {c->bk.data(), d.kv_dim, w.wk}, {c->bv.data(), d.kv_dim, w.wv}};
    acts_matmul_group(c, qkv, 3, c->bxb.data(), d.dim, b);
    for (size_t i = 0; i < b; i++) {
      size_t pos = base + i;
      float* q = c->bq.data() + i * d.att_dim;
      float* k = c->bk.data() + i * d.kv_dim;
      if (w.q_norm && w.k_norm) {
        for (size_t h = 0; h < d.n_heads; h++) rmsnorm_inplace(q + h * d.head_dim, w.q_norm, d.head_dim, c->norm_eps);
        for (size_t h = 0; h < d.n_kv_heads; h++) rmsnorm_inplace(k + h * d.head_dim, w.k_norm, d.head_dim, c->norm_eps);
      }
      rope_apply(q, d.att_dim, d.head_dim, c->freqs.data(), pos, c->rope_style);
      rope_apply(k, d.kv_dim, d.head_dim, c->freqs.data(), pos, c->rope_style);
      size_t cache_row = (l * d.ctx + pos) * d.kv_dim;
      for (size_t j = 0; j < d.kv_dim; j++) {
        c->key_cache[cache_row + j] = f32_to_f16(k[j]);
        c->val_cache[cache_row + j] = f32_to_f16(c->bv[i * d.kv_dim + j]);
      }
    }
    for (size_t i = 0; i < b; i++)
      attend(c, l, c->bq.data() + i * d.att_dim, c->battn.data() + i * d.att_dim, base + i);
    acts_matmul(c, c->bxb.data(), d.dim, w.wo, c->battn.data(), d.att_dim, b);
    for (size_t i = 0; i < b; i++) saxpy(c->bx.data() + i * d.dim, c->residual_scale, c->bxb.data() + i * d.dim, d.dim);
    for (size_t i = 0; i < b; i++)
      rmsnorm(c->bxb.data() + i * d.dim, c->bx.data() + i * d.dim, w.ffn_norm, d.dim, c->norm_eps);
    Job gu[2] = {{c->bgate.data(), d.ffn_dim, w.w_gate}, {c->bup.data(), d.ffn_dim, w.w_up}};
    acts_matmul_group(c, gu, 2, c->bxb.data(), d.dim, b);
    for (size_t i = 0; i < b; i++) swiglu(c->bgate.data() + i * d.ffn_dim, c->bup.data() + i * d.ffn_dim, d.ffn_dim);
    acts_matmul(c, c->bxb.data(), d.dim, w.w_down, c->bgate.data(), d.ffn_dim, b);
    for (size_t i = 0; i < b; i++) saxpy(c->bx.data() + i * d.dim, c->residual_scale, c->bxb.data() + i * d.dim, d.dim);
  }
  const float* last = c->bx.data() + (b - 1) * d.dim;
  rmsnorm(c->xb.data(), last, c->out_norm, d.dim, c->norm_eps);
  acts_matvec(c, c->logits.data(), d.vocab, c->output, c->xb.data(), d.dim);
  if (c->logit_recip != 1.0f) scale_inplace(c->logits.data(), d.vocab, c->logit_recip);
  c->pos += b;
  return PE_OK;
}

// ------------------------------------------------------------ infer.rs:752-759
int ctx_prefill(Ctx* c, const uint32_t* tokens, size_t n) {
  if (n == 0) return PE_BAD_BATCH;
  for (size_t i = 0; i < n; i += MAX_BATCH) {
    size_t b = n - i < (size_t)MAX_BATCH ? n - i : (size_t)MAX_BATCH;
    int rc = ctx_prefill_chunk(c, tokens + i, b);
    if (rc) return rc;
  }
  return PE_OK;
}

// ------------------------------------------------------------- sample.rs:5-96
static float sampler_next_f32(Sampler* s) {
  uint64_t x = s->rng;
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  s->rng = x;
  return (float)(x >> 40) / (float)(1ull << 24);
}

uint32_t sampler_sample(Sampler* s, const float* logits, size_t n) {
  if (s->temperature <= 0.0f) return (uint32_t)argmax(logits, n);
  const int TOP_K = 64;
  float hv[TOP_K];
  uint32_t hi[TOP_K];
  for (int i = 0; i < TOP_K; i++) {
    hv[i] = -INFINITY;
    hi[i] = 0;
  }
  for (size_t i = 0; i < n; i++) {
    float v = logits[i];
    if (v > hv[0]) {
      hv[0] = v;
      hi[0] = (uint32_t)i;
      int k = 0;
      for (;;) {
        int l = 2 * k + 1, r = 2 * k + 2, small = k;
        if (l < TOP_K && hv[l] < hv[small]) small = l;
        if (r < TOP_K && hv[r] < hv[small]) small = r;
        if (small == k) break;
        float tv = hv[k]; hv[k] = hv[small]; hv[small] = tv;
        uint32_t ti = hi[k]; hi[k] = hi[small]; hi[small] = ti;
        k = small;
      }
    }
  }
  // sort_unstable_by descending (sample.rs:66-67): the order among equal
  // logits is unspecified in the reference; here equal logits are ordered by
  // ascending token index (the order the device sampler uses).
  for (int i = 1; i < TOP_K; i++) {
    float v = hv[i];
    uint32_t id = hi[i];
    int j = i - 1;
    while (j >= 0 && (hv[j] < v || (hv[j] == v && hi[j] > id))) {
      hv[j + 1] = hv[j];
      hi[j + 1] = hi[j];
      j--;
    }
    hv[j + 1] = v;
    hi[j + 1] = id;
  }
  float max = hv[0], sum = 0.0f, probs[TOP_K];
  for (int i = 0; i < TOP_K; i++) {
    probs[i] = expf_cr((hv[i] - max) / s->temperature);  // libm::expf (sample.rs:70)
    sum += probs[i];
  }
  float cut = s->top_p * sum, cum = 0.0f;
  int nk = TOP_K;
  for (int i = 0; i < TOP_K; i++) {
    cum += probs[i];
    if (cum >= cut) {
      nk = i + 1;
      break;
    }
  }
  float r = sampler_next_f32(s) * cum, acc = 0.0f;
  for (int i = 0; i < nk; i++) {
    acc += probs[i];
    if (r <= acc) return hi[i];
  }
  return hi[nk - 1];
}

}  // namespace oracle
