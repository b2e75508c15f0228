// TEST INFRASTRUCTURE ONLY — flat C surface of the oracle for ctypes
// (oracle/oracle.py). Each entry forwards to the restated reference function
// named in its comment.
#include <vector>

#include "expf_cr.h"
#include "model.h"
#include "synth.h"

using namespace oracle;

extern "C" {

void or_set_mode(int fast_path, int fast_f16) {  // cpu.rs:46-55
  g_fast_path = fast_path != 0;
  g_fast_f16 = fast_f16 != 0;
}
void or_pool_start(int threads) { pool_start(threads); }

// expf as called by vec.rs:34,47 and sample.rs:70 (correctly rounded).
void or_expf(const float* x, float* y, size_t n) {
  for (size_t i = 0; i < n; i++) y[i] = expf_cr(x[i]);
}
// Per-chunk hashes of expf_cr's output bits over every binary32 input, 2^20
// inputs per chunk (the mixing of oracle/check_expf.cpp).
void or_expf_hash(uint64_t* out, int chunk0, int nchunks) {
  for (int c = chunk0; c < chunk0 + nchunks; c++) {
    uint64_t h = 0;
    for (uint32_t i = 0; i < (1u << 20); i++) {
      const uint32_t bits = ((uint32_t)c << 20) | i;
      float x, y;
      memcpy(&x, &bits, 4);
      y = expf_cr(x);
      uint32_t yb;
      memcpy(&yb, &y, 4);
      h ^= yb + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
      h *= 0xBF58476D1CE4E5B9ull;
    }
    out[c - chunk0] = h;
  }
}
int or_pool_threads() { return pool_threads(); }

void or_f16_to_f32(const uint16_t* in, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = f16_to_f32(in[i]);
}
void or_f32_to_f16(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = f32_to_f16(in[i]);
}

void or_q8_quantize(const float* src, size_t n, void* out) { q8_quantize(src, n, (BlockQ8_0*)out); }
void or_q8_dequantize(const void* b, size_t n, float* out) { q8_dequantize((const BlockQ8_0*)b, n, out); }
void or_quantize_q8k(const float* src, size_t n, void* out) { quantize_q8k(src, n, (BlockQ8K*)out); }
void or_dequant_q4k(const void* b, size_t nb, float* out) {
  for (size_t i = 0; i < nb; i++) dequant_q4k((const BlockQ4K*)b + i, out + i * QK_K);
}
void or_dequant_q6k(const void* b, size_t nb, float* out) {
  for (size_t i = 0; i < nb; i++) dequant_q6k((const BlockQ6K*)b + i, out + i * QK_K);
}
void or_quantize_q4k_ref(const float* src, size_t nb, void* out) {
  for (size_t i = 0; i < nb; i++) ((BlockQ4K*)out)[i] = quantize_q4k_ref(src + i * QK_K);
}
void or_quantize_q6k_ref(const float* src, size_t nb, void* out) {
  for (size_t i = 0; i < nb; i++) ((BlockQ6K*)out)[i] = quantize_q6k_ref(src + i * QK_K);
}

// mode 0: scalar reference dot, 1: AVX2 dot.
float or_dot_q8(const void* w, const void* x, size_t nb, int mode) {
  return mode ? dot_q8_avx2((const BlockQ8_0*)w, (const BlockQ8_0*)x, nb)
              : dot_q8_scalar((const BlockQ8_0*)w, (const BlockQ8_0*)x, nb);
}
float or_dot_q4k(const void* w, const void* x, size_t nb, int mode) {
  return mode ? dot_q4k_avx2((const BlockQ4K*)w, (const BlockQ8K*)x, nb)
              : dot_q4k_scalar((const BlockQ4K*)w, (const BlockQ8K*)x, nb);
}
float or_dot_q6k(const void* w, const void* x, size_t nb, int mode) {
  return mode ? dot_q6k_avx2((const BlockQ6K*)w, (const BlockQ8K*)x, nb)
              : dot_q6k_scalar((const BlockQ6K*)w, (const BlockQ8K*)x, nb);
}
void or_matvec_q8(float* y, const void* w, const void* x, size_t rows, size_t cols) {
  matvec_q8(y, (const BlockQ8_0*)w, (const BlockQ8_0*)x, rows, cols);
}
void or_matmul_q8(float* y, const void* w, const void* xs, size_t rows, size_t cols, size_t batch) {
  matmul_q8(y, (const BlockQ8_0*)w, (const BlockQ8_0*)xs, rows, cols, batch);
}
void or_matvec_q4k(float* y, const void* w, const void* x, size_t rows, size_t cols) {
  matvec_q4k(y, (const BlockQ4K*)w, (const BlockQ8K*)x, rows, cols);
}
void or_matvec_q6k(float* y, const void* w, const void* x, size_t rows, size_t cols) {
  matvec_q6k(y, (const BlockQ6K*)w, (const BlockQ8K*)x, rows, cols);
}
void or_matmul_q4k(float* y, const void* w, const void* xs, size_t rows, size_t cols, size_t batch) {
  matmul_q4k(y, (const BlockQ4K*)w, (const BlockQ8K*)xs, rows, cols, batch);
}
void or_matmul_q6k(float* y, const void* w, const void* xs, size_t rows, size_t cols, size_t batch) {
  matmul_q6k(y, (const BlockQ6K*)w, (const BlockQ8K*)xs, rows, cols, batch);
}
float or_dot_f16(const uint16_t* k, const float* q, size_t n) { return dot_f16(k, q, n); }
void or_axpy_f16(float* out, float a, const uint16_t* v, size_t n) { axpy_f16(out, a, v, n); }

void or_rmsnorm(float* out, const float* x, const float* w, size_t n, float eps) { rmsnorm(out, x, w, n, eps); }
void or_rmsnorm_inplace(float* x, const float* w, size_t n, float eps) { rmsnorm_inplace(x, w, n, eps); }
void or_softmax(float* x, size_t n) { softmax(x, n); }
void or_swiglu(float* g, const float* u, size_t n) { swiglu(g, u, n); }
size_t or_argmax(const float* x, size_t n) { return argmax(x, n); }
void or_saxpy(float* y, float a, const float* x, size_t n) { saxpy(y, a, x, n); }
void or_scale_inplace(float* x, size_t n, float s) { scale_inplace(x, n, s); }
void or_rope_freqs(float* out, size_t head_dim, float theta, float factor, float low, float high, float orig) {
  Llama3Scaling s{factor, low, high, orig};
  rope_freqs(out, head_dim, theta, factor > 0.0f ? &s : nullptr);
}
void or_rope_apply(float* x, size_t len, size_t head_dim, const float* freqs, size_t pos, int style) {
  rope_apply(x, len, head_dim, freqs, pos, style);
}
uint32_t or_crc32(const uint8_t* d, size_t n) { return crc32(d, n); }

// ---- model ----
int or_model_parse(const uint8_t* blob, size_t len, void** out) {
  Model* m = new Model();
  int rc = model_parse(blob, len, m);
  if (rc) {
    delete m;
    *out = nullptr;
    return rc;
  }
  *out = m;
  return 0;
}
void or_model_free(void* m) { delete (Model*)m; }
void or_model_meta(const void* m, Meta* out) { *out = ((const Model*)m)->meta; }
int or_model_verify(const void* m) { return model_verify_data((const Model*)m) ? 1 : 0; }
size_t or_model_tensor_count(const void* m) { return ((const Model*)m)->entries.size(); }
int or_model_tensor(const void* m, size_t i, TensorEntry* out) {
  const Model* mm = (const Model*)m;
  if (i >= mm->entries.size()) return -1;
  *out = mm->entries[i];
  return 0;
}

int or_ctx_new(const void* model, size_t ctx, void** out) {
  Ctx* c = new Ctx();
  int rc = ctx_new((const Model*)model, ctx, c);
  if (rc) {
    delete c;
    *out = nullptr;
    return rc;
  }
  *out = c;
  return 0;
}
void or_ctx_free(void* c) { delete (Ctx*)c; }
int or_ctx_forward(void* c, uint32_t token, float* logits_out) {
  Ctx* cc = (Ctx*)c;
  int rc = ctx_forward(cc, token);
  if (!rc && logits_out) memcpy(logits_out, cc->logits.data(), cc->logits.size() * 4);
  return rc;
}
int or_ctx_prefill_chunk(void* c, const uint32_t* t, size_t n, float* logits_out) {
  Ctx* cc = (Ctx*)c;
  int rc = ctx_prefill_chunk(cc, t, n);
  if (!rc && logits_out) memcpy(logits_out, cc->logits.data(), cc->logits.size() * 4);
  return rc;
}
int or_ctx_prefill(void* c, const uint32_t* t, size_t n, float* logits_out) {
  Ctx* cc = (Ctx*)c;
  int rc = ctx_prefill(cc, t, n);
  if (!rc && logits_out) memcpy(logits_out, cc->logits.data(), cc->logits.size() * 4);
  return rc;
}
void or_ctx_reset(void* c) { ((Ctx*)c)->pos = 0; }       // infer.rs:494-496
size_t or_ctx_pos(const void* c) { return ((const Ctx*)c)->pos; }
// Copy the f16 K and V rows of (layer, pos) (kv_dim values each).
int or_ctx_kv(const void* c, size_t layer, size_t pos, uint16_t* k, uint16_t* v) {
  const Ctx* cc = (const Ctx*)c;
  const Dims& d = cc->dims;
  if (layer >= d.n_layers || pos >= d.ctx) return -1;
  size_t row = (layer * d.ctx + pos) * d.kv_dim;
  memcpy(k, cc->key_cache.data() + row, d.kv_dim * 2);
  memcpy(v, cc->val_cache.data() + row, d.kv_dim * 2);
  return 0;
}

uint32_t or_sampler_sample(float temperature, float top_p, uint64_t* rng, const float* logits, size_t n) {
  Sampler s{temperature, top_p, *rng};
  uint32_t r = sampler_sample(&s, logits, n);
  *rng = s.rng;
  return r;
}

// ---- synthetic models ----
uint64_t or_synth_size(const SynthCfg* cfg) { return synth_nrm_size(*cfg); }
int or_synth_write(const SynthCfg* cfg, uint64_t seed, uint8_t* out, uint64_t cap, int threads) {
  return synth_nrm_write(*cfg, seed, out, cap, threads);
}
float or_synth_gauss(uint64_t key, uint64_t idx) { return synth_gauss(key, idx); }

}  // extern "C"
