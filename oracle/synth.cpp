// TEST INFRASTRUCTURE ONLY — CPU generator of the seeded synthetic .nrm models.
//
// The product library generates the same models on the GPU
// (nightrun_b200/csrc/synth.cu); tests check the two are byte-identical, so a
// fixture computed here without a GPU applies to a model built on the GPU.
// The recipe uses only integer hashing and IEEE basic operations (no libm):
//   key(kind, layer) = mix64(seed ^ mix64(kind << 32 | layer))
//   gauss(key, i)    = (sum of 12 24-bit uniforms from mix64(key + (6i+j)·φ), j=1..6) − 6·2^24,
//                      converted to f32 and scaled by 2^-24 (Irwin–Hall approximation of N(0,1))
//   linear weight    = gauss · 0.02, quantized with the reference quantizer of its dtype
//                      (q8.rs:27-44, kquant.rs:647-712, kquant.rs:715-771)
//   norm weight      = 1 + gauss · 0.01   (f32)
// The file layout follows tools/nrconvert/src/main.rs:180-453 (tensor order,
// 64-byte alignment, CRCs) with an empty tokenizer blob.
#include <thread>
#include <vector>

#include "model.h"
#include "synth.h"

namespace oracle {

static inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static const uint64_t GOLDEN = 0x9E3779B97F4A7C15ull;

static inline uint64_t tensor_key(uint64_t seed, uint32_t kind, uint32_t layer) {
  return mix64(seed ^ mix64(((uint64_t)kind << 32) | layer));
}

float synth_gauss(uint64_t key, uint64_t idx) {
  uint32_t s = 0;
  uint64_t base = key + idx * 6 * GOLDEN;
  for (uint64_t j = 1; j <= 6; j++) {
    uint64_t h = mix64(base + j * GOLDEN);
    s += (uint32_t)(h >> 40) + (uint32_t)((h >> 16) & 0xFFFFFF);
  }
  int32_t t = (int32_t)s - 100663296;
  return (float)t * 5.9604644775390625e-08f;
}

void synth_tensor_list(const SynthCfg& cfg, std::vector<SynthTensor>& out) {
  out.clear();
  uint32_t att = cfg.n_heads * cfg.head_dim, kv = cfg.n_kv_heads * cfg.head_dim;
  bool mix = cfg.quant == 1;
  auto lin = [&](uint16_t kind, uint16_t layer, uint32_t rows, uint32_t cols, bool q6) {
    uint16_t dt = mix ? (q6 ? DT_Q6K : DT_Q4K) : DT_Q8_0;
    out.push_back({kind, layer, dt, rows, cols, 0, 0});
  };
  auto f32 = [&](uint16_t kind, uint16_t layer, uint32_t n) {
    out.push_back({kind, layer, DT_F32, 1, n, 0, 0});
  };
  lin(TK_TOK_EMBED, 0, cfg.vocab, cfg.dim, true);
  if (cfg.rope_freqs_tensor) f32(TK_ROPE_FREQS, 0, cfg.head_dim / 2);
  for (uint32_t l = 0; l < cfg.n_layers; l++) {
    bool even = (l % 2) == 0;
    f32(TK_ATTN_NORM, (uint16_t)l, cfg.dim);
    if (cfg.arch == ARCH_QWEN3) {
      f32(TK_ATTN_Q_NORM, (uint16_t)l, cfg.head_dim);
      f32(TK_ATTN_K_NORM, (uint16_t)l, cfg.head_dim);
    }
    lin(TK_ATTN_Q, (uint16_t)l, att, cfg.dim, false);
    lin(TK_ATTN_K, (uint16_t)l, kv, cfg.dim, false);
    lin(TK_ATTN_V, (uint16_t)l, kv, cfg.dim, even);
    lin(TK_ATTN_O, (uint16_t)l, cfg.dim, att, false);
    f32(TK_FFN_NORM, (uint16_t)l, cfg.dim);
    lin(TK_FFN_GATE, (uint16_t)l, cfg.ffn_dim, cfg.dim, false);
    lin(TK_FFN_UP, (uint16_t)l, cfg.ffn_dim, cfg.dim, false);
    lin(TK_FFN_DOWN, (uint16_t)l, cfg.dim, cfg.ffn_dim, even);
  }
  f32(TK_OUTPUT_NORM, 0, cfg.dim);
  if (!cfg.tied) lin(TK_OUTPUT, 0, cfg.vocab, cfg.dim, true);
  uint64_t cursor = 0;
  for (auto& t : out) {
    cursor = (cursor + DATA_ALIGN - 1) / DATA_ALIGN * DATA_ALIGN;
    t.offset = cursor;
    uint64_t n = (uint64_t)t.rows * t.cols, bs = 0;
    dtype_byte_size(t.dtype, n, &bs);
    t.size = bs;
    cursor += bs;
  }
}

static uint64_t data_size_of(const std::vector<SynthTensor>& ts) {
  return ts.empty() ? 0 : ts.back().offset + ts.back().size;
}

uint64_t synth_nrm_size(const SynthCfg& cfg) {
  std::vector<SynthTensor> ts;
  synth_tensor_list(cfg, ts);
  uint64_t table_off = HEADER_SIZE;  // empty tokenizer blob
  uint64_t data_off = (table_off + ts.size() * ENTRY_SIZE + DATA_ALIGN - 1) / DATA_ALIGN * DATA_ALIGN;
  return data_off + data_size_of(ts);
}

// Fill one tensor's bytes (rows [r0, r1)).
static void gen_rows(const SynthCfg& cfg, uint64_t seed, const SynthTensor& t, uint8_t* dst,
                     uint32_t r0, uint32_t r1) {
  uint64_t key = tensor_key(seed, t.kind, t.layer);
  std::vector<float> row(t.cols);
  for (uint32_t r = r0; r < r1; r++) {
    if (t.dtype == DT_F32) {
      float* out = (float*)(dst + (uint64_t)r * t.cols * 4);
      for (uint32_t c = 0; c < t.cols; c++) {
        uint64_t idx = (uint64_t)r * t.cols + c;
        if (t.kind == TK_ROPE_FREQS)
          out[c] = 1.0f + 0.5f * (float)(idx % 3);
        else
          out[c] = 1.0f + synth_gauss(key, idx) * 0.01f;
      }
      continue;
    }
    for (uint32_t c = 0; c < t.cols; c++) row[c] = synth_gauss(key, (uint64_t)r * t.cols + c) * 0.02f;
    if (t.dtype == DT_Q8_0) {
      q8_quantize(row.data(), t.cols, (BlockQ8_0*)(dst + (uint64_t)r * (t.cols / 32) * 34));
    } else if (t.dtype == DT_Q4K) {
      BlockQ4K* o = (BlockQ4K*)(dst + (uint64_t)r * (t.cols / 256) * 144);
      for (uint32_t b = 0; b < t.cols / 256; b++) o[b] = quantize_q4k_ref(row.data() + b * 256);
    } else {
      BlockQ6K* o = (BlockQ6K*)(dst + (uint64_t)r * (t.cols / 256) * 210);
      for (uint32_t b = 0; b < t.cols / 256; b++) o[b] = quantize_q6k_ref(row.data() + b * 256);
    }
  }
  (void)cfg;
}

static void put32(uint8_t* b, size_t off, uint32_t v) { memcpy(b + off, &v, 4); }
static void put64(uint8_t* b, size_t off, uint64_t v) { memcpy(b + off, &v, 8); }
static void putf(uint8_t* b, size_t off, float v) { memcpy(b + off, &v, 4); }

int synth_nrm_write(const SynthCfg& cfg, uint64_t seed, uint8_t* out, uint64_t cap, int threads) {
  std::vector<SynthTensor> ts;
  synth_tensor_list(cfg, ts);
  uint64_t table_off = HEADER_SIZE;
  uint64_t table_len = ts.size() * ENTRY_SIZE;
  uint64_t data_off = (table_off + table_len + DATA_ALIGN - 1) / DATA_ALIGN * DATA_ALIGN;
  uint64_t dsize = data_size_of(ts);
  if (cap < data_off + dsize) return -1;
  memset(out, 0, data_off + dsize);
  uint8_t* data = out + data_off;
  // Tensor data, rows split over threads.
  if (threads < 1) threads = 1;
  for (const auto& t : ts) {
    std::vector<std::thread> th;
    uint32_t per = (t.rows + threads - 1) / threads;
    for (int i = 0; i < threads; i++) {
      uint32_t r0 = i * per, r1 = r0 + per < t.rows ? r0 + per : t.rows;
      if (r0 >= r1) break;
      th.emplace_back(gen_rows, std::cref(cfg), seed, std::cref(t), data + t.offset, r0, r1);
    }
    for (auto& x : th) x.join();
  }
  // Header (format.rs:260-310 field order).
  memcpy(out, "NRUN", 4);
  put32(out, 4, 3);
  put32(out, 8, cfg.arch);
  uint32_t dims[8] = {cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab, cfg.ctx_train};
  for (int i = 0; i < 8; i++) put32(out, 12 + 4 * i, dims[i]);
  float rp[6] = {cfg.rope_theta, cfg.norm_eps, cfg.rope_factor, cfg.rope_low, cfg.rope_high, cfg.rope_orig_ctx};
  for (int i = 0; i < 6; i++) putf(out, 44 + 4 * i, rp[i]);
  put32(out, 68, cfg.tied ? FLAG_TIED_EMBEDDINGS : 0);
  putf(out, 72, cfg.embed_scale);
  putf(out, 76, cfg.attn_scale);
  putf(out, 80, cfg.residual_scale);
  putf(out, 84, cfg.logit_scale);
  memcpy(out + 88, cfg.name, NAME_LEN);
  put64(out, 136, HEADER_SIZE);  // tok_off
  put64(out, 144, 0);            // tok_size
  put64(out, 152, table_off);
  put32(out, 160, (uint32_t)ts.size());
  put64(out, 168, data_off);
  put64(out, 176, dsize);
  // Tensor table (main.rs:316-345).
  for (size_t i = 0; i < ts.size(); i++) {
    uint8_t* e = out + table_off + i * ENTRY_SIZE;
    const SynthTensor& t = ts[i];
    memcpy(e + 0, &t.kind, 2);
    memcpy(e + 2, &t.layer, 2);
    memcpy(e + 4, &t.dtype, 2);
    put64(e, 8, t.offset);
    put64(e, 16, t.size);
    put32(e, 24, t.rows);
    put32(e, 28, t.cols);
  }
  put32(out, 184, crc32(data, dsize));
  uint32_t crc = 0xffffffffu;
  crc = crc32_update(crc, out, HEADER_SIZE - 8);
  const uint8_t zeros[8] = {0};
  crc = crc32_update(crc, zeros, 8);
  crc = crc32_update(crc, out + table_off, table_len);
  put32(out, 188, crc ^ 0xffffffffu);
  return 0;
}

}  // namespace oracle
