// nrcuda engine: .nrm parsing and upload, synthetic models, the inference
// context (crates/nr-model/src/infer.rs InferCtx) and the C ABI of
// include/nrcuda.h.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemv.cuh"
#include "mma.cuh"
#include "nrcuda.h"
#include "ops.cuh"
#include "sample.cuh"
#include "synth.cuh"
#include "tp.cuh"

using namespace nrc;

// ------------------------------------------------------------------ errors
static thread_local std::string g_err;
static int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}
#define CU(call)                                                                          \
  do {                                                                                    \
    cudaError_t e_ = (call);                                                              \
    if (e_ != cudaSuccess) return fail(NRC_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

int nrc_fail_api(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

extern "C" const char* nrc_last_error(void) { return g_err.c_str(); }
extern "C" int nrc_version(void) { return 100; }

// ---------------------------------------------------- CRC-32 (crc32.rs:6-79)
namespace {
struct Crc {
  uint32_t t[8][256];
  Crc() {
    for (uint32_t i = 0; i < 256; i++) {
      uint32_t c = i;
      for (int k = 0; k < 8; k++) c = (c & 1) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
      t[0][i] = c;
    }
    for (int s = 1; s < 8; s++)
      for (int i = 0; i < 256; i++) t[s][i] = t[0][t[s - 1][i] & 0xff] ^ (t[s - 1][i] >> 8);
  }
  uint32_t update(uint32_t c, const uint8_t* w, size_t n) const {
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
      const uint32_t lo = ((uint32_t)w[i] | ((uint32_t)w[i + 1] << 8) | ((uint32_t)w[i + 2] << 16) |
                           ((uint32_t)w[i + 3] << 24)) ^ c;
      c = t[7][lo & 0xff] ^ t[6][(lo >> 8) & 0xff] ^ t[5][(lo >> 16) & 0xff] ^ t[4][lo >> 24] ^ t[3][w[i + 4]] ^
          t[2][w[i + 5]] ^ t[1][w[i + 6]] ^ t[0][w[i + 7]];
    }
    for (; i < n; i++) c = t[0][(c ^ w[i]) & 0xff] ^ (c >> 8);
    return c;
  }
};
const Crc& crc_tables() {
  static Crc c;
  return c;
}
uint32_t crc32_host(const uint8_t* d, size_t n) { return crc_tables().update(0xffffffffu, d, n) ^ 0xffffffffu; }

// ------------------------------------------------------ .nrm format (format.rs)
constexpr size_t HEADER_SIZE = 192, NAME_LEN = 48, ENTRY_SIZE = 32, DATA_ALIGN = 64;
constexpr uint32_t FLAG_TIED = 1;
enum { TK_TOK_EMBED = 1, TK_OUTPUT_NORM = 2, TK_OUTPUT = 3, TK_ROPE_FREQS = 4, TK_ATTN_NORM = 10, TK_ATTN_Q = 11,
       TK_ATTN_K = 12, TK_ATTN_V = 13, TK_ATTN_O = 14, TK_FFN_NORM = 15, TK_FFN_GATE = 16, TK_FFN_UP = 17,
       TK_FFN_DOWN = 18, TK_ATTN_Q_NORM = 19, TK_ATTN_K_NORM = 20 };
enum { DT_F32 = 0, DT_Q8_0 = 1, DT_Q4K = 2, DT_Q6K = 3 };

struct Entry {
  uint16_t kind, layer, dtype;
  uint64_t offset, size;
  uint32_t rows, cols;
};

// TensorDtype::byte_size (format.rs:104-124), checked.
bool byte_size(int dtype, uint64_t n, uint64_t* out) {
  uint64_t b, per;
  switch (dtype) {
    case DT_F32: return !__builtin_mul_overflow(n, (uint64_t)4, out);
    case DT_Q8_0: if (n % 32) return false; b = n / 32; per = 34; break;
    case DT_Q4K: if (n % 256) return false; b = n / 256; per = 144; break;
    case DT_Q6K: if (n % 256) return false; b = n / 256; per = 210; break;
    default: return false;
  }
  return !__builtin_mul_overflow(b, per, out);
}

template <typename T>
T rd(const uint8_t* p) {
  T v;
  memcpy(&v, p, sizeof(T));
  return v;
}
template <typename T>
void wr(uint8_t* p, T v) {
  memcpy(p, &v, sizeof(T));
}

int dtype_fmt(int dt) { return dt == DT_Q8_0 ? FMT_Q8_0 : (dt == DT_Q4K ? FMT_Q4K : FMT_Q6K); }
}  // namespace
namespace nrc {
uint32_t crc32_bytes(const uint8_t* d, size_t n) { return crc32_host(d, n); }
uint32_t crc32_update(uint32_t state, const uint8_t* d, size_t n) { return crc_tables().update(state, d, n); }
}  // namespace nrc

struct nrc_model {
  int device = 0;
  nrc_meta meta{};
  std::vector<Entry> entries;
  std::vector<uint8_t> prefix;  // header | tokenizer | table | padding  (bytes [0, data_off))
  uint8_t* d_data = nullptr;
  uint64_t data_size = 0;
  bool crc_known = false;
  uint32_t data_crc = 0;

  const Entry* find(int kind, int layer) const {
    for (const auto& e : entries)
      if (e.kind == kind && e.layer == layer) return &e;
    return nullptr;
  }
  bool has(int kind) const {
    for (const auto& e : entries)
      if (e.kind == kind) return true;
    return false;
  }
};

// Model::parse (format.rs:260-406).
static int parse_nrm(const uint8_t* blob, size_t len, nrc_model* m, uint64_t* data_off_out) {
  if (len < HEADER_SIZE) return fail(NRC_ERR_TOO_SHORT, "blob shorter than the 192-byte header");
  if (memcmp(blob, "NRUN", 4) != 0) return fail(NRC_ERR_BAD_MAGIC, "bad magic");
  const uint32_t version = rd<uint32_t>(blob + 4);
  if (version != 3) return fail(NRC_ERR_BAD_VERSION, "unsupported version %u", version);
  nrc_meta& mt = m->meta;
  mt.arch = (int32_t)rd<uint32_t>(blob + 8);
  if (mt.arch < 1 || mt.arch > 3) return fail(NRC_ERR_BAD_TABLE, "unknown arch %d", mt.arch);
  uint32_t* dims[8] = {&mt.dim, &mt.n_layers, &mt.n_heads, &mt.n_kv_heads, &mt.head_dim, &mt.ffn_dim, &mt.vocab,
                       &mt.ctx_train};
  for (int i = 0; i < 8; i++) *dims[i] = rd<uint32_t>(blob + 12 + 4 * i);
  float* rp[6] = {&mt.rope_theta, &mt.norm_eps, &mt.rope_factor, &mt.rope_low, &mt.rope_high, &mt.rope_orig_ctx};
  for (int i = 0; i < 6; i++) *rp[i] = rd<float>(blob + 44 + 4 * i);
  mt.flags = rd<uint32_t>(blob + 68);
  mt.embed_scale = rd<float>(blob + 72);
  mt.attn_scale = rd<float>(blob + 76);
  mt.residual_scale = rd<float>(blob + 80);
  mt.logit_scale = rd<float>(blob + 84);
  memcpy(mt.name, blob + 88, NAME_LEN);
  const uint64_t tok_off = rd<uint64_t>(blob + 136), tok_size = rd<uint64_t>(blob + 144);
  const uint64_t table_off = rd<uint64_t>(blob + 152);
  const uint64_t count = rd<uint32_t>(blob + 160);
  const uint64_t data_off = rd<uint64_t>(blob + 168), data_size = rd<uint64_t>(blob + 176);
  const uint32_t data_crc = rd<uint32_t>(blob + 184), meta_crc = rd<uint32_t>(blob + 188);
  if (!isfinite(mt.embed_scale) || !isfinite(mt.attn_scale) || mt.attn_scale < 0.0f ||
      !isfinite(mt.residual_scale) || mt.residual_scale <= 0.0f || !isfinite(mt.logit_scale) ||
      mt.logit_scale <= 0.0f)
    return fail(NRC_ERR_BAD_TABLE, "nonsensical muP scalars");
  uint64_t table_len, table_end, data_end, tok_end;
  if (__builtin_mul_overflow(count, (uint64_t)ENTRY_SIZE, &table_len)) return fail(NRC_ERR_BAD_TABLE, "table size overflow");
  if (__builtin_add_overflow(table_off, table_len, &table_end) || __builtin_add_overflow(data_off, data_size, &data_end) ||
      __builtin_add_overflow(tok_off, tok_size, &tok_end))
    return fail(NRC_ERR_TOO_SHORT, "region bounds overflow");
  if (len < table_end || len < data_end || len < tok_end) return fail(NRC_ERR_TOO_SHORT, "region past end of blob");
  const Crc& C = crc_tables();
  uint32_t c = 0xffffffffu;
  c = C.update(c, blob, HEADER_SIZE - 8);
  const uint8_t zeros[8] = {0};
  c = C.update(c, zeros, 8);
  c = C.update(c, blob + tok_off, tok_size);
  c = C.update(c, blob + table_off, table_len);
  if ((c ^ 0xffffffffu) != meta_crc) return fail(NRC_ERR_META_CRC, "meta crc mismatch");
  m->entries.clear();
  for (uint64_t i = 0; i < count; i++) {
    const uint8_t* e = blob + table_off + i * ENTRY_SIZE;
    Entry t;
    t.kind = rd<uint16_t>(e);
    t.layer = rd<uint16_t>(e + 2);
    t.dtype = rd<uint16_t>(e + 4);
    if (t.dtype > 3) return fail(NRC_ERR_BAD_TABLE, "bad dtype");
    t.offset = rd<uint64_t>(e + 8);
    t.size = rd<uint64_t>(e + 16);
    t.rows = rd<uint32_t>(e + 24);
    t.cols = rd<uint32_t>(e + 28);
    uint64_t end, bs;
    if (__builtin_add_overflow(t.offset, t.size, &end) || end > data_size)
      return fail(NRC_ERR_BAD_TABLE, "tensor outside the data section");
    if (t.offset % DATA_ALIGN) return fail(NRC_ERR_BAD_TABLE, "misaligned tensor offset");
    const uint64_t n = (uint64_t)t.rows * (uint64_t)t.cols;
    if (!byte_size(t.dtype, n, &bs) || bs != t.size) return fail(NRC_ERR_BAD_TABLE, "size/dtype mismatch");
    m->entries.push_back(t);
  }
  m->data_size = data_size;
  m->data_crc = data_crc;
  m->crc_known = true;
  *data_off_out = data_off;
  return NRC_OK;
}

extern "C" int nrc_model_load(const uint8_t* blob, size_t len, int device, int verify_crc, nrc_model** out) {
  if (!blob || !out) return fail(NRC_ERR_INVALID, "null argument");
  *out = nullptr;
  nrc_model* m = new nrc_model();
  uint64_t data_off = 0;
  int rc = parse_nrm(blob, len, m, &data_off);
  if (rc) {
    delete m;
    return rc;
  }
  if (verify_crc && crc32_host(blob + data_off, m->data_size) != m->data_crc) {
    delete m;
    return fail(NRC_ERR_DATA_CRC, "data crc mismatch");
  }
  m->device = device;
  m->prefix.assign(blob, blob + data_off);
  if (cudaSetDevice(device) != cudaSuccess) {
    delete m;
    return fail(NRC_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  }
  // +256: slack so no kernel ever needs to read past the allocation.
  if (cudaMalloc(&m->d_data, m->data_size + 256) != cudaSuccess) {
    delete m;
    return fail(NRC_ERR_ALLOC, "cannot allocate %llu bytes of weights", (unsigned long long)m->data_size);
  }
  if (cudaMemcpy(m->d_data, blob + data_off, m->data_size, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(m->d_data);
    delete m;
    return fail(NRC_ERR_CUDA, "weight upload failed");
  }
  *out = m;
  return NRC_OK;
}

// Tensor list of a synthetic model, in the order tools/nrconvert writes them
// (tools/nrconvert/src/main.rs:231-277), 64-byte aligned.
static void synth_entries(const nrc_synth_cfg& c, std::vector<Entry>& out) {
  out.clear();
  const uint32_t att = c.n_heads * c.head_dim, kv = c.n_kv_heads * c.head_dim;
  const bool mix = c.quant == 1;
  auto lin = [&](uint16_t kind, uint16_t layer, uint32_t rows, uint32_t cols, bool q6) {
    out.push_back({kind, layer, (uint16_t)(mix ? (q6 ? DT_Q6K : DT_Q4K) : DT_Q8_0), 0, 0, rows, cols});
  };
  auto f32 = [&](uint16_t kind, uint16_t layer, uint32_t n) { out.push_back({kind, layer, DT_F32, 0, 0, 1, n}); };
  lin(TK_TOK_EMBED, 0, c.vocab, c.dim, true);
  if (c.rope_freqs_tensor) f32(TK_ROPE_FREQS, 0, c.head_dim / 2);
  for (uint32_t l = 0; l < c.n_layers; l++) {
    const bool even = (l % 2) == 0;
    const uint16_t L = (uint16_t)l;
    f32(TK_ATTN_NORM, L, c.dim);
    if (c.arch == 2) {
      f32(TK_ATTN_Q_NORM, L, c.head_dim);
      f32(TK_ATTN_K_NORM, L, c.head_dim);
    }
    lin(TK_ATTN_Q, L, att, c.dim, false);
    lin(TK_ATTN_K, L, kv, c.dim, false);
    lin(TK_ATTN_V, L, kv, c.dim, even);
    lin(TK_ATTN_O, L, c.dim, att, false);
    f32(TK_FFN_NORM, L, c.dim);
    lin(TK_FFN_GATE, L, c.ffn_dim, c.dim, false);
    lin(TK_FFN_UP, L, c.ffn_dim, c.dim, false);
    lin(TK_FFN_DOWN, L, c.dim, c.ffn_dim, even);
  }
  f32(TK_OUTPUT_NORM, 0, c.dim);
  if (!c.tied) lin(TK_OUTPUT, 0, c.vocab, c.dim, true);
  uint64_t cur = 0;
  for (auto& e : out) {
    cur = (cur + DATA_ALIGN - 1) / DATA_ALIGN * DATA_ALIGN;
    e.offset = cur;
    uint64_t bs = 0;
    byte_size(e.dtype, (uint64_t)e.rows * e.cols, &bs);
    e.size = bs;
    cur += bs;
  }
}

extern "C" int nrc_model_synth(const nrc_synth_cfg* cfg, uint64_t seed, int device, nrc_model** out) {
  if (!cfg || !out) return fail(NRC_ERR_INVALID, "null argument");
  *out = nullptr;
  const nrc_synth_cfg& c = *cfg;
  if (c.arch < 1 || c.arch > 3 || !c.dim || !c.n_layers || !c.n_heads || !c.n_kv_heads || !c.head_dim ||
      c.n_heads % c.n_kv_heads)
    return fail(NRC_ERR_INVALID, "bad synthetic config");
  nrc_model* m = new nrc_model();
  m->device = device;
  synth_entries(c, m->entries);
  m->data_size = m->entries.empty() ? 0 : m->entries.back().offset + m->entries.back().size;
  const uint64_t table_off = HEADER_SIZE, table_len = m->entries.size() * ENTRY_SIZE;
  const uint64_t data_off = (table_off + table_len + DATA_ALIGN - 1) / DATA_ALIGN * DATA_ALIGN;
  std::vector<uint8_t>& p = m->prefix;
  p.assign(data_off, 0);
  memcpy(p.data(), "NRUN", 4);
  wr<uint32_t>(&p[4], 3);
  wr<uint32_t>(&p[8], c.arch);
  const uint32_t dims[8] = {c.dim, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn_dim, c.vocab, c.ctx_train};
  for (int i = 0; i < 8; i++) wr<uint32_t>(&p[12 + 4 * i], dims[i]);
  const float rp[6] = {c.rope_theta, c.norm_eps, c.rope_factor, c.rope_low, c.rope_high, c.rope_orig_ctx};
  for (int i = 0; i < 6; i++) wr<float>(&p[44 + 4 * i], rp[i]);
  wr<uint32_t>(&p[68], c.tied ? FLAG_TIED : 0);
  wr<float>(&p[72], c.embed_scale);
  wr<float>(&p[76], c.attn_scale);
  wr<float>(&p[80], c.residual_scale);
  wr<float>(&p[84], c.logit_scale);
  memcpy(&p[88], c.name, NAME_LEN);
  wr<uint64_t>(&p[136], HEADER_SIZE);
  wr<uint64_t>(&p[144], 0);
  wr<uint64_t>(&p[152], table_off);
  wr<uint32_t>(&p[160], (uint32_t)m->entries.size());
  wr<uint64_t>(&p[168], data_off);
  wr<uint64_t>(&p[176], m->data_size);
  for (size_t i = 0; i < m->entries.size(); i++) {
    uint8_t* e = &p[table_off + i * ENTRY_SIZE];
    const Entry& t = m->entries[i];
    wr<uint16_t>(e, t.kind);
    wr<uint16_t>(e + 2, t.layer);
    wr<uint16_t>(e + 4, t.dtype);
    wr<uint64_t>(e + 8, t.offset);
    wr<uint64_t>(e + 16, t.size);
    wr<uint32_t>(e + 24, t.rows);
    wr<uint32_t>(e + 28, t.cols);
  }
  const Crc& C = crc_tables();
  uint32_t mc = 0xffffffffu;
  mc = C.update(mc, p.data(), HEADER_SIZE - 8);
  const uint8_t zeros[8] = {0};
  mc = C.update(mc, zeros, 8);
  mc = C.update(mc, p.data() + table_off, table_len);
  wr<uint32_t>(&p[188], mc ^ 0xffffffffu);
  m->meta.arch = (int32_t)c.arch;
  m->meta.dim = c.dim;
  m->meta.n_layers = c.n_layers;
  m->meta.n_heads = c.n_heads;
  m->meta.n_kv_heads = c.n_kv_heads;
  m->meta.head_dim = c.head_dim;
  m->meta.ffn_dim = c.ffn_dim;
  m->meta.vocab = c.vocab;
  m->meta.ctx_train = c.ctx_train;
  m->meta.rope_theta = c.rope_theta;
  m->meta.norm_eps = c.norm_eps;
  m->meta.rope_factor = c.rope_factor;
  m->meta.rope_low = c.rope_low;
  m->meta.rope_high = c.rope_high;
  m->meta.rope_orig_ctx = c.rope_orig_ctx;
  m->meta.flags = c.tied ? FLAG_TIED : 0;
  m->meta.embed_scale = c.embed_scale;
  m->meta.attn_scale = c.attn_scale;
  m->meta.residual_scale = c.residual_scale;
  m->meta.logit_scale = c.logit_scale;
  memcpy(m->meta.name, c.name, NAME_LEN);
  if (cudaSetDevice(device) != cudaSuccess) {
    delete m;
    return fail(NRC_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  }
  if (cudaMalloc(&m->d_data, m->data_size + 256) != cudaSuccess) {
    delete m;
    return fail(NRC_ERR_ALLOC, "cannot allocate %llu bytes of weights", (unsigned long long)m->data_size);
  }
  cudaMemset(m->d_data, 0, m->data_size + 256);
  for (const auto& e : m->entries) {
    cudaError_t err = synth_fill(m->d_data + e.offset, e.dtype, e.kind, e.rows, e.cols,
                                 synth_tensor_key(seed, e.kind, e.layer), 0);
    if (err != cudaSuccess) {
      cudaFree(m->d_data);
      delete m;
      return fail(NRC_ERR_CUDA, "synthetic fill failed: %s", cudaGetErrorString(err));
    }
  }
  if (cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(m->d_data);
    delete m;
    return fail(NRC_ERR_CUDA, "synthetic fill failed");
  }
  *out = m;
  return NRC_OK;
}

extern "C" int nrc_model_meta(const nrc_model* m, nrc_meta* out) {
  if (!m || !out) return fail(NRC_ERR_INVALID, "null argument");
  *out = m->meta;
  return NRC_OK;
}

extern "C" size_t nrc_model_nrm_size(const nrc_model* m) { return m ? m->prefix.size() + m->data_size : 0; }

static int ensure_crc(nrc_model* m, const uint8_t* host_data) {
  if (m->crc_known) return NRC_OK;
  std::vector<uint8_t> tmp;
  if (!host_data) {
    tmp.resize(m->data_size);
    CU(cudaSetDevice(m->device));
    CU(cudaMemcpy(tmp.data(), m->d_data, m->data_size, cudaMemcpyDeviceToHost));
    host_data = tmp.data();
  }
  m->data_crc = crc32_host(host_data, m->data_size);
  m->crc_known = true;
  wr<uint32_t>(&m->prefix[184], m->data_crc);
  return NRC_OK;
}

extern "C" int nrc_model_export(const nrc_model* mc, uint8_t* out, size_t cap) {
  nrc_model* m = const_cast<nrc_model*>(mc);
  if (!m || !out) return fail(NRC_ERR_INVALID, "null argument");
  if (cap < m->prefix.size() + m->data_size) return fail(NRC_ERR_INVALID, "export buffer too small");
  CU(cudaSetDevice(m->device));
  CU(cudaMemcpy(out + m->prefix.size(), m->d_data, m->data_size, cudaMemcpyDeviceToHost));
  int rc = ensure_crc(m, out + m->prefix.size());
  if (rc) return rc;
  memcpy(out, m->prefix.data(), m->prefix.size());
  return NRC_OK;
}

extern "C" int nrc_model_data_crc(const nrc_model* mc, uint32_t* out) {
  nrc_model* m = const_cast<nrc_model*>(mc);
  if (!m || !out) return fail(NRC_ERR_INVALID, "null argument");
  // Recomputed from the device copy (checks what the kernels will read).
  std::vector<uint8_t> tmp(m->data_size);
  CU(cudaSetDevice(m->device));
  CU(cudaMemcpy(tmp.data(), m->d_data, m->data_size, cudaMemcpyDeviceToHost));
  *out = crc32_host(tmp.data(), m->data_size);
  return NRC_OK;
}

extern "C" int nrc_model_free(nrc_model* m) {
  if (!m) return NRC_OK;
  cudaSetDevice(m->device);
  if (m->d_data) cudaFree(m->d_data);
  delete m;
  return NRC_OK;
}

// ------------------------------------------------------------ inference context
namespace {
struct LayerW {
  const uint8_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
  int fq, fk, fv, fo, fg, fu, fd;
  const float *attn_norm, *ffn_norm, *q_norm, *k_norm;
};

// Device-resident step state (positions and tokens are read by the kernels
// so one captured graph serves every decode step).
struct Status {
  uint32_t pos;
  uint32_t next;
  uint32_t err;
  uint32_t pad;
  unsigned long long key;
  unsigned long long rng;  // Sampler::rng (sample.rs:9), advanced once per draw
  uint32_t tok[NRC_MAX_BATCH];
};

// This rank's part of the model under tensor parallelism over n ranks (n = 1:
// everything). Query heads and KV heads go by whole KV groups; the rows of
// wo / ffn_down (model dim), ffn_gate / ffn_up and the classifier (vocab) in
// equal contiguous ranges. Every output element is computed whole, with the
// full K, by exactly one rank; ranks exchange activations (all-gather), never
// partial sums, so results are bit-identical to one GPU.
struct Shard {
  int n = 1, r = 0;
  int h0 = 0, nh = 0;    // query heads
  int kv0 = 0, nkv = 0;  // KV heads
  int d0 = 0, dn = 0;    // model-dim rows (wo, ffn_down)
  int f0 = 0, fn = 0;    // ffn rows (ffn_gate, ffn_up)
  int v0 = 0, vn = 0;    // vocabulary rows (classifier)
};

int shard_for(const nrc_meta& mt, int n, int r, Shard* sh) {
  if (n < 1 || r < 0 || r >= n) return NRC_ERR_INVALID;
  if (mt.n_kv_heads % n || mt.dim % n || mt.ffn_dim % n || mt.vocab % n) return NRC_ERR_INVALID;
  const int gqa = (int)(mt.n_heads / mt.n_kv_heads);
  sh->n = n;
  sh->r = r;
  sh->nkv = (int)mt.n_kv_heads / n;
  sh->kv0 = r * sh->nkv;
  sh->nh = sh->nkv * gqa;
  sh->h0 = sh->kv0 * gqa;
  sh->dn = (int)mt.dim / n;
  sh->d0 = r * sh->dn;
  sh->fn = (int)mt.ffn_dim / n;
  sh->f0 = r * sh->fn;
  sh->vn = (int)mt.vocab / n;
  sh->v0 = r * sh->vn;
  return NRC_OK;
}

struct Layout {
  size_t kc, vc, x, q, k, v, att, g, u, logits, cos_t, sin_t, mxq, mxd, mxb, xsh, status, hist, samp, tps, tpr;
  // Several sequences: per-sequence positions / next input / last choice,
  // 0..S-1, the pass's per-token ids / positions / sequences, classifier
  // rows, gathered final rows, their logits, per-sequence token history.
  size_t bpos, btok, bnext, biota, ctok, cpos, cseq, crow, xl, blogits, bhist;
  size_t total;
};

size_t al(size_t v) { return (v + 255) & ~(size_t)255; }

// Tokens per forward pass of a context of n_seqs sequences.
size_t pass_tokens(size_t n_seqs) { return n_seqs > NRC_MAX_BATCH ? n_seqs : NRC_MAX_BATCH; }

Layout layout_for(const nrc_meta& mt, size_t ctx, size_t n_seqs = 1, bool batch = false, int tp = 1) {
  Layout L{};
  const size_t dim = mt.dim, att = (size_t)mt.n_heads * mt.head_dim;
  const size_t kv = (size_t)mt.n_kv_heads * mt.head_dim / (size_t)tp;  // this rank's KV heads
  const size_t B = pass_tokens(n_seqs);
  const size_t BM = (B + 63) / 64 * 64;  // tensor-core token groups
  size_t maxk = dim > att ? dim : att;
  if (mt.ffn_dim > maxk) maxk = mt.ffn_dim;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t r = o;
    o = al(o + bytes);
    return r;
  };
  // KV caches f16 [layer][sequence][ctx][kv_dim].
  L.kc = take((size_t)mt.n_layers * n_seqs * ctx * kv * 2);
  L.vc = take((size_t)mt.n_layers * n_seqs * ctx * kv * 2);
  L.x = take(B * dim * 4);
  L.q = take(B * att * 4);
  L.k = take(B * kv * 4);
  L.v = take(B * kv * 4);
  L.att = take(B * att * 4);
  L.g = take(B * mt.ffn_dim * 4);
  L.u = take(B * mt.ffn_dim * 4);
  L.logits = take((size_t)mt.vocab * 4);
  L.cos_t = take(ctx * (mt.head_dim / 2) * 4);
  L.sin_t = take(ctx * (mt.head_dim / 2) * 4);
  L.mxq = take(BM * maxk * 2);        // tensor-core activation tiles (x 2: the Q6_K masked halves)
  L.mxd = take(BM * (maxk / 32) * 4);  // and their block scales
  L.mxb = take(BM * (maxk / 256) * 8 * 4);  // and the chunk sums of the K-quant tiles
  // Quantized activations of up to 8 tokens handed from one kernel to the
  // next: the attention-norm input shared by the QKV launches of one layer
  // (Q8_0 or Q8_K blocks), the attention output for the output projection and
  // the SwiGLU output for the down projection (Q8_0 blocks).
  const size_t q8_max = std::max(std::max(dim, att), (size_t)mt.ffn_dim) / 32 * 34;
  L.xsh = take(8 * std::max(q8_max, dim / 256 * 292 + 292));
  L.status = take(sizeof(Status));
  L.hist = take((ctx + 1) * 4);
  L.samp = take(sample_scratch_bytes((int)mt.vocab));  // sampler candidates
  if (tp > 1) {
    // Tensor parallelism: this rank's compact part of an activation [B][part]
    // and the all-gathered parts of every rank [tp][B][part].
    size_t part = att / tp;
    part = std::max(part, dim / tp);
    part = std::max(part, (size_t)mt.ffn_dim / tp);
    const size_t send = std::max(B * part, (size_t)mt.vocab / tp);
    L.tps = take(send * 4);
    L.tpr = take(send * tp * 4);
  }
  if (batch) {
    const size_t S = n_seqs;
    L.bpos = take(S * 4);
    L.btok = take(S * 4);
    L.bnext = take(S * 4);
    L.biota = take(S * 4);
    L.ctok = take(B * 4);
    L.cpos = take(B * 4);
    L.cseq = take(B * 4);
    L.crow = take(S * 4);
    L.xl = take(S * dim * 4);
    L.blogits = take(S * (size_t)mt.vocab * 4);
    L.bhist = take(S * ctx * 4);
  }
  L.total = o;
  return L;
}

// rope::rope_freqs (crates/nr-tensor/src/rope.rs:14-34) with glibc powf.
void host_rope_freqs(float* out, size_t head_dim, float theta, bool scaled, float factor, float low, float high,
                     float orig) {
  const size_t half = head_dim / 2;
  const float PI = 3.14159265358979323846f;
  for (size_t i = 0; i < half; i++) {
    volatile float exponent = -2.0f * (float)i / (float)head_dim;
    float freq = powf(theta, exponent);
    if (scaled) {
      const float wavelen = 2.0f * PI / freq;
      const float low_wavelen = orig / low;
      const float high_wavelen = orig / high;
      if (wavelen > low_wavelen) {
        freq /= factor;
      } else if (wavelen > high_wavelen) {
        volatile float smooth = (orig / wavelen - low) / (high - low);
        volatile float a = (1.0f - smooth) * freq;
        volatile float b = a / factor;
        volatile float c2 = smooth * freq;
        freq = b + c2;
      }
    }
    out[i] = freq;
  }
}
}  // namespace

struct nrc_ctx {
  const nrc_model* m = nullptr;
  int device = 0;
  cudaStream_t stream = nullptr;
  size_t ctx = 0;
  int dim, att_dim, n_layers, n_heads, n_kv, hd, kv_dim, ffn, vocab;
  int style;
  float eps, embed_scale, att_scale, rs, logit_recip;
  std::vector<LayerW> L;
  const uint8_t* embed;
  int f_embed;
  const uint8_t* out_w;
  int f_out;
  const float* out_norm;
  uint8_t* arena = nullptr;
  Layout lay;
  uint16_t *kc, *vc;
  float *x, *q, *k, *v, *att, *g, *u, *logits, *cos_t, *sin_t;
  uint8_t* mxq;  // tensor-core activation tiles (prefill)
  float* mxd;
  int* mxb;
  uint8_t* xsh;
  Status* st;
  uint32_t* hist;
  uint32_t* h_stage = nullptr;  // pinned host staging: tokens in, status out
  size_t pos = 0;
  size_t pending = 0;  // decode steps enqueued by nrc_ctx_decode_async, not yet synced
  cudaGraphExec_t gexec = nullptr;
  bool pdl = true;
  // Sampler attached by nrc_ctx_set_sampler (greedy when temperature <= 0).
  float temperature = 0.0f, top_p = 1.0f;
  bool sampling = false;
  unsigned long long* samp = nullptr;
  // Tolerance mode (nrc_ctx_set_mode): decode steps use tree reductions.
  bool fast = false;
  // Tensor parallelism (nrc_tp_ctx_new): this rank's shard, its KV width, NCCL.
  Shard sh;
  int kvl = 0;  // KV cache row width of this rank (n_kv_heads / tp * head_dim)
  ncclComm_t comm = nullptr;
  float *tp_send = nullptr, *tp_recv = nullptr;
  // Several sequences (nrc_batch_new): each has its own KV cache and position.
  size_t n_seqs = 1, max_tok = NRC_MAX_BATCH;
  bool batch = false;  // created by nrc_batch_new: the nrc_batch_* entry points drive it
  uint32_t *bpos = nullptr, *btok = nullptr, *bnext = nullptr, *biota = nullptr;
  uint32_t *ctok = nullptr, *cpos = nullptr, *cseq = nullptr, *crow = nullptr;
  float *xl = nullptr, *blogits = nullptr;
  uint32_t* bhist = nullptr;
  std::vector<size_t> hpos;  // host copy of every sequence's position
  uint32_t* h_big = nullptr;  // pinned staging for pass arrays (4 x max_tok words)
};

extern "C" int nrc_ctx_required_bytes(const nrc_model* m, size_t ctx, size_t* out) {
  if (!m || !out) return fail(NRC_ERR_INVALID, "null argument");
  *out = layout_for(m->meta, ctx).total;
  return NRC_OK;
}

// InferCtx::new (infer.rs:352-492): shape-checked binding of every tensor;
// n_seqs independent sequences (each its own KV cache and position).
static int ctx_create(const nrc_model* m, size_t ctx, size_t n_seqs, bool batch, nrc_ctx** out, int tp_n = 1,
                      int tp_r = 0, const uint8_t* tp_id = nullptr) {
  if (!m || !out) return fail(NRC_ERR_INVALID, "null argument");
  if (ctx == 0) return fail(NRC_ERR_INVALID, "ctx must be > 0");
  if (n_seqs == 0 || n_seqs > 4096) return fail(NRC_ERR_INVALID, "n_seqs must be in 1..4096");
  *out = nullptr;
  const nrc_meta& mt = m->meta;
  if (mt.head_dim % 32 || mt.head_dim > 128 || mt.n_kv_heads == 0 || mt.n_heads % mt.n_kv_heads)
    return fail(NRC_ERR_INVALID, "unsupported attention shape (head_dim %u, heads %u/%u)", mt.head_dim, mt.n_heads,
                mt.n_kv_heads);
  if (attention_smem_bytes(mt.n_heads, mt.n_kv_heads, mt.head_dim, (int)ctx, 1) > ATTN_MAX_SMEM)
    return fail(NRC_ERR_INVALID, "context of %zu positions exceeds the attention kernel's score buffer", ctx);
  nrc_ctx* c = new nrc_ctx();
  c->m = m;
  c->device = m->device;
  c->ctx = ctx;
  c->dim = mt.dim;
  c->att_dim = mt.n_heads * mt.head_dim;
  c->n_layers = mt.n_layers;
  c->n_heads = mt.n_heads;
  c->n_kv = mt.n_kv_heads;
  c->hd = mt.head_dim;
  c->kv_dim = mt.n_kv_heads * mt.head_dim;
  c->ffn = mt.ffn_dim;
  c->vocab = mt.vocab;
  std::unique_ptr<nrc_ctx, int (*)(nrc_ctx*)> guard(c, nrc_ctx_free);
  const uint8_t* base = m->d_data;
  auto mat = [&](int kind, int layer, uint32_t rows, uint32_t cols, const uint8_t** p, int* fmt) -> int {
    const Entry* e = m->find(kind, layer);
    if (!e) return fail(NRC_ERR_MISSING, "missing tensor kind %d layer %d", kind, layer);
    if (e->rows != rows || e->cols != cols) return fail(NRC_ERR_MISSING, "bad matrix shape (kind %d layer %d)", kind, layer);
    if (e->dtype == DT_F32) return fail(NRC_ERR_BAD_TABLE, "f32 matrix (kind %d)", kind);
    *p = base + e->offset;
    *fmt = dtype_fmt(e->dtype);
    return NRC_OK;
  };
  auto f32t = [&](int kind, int layer, uint32_t n, const float** p) -> int {
    const Entry* e = m->find(kind, layer);
    if (!e) return fail(NRC_ERR_MISSING, "missing tensor kind %d layer %d", kind, layer);
    if (e->dtype != DT_F32 || (uint64_t)e->rows * e->cols != n) return fail(NRC_ERR_MISSING, "bad f32 tensor shape");
    *p = reinterpret_cast<const float*>(base + e->offset);
    return NRC_OK;
  };
  int rc;
  if ((rc = mat(TK_TOK_EMBED, 0, mt.vocab, mt.dim, &c->embed, &c->f_embed))) return rc;
  const bool qwen = mt.arch == 2;
  if (!qwen && m->has(TK_ATTN_Q_NORM)) return fail(NRC_ERR_MISSING, "unexpected attn_q_norm for this arch");
  c->L.resize(mt.n_layers);
  for (uint32_t l = 0; l < mt.n_layers; l++) {
    LayerW& w = c->L[l];
    if ((rc = f32t(TK_ATTN_NORM, l, mt.dim, &w.attn_norm))) return rc;
    w.q_norm = w.k_norm = nullptr;
    if (qwen) {
      if ((rc = f32t(TK_ATTN_Q_NORM, l, mt.head_dim, &w.q_norm))) return rc;
      if ((rc = f32t(TK_ATTN_K_NORM, l, mt.head_dim, &w.k_norm))) return rc;
    }
    if ((rc = mat(TK_ATTN_Q, l, c->att_dim, mt.dim, &w.wq, &w.fq))) return rc;
    if ((rc = mat(TK_ATTN_K, l, c->kv_dim, mt.dim, &w.wk, &w.fk))) return rc;
    if ((rc = mat(TK_ATTN_V, l, c->kv_dim, mt.dim, &w.wv, &w.fv))) return rc;
    if ((rc = mat(TK_ATTN_O, l, mt.dim, c->att_dim, &w.wo, &w.fo))) return rc;
    if ((rc = f32t(TK_FFN_NORM, l, mt.dim, &w.ffn_norm))) return rc;
    if ((rc = mat(TK_FFN_GATE, l, mt.ffn_dim, mt.dim, &w.wg, &w.fg))) return rc;
    if ((rc = mat(TK_FFN_UP, l, mt.ffn_dim, mt.dim, &w.wu, &w.fu))) return rc;
    if ((rc = mat(TK_FFN_DOWN, l, mt.dim, mt.ffn_dim, &w.wd, &w.fd))) return rc;
  }
  if ((rc = f32t(TK_OUTPUT_NORM, 0, mt.dim, &c->out_norm))) return rc;
  if (mt.flags & FLAG_TIED) {
    c->out_w = c->embed;
    c->f_out = c->f_embed;
  } else if ((rc = mat(TK_OUTPUT, 0, mt.vocab, mt.dim, &c->out_w, &c->f_out))) {
    return rc;
  }
  c->style = qwen ? 1 : 0;
  c->eps = mt.norm_eps;
  c->embed_scale = mt.embed_scale;
  c->att_scale = mt.attn_scale != 0.0f ? mt.attn_scale : 1.0f / sqrtf((float)mt.head_dim);
  c->rs = mt.residual_scale;
  c->logit_recip = 1.0f / mt.logit_scale;

  CU(cudaSetDevice(c->device));
  if (shard_for(mt, tp_n, tp_r, &c->sh))
    return fail(NRC_ERR_INVALID, "model does not split over %d ranks (KV heads %u, dim %u, ffn %u, vocab %u)", tp_n,
                mt.n_kv_heads, mt.dim, mt.ffn_dim, mt.vocab);
  if (tp_n > 1 && batch) return fail(NRC_ERR_INVALID, "tensor parallelism serves single-sequence contexts");
  c->kvl = c->sh.nkv * c->hd;
  c->n_seqs = n_seqs;
  c->batch = batch;
  c->max_tok = pass_tokens(n_seqs);
  c->lay = layout_for(mt, ctx, n_seqs, batch, tp_n);
  if (cudaMalloc(&c->arena, c->lay.total) != cudaSuccess)
    return fail(NRC_ERR_ALLOC, "inference arena exhausted (%llu bytes)", (unsigned long long)c->lay.total);
  CU(cudaMemset(c->arena, 0, c->lay.total));
  uint8_t* A = c->arena;
  c->kc = reinterpret_cast<uint16_t*>(A + c->lay.kc);
  c->vc = reinterpret_cast<uint16_t*>(A + c->lay.vc);
  c->x = reinterpret_cast<float*>(A + c->lay.x);
  c->q = reinterpret_cast<float*>(A + c->lay.q);
  c->k = reinterpret_cast<float*>(A + c->lay.k);
  c->v = reinterpret_cast<float*>(A + c->lay.v);
  c->att = reinterpret_cast<float*>(A + c->lay.att);
  c->g = reinterpret_cast<float*>(A + c->lay.g);
  c->u = reinterpret_cast<float*>(A + c->lay.u);
  c->logits = reinterpret_cast<float*>(A + c->lay.logits);
  c->cos_t = reinterpret_cast<float*>(A + c->lay.cos_t);
  c->sin_t = reinterpret_cast<float*>(A + c->lay.sin_t);
  c->mxq = A + c->lay.mxq;
  c->mxd = reinterpret_cast<float*>(A + c->lay.mxd);
  c->mxb = reinterpret_cast<int*>(A + c->lay.mxb);
  c->xsh = A + c->lay.xsh;
  c->st = reinterpret_cast<Status*>(A + c->lay.status);
  c->hist = reinterpret_cast<uint32_t*>(A + c->lay.hist);
  c->samp = reinterpret_cast<unsigned long long*>(A + c->lay.samp);
  if (tp_n > 1) {
    c->tp_send = reinterpret_cast<float*>(A + c->lay.tps);
    c->tp_recv = reinterpret_cast<float*>(A + c->lay.tpr);
    const NcclApi* api = nccl_api();
    if (!api) return fail(NRC_ERR_CUDA, "tensor parallelism needs NCCL (libnccl.so.2 not found)");
    ncclUniqueId id;
    memcpy(&id, tp_id, sizeof id);
    const ncclResult_t nr = api->comm_init_rank(&c->comm, tp_n, id, tp_r);
    if (nr != ncclSuccess) {
      c->comm = nullptr;
      return fail(NRC_ERR_CUDA, "ncclCommInitRank: %s", api->error_string(nr));
    }
  }
  if (batch) {
    c->bpos = reinterpret_cast<uint32_t*>(A + c->lay.bpos);
    c->btok = reinterpret_cast<uint32_t*>(A + c->lay.btok);
    c->bnext = reinterpret_cast<uint32_t*>(A + c->lay.bnext);
    c->biota = reinterpret_cast<uint32_t*>(A + c->lay.biota);
    c->ctok = reinterpret_cast<uint32_t*>(A + c->lay.ctok);
    c->cpos = reinterpret_cast<uint32_t*>(A + c->lay.cpos);
    c->cseq = reinterpret_cast<uint32_t*>(A + c->lay.cseq);
    c->crow = reinterpret_cast<uint32_t*>(A + c->lay.crow);
    c->xl = reinterpret_cast<float*>(A + c->lay.xl);
    c->blogits = reinterpret_cast<float*>(A + c->lay.blogits);
    c->bhist = reinterpret_cast<uint32_t*>(A + c->lay.bhist);
    c->hpos.assign(n_seqs, 0);
    std::vector<uint32_t> iota(n_seqs);
    for (size_t i = 0; i < n_seqs; i++) iota[i] = (uint32_t)i;
    CU(cudaMemcpy(c->biota, iota.data(), n_seqs * 4, cudaMemcpyHostToDevice));
    CU(cudaMallocHost(&c->h_big, (c->max_tok * 3 + n_seqs) * 4));
  }

  // RoPE tables (infer.rs:427-445; rope.rs:49-65): cos/sin of pos * freq.
  const size_t half = mt.head_dim / 2;
  std::vector<float> freqs(half);
  if (m->has(TK_ROPE_FREQS)) {
    host_rope_freqs(freqs.data(), mt.head_dim, mt.rope_theta, false, 0, 0, 0, 0);
    const Entry* e = m->find(TK_ROPE_FREQS, 0);
    std::vector<float> fac((size_t)e->rows * e->cols);
    CU(cudaMemcpy(fac.data(), base + e->offset, fac.size() * 4, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < half && i < fac.size(); i++) freqs[i] /= fac[i];
  } else {
    host_rope_freqs(freqs.data(), mt.head_dim, mt.rope_theta, mt.rope_factor > 0.0f, mt.rope_factor, mt.rope_low,
                    mt.rope_high, mt.rope_orig_ctx);
  }
  std::vector<float> ct(ctx * half), stab(ctx * half);
  for (size_t p = 0; p < ctx; p++)
    for (size_t i = 0; i < half; i++) {
      volatile float angle = (float)p * freqs[i];
      float s, co;
      sincosf(angle, &s, &co);
      ct[p * half + i] = co;
      stab[p * half + i] = s;
    }
  CU(cudaMemcpy(c->cos_t, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice));
  CU(cudaMemcpy(c->sin_t, stab.data(), stab.size() * 4, cudaMemcpyHostToDevice));
  CU(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  CU(cudaMallocHost(&c->h_stage, 4096));
  *out = guard.release();
  return NRC_OK;
}

extern "C" int nrc_ctx_new(const nrc_model* m, size_t ctx, nrc_ctx** out) { return ctx_create(m, ctx, 1, false, out); }

extern "C" int nrc_ctx_free(nrc_ctx* c) {
  if (!c) return NRC_OK;
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  // A graph holding NCCL calls is released before its communicator.
  if (c->gexec) cudaGraphExecDestroy(c->gexec);
  if (c->comm) nccl_api()->comm_destroy(c->comm);
  if (c->stream) cudaStreamDestroy(c->stream);
  if (c->h_stage) cudaFreeHost(c->h_stage);
  if (c->h_big) cudaFreeHost(c->h_big);
  if (c->arena) cudaFree(c->arena);
  delete c;
  return NRC_OK;
}

namespace {
// One GEMV over up to 64 tokens (groups of 8 per launch).
cudaError_t gemv_tokens(GemvArgs a, int nt, int x_ld_f, cudaStream_t s, bool pdl) {
  for (int t0 = 0; t0 < nt; t0 += 8) {
    GemvArgs b = a;
    b.nt = nt - t0 < 8 ? nt - t0 : 8;
    if (b.xf) b.xf = a.xf + (size_t)t0 * x_ld_f;
    if (a.xq) {
      const size_t blk = a.fmt == FMT_Q8_0 ? (size_t)(a.K / 32) * 34 : (size_t)(a.K / 256) * 292;
      b.xq = static_cast<const uint8_t*>(a.xq) + (size_t)t0 * blk;
    }
    if (t0 > 0) b.xq_out = nullptr;  // the sharing serves one group of at most 8 tokens
    if (nt > 8) b.yq_out = nullptr;  // and so does the SwiGLU output export
    for (int i = 0; i < b.nseg; i++)
      if (b.seg[i].y) b.seg[i].y = a.seg[i].y + (size_t)t0 * a.seg[i].ld;
    if (b.resid) b.resid = a.resid + (size_t)t0 * a.resid_ld;
    cudaError_t e = gemv_run(b, s, pdl);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

GemvArgs gemv_base(nrc_ctx* c, int fmt, int K) {
  GemvArgs a{};
  a.fmt = fmt;
  a.K = K;
  a.scale = 1.0f;
  a.err = &c->st->err;
  a.eps = c->eps;
  return a;
}

// One linear layer over nt tokens: x [nt][K] f32 (optionally RMS-normalised
// with norm_w) times up to three weight matrices of one format. EPI_SWIGLU
// takes gate = w[0] -> y[0] and up = w[1] (-> y[1] on the tensor-core path)
// and leaves silu(gate)*up in y[0]; EPI_RESID adds rs * result into c->x.
// Prefill chunks of more than 8 tokens over Q8_0 weights run on the tensor
// cores (mma.cu), everything else on the streaming GEMV (gemv.cu); both are
// bit-identical to the reference's scalar dots.
struct Lin {
  int fmt, K;
  const float* x;
  const float* norm_w;
  const uint8_t* w[3];
  float* y[3];
  int rows[3];
  int nseg;
  int epi;
  float scale = 1.0f;  // EPI_STORE: y = sum * scale
  // Streaming GEMV only: export the quantized input (xq_out), or take it
  // already quantized (xq, then x / norm_w are not read).
  uint8_t* xq_out = nullptr;
  const uint8_t* xq = nullptr;
  // EPI_SWIGLU on the streaming GEMV: also store the output as Q8_0 blocks in
  // yq_out when the launch can; *yq_done (set to 0 or 1) says whether it did.
  uint8_t* yq_out = nullptr;
  int* yq_done = nullptr;
  // Weights of the next linear layer, prefetched into L2 while this one runs.
  const uint8_t* pf;
  size_t pf_bytes;
};

// Bytes of a rows x K matrix of format fmt.
size_t mat_bytes(int fmt, int rows, int K) {
  const size_t bb = fmt == FMT_Q8_0 ? 34 : (fmt == FMT_Q4K ? 144 : 210);
  const size_t blk = fmt == FMT_Q8_0 ? 32 : 256;
  return (size_t)rows * (K / blk) * bb;
}
// One byte range covering matrices a and b when they sit back to back (the
// .nrm layout keeps a layer's tensors together), else just a.
void span2(const uint8_t* a, size_t na, const uint8_t* b, size_t nb, const uint8_t** p, size_t* n) {
  *p = a;
  *n = (b >= a && b <= a + na + 256) ? (size_t)(b - a) + nb : na;
}

cudaError_t linear(nrc_ctx* c, const Lin& L, int nt) {
  cudaStream_t s = c->stream;
  const bool pdl = c->pdl;
  // K-quant chunks of more than 8 tokens: tensor cores (mma_kq.cu), one launch per matrix.
  bool kq = nt > 8 && L.fmt != FMT_Q8_0 && L.K % 256 == 0 && (size_t)L.K * 4 <= 64 * 1024;
  for (int i = 0; i < L.nseg; i++) kq = kq && (reinterpret_cast<uintptr_t>(L.w[i]) & 15) == 0;
  if (kq) {
    const int NS = mma_kq_ns(L.fmt), ntg = (nt + NS - 1) / NS;
    MmaKqActArgs qa{L.x, L.K, L.norm_w, c->eps, nt, L.K, NS, ntg, c->mxq, c->mxd, c->mxb, L.fmt == FMT_Q6K ? 1 : 0};
    cudaError_t e = mma_kq_act_run(qa, s, pdl);
    if (e) return e;
    MmaKqArgs m{};
    m.fmt = L.fmt;
    for (int i = 0; i < L.nseg; i++) m.seg[i] = MmaSeg{L.w[i], L.y[i], L.rows[i], L.rows[i]};
    m.nseg = L.nseg;
    m.K = L.K;
    m.xq = c->mxq;
    m.xd = c->mxd;
    m.xb = c->mxb;
    m.nt = nt;
    m.NS = NS;
    m.ntg = ntg;
    m.epi = L.epi == EPI_RESID ? EPI_RESID : EPI_STORE;
    m.scale = L.scale;
    m.resid = c->x;
    m.resid_ld = c->dim;
    m.rs = c->rs;
    m.err = &c->st->err;
    if ((e = mma_kq_run(m, s, pdl))) return e;
    if (L.epi == EPI_SWIGLU) return op_swiglu(L.y[0], L.y[1], (size_t)nt * L.rows[0], s);
    return cudaSuccess;
  }
  bool mma = nt > 8 && L.fmt == FMT_Q8_0 && L.K % 256 == 0 && L.K <= 16384;
  for (int i = 0; i < L.nseg; i++) mma = mma && (reinterpret_cast<uintptr_t>(L.w[i]) & 15) == 0;
  if (mma) {
    int tiles = 0;
    for (int i = 0; i < L.nseg; i++) tiles += (L.rows[i] + 127) / 128;
    int NS, ntg;
    mma_choose(tiles, nt, &NS, &ntg);
    MmaActArgs qa{L.x, L.K, L.norm_w, c->eps, nt, L.K, NS, ntg, c->mxq, c->mxd};
    cudaError_t e = mma_quant_act_run(qa, s, pdl);
    if (e) return e;
    MmaArgs m{};
    for (int i = 0; i < L.nseg; i++) m.seg[i] = MmaSeg{L.w[i], L.y[i], L.rows[i], L.rows[i]};
    m.nseg = L.nseg;
    m.K = L.K;
    m.xq = c->mxq;
    m.xd = c->mxd;
    m.nt = nt;
    m.NS = NS;
    m.ntg = ntg;
    m.epi = L.epi == EPI_RESID ? EPI_RESID : EPI_STORE;
    m.scale = L.scale;
    m.resid = c->x;
    m.resid_ld = c->dim;
    m.rs = c->rs;
    m.err = &c->st->err;
    if ((e = mma_q8_run(m, s, pdl))) return e;
    if (L.epi == EPI_SWIGLU) return op_swiglu(L.y[0], L.y[1], (size_t)nt * L.rows[0], s);
    return cudaSuccess;
  }
  GemvArgs a = gemv_base(c, L.fmt, L.K);
  a.scale = L.scale;
  if (L.xq) {
    a.xq = L.xq;
  } else {
    a.xf = L.x;
    a.xf_ld = L.K;
    a.norm_w = L.norm_w;
    a.xq_out = L.xq_out;
  }
  a.epi = L.epi;
  for (int i = 0; i < L.nseg; i++) a.seg[i] = GemvSegArg{L.w[i], L.y[i], L.rows[i], L.rows[i]};
  a.nseg = L.nseg;
  if (L.epi == EPI_SWIGLU) {
    a.pair = 1;
    a.seg[1].y = nullptr;
    a.yq_out = L.yq_out;
    a.yq_done = L.yq_done;
  }
  if (L.epi == EPI_RESID) {
    a.resid = c->x;
    a.resid_ld = c->dim;
    a.rs = c->rs;
  }
  a.pf = L.pf;
  a.pf_bytes = L.pf_bytes;
  a.fast_norm = c->fast && nt == 1;
  return gemv_tokens(a, nt, L.K, s, pdl);
}

// The tokens of one pass of a context of several sequences: token t is id
// ids[t] at position pos[t] of sequence seq[t]; the classifier runs on the
// nrows tokens rows[0..nrows) (the last token of each sequence that ends in
// this pass), whose sequences advance to position pos + 1.
struct Pass {
  const uint32_t* ids;
  const uint32_t* pos;
  const uint32_t* seq;
  const uint32_t* rows;
  int nrows;
};

// Enqueue one forward pass over nt tokens (infer.rs:510-595 for nt == 1,
// infer.rs:601-750 otherwise): one sequence at positions st->pos .. +nt-1
// (bp null), or the tokens of `bp` over several sequences.
// Bytes of one row of a K-column matrix of format fmt.
size_t row_bytes(int fmt, int K) { return mat_bytes(fmt, 1, K); }

// Tensor parallelism: all-gather this rank's compact part [nt][chunk] (in
// tp_send) and spread every rank's part into dst [nt][ld] (resid: dst +=
// rs * part, the residual add of the single-GPU epilogue).
cudaError_t tp_gather(nrc_ctx* c, float* dst, int ld, int chunk, int nt, int resid) {
  const NcclApi* api = nccl_api();
  const ncclResult_t r =
      api->all_gather(c->tp_send, c->tp_recv, (size_t)nt * chunk, ncclFloat32, c->comm, c->stream);
  if (r != ncclSuccess) {
    fail(NRC_ERR_CUDA, "ncclAllGather: %s", api->error_string(r));
    return cudaErrorUnknown;
  }
  return tp_unpack_run(c->tp_recv, dst, ld, chunk, nt, c->sh.n, resid, c->rs, c->stream);
}

// Enqueue one forward pass over nt tokens (infer.rs:510-595 for nt == 1,
// infer.rs:601-750 otherwise): one sequence at positions st->pos .. +nt-1
// (bp null), or the tokens of `bp` over several sequences. Under tensor
// parallelism every linear layer computes this rank's rows (Shard) and the
// activations the next layer needs whole are all-gathered.
cudaError_t enqueue_step(nrc_ctx* c, int nt, bool draw, const Pass* bp = nullptr) {
  cudaStream_t s = c->stream;
  const bool pdl = c->pdl;
  const Shard& sh = c->sh;
  const bool tp = sh.n > 1;
  const int hd = c->hd, ql = sh.nh * hd;
  cudaError_t e;
  EmbedArgs ea{c->embed, c->f_embed, c->dim, c->embed_scale, bp ? bp->ids : c->st->tok, nt, c->x, &c->st->key};
  if ((e = embed_run(ea, s, pdl))) return e;
  // Weight regions of each layer's linear layers, for the L2 prefetch hints.
  auto qkv_region = [&](const LayerW& w, const uint8_t** p, size_t* n) {
    if (tp) {
      *p = w.wq + (size_t)sh.h0 * hd * row_bytes(w.fq, c->dim);
      *n = mat_bytes(w.fq, ql, c->dim);
      return;
    }
    const uint8_t* pq;
    size_t nq;
    span2(w.wq, mat_bytes(w.fq, c->att_dim, c->dim), w.wk, mat_bytes(w.fk, c->kv_dim, c->dim), &pq, &nq);
    span2(pq, nq, w.wv, mat_bytes(w.fv, c->kv_dim, c->dim), p, n);
  };
  for (int l = 0; l < c->n_layers; l++) {
    const LayerW& w = c->L[l];
    const uint8_t* wo = w.wo + (size_t)sh.d0 * row_bytes(w.fo, c->att_dim);
    const uint8_t* wg = w.wg + (size_t)sh.f0 * row_bytes(w.fg, c->dim);
    const uint8_t* wu = w.wu + (size_t)sh.f0 * row_bytes(w.fu, c->dim);
    const uint8_t* wd = w.wd + (size_t)sh.d0 * row_bytes(w.fd, c->ffn);
    const uint8_t *pf_o = wo, *pf_gu, *pf_d = wd, *pf_next;
    size_t n_o = mat_bytes(w.fo, sh.dn, c->att_dim), n_gu, n_d = mat_bytes(w.fd, sh.dn, c->ffn), n_next;
    span2(wg, mat_bytes(w.fg, sh.fn, c->dim), wu, mat_bytes(w.fu, sh.fn, c->dim), &pf_gu, &n_gu);
    if (l + 1 < c->n_layers) {
      qkv_region(c->L[l + 1], &pf_next, &n_next);
    } else {
      pf_next = c->out_w + (size_t)sh.v0 * row_bytes(c->f_out, c->dim);  // the classifier: its first 48 MB
      n_next = std::min(mat_bytes(c->f_out, sh.vn, c->dim), (size_t)48 << 20);
    }
    // QKV (infer.rs:527-531 / 620-637): rmsnorm + activation quantization fused
    // into the consumer; one launch per weight format; this rank's heads.
    {
      const uint8_t* ws[3] = {w.wq + (size_t)sh.h0 * hd * row_bytes(w.fq, c->dim),
                              w.wk + (size_t)sh.kv0 * hd * row_bytes(w.fk, c->dim),
                              w.wv + (size_t)sh.kv0 * hd * row_bytes(w.fv, c->dim)};
      const int fs[3] = {w.fq, w.fk, w.fv};
      float* ys[3] = {c->q, c->k, c->v};
      const int rows[3] = {ql, c->kvl, c->kvl};
      bool done[3] = {false, false, false};
      // Q4_K and Q6_K launches both read Q8_K activations: the first launch
      // exports them (at most 8 tokens), the next one reads them back.
      const bool kq_mix = nt <= 8 && fs[0] != FMT_Q8_0 && fs[1] != FMT_Q8_0 && fs[2] != FMT_Q8_0 &&
                          !(fs[0] == fs[1] && fs[1] == fs[2]);
      bool first = true;
      for (int i = 0; i < 3; i++) {
        if (done[i]) continue;
        Lin L{};
        L.fmt = fs[i];
        L.K = c->dim;
        L.x = c->x;
        L.norm_w = w.attn_norm;
        L.epi = EPI_STORE;
        L.pf = pf_o;
        L.pf_bytes = n_o;
        if (kq_mix) {
          if (first)
            L.xq_out = c->xsh;
          else
            L.xq = c->xsh;
          first = false;
        }
        for (int j = i; j < 3; j++)
          if (!done[j] && fs[j] == fs[i]) {
            L.w[L.nseg] = ws[j];
            L.y[L.nseg] = ys[j];
            L.rows[L.nseg++] = rows[j];
            done[j] = true;
          }
        if ((e = linear(c, L, nt))) return e;
      }
    }
    const size_t seq_stride = c->ctx * (size_t)c->kvl;
    uint16_t* kc_l = c->kc + (size_t)l * c->n_seqs * seq_stride;
    uint16_t* vc_l = c->vc + (size_t)l * c->n_seqs * seq_stride;
    AttnArgs aa{};
    aa.q = c->q;
    aa.out = tp ? c->tp_send : c->att;
    aa.kcache = kc_l;
    aa.vcache = vc_l;
    aa.scale = c->att_scale;
    aa.nt = nt;
    aa.n_heads = sh.nh;
    aa.n_kv_heads = sh.nkv;
    aa.head_dim = hd;
    aa.ctx = (int)c->ctx;
    aa.pos_dev = &c->st->pos;
    if (bp) {
      aa.pos_tok = bp->pos;
      aa.seq_tok = bp->seq;
      aa.seq_stride = seq_stride;
    }
    if (nt == 1 && !bp) {
      // Decode: per-head norms, RoPE and the KV append fused into attention.
      aa.fused = 1;
      aa.k = c->k;
      aa.v = c->v;
      aa.q_norm = w.q_norm;
      aa.k_norm = w.k_norm;
      aa.eps = c->eps;
      aa.cos_tab = c->cos_t;
      aa.sin_tab = c->sin_t;
      aa.style = c->style;
      // A Q8_0 output projection takes the attention output already quantized.
      if (w.fo == FMT_Q8_0 && !tp) aa.xq_out = c->xsh;
    } else {
      RopeArgs ra{c->q, c->k, c->v, w.q_norm, w.k_norm, c->eps, c->cos_t, c->sin_t, c->style, kc_l, vc_l,
                  nt, sh.nh, sh.nkv, hd, (int)c->ctx, &c->st->pos};
      if (bp) {
        ra.pos_tok = bp->pos;
        ra.seq_tok = bp->seq;
        ra.seq_stride = seq_stride;
      }
      if ((e = rope_append_run(ra, s, pdl))) return e;
    }
    if ((e = attention_run(aa, s, pdl, c->fast && nt == 1 && !bp))) return e;
    if (tp && (e = tp_gather(c, c->att, c->att_dim, ql, nt, 0))) return e;
    {  // output projection + residual (infer.rs:574-575)
      Lin L{};
      L.fmt = w.fo;
      L.K = c->att_dim;
      L.x = c->att;
      L.xq = aa.xq_out;  // quantized by the attention kernel (fused decode, Q8_0), else null
      L.w[0] = wo;
      L.y[0] = c->tp_send;
      L.rows[0] = sh.dn;
      L.nseg = 1;
      L.epi = tp ? EPI_STORE : EPI_RESID;
      L.pf = pf_gu;
      L.pf_bytes = n_gu;
      if ((e = linear(c, L, nt))) return e;
      if (tp && (e = tp_gather(c, c->x, c->dim, sh.dn, nt, 1))) return e;
    }
    int h_quantized = 0;  // the SwiGLU output also left in xsh as Q8_0 blocks
    {  // SwiGLU MLP gate/up (infer.rs:577-581)
      float* g = tp ? c->tp_send : c->g;
      Lin L{};
      L.fmt = w.fg;
      L.K = c->dim;
      L.x = c->x;
      L.norm_w = w.ffn_norm;
      L.w[0] = wg;
      L.y[0] = g;
      L.rows[0] = sh.fn;
      L.nseg = 1;
      L.epi = EPI_STORE;
      L.pf = pf_d;
      L.pf_bytes = n_d;
      if (w.fg == w.fu) {
        L.w[1] = wu;
        L.y[1] = c->u;
        L.rows[1] = sh.fn;
        L.nseg = 2;
        L.epi = EPI_SWIGLU;
        if (w.fd == FMT_Q8_0 && !tp) {  // a Q8_0 down projection takes it quantized
          L.yq_out = c->xsh;
          L.yq_done = &h_quantized;
        }
        if ((e = linear(c, L, nt))) return e;
      } else {
        if ((e = linear(c, L, nt))) return e;
        L.fmt = w.fu;
        L.w[0] = wu;
        L.y[0] = c->u;
        if ((e = linear(c, L, nt))) return e;
        if ((e = op_swiglu(g, c->u, (size_t)nt * sh.fn, s))) return e;
      }
      if (tp && (e = tp_gather(c, c->g, c->ffn, sh.fn, nt, 0))) return e;
    }
    {  // down projection + residual (infer.rs:582-583)
      Lin L{};
      L.fmt = w.fd;
      L.K = c->ffn;
      L.x = c->g;
      L.xq = h_quantized ? c->xsh : nullptr;
      L.w[0] = wd;
      L.y[0] = c->tp_send;
      L.rows[0] = sh.dn;
      L.nseg = 1;
      L.epi = tp ? EPI_STORE : EPI_RESID;
      L.pf = pf_next;
      L.pf_bytes = n_next;
      if ((e = linear(c, L, nt))) return e;
      if (tp && (e = tp_gather(c, c->x, c->dim, sh.dn, nt, 1))) return e;
    }
  }
  if (bp && bp->nrows == 0) return cudaSuccess;
  if (bp) {
    // Final norm + classifier on every sequence's last token of the pass, then
    // each row's greedy argmax (infer.rs:586-591, 740-746; sample.rs:33-35).
    if ((e = gather_rows_run(c->x, c->dim, bp->rows, bp->nrows, c->xl, s, pdl))) return e;
    Lin L{};
    L.fmt = c->f_out;
    L.K = c->dim;
    L.x = c->xl;
    L.norm_w = c->out_norm;
    L.w[0] = c->out_w;
    L.y[0] = c->blogits;
    L.rows[0] = c->vocab;
    L.nseg = 1;
    L.epi = EPI_STORE;
    L.scale = c->logit_recip;
    if ((e = linear(c, L, bp->nrows))) return e;
    return rows_argmax_run(c->blogits, c->vocab, bp->nrows, bp->rows, bp->seq, bp->pos, c->bpos, c->btok, c->bnext,
                           c->bhist, (int)c->ctx, s, pdl);
  }
  // Final norm + classifier on the last token, fused greedy argmax (infer.rs:586-591, 740-746);
  // under tensor parallelism this rank's vocabulary rows, then the logits
  // all-gathered and the greedy key reduced (max) over ranks.
  {
    GemvArgs a = gemv_base(c, c->f_out, c->dim);
    a.xf = c->x + (size_t)(nt - 1) * c->dim;
    a.xf_ld = c->dim;
    a.norm_w = c->out_norm;
    float* lg = tp ? c->tp_send : c->logits;
    a.seg[0] = GemvSegArg{c->out_w + (size_t)sh.v0 * row_bytes(c->f_out, c->dim), lg, sh.vn, sh.vn};
    a.nseg = 1;
    a.epi = EPI_ARGMAX;
    a.scale = c->logit_recip;
    a.argmax_key = &c->st->key;
    a.argmax_base = sh.v0;
    a.nt = 1;
    a.fast_norm = c->fast && nt == 1;
    if ((e = gemv_run(a, s, pdl))) return e;
    if (tp) {
      if ((e = tp_gather(c, c->logits, c->vocab, sh.vn, 1, 0))) return e;
      const NcclApi* api = nccl_api();
      const ncclResult_t r = api->all_reduce(&c->st->key, &c->st->key, 1, ncclUint64, ncclMax, c->comm, s);
      if (r != ncclSuccess) {
        fail(NRC_ERR_CUDA, "ncclAllReduce: %s", api->error_string(r));
        return cudaErrorUnknown;
      }
    }
  }
  if (c->sampling && draw) {
    // Sampler::sample (sample.rs:32-96) replaces the greedy key with its draw.
    SampleArgs sa{c->logits, c->vocab, c->temperature, c->top_p, &c->st->rng, c->samp, nullptr, &c->st->key};
    if ((e = sample_run(sa, s, pdl))) return e;
  }
  return step_finish_run(&c->st->pos, (uint32_t)nt, &c->st->key, &c->st->next, c->st->tok, c->hist, s, pdl);
}

int finish_sync(nrc_ctx* c, float* logits_host, uint32_t* next_host, size_t advance) {
  if (logits_host)
    CU(cudaMemcpyAsync(logits_host, c->logits, (size_t)c->vocab * 4, cudaMemcpyDeviceToHost, c->stream));
  CU(cudaMemcpyAsync(c->h_stage, &c->st->next, 8, cudaMemcpyDeviceToHost, c->stream));
  CU(cudaStreamSynchronize(c->stream));
  const uint32_t next = c->h_stage[0], err = c->h_stage[1];
  c->pos += advance;
  if (err) return fail(NRC_ERR_DEVICE, "kernel wait expired (error bits 0x%x)", err);
  if (next_host) *next_host = next;
  return NRC_OK;
}

int ensure_graph(nrc_ctx* c) {
  if (c->gexec) return NRC_OK;
  cudaGraph_t g = nullptr;
  CU(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  cudaError_t e = enqueue_step(c, 1, true);
  cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
  if (e != cudaSuccess || e2 != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    return fail(NRC_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(e != cudaSuccess ? e : e2));
  }
  e = cudaGraphInstantiate(&c->gexec, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    c->gexec = nullptr;
    return fail(NRC_ERR_CUDA, "graph instantiate failed: %s", cudaGetErrorString(e));
  }
  return NRC_OK;
}
}  // namespace

static int not_batch(const nrc_ctx* c) {
  if (!c) return fail(NRC_ERR_INVALID, "null context");
  if (c->batch) return fail(NRC_ERR_INVALID, "multi-sequence context: use the nrc_batch_* entry points");
  return NRC_OK;
}

extern "C" int nrc_ctx_forward(nrc_ctx* c, uint32_t token, float* logits_host, uint32_t* next_host) {
  if (int rc = not_batch(c)) return rc;
  if (c->pos + c->pending >= c->ctx) return fail(NRC_ERR_CTX_FULL, "context window exhausted");
  if (token >= (uint32_t)c->vocab) return fail(NRC_ERR_BAD_TOKEN, "token %u >= vocab %d", token, c->vocab);
  CU(cudaSetDevice(c->device));
  if (!c->gexec) {
    // First step runs eagerly (warms per-kernel caches), later ones replay the graph.
    c->h_stage[16] = token;
    CU(cudaMemcpyAsync(c->st->tok, &c->h_stage[16], 4, cudaMemcpyHostToDevice, c->stream));
    CU(enqueue_step(c, 1, true));
    int rc = finish_sync(c, logits_host, next_host, 1);
    if (rc) return rc;
    return ensure_graph(c);
  }
  c->h_stage[16] = token;
  CU(cudaMemcpyAsync(c->st->tok, &c->h_stage[16], 4, cudaMemcpyHostToDevice, c->stream));
  CU(cudaGraphLaunch(c->gexec, c->stream));
  return finish_sync(c, logits_host, next_host, 1);
}

static int prefill_chunk_impl(nrc_ctx* c, const uint32_t* tokens, size_t n, float* logits_host, uint32_t* next_host,
                              bool draw) {
  if (int rc = not_batch(c)) return rc;
  if (!tokens) return fail(NRC_ERR_INVALID, "null argument");
  if (n < 1 || n > NRC_MAX_BATCH) return fail(NRC_ERR_BAD_BATCH, "prefill chunk of %zu tokens", n);
  if (c->pos + c->pending + n > c->ctx) return fail(NRC_ERR_CTX_FULL, "context window exhausted");
  for (size_t i = 0; i < n; i++)
    if (tokens[i] >= (uint32_t)c->vocab) return fail(NRC_ERR_BAD_TOKEN, "token %u >= vocab %d", tokens[i], c->vocab);
  CU(cudaSetDevice(c->device));
  memcpy(&c->h_stage[16], tokens, n * 4);
  CU(cudaMemcpyAsync(c->st->tok, &c->h_stage[16], n * 4, cudaMemcpyHostToDevice, c->stream));
  CU(enqueue_step(c, (int)n, draw));
  int rc = finish_sync(c, logits_host, next_host, n);
  if (rc) return rc;
  return ensure_graph(c);
}

extern "C" int nrc_ctx_prefill_chunk(nrc_ctx* c, const uint32_t* tokens, size_t n, float* logits_host,
                                     uint32_t* next_host) {
  return prefill_chunk_impl(c, tokens, n, logits_host, next_host, true);
}

extern "C" int nrc_ctx_prefill(nrc_ctx* c, const uint32_t* tokens, size_t n, float* logits_host, uint32_t* next_host) {
  if (int rc = not_batch(c)) return rc;
  if (!tokens) return fail(NRC_ERR_INVALID, "null argument");
  if (n == 0) return fail(NRC_ERR_BAD_BATCH, "empty prompt");
  if (c->pos + c->pending + n > c->ctx) return fail(NRC_ERR_CTX_FULL, "context window exhausted");
  for (size_t i = 0; i < n; i += NRC_MAX_BATCH) {
    const size_t b = n - i < (size_t)NRC_MAX_BATCH ? n - i : (size_t)NRC_MAX_BATCH;
    const bool last = i + b == n;
    int rc = prefill_chunk_impl(c, tokens + i, b, last ? logits_host : nullptr, last ? next_host : nullptr, last);
    if (rc) return rc;
  }
  return NRC_OK;
}

extern "C" int nrc_ctx_generate(nrc_ctx* c, uint32_t first, size_t n, uint32_t* out_host) {
  if (int rc = not_batch(c)) return rc;
  if (!out_host && n) return fail(NRC_ERR_INVALID, "null argument");
  if (n == 0) return NRC_OK;
  if (c->pos + c->pending + n > c->ctx) return fail(NRC_ERR_CTX_FULL, "context window exhausted");
  if (first >= (uint32_t)c->vocab) return fail(NRC_ERR_BAD_TOKEN, "token %u >= vocab %d", first, c->vocab);
  CU(cudaSetDevice(c->device));
  const size_t p0 = c->pos;
  uint32_t next = 0;
  int rc = nrc_ctx_forward(c, first, nullptr, &next);  // eager first step + graph capture
  if (rc) return rc;
  for (size_t i = 1; i < n; i++) CU(cudaGraphLaunch(c->gexec, c->stream));
  CU(cudaMemcpyAsync(out_host, c->hist + p0, n * 4, cudaMemcpyDeviceToHost, c->stream));
  rc = finish_sync(c, nullptr, nullptr, n - 1);
  return rc;
}

extern "C" int nrc_ctx_decode_async(nrc_ctx* c, size_t n) {
  if (int rc = not_batch(c)) return rc;
  if (c->pos + c->pending + n > c->ctx) return fail(NRC_ERR_CTX_FULL, "context window exhausted");
  if (!c->gexec) return fail(NRC_ERR_INVALID, "no decode step yet: call nrc_ctx_forward or nrc_ctx_prefill first");
  CU(cudaSetDevice(c->device));
  for (size_t i = 0; i < n; i++) CU(cudaGraphLaunch(c->gexec, c->stream));
  c->pending += n;
  return NRC_OK;
}

extern "C" int nrc_ctx_sync(nrc_ctx* c, uint32_t* next_host) {
  if (!c) return fail(NRC_ERR_INVALID, "null context");
  CU(cudaSetDevice(c->device));
  const size_t adv = c->pending;
  c->pending = 0;
  return finish_sync(c, nullptr, next_host, adv);
}

// Decode arithmetic: NRC_MODE_EXACT (the reference's summation order, bit for
// bit) or NRC_MODE_FAST (tree reductions within the north star's tolerance).
extern "C" int nrc_ctx_set_mode(nrc_ctx* c, int mode) {
  if (int rc = not_batch(c)) return rc;
  if (mode != NRC_MODE_EXACT && mode != NRC_MODE_FAST) return fail(NRC_ERR_INVALID, "unknown mode %d", mode);
  CU(cudaSetDevice(c->device));
  CU(cudaStreamSynchronize(c->stream));
  const bool fast = mode == NRC_MODE_FAST;
  if (fast == c->fast) return NRC_OK;
  c->fast = fast;
  if (c->gexec) {
    cudaGraphExecDestroy(c->gexec);
    c->gexec = nullptr;
    return ensure_graph(c);
  }
  return NRC_OK;
}

// Sampler::new (sample.rs:15-21) attached to the context: rng = seed | 1.
extern "C" int nrc_ctx_set_sampler(nrc_ctx* c, float temperature, float top_p, uint64_t seed) {
  if (int rc = not_batch(c)) return rc;
  if (c->vocab > SAMPLE_MAX_N) return fail(NRC_ERR_INVALID, "vocabulary of %d exceeds the sampler's %d", c->vocab, SAMPLE_MAX_N);
  CU(cudaSetDevice(c->device));
  CU(cudaStreamSynchronize(c->stream));
  c->temperature = temperature;
  c->top_p = top_p;
  c->sampling = !(temperature <= 0.0f);
  const unsigned long long rng = (unsigned long long)(seed | 1ull);
  CU(cudaMemcpy(&c->st->rng, &rng, 8, cudaMemcpyHostToDevice));
  // The decode graph is recaptured with (or without) the sampler kernels.
  if (c->gexec) {
    cudaGraphExecDestroy(c->gexec);
    c->gexec = nullptr;
    return ensure_graph(c);
  }
  return NRC_OK;
}

extern "C" int nrc_ctx_reset(nrc_ctx* c) {
  if (!c) return fail(NRC_ERR_INVALID, "null context");
  CU(cudaSetDevice(c->device));
  CU(cudaStreamSynchronize(c->stream));
  c->pos = 0;
  c->pending = 0;
  CU(cudaMemsetAsync(&c->st->pos, 0, 4, c->stream));
  if (c->batch) {
    std::fill(c->hpos.begin(), c->hpos.end(), (size_t)0);
    CU(cudaMemsetAsync(c->bpos, 0, c->n_seqs * 4, c->stream));
  }
  CU(cudaStreamSynchronize(c->stream));
  return NRC_OK;
}
extern "C" size_t nrc_ctx_pos(const nrc_ctx* c) { return c ? c->pos : 0; }
extern "C" size_t nrc_ctx_remaining(const nrc_ctx* c) { return c ? c->ctx - c->pos - c->pending : 0; }
extern "C" int nrc_ctx_logits_device(const nrc_ctx* c, const float** out) {
  if (!c || !out) return fail(NRC_ERR_INVALID, "null argument");
  *out = c->logits;
  return NRC_OK;
}
extern "C" void* nrc_ctx_stream(const nrc_ctx* c) { return c ? (void*)c->stream : nullptr; }
extern "C" int nrc_ctx_kv(nrc_ctx* c, size_t layer, size_t pos, uint16_t* k_host, uint16_t* v_host) {
  if (!c || !k_host || !v_host) return fail(NRC_ERR_INVALID, "null argument");
  if (layer >= (size_t)c->n_layers || pos >= c->ctx) return fail(NRC_ERR_INVALID, "kv index out of range");
  CU(cudaSetDevice(c->device));
  const size_t off = (layer * c->ctx + pos) * c->kvl;
  CU(cudaMemcpyAsync(k_host, c->kc + off, c->kvl * 2, cudaMemcpyDeviceToHost, c->stream));
  CU(cudaMemcpyAsync(v_host, c->vc + off, c->kvl * 2, cudaMemcpyDeviceToHost, c->stream));
  CU(cudaStreamSynchronize(c->stream));
  return NRC_OK;
}

// ------------------------------------------------------------ several sequences
// Independent sequences decoded together (the batched-stream workload): every
// linear layer runs once per pass over all the pass's tokens, attention runs
// per (sequence, head) over that sequence's own KV cache. Results per
// sequence are bit-identical to a single-sequence context (every per-token
// reduction keeps the reference's order; nothing mixes tokens).
extern "C" int nrc_batch_new(const nrc_model* m, size_t ctx, size_t n_seqs, nrc_ctx** out) {
  return ctx_create(m, ctx, n_seqs, true, out);
}

static int is_batch(const nrc_ctx* c) {
  if (!c) return fail(NRC_ERR_INVALID, "null context");
  if (!c->batch) return fail(NRC_ERR_INVALID, "not a multi-sequence context (nrc_batch_new)");
  return NRC_OK;
}

static int batch_sync(nrc_ctx* c) {
  CU(cudaMemcpyAsync(c->h_stage, &c->st->err, 4, cudaMemcpyDeviceToHost, c->stream));
  CU(cudaStreamSynchronize(c->stream));
  if (c->h_stage[0]) return fail(NRC_ERR_DEVICE, "kernel wait expired (error bits 0x%x)", c->h_stage[0]);
  return NRC_OK;
}

// Prefill of every sequence: prompts back to back in `tokens`, lens[s] >= 1
// tokens for sequence s (continuing at its current position). Tokens are
// packed into passes of up to the context's pass size, several sequences per
// pass (infer.rs:601-750 per sequence). next_host[s] (optional) receives
// each sequence's greedy choice after its prompt.
extern "C" int nrc_batch_prefill(nrc_ctx* c, const uint32_t* tokens, const uint32_t* lens, uint32_t* next_host) {
  if (int rc = is_batch(c)) return rc;
  if (!tokens || !lens) return fail(NRC_ERR_INVALID, "null argument");
  const size_t S = c->n_seqs, B = c->max_tok;
  size_t total = 0;
  for (size_t q = 0; q < S; q++) {
    if (lens[q] < 1) return fail(NRC_ERR_BAD_BATCH, "sequence %zu: empty prompt", q);
    if (c->hpos[q] + lens[q] > c->ctx) return fail(NRC_ERR_CTX_FULL, "sequence %zu: context window exhausted", q);
    total += lens[q];
  }
  for (size_t i = 0; i < total; i++)
    if (tokens[i] >= (uint32_t)c->vocab) return fail(NRC_ERR_BAD_TOKEN, "token %u >= vocab %d", tokens[i], c->vocab);
  CU(cudaSetDevice(c->device));
  uint32_t* hid = c->h_big;
  uint32_t* hp = hid + B;
  uint32_t* hs = hp + B;
  uint32_t* hr = hs + B;
  size_t q = 0, j = 0, off = 0;  // sequence, token within it, offset in `tokens`
  while (q < S) {
    int nt = 0, nrows = 0;
    while (q < S && (size_t)nt < B) {
      hid[nt] = tokens[off];
      hp[nt] = (uint32_t)(c->hpos[q] + j);
      hs[nt] = (uint32_t)q;
      nt++;
      off++;
      if (++j == lens[q]) {
        hr[nrows++] = (uint32_t)(nt - 1);
        c->hpos[q] += lens[q];
        q++;
        j = 0;
      }
    }
    CU(cudaMemcpyAsync(c->ctok, hid, nt * 4, cudaMemcpyHostToDevice, c->stream));
    CU(cudaMemcpyAsync(c->cpos, hp, nt * 4, cudaMemcpyHostToDevice, c->stream));
    CU(cudaMemcpyAsync(c->cseq, hs, nt * 4, cudaMemcpyHostToDevice, c->stream));
    if (nrows) CU(cudaMemcpyAsync(c->crow, hr, nrows * 4, cudaMemcpyHostToDevice, c->stream));
    const Pass pass{c->ctok, c->cpos, c->cseq, c->crow, nrows};
    CU(enqueue_step(c, nt, false, &pass));
    if (int rc = batch_sync(c)) return rc;  // the staging buffer is refilled by the next pass
  }
  if (next_host) {
    CU(cudaMemcpyAsync(next_host, c->bnext, S * 4, cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
  }
  return NRC_OK;
}

static int ensure_batch_graph(nrc_ctx* c) {
  if (c->gexec) return NRC_OK;
  const Pass pass{c->btok, c->bpos, c->biota, c->biota, (int)c->n_seqs};
  cudaGraph_t g = nullptr;
  CU(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  cudaError_t e = enqueue_step(c, (int)c->n_seqs, false, &pass);
  cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
  if (e != cudaSuccess || e2 != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    return fail(NRC_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(e != cudaSuccess ? e : e2));
  }
  e = cudaGraphInstantiate(&c->gexec, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    c->gexec = nullptr;
    return fail(NRC_ERR_CUDA, "graph instantiate failed: %s", cudaGetErrorString(e));
  }
  return NRC_OK;
}

static int batch_check_step(nrc_ctx* c, size_t n) {
  for (size_t q = 0; q < c->n_seqs; q++) {
    if (c->hpos[q] == 0) return fail(NRC_ERR_INVALID, "sequence %zu has no prompt yet: call nrc_batch_prefill", q);
    if (c->hpos[q] + n > c->ctx) return fail(NRC_ERR_CTX_FULL, "sequence %zu: context window exhausted", q);
  }
  return NRC_OK;
}

// One decode step of every sequence (InferCtx::forward per sequence,
// infer.rs:510-595): each consumes the token it chose last, on the device.
// logits_host (optional) receives [n_seqs][vocab], next_host [n_seqs].
extern "C" int nrc_batch_step(nrc_ctx* c, float* logits_host, uint32_t* next_host) {
  if (int rc = is_batch(c)) return rc;
  if (int rc = batch_check_step(c, 1)) return rc;
  CU(cudaSetDevice(c->device));
  if (int rc = ensure_batch_graph(c)) return rc;
  CU(cudaGraphLaunch(c->gexec, c->stream));
  for (auto& p : c->hpos) p++;
  if (logits_host)
    CU(cudaMemcpyAsync(logits_host, c->blogits, c->n_seqs * (size_t)c->vocab * 4, cudaMemcpyDeviceToHost,
                       c->stream));
  if (next_host) CU(cudaMemcpyAsync(next_host, c->bnext, c->n_seqs * 4, cudaMemcpyDeviceToHost, c->stream));
  return batch_sync(c);
}

// n greedy decode steps of every sequence on the device (one graph replay per
// step); out_host[s * n + i] = sequence s's choice after step i.
extern "C" int nrc_batch_generate(nrc_ctx* c, size_t n, uint32_t* out_host) {
  if (int rc = is_batch(c)) return rc;
  if (!out_host && n) return fail(NRC_ERR_INVALID, "null argument");
  if (n == 0) return NRC_OK;
  if (int rc = batch_check_step(c, n)) return rc;
  CU(cudaSetDevice(c->device));
  if (int rc = ensure_batch_graph(c)) return rc;
  std::vector<size_t> p0 = c->hpos;
  for (size_t i = 0; i < n; i++) CU(cudaGraphLaunch(c->gexec, c->stream));
  for (size_t q = 0; q < c->n_seqs; q++) {
    CU(cudaMemcpyAsync(out_host + q * n, c->bhist + q * c->ctx + p0[q], n * 4, cudaMemcpyDeviceToHost, c->stream));
    c->hpos[q] += n;
  }
  return batch_sync(c);
}

// Enqueue n decode steps of every sequence without waiting (pair with
// nrc_batch_sync): the device-resident loop the batched throughput is timed on.
extern "C" int nrc_batch_decode_async(nrc_ctx* c, size_t n) {
  if (int rc = is_batch(c)) return rc;
  if (int rc = batch_check_step(c, n)) return rc;
  CU(cudaSetDevice(c->device));
  if (int rc = ensure_batch_graph(c)) return rc;
  for (size_t i = 0; i < n; i++) CU(cudaGraphLaunch(c->gexec, c->stream));
  for (auto& p : c->hpos) p += n;
  return NRC_OK;
}
extern "C" int nrc_batch_sync(nrc_ctx* c, uint32_t* next_host) {
  if (int rc = is_batch(c)) return rc;
  CU(cudaSetDevice(c->device));
  if (next_host) CU(cudaMemcpyAsync(next_host, c->bnext, c->n_seqs * 4, cudaMemcpyDeviceToHost, c->stream));
  return batch_sync(c);
}

extern "C" size_t nrc_batch_size(const nrc_ctx* c) { return c ? c->n_seqs : 0; }
extern "C" size_t nrc_batch_pos(const nrc_ctx* c, size_t seq) {
  return (c && c->batch && seq < c->n_seqs) ? c->hpos[seq] : 0;
}
extern "C" int nrc_batch_kv(nrc_ctx* c, size_t seq, size_t layer, size_t pos, uint16_t* k_host, uint16_t* v_host) {
  if (int rc = is_batch(c)) return rc;
  if (!k_host || !v_host) return fail(NRC_ERR_INVALID, "null argument");
  if (seq >= c->n_seqs || layer >= (size_t)c->n_layers || pos >= c->ctx) return fail(NRC_ERR_INVALID, "kv index out of range");
  CU(cudaSetDevice(c->device));
  const size_t off = ((layer * c->n_seqs + seq) * c->ctx + pos) * c->kvl;
  CU(cudaMemcpyAsync(k_host, c->kc + off, c->kvl * 2, cudaMemcpyDeviceToHost, c->stream));
  CU(cudaMemcpyAsync(v_host, c->vc + off, c->kvl * 2, cudaMemcpyDeviceToHost, c->stream));
  CU(cudaStreamSynchronize(c->stream));
  return NRC_OK;
}

// ------------------------------------------------------------ tensor parallelism
extern "C" int nrc_tp_unique_id(uint8_t* out) {
  if (!out) return fail(NRC_ERR_INVALID, "null argument");
  const NcclApi* api = nccl_api();
  if (!api) return fail(NRC_ERR_CUDA, "tensor parallelism needs NCCL (libnccl.so.2 not found)");
  ncclUniqueId id;
  const ncclResult_t r = api->get_unique_id(&id);
  if (r != ncclSuccess) return fail(NRC_ERR_CUDA, "ncclGetUniqueId: %s", api->error_string(r));
  memcpy(out, &id, sizeof id);
  return NRC_OK;
}

extern "C" int nrc_tp_ctx_new(const nrc_model* m, size_t ctx, int nranks, int rank, const uint8_t* id, nrc_ctx** out) {
  if (!id) return fail(NRC_ERR_INVALID, "null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(NRC_ERR_INVALID, "rank %d of %d", rank, nranks);
  if (nranks == 1) return ctx_create(m, ctx, 1, false, out);
  return ctx_create(m, ctx, 1, false, out, nranks, rank, id);
}

extern "C" int nrc_tp_shard(const nrc_ctx* c, int32_t* out) {
  if (!c || !out) return fail(NRC_ERR_INVALID, "null argument");
  const Shard& sh = c->sh;
  const int32_t v[12] = {sh.n, sh.r, sh.h0, sh.nh, sh.kv0, sh.nkv, sh.d0, sh.dn, sh.f0, sh.fn, sh.v0, sh.vn};
  memcpy(out, v, sizeof v);
  return NRC_OK;
}
