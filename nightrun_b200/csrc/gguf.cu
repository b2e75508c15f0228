// GGUF ingestion: a GGUF v2/v3 file of a dense llama / qwen3 / granite model
// as a .nrm v3 blob, and a loader that converts and uploads it. Host code
// only; it follows the reference's converter (tools/nrconvert/src/gguf.rs:
// the GGUF reader; tools/nrconvert/src/main.rs:63-110 arch_verdict, 180-453
// the conversion) with two differences:
//   - the tokenizer section is left empty (tokenizer length 0): tokenization
//     is outside this library's path, and nothing on the forward path reads
//     the section;
//   - every condition the converter meets with a panic or exit(1) returns a
//     status code instead (NRC_ERR_TOO_SHORT for a truncated file,
//     NRC_ERR_BAD_MAGIC / NRC_ERR_BAD_VERSION for the GGUF header,
//     NRC_ERR_MISSING for a missing key or tensor, NRC_ERR_UNSUPPORTED for an
//     architecture, SSM/MoE feature or tensor type the converter rejects).
// The .nrm layout, tensor order, 64-byte data alignment and both CRCs are the
// converter's, so the data section and tensor table equal what it writes.
#include <stdint.h>
#include <string.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "nrcuda.h"

int nrc_fail_api(int code, const char* fmt, ...);  // the library's error slot (engine.cu)
namespace nrc {
uint32_t crc32_bytes(const uint8_t* d, size_t n);                    // crc32.rs:6-79 (engine.cu)
uint32_t crc32_update(uint32_t state, const uint8_t* d, size_t n);  // raw state, no final xor
}  // namespace nrc

namespace {

// GGML tensor types (gguf.rs:58-63).
constexpr uint32_t GGML_F32 = 0, GGML_F16 = 1, GGML_Q8_0 = 8, GGML_Q4_K = 12, GGML_Q5_K = 13, GGML_Q6_K = 14;
// .nrm v3 (crates/nr-model/src/format.rs): sizes, tensor kinds and dtypes.
constexpr size_t HEADER_SIZE = 192, NAME_LEN = 48, ENTRY_SIZE = 32, DATA_ALIGN = 64;
enum : uint16_t {
  TK_TOK_EMBED = 1, TK_OUTPUT_NORM = 2, TK_OUTPUT = 3, TK_ROPE_FREQS = 4, TK_ATTN_NORM = 10, TK_ATTN_Q = 11,
  TK_ATTN_K = 12, TK_ATTN_V = 13, TK_ATTN_O = 14, TK_FFN_NORM = 15, TK_FFN_GATE = 16, TK_FFN_UP = 17,
  TK_FFN_DOWN = 18, TK_ATTN_Q_NORM = 19, TK_ATTN_K_NORM = 20
};
enum : uint16_t { DT_F32 = 0, DT_Q8_0 = 1, DT_Q4K = 2, DT_Q6K = 3 };

// A metadata value: integers, floats and strings as read; arrays keep only
// their length (the converter reads no array element, only the token count).
struct Value {
  enum Kind { INT, UINT, FLOAT, STR, ARR, BOOL } kind = UINT;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  std::string s;
  uint64_t count = 0;
  uint32_t width = 0;  // bytes of the scalar as stored (the u32 view accepts u8/u16/u32/i32/u64)
  bool as_u32(uint32_t* out) const {  // gguf.rs:24-33
    if (kind == UINT && width <= 4) { *out = (uint32_t)u; return true; }
    if (kind == UINT && width == 8) {
      if (u > 0xffffffffull) return false;
      *out = (uint32_t)u;
      return true;
    }
    if (kind == INT && width == 4) {
      if (i < 0) return false;
      *out = (uint32_t)i;
      return true;
    }
    return false;
  }
  bool as_f32(float* out) const {  // gguf.rs:35-41
    if (kind != FLOAT) return false;
    *out = (float)f;
    return true;
  }
};

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;  // dims[0] = fastest (cols)
  uint32_t type = 0;
  uint64_t offset = 0;  // absolute offset in the file
  uint64_t size = 0;
};

struct Reader {
  const uint8_t* b;
  size_t n, pos = 0;
  bool ok = true;
  bool take(size_t k, const uint8_t** p) {
    if (!ok || k > n - pos) return ok = false;
    *p = b + pos;
    pos += k;
    return true;
  }
  template <class T>
  T get() {
    const uint8_t* p = nullptr;
    T v{};
    if (take(sizeof(T), &p)) memcpy(&v, p, sizeof(T));
    return v;
  }
  std::string str() {  // v2/v3: u64 length, then bytes
    const uint64_t len = get<uint64_t>();
    const uint8_t* p = nullptr;
    if (!ok || len > n - pos || !take((size_t)len, &p)) {
      ok = false;
      return {};
    }
    return std::string(reinterpret_cast<const char*>(p), (size_t)len);
  }
  // One value of GGUF type `ty` (gguf.rs:121-150); arrays recurse over their
  // elements (to move past them) and keep the count. `depth` bounds nesting.
  bool value(uint32_t ty, Value* v, int depth) {
    switch (ty) {
      case 0: v->kind = Value::UINT; v->width = 1; v->u = get<uint8_t>(); break;
      case 1: v->kind = Value::INT; v->width = 1; v->i = get<int8_t>(); break;
      case 2: v->kind = Value::UINT; v->width = 2; v->u = get<uint16_t>(); break;
      case 3: v->kind = Value::INT; v->width = 2; v->i = get<int16_t>(); break;
      case 4: v->kind = Value::UINT; v->width = 4; v->u = get<uint32_t>(); break;
      case 5: v->kind = Value::INT; v->width = 4; v->i = get<int32_t>(); break;
      case 6: v->kind = Value::FLOAT; v->width = 4; v->f = get<float>(); break;
      case 7: v->kind = Value::BOOL; v->width = 1; v->u = get<uint8_t>() != 0; break;
      case 8: v->kind = Value::STR; v->s = str(); break;
      case 9: {
        if (depth > 4) return ok = false;
        const uint32_t et = get<uint32_t>();
        const uint64_t count = get<uint64_t>();
        if (!ok) return false;
        v->kind = Value::ARR;
        v->count = count;
        Value e;
        for (uint64_t k = 0; k < count && ok; k++)
          if (!value(et, &e, depth + 1)) return false;
        break;
      }
      case 10: v->kind = Value::UINT; v->width = 8; v->u = get<uint64_t>(); break;
      case 11: v->kind = Value::INT; v->width = 8; v->i = get<int64_t>(); break;
      case 12: v->kind = Value::FLOAT; v->width = 8; v->f = get<double>(); break;
      default: return ok = false;  // the reference panics on an unknown type
    }
    return ok;
  }
};

// gguf.rs:82-92; 0 for a type the reference does not size.
bool tensor_bytes(uint32_t type, uint64_t nelem, uint64_t* out) {
  uint64_t per, blk;
  switch (type) {
    case GGML_F32: per = 4; blk = 1; break;
    case GGML_F16: per = 2; blk = 1; break;
    case GGML_Q8_0: per = 34; blk = 32; break;
    case GGML_Q4_K: per = 144; blk = 256; break;
    case GGML_Q5_K: per = 176; blk = 256; break;
    case GGML_Q6_K: per = 210; blk = 256; break;
    default: return false;
  }
  return !__builtin_mul_overflow(nelem / blk, per, out);
}

struct Gguf {
  std::unordered_map<std::string, Value> kv;
  std::vector<TensorInfo> tensors;
};

// gguf.rs:153-213.
int parse(const uint8_t* b, size_t n, Gguf* g) {
  Reader r{b, n};
  const uint8_t* magic = nullptr;
  if (!r.take(4, &magic)) return nrc_fail_api(NRC_ERR_TOO_SHORT, "GGUF: shorter than its magic");
  if (memcmp(magic, "GGUF", 4) != 0) return nrc_fail_api(NRC_ERR_BAD_MAGIC, "not a GGUF file");
  const uint32_t version = r.get<uint32_t>();
  if (!r.ok) return nrc_fail_api(NRC_ERR_TOO_SHORT, "GGUF: truncated header");
  if (version < 2 || version > 3) return nrc_fail_api(NRC_ERR_BAD_VERSION, "unsupported GGUF version %u", version);
  const uint64_t n_tensors = r.get<uint64_t>();
  const uint64_t n_kv = r.get<uint64_t>();
  if (!r.ok) return nrc_fail_api(NRC_ERR_TOO_SHORT, "GGUF: truncated header");
  for (uint64_t k = 0; k < n_kv; k++) {
    std::string key = r.str();
    const uint32_t ty = r.get<uint32_t>();
    Value v;
    if (!r.ok || !r.value(ty, &v, 0)) return nrc_fail_api(NRC_ERR_TOO_SHORT, "GGUF: truncated or bad metadata");
    g->kv[key] = v;
  }
  uint32_t alignment = 32;
  auto ia = g->kv.find("general.alignment");
  if (ia != g->kv.end()) {
    uint32_t a = 0;
    if (ia->second.as_u32(&a)) alignment = a;
  }
  if (alignment == 0) return nrc_fail_api(NRC_ERR_BAD_TABLE, "GGUF: zero alignment");
  for (uint64_t k = 0; k < n_tensors; k++) {
    TensorInfo t;
    t.name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    if (!r.ok || nd > 8) return nrc_fail_api(NRC_ERR_TOO_SHORT, "GGUF: truncated or bad tensor info");
    for (uint32_t d = 0; d < nd; d++) t.dims.push_back(r.get<uint64_t>());
    t.type = r.get<uint32_t>();
    t.offset = r.get<uint64_t>();  // relative to the data section for now
    if (!r.ok) return nrc_fail_api(NRC_ERR_TOO_SHORT, "GGUF: truncated tensor info");
    g->tensors.push_back(std::move(t));
  }
  const uint64_t data_start = ((uint64_t)r.pos + alignment - 1) / alignment * alignment;
  for (auto& t : g->tensors) {
    uint64_t nelem = 1;
    for (uint64_t d : t.dims)
      if (__builtin_mul_overflow(nelem, d, &nelem)) return nrc_fail_api(NRC_ERR_BAD_TABLE, "GGUF: %s: size overflow", t.name.c_str());
    if (!tensor_bytes(t.type, nelem, &t.size))
      return nrc_fail_api(NRC_ERR_UNSUPPORTED, "unsupported ggml dtype %u (%s)", t.type, t.name.c_str());
    if (__builtin_add_overflow(t.offset, data_start, &t.offset) || t.offset > n || t.size > n - t.offset)
      return nrc_fail_api(NRC_ERR_TOO_SHORT, "GGUF: tensor %s lies outside the file", t.name.c_str());
  }
  return NRC_OK;
}

// main.rs:63-110.
int arch_verdict(const Gguf& g, const std::string& arch) {
  if (arch == "granitehybrid" || arch == "granitemoehybrid")
    return nrc_fail_api(NRC_ERR_UNSUPPORTED,
                       "unsupported Granite artifact: architecture %s (hybrid transformer + state-space); "
                       "use a dense Granite GGUF (general.architecture == \"granite\")",
                       arch.c_str());
  if (arch != "llama" && arch != "qwen3" && arch != "granite")
    return nrc_fail_api(NRC_ERR_UNSUPPORTED, "unsupported architecture \"%s\" (supported: llama, qwen3, granite)",
                       arch.c_str());
  for (const char* key : {"ssm_conv_kernel", "ssm_state_size", "expert_count", "expert_used_count"}) {
    auto it = g.kv.find(arch + "." + key);
    uint32_t v = 0;
    if (it != g.kv.end() && it->second.as_u32(&v) && v != 0)
      return nrc_fail_api(NRC_ERR_UNSUPPORTED, "unsupported architecture feature: %s.%s = %u (SSM/MoE models are out of scope)",
                         arch.c_str(), key, v);
  }
  for (const auto& t : g.tensors)
    if (t.name.find(".ssm_") != std::string::npos || t.name.find("ffn_gate_exps") != std::string::npos)
      return nrc_fail_api(NRC_ERR_UNSUPPORTED, "unsupported tensor \"%s\": SSM/MoE layers detected", t.name.c_str());
  return NRC_OK;
}

// main.rs:27-37.
const char* quant_label(const Gguf& g) {
  auto it = g.kv.find("general.file_type");
  uint32_t v = 0;
  if (it == g.kv.end() || !it->second.as_u32(&v)) return "quantized";
  switch (v) {
    case 7: return "Q8_0";
    case 14: return "Q4_K_S";
    case 15: return "Q4_K_M";
    case 17: return "Q5_K_M";
    case 18: return "Q6_K";
    default: return "quantized";
  }
}

struct Out {
  uint16_t kind, layer, dtype;
  uint32_t rows, cols;
  const uint8_t* bytes;
  uint64_t size, offset;
};

template <class T>
void put(std::vector<uint8_t>& v, T x) {
  const size_t o = v.size();
  v.resize(o + sizeof(T));
  memcpy(v.data() + o, &x, sizeof(T));
}

// main.rs:180-426: the .nrm blob.
int convert(const uint8_t* b, size_t n, std::vector<uint8_t>* file) {
  Gguf g;
  if (int rc = parse(b, n, &g)) return rc;
  auto ia = g.kv.find("general.architecture");
  if (ia == g.kv.end() || ia->second.kind != Value::STR) return nrc_fail_api(NRC_ERR_MISSING, "missing general.architecture");
  const std::string arch = ia->second.s;
  if (int rc = arch_verdict(g, arch)) return rc;
  const uint32_t arch_id = arch == "llama" ? 1u : (arch == "qwen3" ? 2u : 3u);
  auto u32 = [&](const std::string& key, uint32_t* out) {
    auto it = g.kv.find(key);
    if (it == g.kv.end() || !it->second.as_u32(out)) return nrc_fail_api(NRC_ERR_MISSING, "missing %s", key.c_str());
    return NRC_OK;
  };
  auto f32 = [&](const std::string& key, float* out) {
    auto it = g.kv.find(key);
    if (it == g.kv.end() || !it->second.as_f32(out)) return nrc_fail_api(NRC_ERR_MISSING, "missing %s", key.c_str());
    return NRC_OK;
  };
  const std::string A = arch + ".";
  uint32_t dim, n_layers, n_heads, n_kv, ffn, ctx_train;
  float rope_theta, norm_eps;
  if (int rc = u32(A + "embedding_length", &dim)) return rc;
  if (int rc = u32(A + "block_count", &n_layers)) return rc;
  if (int rc = u32(A + "attention.head_count", &n_heads)) return rc;
  if (int rc = u32(A + "attention.head_count_kv", &n_kv)) return rc;
  if (int rc = u32(A + "feed_forward_length", &ffn)) return rc;
  if (int rc = u32(A + "context_length", &ctx_train)) return rc;
  if (int rc = f32(A + "rope.freq_base", &rope_theta)) return rc;
  if (int rc = f32(A + "attention.layer_norm_rms_epsilon", &norm_eps)) return rc;
  if (n_heads == 0) return nrc_fail_api(NRC_ERR_INVALID, "zero attention heads");
  uint32_t head_dim = dim / n_heads;
  {
    auto it = g.kv.find(A + "attention.key_length");
    uint32_t v = 0;
    if (it != g.kv.end() && it->second.as_u32(&v)) head_dim = v;
  }
  auto itok = g.kv.find("tokenizer.ggml.tokens");
  if (itok == g.kv.end() || itok->second.kind != Value::ARR) return nrc_fail_api(NRC_ERR_MISSING, "missing tokenizer.ggml.tokens");
  if (itok->second.count > 0xffffffffull) return nrc_fail_api(NRC_ERR_INVALID, "vocabulary too large");
  const uint32_t vocab = (uint32_t)itok->second.count;

  // Tensors in the converter's order (main.rs:231-277).
  std::vector<Out> out;
  auto find = [&](const std::string& name) -> const TensorInfo* {
    for (const auto& t : g.tensors)
      if (t.name == name) return &t;
    return nullptr;
  };
  int err = NRC_OK;
  auto push = [&](const TensorInfo* t, uint16_t kind, uint16_t layer) {
    uint16_t dt;
    switch (t->type) {
      case GGML_F32: dt = DT_F32; break;
      case GGML_Q8_0: dt = DT_Q8_0; break;
      case GGML_Q4_K: dt = DT_Q4K; break;
      case GGML_Q6_K: dt = DT_Q6K; break;
      default:
        err = nrc_fail_api(NRC_ERR_UNSUPPORTED, "%s: unsupported dtype %u (supported: F32, Q8_0, Q4_K, Q6_K)",
                          t->name.c_str(), t->type);
        return;
    }
    const uint32_t cols = t->dims.empty() ? 1u : (uint32_t)t->dims[0];
    const uint32_t rows = t->dims.size() > 1 ? (uint32_t)t->dims[1] : 1u;
    out.push_back({kind, layer, dt, rows, cols, b + t->offset, t->size, 0});
  };
  auto expect = [&](const std::string& name, uint16_t kind, uint16_t layer) {
    if (err) return;
    const TensorInfo* t = find(name);
    if (!t) {
      err = nrc_fail_api(NRC_ERR_MISSING, "gguf missing tensor %s", name.c_str());
      return;
    }
    push(t, kind, layer);
  };
  expect("token_embd.weight", TK_TOK_EMBED, 0);
  if (!err)
    if (const TensorInfo* t = find("rope_freqs.weight")) push(t, TK_ROPE_FREQS, 0);
  for (uint32_t l = 0; l < n_layers && !err; l++) {
    const std::string p = "blk." + std::to_string(l) + ".";
    const uint16_t L = (uint16_t)l;
    expect(p + "attn_norm.weight", TK_ATTN_NORM, L);
    if (arch_id == 2) {
      expect(p + "attn_q_norm.weight", TK_ATTN_Q_NORM, L);
      expect(p + "attn_k_norm.weight", TK_ATTN_K_NORM, L);
    }
    expect(p + "attn_q.weight", TK_ATTN_Q, L);
    expect(p + "attn_k.weight", TK_ATTN_K, L);
    expect(p + "attn_v.weight", TK_ATTN_V, L);
    expect(p + "attn_output.weight", TK_ATTN_O, L);
    expect(p + "ffn_norm.weight", TK_FFN_NORM, L);
    expect(p + "ffn_gate.weight", TK_FFN_GATE, L);
    expect(p + "ffn_up.weight", TK_FFN_UP, L);
    expect(p + "ffn_down.weight", TK_FFN_DOWN, L);
  }
  expect("output_norm.weight", TK_OUTPUT_NORM, 0);
  if (err) return err;
  bool tied = true;
  if (const TensorInfo* t = find("output.weight")) {
    push(t, TK_OUTPUT, 0);
    tied = false;
    if (err) return err;
  }

  // main.rs:282-315: Llama-3 rope factor (the literal llama key), Granite muP scalars.
  float rope_factor = 0.0f;
  {
    auto it = g.kv.find("llama.rope.scaling.factor");
    if (it != g.kv.end()) it->second.as_f32(&rope_factor);
  }
  float embed_scale = 1.0f, attn_scale = 0.0f, residual_scale = 1.0f, logit_scale = 1.0f;
  if (arch_id == 3) {
    const char* keys[4] = {"embedding_scale", "attention.scale", "residual_scale", "logit_scale"};
    float* dst[4] = {&embed_scale, &attn_scale, &residual_scale, &logit_scale};
    for (int k = 0; k < 4; k++) {
      auto it = g.kv.find(A + keys[k]);
      if (it == g.kv.end() || !it->second.as_f32(dst[k]))
        return nrc_fail_api(NRC_ERR_MISSING, "granite artifact missing required scalar %s%s", A.c_str(), keys[k]);
    }
  }

  // 64-byte aligned data offsets; layout header | tokenizer (empty) | table | data.
  uint64_t cursor = 0;
  for (auto& t : out) {
    cursor = (cursor + DATA_ALIGN - 1) / DATA_ALIGN * DATA_ALIGN;
    t.offset = cursor;
    cursor += t.size;
  }
  const uint64_t data_size = cursor;
  const uint64_t tok_off = HEADER_SIZE, tok_len = 0;
  const uint64_t table_off = tok_off + tok_len;
  const uint64_t table_size = out.size() * ENTRY_SIZE;
  const uint64_t data_off = (table_off + table_size + DATA_ALIGN - 1) / DATA_ALIGN * DATA_ALIGN;

  std::vector<uint8_t> table;
  table.reserve(table_size);
  for (const auto& t : out) {
    put<uint16_t>(table, t.kind);
    put<uint16_t>(table, t.layer);
    put<uint16_t>(table, t.dtype);
    put<uint16_t>(table, 0);
    put<uint64_t>(table, t.offset);
    put<uint64_t>(table, t.size);
    put<uint32_t>(table, t.rows);
    put<uint32_t>(table, t.cols);
  }

  file->assign(data_off + data_size, 0);
  uint8_t* f = file->data();
  for (const auto& t : out) memcpy(f + data_off + t.offset, t.bytes, t.size);
  const uint32_t data_crc = nrc::crc32_bytes(f + data_off, data_size);  // zero padding included

  std::vector<uint8_t> h;
  h.reserve(HEADER_SIZE);
  h.insert(h.end(), {'N', 'R', 'U', 'N'});
  put<uint32_t>(h, 3);
  put<uint32_t>(h, arch_id);
  for (uint32_t v : {dim, n_layers, n_heads, n_kv, head_dim, ffn, vocab, ctx_train}) put<uint32_t>(h, v);
  for (float v : {rope_theta, norm_eps, rope_factor, 0.0f, 0.0f, 0.0f}) put<float>(h, v);
  put<uint32_t>(h, tied ? 1u : 0u);
  for (float v : {embed_scale, attn_scale, residual_scale, logit_scale}) put<float>(h, v);
  std::string name = "Unknown Model";
  {
    auto it = g.kv.find("general.name");
    if (it != g.kv.end() && it->second.kind == Value::STR) name = it->second.s;
  }
  name += " ";
  name += quant_label(g);
  uint8_t nb[NAME_LEN] = {0};
  memcpy(nb, name.data(), name.size() < NAME_LEN ? name.size() : NAME_LEN);
  h.insert(h.end(), nb, nb + NAME_LEN);
  put<uint64_t>(h, tok_off);
  put<uint64_t>(h, tok_len);
  put<uint64_t>(h, table_off);
  put<uint32_t>(h, (uint32_t)out.size());
  put<uint32_t>(h, 0);
  put<uint64_t>(h, data_off);
  put<uint64_t>(h, data_size);
  put<uint32_t>(h, data_crc);
  // Metadata CRC: header with both CRC fields zeroed, tokenizer, table (main.rs:401-408).
  uint32_t mc = 0xffffffffu;
  mc = nrc::crc32_update(mc, h.data(), HEADER_SIZE - 8);
  const uint8_t zeros[8] = {0};
  mc = nrc::crc32_update(mc, zeros, 8);
  mc = nrc::crc32_update(mc, table.data(), table.size());
  put<uint32_t>(h, mc ^ 0xffffffffu);
  memcpy(f, h.data(), HEADER_SIZE);
  memcpy(f + table_off, table.data(), table.size());
  return NRC_OK;
}

}  // namespace

extern "C" int nrc_gguf_to_nrm(const uint8_t* gguf, size_t len, uint8_t* out, size_t out_cap, size_t* out_len) {
  if (!gguf || !out_len) return nrc_fail_api(NRC_ERR_INVALID, "null argument");
  std::vector<uint8_t> file;
  if (int rc = convert(gguf, len, &file)) return rc;
  *out_len = file.size();
  if (!out) return NRC_OK;
  if (out_cap < file.size()) return nrc_fail_api(NRC_ERR_INVALID, "output buffer of %zu bytes, %zu needed", out_cap, file.size());
  memcpy(out, file.data(), file.size());
  return NRC_OK;
}

extern "C" int nrc_model_load_gguf(const uint8_t* gguf, size_t len, int device, nrc_model** out) {
  if (!gguf || !out) return nrc_fail_api(NRC_ERR_INVALID, "null argument");
  *out = nullptr;
  std::vector<uint8_t> file;
  if (int rc = convert(gguf, len, &file)) return rc;
  return nrc_model_load(file.data(), file.size(), device, 1, out);
}
