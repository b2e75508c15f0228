// TEST INFRASTRUCTURE ONLY — CPU oracle for the NIGHTRUN quantized forward path.
//
// This is a C++ restatement of the reference's Rust code (crates/nr-tensor and
// crates/nr-model of NicoAvanzDev/NIGHTRUN). It is the checker for the CUDA
// library in nightrun_b200/ and the timed CPU baseline in bench.py. Nothing in
// the product path links, loads or calls it: only tests/, __graft_entry__.smoke()
// and bench.py's cpu_baseline / --impl reference legs do.
//
// Parity pinning: the reference cannot be built here (no Rust toolchain), so the
// restatement is pinned against the reference's own known-answer tests
// (crates/nr-tensor/tests/kernels.rs, crates/nr-tensor/tests/kquant.rs,
// crates/nr-model/tests/format_malformed.rs), restated in tests/test_oracle.py.
// libm's expf/powf/sincosf (crate libm 0.2.16, not vendored) are replaced by
// glibc's; they may differ by an ulp, so parity at that level is unpinned.
//
// Build: oracle/build.sh (g++ -O2 -mavx2 -mfma -mf16c -ffp-contract=off).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>

namespace oracle {

// ---- block layouts (crates/nr-tensor/src/q8.rs:9-17, kquant.rs:24-56) ----
constexpr int QK8_0 = 32;
constexpr int QK_K = 256;

#pragma pack(push, 1)
struct BlockQ8_0 {  // q8.rs:11-14 — 34 bytes
  uint16_t d;
  int8_t qs[QK8_0];
};
struct BlockQ4K {  // kquant.rs:26-31 — 144 bytes
  uint16_t d;
  uint16_t dmin;
  uint8_t scales[12];
  uint8_t qs[128];
};
struct BlockQ6K {  // kquant.rs:37-42 — 210 bytes
  uint8_t ql[128];
  uint8_t qh[64];
  int8_t scales[16];
  uint16_t d;
};
#pragma pack(pop)
struct BlockQ8K {  // kquant.rs:46-52 — repr(C): f32 d, 256 i8, 16 i16 = 292 bytes
  float d;
  int8_t qs[QK_K];
  int16_t bsums[QK_K / 16];
};
static_assert(sizeof(BlockQ8_0) == 34, "q8_0");
static_assert(sizeof(BlockQ4K) == 144, "q4k");
static_assert(sizeof(BlockQ6K) == 210, "q6k");
static_assert(sizeof(BlockQ8K) == 292, "q8k");

// Rust `f as i32`: truncation toward zero, saturating, NaN -> 0.
inline int32_t rust_f32_to_i32(float f) {
  if (f != f) return 0;
  if (f >= 2147483648.0f) return INT32_MAX;
  if (f <= -2147483648.0f) return INT32_MIN;
  return (int32_t)f;
}
// Rust f32::max / f32::min: NaN loses.
inline float rust_max(float a, float b) {
  if (a != a) return b;
  if (b != b) return a;
  return a > b ? a : b;
}
inline float rust_min(float a, float b) {
  if (a != a) return b;
  if (b != b) return a;
  return a < b ? a : b;
}
inline int32_t clampi(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }
inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

// ---- f16.rs ----
float f16_to_f32(uint16_t bits);
uint16_t f32_to_f16(float v);

// ---- cpu.rs: the fast-path gate; the oracle lets tests choose the path ----
extern bool g_fast_path;  // AVX2+FMA kernels (cpu.rs:46-49)
extern bool g_fast_f16;   // F16C dot/axpy (cpu.rs:52-55)

// ---- parallel.rs ----
typedef void (*RangeFn)(void* ctx, size_t r0, size_t r1);
void pool_start(int threads);  // nrhost main.rs:41-51 (threads-1 workers)
void pool_run(size_t total, RangeFn fn, void* ctx);  // parallel.rs:88-105
int pool_threads();

// ---- q8.rs ----
void q8_quantize(const float* src, size_t n, BlockQ8_0* out);
void q8_dequantize(const BlockQ8_0* blocks, size_t n, float* out);

// ---- kquant.rs ----
void q4k_scale_min(const uint8_t* scales, int j, uint8_t* sc, uint8_t* m);
void dequant_q4k(const BlockQ4K* b, float* out);
void dequant_q6k(const BlockQ6K* b, float* out);
void quantize_q8k(const float* src, size_t n, BlockQ8K* out);
float dot_q4k_scalar(const BlockQ4K* w, const BlockQ8K* x, size_t nb);
float dot_q6k_scalar(const BlockQ6K* w, const BlockQ8K* x, size_t nb);
float dot_q4k_avx2(const BlockQ4K* w, const BlockQ8K* x, size_t nb);
float dot_q6k_avx2(const BlockQ6K* w, const BlockQ8K* x, size_t nb);
void dot_q4k_avx2_x4(const BlockQ4K* w, const BlockQ8K* const xs[4], size_t nb, float out[4]);
void dot_q6k_avx2_x4(const BlockQ6K* w, const BlockQ8K* const xs[4], size_t nb, float out[4]);
void matvec_q4k(float* y, const BlockQ4K* w, const BlockQ8K* x, size_t rows, size_t cols);
void matvec_q6k(float* y, const BlockQ6K* w, const BlockQ8K* x, size_t rows, size_t cols);
void matmul_q4k(float* y, const BlockQ4K* w, const BlockQ8K* xs, size_t rows, size_t cols, size_t batch);
void matmul_q6k(float* y, const BlockQ6K* w, const BlockQ8K* xs, size_t rows, size_t cols, size_t batch);
BlockQ4K quantize_q4k_ref(const float* src);
BlockQ6K quantize_q6k_ref(const float* src);

// ---- kernels.rs ----
float dot_q8_scalar(const BlockQ8_0* w, const BlockQ8_0* x, size_t nb);
float dot_q8_avx2(const BlockQ8_0* w, const BlockQ8_0* x, size_t nb);
void dot_q8_avx2_x4(const BlockQ8_0* w, const BlockQ8_0* const xs[4], size_t nb, float out[4]);
void matvec_q8(float* y, const BlockQ8_0* w, const BlockQ8_0* x, size_t rows, size_t cols);
void matmul_q8(float* y, const BlockQ8_0* w, const BlockQ8_0* xs, size_t rows, size_t cols, size_t batch);
float dot_f16(const uint16_t* k, const float* q, size_t n);
void axpy_f16(float* out, float a, const uint16_t* v, size_t n);

// ---- vec.rs ----
void rmsnorm(float* out, const float* x, const float* w, size_t n, float eps);
void rmsnorm_inplace(float* x, const float* w, size_t n, float eps);
void softmax(float* x, size_t n);
void swiglu(float* gate, const float* up, size_t n);
float vdot(const float* a, const float* b, size_t n);
void scale_inplace(float* x, size_t n, float s);
void saxpy(float* y, float a, const float* x, size_t n);
size_t argmax(const float* x, size_t n);

// ---- rope.rs ----
struct Llama3Scaling { float factor, low_freq_factor, high_freq_factor, original_context; };
void rope_freqs(float* out, size_t head_dim, float theta, const Llama3Scaling* scaling);
enum RopeStyle { ROPE_ADJACENT = 0, ROPE_NEOX = 1 };
void rope_apply(float* x, size_t len, size_t head_dim, const float* freqs, size_t pos, int style);

// ---- crc32.rs ----
uint32_t crc32_update(uint32_t state, const uint8_t* data, size_t n);  // state starts at 0xffffffff
uint32_t crc32(const uint8_t* data, size_t n);

}  // namespace oracle
