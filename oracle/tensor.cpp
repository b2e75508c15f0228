// TEST INFRASTRUCTURE ONLY — restatement of crates/nr-tensor/src/*.rs
// (f16.rs, q8.rs, kquant.rs, kernels.rs, vec.rs, rope.rs, parallel.rs) and
// crates/nr-model/src/crc32.rs. Compiled with -ffp-contract=off so that every
// `a * b + c` rounds twice, as Rust does. See oracle.h for the pinning status.
#include <immintrin.h>
#include <math.h>

#include <atomic>
#include <thread>
#include <vector>

#include "oracle.h"
#include "expf_cr.h"

namespace oracle {

bool g_fast_path = false;
bool g_fast_f16 = false;

// ------------------------------------------------------------------ f16.rs:3-23
float f16_to_f32(uint16_t bits) {
  uint32_t sign = ((uint32_t)(bits >> 15)) << 31;
  uint32_t exp = (bits >> 10) & 0x1f;
  uint32_t frac = bits & 0x3ff;
  uint32_t out;
  if (exp == 0) {
    if (frac == 0) {
      out = sign;
    } else {
      uint32_t msb = 31 - __builtin_clz(frac);  // 0..=9
      uint32_t e = 127 - 24 + msb;
      uint32_t f = (frac << (23 - msb)) & 0x7fffff;
      out = sign | (e << 23) | f;
    }
  } else if (exp == 0x1f) {
    out = sign | 0x7f800000u | (frac << 13);
  } else {
    out = sign | ((exp + 127 - 15) << 23) | (frac << 13);
  }
  return bits_f32(out);
}

// ------------------------------------------------------------------ f16.rs:25-56
uint16_t f32_to_f16(float v) {
  uint32_t bits = f32_bits(v);
  uint16_t sign = (uint16_t)((bits >> 31) << 15);
  int32_t exp = (int32_t)((bits >> 23) & 0xff);
  uint32_t frac = bits & 0x7fffff;
  if (exp == 0xff) return (uint16_t)(sign | 0x7c00 | (frac != 0 ? 0x200 : 0));
  int32_t e = exp - 127 + 15;
  if (e >= 0x1f) return (uint16_t)(sign | 0x7c00);
  if (e <= 0) {
    if (e < -10) return sign;
    uint32_t f = frac | 0x800000;
    uint32_t shift = (uint32_t)(14 - e);
    uint32_t half = 1u << (shift - 1);
    return (uint16_t)(sign | (uint16_t)((f + half) >> shift));  // half-up, as the reference
  }
  uint32_t out = (uint32_t)sign | ((uint32_t)e << 10) | (frac >> 13);
  uint32_t round = frac & 0x1fff;
  if (round > 0x1000 || (round == 0x1000 && (out & 1) != 0)) out += 1;
  return (uint16_t)out;
}

// ------------------------------------------------------------ parallel.rs:14-105
// Same protocol as the reference's spin pool: workers spin on a sequence
// counter and pull `chunk`-sized row ranges from an atomic cursor; the caller
// participates; inline when there are no workers or total < 128.
namespace {
struct Pool {
  std::atomic<size_t> seq{0}, cursor{0}, total{0}, chunk{1}, done{0}, workers{0}, ready{0};
  std::atomic<RangeFn> fn{nullptr};
  std::atomic<void*> ctx{nullptr};
  std::vector<std::thread> threads;
};
Pool g_pool;

void pool_drain() {
  size_t total = g_pool.total.load();
  size_t chunk = g_pool.chunk.load();
  if (chunk < 1) chunk = 1;
  RangeFn fn = g_pool.fn.load();
  void* ctx = g_pool.ctx.load();
  for (;;) {
    size_t start = g_pool.cursor.fetch_add(chunk);
    if (start >= total) break;
    size_t end = start + chunk < total ? start + chunk : total;
    fn(ctx, start, end);
  }
}

void worker_loop() {  // parallel.rs:57-72 (exits when workers is set to 0)
  g_pool.ready.fetch_add(1);
  size_t last = g_pool.seq.load();
  for (;;) {
    size_t s = g_pool.seq.load();
    if (s == (size_t)-1) return;
    if (s != last) {
      last = s;
      pool_drain();
      g_pool.done.fetch_add(1);
    }
    _mm_pause();
  }
}
}  // namespace

void pool_start(int threads) {
  if (!g_pool.threads.empty() || threads <= 1) return;
  size_t workers = (size_t)threads - 1;
  for (size_t i = 0; i < workers; i++) g_pool.threads.emplace_back(worker_loop);
  while (g_pool.ready.load() < workers) std::this_thread::yield();
  g_pool.workers.store(workers);
  for (auto& t : g_pool.threads) t.detach();
}

int pool_threads() { return (int)g_pool.workers.load() + 1; }

void pool_run(size_t total, RangeFn fn, void* ctx) {
  size_t n = g_pool.workers.load();
  if (n == 0 || total < 128) {
    fn(ctx, 0, total);
    return;
  }
  g_pool.total.store(total);
  g_pool.cursor.store(0);
  size_t chunk = total / ((n + 1) * 4);
  g_pool.chunk.store(chunk > 16 ? chunk : 16);
  g_pool.done.store(0);
  g_pool.fn.store(fn);
  g_pool.ctx.store(ctx);
  g_pool.seq.fetch_add(1);
  pool_drain();
  while (g_pool.done.load() < n) _mm_pause();
}

// ------------------------------------------------------------------- q8.rs:27-55
void q8_quantize(const float* src, size_t n, BlockQ8_0* out) {
  for (size_t b = 0; b < n / QK8_0; b++) {
    const float* chunk = src + b * QK8_0;
    float amax = 0.0f;
    for (int i = 0; i < QK8_0; i++) amax = rust_max(amax, fabsf(chunk[i]));
    uint16_t d_bits = f32_to_f16(amax / 127.0f);
    float d = f16_to_f32(d_bits);
    float inv = d > 0.0f ? 1.0f / d : 0.0f;
    out[b].d = d_bits;
    for (int i = 0; i < QK8_0; i++) {
      float x = chunk[i] * inv;
      float r = x >= 0.0f ? x + 0.5f : x - 0.5f;
      out[b].qs[i] = (int8_t)clampi(rust_f32_to_i32(r), -127, 127);
    }
  }
}

void q8_dequantize(const BlockQ8_0* blocks, size_t n, float* out) {
  for (size_t b = 0; b < n / QK8_0; b++) {
    float d = f16_to_f32(blocks[b].d);
    for (int i = 0; i < QK8_0; i++) out[b * QK8_0 + i] = (float)blocks[b].qs[i] * d;
  }
}

// --------------------------------------------------------------- kquant.rs:83-92
void q4k_scale_min(const uint8_t* scales, int j, uint8_t* sc, uint8_t* m) {
  if (j < 4) {
    *sc = scales[j] & 63;
    *m = scales[j + 4] & 63;
  } else {
    *sc = (uint8_t)((scales[j + 4] & 0x0F) | ((scales[j - 4] >> 6) << 4));
    *m = (uint8_t)((scales[j + 4] >> 4) | ((scales[j] >> 6) << 4));
  }
}

// -------------------------------------------------------------- kquant.rs:95-118
void dequant_q4k(const BlockQ4K* b, float* out) {
  float d = f16_to_f32(b->d);
  float dmin = f16_to_f32(b->dmin);
  int is = 0, y = 0;
  for (int chunk = 0; chunk < 4; chunk++) {
    const uint8_t* q = b->qs + chunk * 32;
    uint8_t sc1, m1, sc2, m2;
    q4k_scale_min(b->scales, is, &sc1, &m1);
    q4k_scale_min(b->scales, is + 1, &sc2, &m2);
    float d1 = d * (float)sc1, min1 = dmin * (float)m1;
    float d2 = d * (float)sc2, min2 = dmin * (float)m2;
    for (int k = 0; k < 32; k++) out[y++] = d1 * (float)(q[k] & 0x0F) - min1;
    for (int k = 0; k < 32; k++) out[y++] = d2 * (float)(q[k] >> 4) - min2;
    is += 2;
  }
}

// ------------------------------------------------------------- kquant.rs:121-142
void dequant_q6k(const BlockQ6K* b, float* out) {
  float d = f16_to_f32(b->d);
  for (int half = 0; half < 2; half++) {
    const uint8_t* ql = b->ql + half * 64;
    const uint8_t* qh = b->qh + half * 32;
    const int8_t* sc = b->scales + half * 8;
    float* y = out + half * 128;
    for (int l = 0; l < 32; l++) {
      int is = l / 16;
      int q1 = (int)((ql[l] & 0x0F) | ((qh[l] & 3) << 4)) - 32;
      int q2 = (int)((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
      int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
      int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
      y[l] = d * (float)sc[is] * (float)q1;
      y[l + 32] = d * (float)sc[is + 2] * (float)q2;
      y[l + 64] = d * (float)sc[is + 4] * (float)q3;
      y[l + 96] = d * (float)sc[is + 6] * (float)q4;
    }
  }
}

// ------------------------------------------------------------- kquant.rs:145-153
static inline int32_t nearest_int(float v) {
  return v >= 0.0f ? rust_f32_to_i32(v + 0.5f) : rust_f32_to_i32(v - 0.5f);
}

// ------------------------------------------------------------- kquant.rs:157-187
void quantize_q8k(const float* src, size_t n, BlockQ8K* out) {
  for (size_t b = 0; b < n / QK_K; b++) {
    const float* chunk = src + b * QK_K;
    BlockQ8K* blk = out + b;
    float amax = 0.0f, max = 0.0f;
    for (int i = 0; i < QK_K; i++) {
      if (fabsf(chunk[i]) > amax) {
        amax = fabsf(chunk[i]);
        max = chunk[i];
      }
    }
    if (amax == 0.0f) {
      blk->d = 0.0f;
      memset(blk->qs, 0, sizeof(blk->qs));
      memset(blk->bsums, 0, sizeof(blk->bsums));
      continue;
    }
    float iscale = -128.0f / max;
    for (int i = 0; i < QK_K; i++) {
      int32_t q = nearest_int(iscale * chunk[i]);
      if (q > 127) q = 127;
      blk->qs[i] = (int8_t)(uint8_t)(q & 0xff);  // `as i8` wraps
    }
    for (int j = 0; j < 16; j++) {
      int32_t s = 0;
      for (int k = 0; k < 16; k++) s += blk->qs[j * 16 + k];
      blk->bsums[j] = (int16_t)s;
    }
    blk->d = 1.0f / iscale;
  }
}

// ------------------------------------------------------------- kquant.rs:192-218
float dot_q4k_scalar(const BlockQ4K* w, const BlockQ8K* x, size_t nb) {
  float sumf = 0.0f;
  for (size_t b = 0; b < nb; b++) {
    const BlockQ4K* bw = w + b;
    const BlockQ8K* bx = x + b;
    float d_all = f16_to_f32(bw->d) * bx->d;
    float dmin_all = f16_to_f32(bw->dmin) * bx->d;
    float sum_q = 0.0f;
    int32_t sum_m = 0;
    for (int j = 0; j < 8; j++) {
      uint8_t sc, m;
      q4k_scale_min(bw->scales, j, &sc, &m);
      int32_t sub = 0;
      int chunk = j / 2;
      bool hi = (j % 2) == 1;
      const uint8_t* q = bw->qs + chunk * 32;
      const int8_t* q8 = bx->qs + j * 32;
      for (int k = 0; k < 32; k++) {
        int32_t qv = hi ? (q[k] >> 4) : (q[k] & 0x0F);
        sub += qv * (int32_t)q8[k];
      }
      sum_q += (float)sc * (float)sub;
      sum_m += (int32_t)m * ((int32_t)bx->bsums[2 * j] + (int32_t)bx->bsums[2 * j + 1]);
    }
    sumf += d_all * sum_q - dmin_all * (float)sum_m;
  }
  return sumf;
}

// ------------------------------------------------------------- kquant.rs:220-250
float dot_q6k_scalar(const BlockQ6K* w, const BlockQ8K* x, size_t nb) {
  float sumf = 0.0f;
  for (size_t b = 0; b < nb; b++) {
    const BlockQ6K* bw = w + b;
    const BlockQ8K* bx = x + b;
    float d_all = f16_to_f32(bw->d) * bx->d;
    float sum = 0.0f;
    for (int half = 0; half < 2; half++) {
      const uint8_t* ql = bw->ql + half * 64;
      const uint8_t* qh = bw->qh + half * 32;
      const int8_t* sc = bw->scales + half * 8;
      const int8_t* q8 = bx->qs + half * 128;
      int32_t gs[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int l = 0; l < 32; l++) {
        int32_t q1 = (int32_t)((ql[l] & 0x0F) | ((qh[l] & 3) << 4)) - 32;
        int32_t q2 = (int32_t)((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
        int32_t q3 = (int32_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
        int32_t q4 = (int32_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
        gs[l / 16] += q1 * q8[l];
        gs[2 + l / 16] += q2 * q8[l + 32];
        gs[4 + l / 16] += q3 * q8[l + 64];
        gs[6 + l / 16] += q4 * q8[l + 96];
      }
      for (int g = 0; g < 8; g++) sum += (float)sc[g] * (float)gs[g];
    }
    sumf += d_all * sum;
  }
  return sumf;
}

// ------------------------------------------------------------- kquant.rs:512-522
__attribute__((target("avx2"))) static inline float hsum256(__m256 v) {
  __m128 hi = _mm256_extractf128_ps(v, 1);
  __m128 lo = _mm256_castps256_ps128(v);
  __m128 s = _mm_add_ps(hi, lo);
  s = _mm_add_ps(s, _mm_movehl_ps(s, s));
  s = _mm_add_ss(s, _mm_shuffle_ps(s, s, 1));
  return _mm_cvtss_f32(s);
}

// ------------------------------------------------------------- kquant.rs:257-305
__attribute__((target("avx2,fma"))) float dot_q4k_avx2(const BlockQ4K* w, const BlockQ8K* x,
                                                       size_t nb) {
  const __m256i m4 = _mm256_set1_epi8(0x0F);
  __m256 acc = _mm256_setzero_ps();
  float acc_min = 0.0f;
  for (size_t b = 0; b < nb; b++) {
    const BlockQ4K* bw = w + b;
    const BlockQ8K* bx = x + b;
    float d = f16_to_f32(bw->d) * bx->d;
    float dmin = f16_to_f32(bw->dmin) * bx->d;
    uint8_t sc[8], mins[8];
    for (int j = 0; j < 8; j++) q4k_scale_min(bw->scales, j, &sc[j], &mins[j]);
    int32_t min_sum = 0;
    for (int j = 0; j < 8; j++)
      min_sum += (int32_t)mins[j] * ((int32_t)bx->bsums[2 * j] + (int32_t)bx->bsums[2 * j + 1]);
    acc_min += dmin * (float)min_sum;
    const uint8_t* qs = bw->qs;
    const int8_t* q8 = bx->qs;
    __m256i sumi = _mm256_setzero_si256();
    for (int j = 0; j < 4; j++) {
      __m256i q4bits = _mm256_loadu_si256((const __m256i*)(qs + j * 32));
      __m256i q4l = _mm256_and_si256(q4bits, m4);
      __m256i q4h = _mm256_and_si256(_mm256_srli_epi16(q4bits, 4), m4);
      __m256i q8l = _mm256_loadu_si256((const __m256i*)(q8 + j * 64));
      __m256i q8h = _mm256_loadu_si256((const __m256i*)(q8 + j * 64 + 32));
      __m256i p16l = _mm256_maddubs_epi16(q4l, q8l);
      p16l = _mm256_madd_epi16(_mm256_set1_epi16((int16_t)sc[2 * j]), p16l);
      __m256i p16h = _mm256_maddubs_epi16(q4h, q8h);
      p16h = _mm256_madd_epi16(_mm256_set1_epi16((int16_t)sc[2 * j + 1]), p16h);
      sumi = _mm256_add_epi32(sumi, _mm256_add_epi32(p16l, p16h));
    }
    acc = _mm256_fmadd_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sumi), acc);
  }
  return hsum256(acc) - acc_min;
}

// ------------------------------------------------------------- kquant.rs:314-374
__attribute__((target("avx2,fma"))) void dot_q4k_avx2_x4(const BlockQ4K* w,
                                                         const BlockQ8K* const xs[4], size_t nb,
                                                         float out[4]) {
  const __m256i m4 = _mm256_set1_epi8(0x0F);
  __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(),
                   _mm256_setzero_ps()};
  float acc_min[4] = {0, 0, 0, 0};
  for (size_t bi = 0; bi < nb; bi++) {
    const BlockQ4K* bw = w + bi;
    float d_w = f16_to_f32(bw->d);
    float dmin_w = f16_to_f32(bw->dmin);
    uint8_t sc[8], mins[8];
    for (int j = 0; j < 8; j++) q4k_scale_min(bw->scales, j, &sc[j], &mins[j]);
    for (int lane = 0; lane < 4; lane++) {
      const BlockQ8K* bx = xs[lane] + bi;
      int32_t min_sum = 0;
      for (int j = 0; j < 8; j++)
        min_sum += (int32_t)mins[j] * ((int32_t)bx->bsums[2 * j] + (int32_t)bx->bsums[2 * j + 1]);
      acc_min[lane] += dmin_w * bx->d * (float)min_sum;
    }
    __m256i sumi[4] = {_mm256_setzero_si256(), _mm256_setzero_si256(), _mm256_setzero_si256(),
                       _mm256_setzero_si256()};
    for (int j = 0; j < 4; j++) {
      __m256i q4bits = _mm256_loadu_si256((const __m256i*)(bw->qs + j * 32));
      __m256i q4l = _mm256_and_si256(q4bits, m4);
      __m256i q4h = _mm256_and_si256(_mm256_srli_epi16(q4bits, 4), m4);
      __m256i scale_l = _mm256_set1_epi16((int16_t)sc[2 * j]);
      __m256i scale_h = _mm256_set1_epi16((int16_t)sc[2 * j + 1]);
      for (int lane = 0; lane < 4; lane++) {
        const int8_t* q8 = xs[lane][bi].qs;
        __m256i q8l = _mm256_loadu_si256((const __m256i*)(q8 + j * 64));
        __m256i q8h = _mm256_loadu_si256((const __m256i*)(q8 + j * 64 + 32));
        __m256i p16l = _mm256_madd_epi16(scale_l, _mm256_maddubs_epi16(q4l, q8l));
        __m256i p16h = _mm256_madd_epi16(scale_h, _mm256_maddubs_epi16(q4h, q8h));
        sumi[lane] = _mm256_add_epi32(sumi[lane], _mm256_add_epi32(p16l, p16h));
      }
    }
    for (int lane = 0; lane < 4; lane++) {
      __m256 d = _mm256_set1_ps(d_w * xs[lane][bi].d);
      acc[lane] = _mm256_fmadd_ps(d, _mm256_cvtepi32_ps(sumi[lane]), acc[lane]);
    }
  }
  for (int lane = 0; lane < 4; lane++) out[lane] = hsum256(acc[lane]) - acc_min[lane];
}

// ----------------------------------------------------- kquant.rs:381-448, 452-510
// Shared Q6_K body: (q6 - 32) * q8 via maddubs(q6, q8) - maddubs(32, q8), then
// madd with the per-16 scale pair (low 128-bit lane = group g, high = g+1).
__attribute__((target("avx2,fma"))) static inline void q6k_planes(const BlockQ6K* bw, int half,
                                                                 __m256i q6[4]) {
  const __m256i m4 = _mm256_set1_epi8(0x0F);
  const __m256i m2 = _mm256_set1_epi8(3);
  const uint8_t* ql = bw->ql + half * 64;
  const uint8_t* qh = bw->qh + half * 32;
  __m256i q4bits1 = _mm256_loadu_si256((const __m256i*)ql);
  __m256i q4bits2 = _mm256_loadu_si256((const __m256i*)(ql + 32));
  __m256i qhbits = _mm256_loadu_si256((const __m256i*)qh);
  __m256i q4h_0 = _mm256_slli_epi16(_mm256_and_si256(qhbits, m2), 4);
  __m256i q4h_1 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qhbits, 2), m2), 4);
  __m256i q4h_2 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qhbits, 4), m2), 4);
  __m256i q4h_3 = _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qhbits, 6), m2), 4);
  q6[0] = _mm256_or_si256(_mm256_and_si256(q4bits1, m4), q4h_0);
  q6[1] = _mm256_or_si256(_mm256_and_si256(q4bits2, m4), q4h_1);
  q6[2] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(q4bits1, 4), m4), q4h_2);
  q6[3] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(q4bits2, 4), m4), q4h_3);
}

__attribute__((target("avx2,fma"))) float dot_q6k_avx2(const BlockQ6K* w, const BlockQ8K* x,
                                                       size_t nb) {
  const __m256i m32s = _mm256_set1_epi8(32);
  __m256 acc = _mm256_setzero_ps();
  for (size_t b = 0; b < nb; b++) {
    const BlockQ6K* bw = w + b;
    const BlockQ8K* bx = x + b;
    float d = f16_to_f32(bw->d) * bx->d;
    __m256i sumi = _mm256_setzero_si256();
    for (int half = 0; half < 2; half++) {
      const int8_t* q8p = bx->qs + half * 128;
      const int8_t* sc = bw->scales + half * 8;
      __m256i q6[4];
      q6k_planes(bw, half, q6);
      for (int n = 0; n < 4; n++) {
        __m256i scale = _mm256_set_m128i(_mm_set1_epi16((int16_t)sc[2 * n + 1]),
                                         _mm_set1_epi16((int16_t)sc[2 * n]));
        __m256i q8 = _mm256_loadu_si256((const __m256i*)(q8p + n * 32));
        __m256i corr = _mm256_maddubs_epi16(m32s, q8);
        __m256i p16 = _mm256_maddubs_epi16(q6[n], q8);
        p16 = _mm256_sub_epi16(p16, corr);
        p16 = _mm256_madd_epi16(scale, p16);
        sumi = _mm256_add_epi32(sumi, p16);
      }
    }
    acc = _mm256_fmadd_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sumi), acc);
  }
  return hsum256(acc);
}

__attribute__((target("avx2,fma"))) void dot_q6k_avx2_x4(const BlockQ6K* w,
                                                         const BlockQ8K* const xs[4], size_t nb,
                                                         float out[4]) {
  const __m256i m32s = _mm256_set1_epi8(32);
  __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(),
                   _mm256_setzero_ps()};
  for (size_t bi = 0; bi < nb; bi++) {
    const BlockQ6K* bw = w + bi;
    float d_w = f16_to_f32(bw->d);
    __m256i sumi[4] = {_mm256_setzero_si256(), _mm256_setzero_si256(), _mm256_setzero_si256(),
                       _mm256_setzero_si256()};
    for (int half = 0; half < 2; half++) {
      const int8_t* sc = bw->scales + half * 8;
      __m256i q6[4];
      q6k_planes(bw, half, q6);
      for (int n = 0; n < 4; n++) {
        __m256i sc_vec = _mm256_set_m128i(_mm_set1_epi16((int16_t)sc[2 * n + 1]),
                                          _mm_set1_epi16((int16_t)sc[2 * n]));
        for (int lane = 0; lane < 4; lane++) {
          const int8_t* q8p = xs[lane][bi].qs + half * 128;
          __m256i q8 = _mm256_loadu_si256((const __m256i*)(q8p + n * 32));
          __m256i corr = _mm256_maddubs_epi16(m32s, q8);
          __m256i p16 = _mm256_maddubs_epi16(q6[n], q8);
          p16 = _mm256_sub_epi16(p16, corr);
          p16 = _mm256_madd_epi16(sc_vec, p16);
          sumi[lane] = _mm256_add_epi32(sumi[lane], p16);
        }
      }
    }
    for (int lane = 0; lane < 4; lane++) {
      __m256 d = _mm256_set1_ps(d_w * xs[lane][bi].d);
      acc[lane] = _mm256_fmadd_ps(d, _mm256_cvtepi32_ps(sumi[lane]), acc[lane]);
    }
  }
  for (int lane = 0; lane < 4; lane++) out[lane] = hsum256(acc[lane]);
}

// ------------------------------------------------- kquant.rs:536-639 (matvec/matmul)
namespace {
template <typename B>
struct KqJob {
  float* y;
  const B* w;
  const BlockQ8K* x;
  size_t rows, bpr, batch;
};

template <typename B>
float kq_dot(const B* w, const BlockQ8K* x, size_t nb, bool fast);
template <>
float kq_dot<BlockQ4K>(const BlockQ4K* w, const BlockQ8K* x, size_t nb, bool fast) {
  return fast ? dot_q4k_avx2(w, x, nb) : dot_q4k_scalar(w, x, nb);
}
template <>
float kq_dot<BlockQ6K>(const BlockQ6K* w, const BlockQ8K* x, size_t nb, bool fast) {
  return fast ? dot_q6k_avx2(w, x, nb) : dot_q6k_scalar(w, x, nb);
}
void kq_dot4(const BlockQ4K* w, const BlockQ8K* const xs[4], size_t nb, float o[4]) {
  dot_q4k_avx2_x4(w, xs, nb, o);
}
void kq_dot4(const BlockQ6K* w, const BlockQ8K* const xs[4], size_t nb, float o[4]) {
  dot_q6k_avx2_x4(w, xs, nb, o);
}

template <typename B>
void kq_matvec_range(void* p, size_t r0, size_t r1) {
  auto* j = (KqJob<B>*)p;
  bool fast = g_fast_path;
  for (size_t r = r0; r < r1; r++) j->y[r] = kq_dot<B>(j->w + r * j->bpr, j->x, j->bpr, fast);
}

template <typename B>
void kq_matmul_range(void* p, size_t r0, size_t r1) {
  auto* j = (KqJob<B>*)p;
  bool fast = g_fast_path;
  size_t bpr = j->bpr, rows = j->rows, batch = j->batch;
  for (size_t r = r0; r < r1; r++) {
    const B* row = j->w + r * bpr;
    size_t b = 0;
    while (fast && b + 4 <= batch) {
      const BlockQ8K* xs[4] = {j->x + b * bpr, j->x + (b + 1) * bpr, j->x + (b + 2) * bpr,
                               j->x + (b + 3) * bpr};
      float o[4];
      kq_dot4(row, xs, bpr, o);
      for (int i = 0; i < 4; i++) j->y[(b + i) * rows + r] = o[i];
      b += 4;
    }
    while (b < batch) {
      j->y[b * rows + r] = kq_dot<B>(row, j->x + b * bpr, bpr, fast);
      b += 1;
    }
  }
}
}  // namespace

void matvec_q4k(float* y, const BlockQ4K* w, const BlockQ8K* x, size_t rows, size_t cols) {
  KqJob<BlockQ4K> j{y, w, x, rows, cols / QK_K, 1};
  pool_run(rows, kq_matvec_range<BlockQ4K>, &j);
}
void matvec_q6k(float* y, const BlockQ6K* w, const BlockQ8K* x, size_t rows, size_t cols) {
  KqJob<BlockQ6K> j{y, w, x, rows, cols / QK_K, 1};
  pool_run(rows, kq_matvec_range<BlockQ6K>, &j);
}
void matmul_q4k(float* y, const BlockQ4K* w, const BlockQ8K* xs, size_t rows, size_t cols,
                size_t batch) {
  KqJob<BlockQ4K> j{y, w, xs, rows, cols / QK_K, batch};
  pool_run(rows, kq_matmul_range<BlockQ4K>, &j);
}
void matmul_q6k(float* y, const BlockQ6K* w, const BlockQ8K* xs, size_t rows, size_t cols,
                size_t batch) {
  KqJob<BlockQ6K> j{y, w, xs, rows, cols / QK_K, batch};
  pool_run(rows, kq_matmul_range<BlockQ6K>, &j);
}

// ------------------------------------------------------------- kquant.rs:647-712
BlockQ4K quantize_q4k_ref(const float* src) {
  float sub_scale[8], sub_min[8];
  for (int j = 0; j < 8; j++) {
    const float* s = src + j * 32;
    float mx = -3.40282347e38f, mn = 3.40282347e38f;  // f32::MIN / f32::MAX
    for (int k = 0; k < 32; k++) {
      mx = rust_max(mx, s[k]);
      mn = rust_min(mn, s[k]);
    }
    sub_min[j] = rust_max(-mn, 0.0f);
    sub_scale[j] = rust_max((mx + sub_min[j]) / 15.0f, 0.0f);
  }
  float max_scale = 0.0f, max_min = 0.0f;
  for (int j = 0; j < 8; j++) {
    max_scale = rust_max(max_scale, sub_scale[j]);
    max_min = rust_max(max_min, sub_min[j]);
  }
  float d = max_scale / 63.0f;
  float dmin = max_min / 63.0f;
  float df = f16_to_f32(f32_to_f16(d));
  float dminf = f16_to_f32(f32_to_f16(dmin));
  uint8_t scales6[8], mins6[8];
  for (int j = 0; j < 8; j++) {
    scales6[j] = df > 0.0f ? (uint8_t)clampi(nearest_int(sub_scale[j] / df), 0, 63) : 0;
    mins6[j] = dminf > 0.0f ? (uint8_t)clampi(nearest_int(sub_min[j] / dminf), 0, 63) : 0;
  }
  BlockQ4K out;
  memset(&out, 0, sizeof(out));
  for (int j = 0; j < 4; j++) {
    out.scales[j] = (uint8_t)((scales6[j] & 63) | ((scales6[j + 4] >> 4) << 6));
    out.scales[j + 4] = (uint8_t)((mins6[j] & 63) | ((mins6[j + 4] >> 4) << 6));
    out.scales[j + 8] = (uint8_t)((scales6[j + 4] & 0x0F) | ((mins6[j + 4] & 0x0F) << 4));
  }
  for (int j = 0; j < 8; j++) {
    float sc = df * (float)scales6[j];
    float m = dminf * (float)mins6[j];
    const float* s = src + j * 32;
    int chunk = j / 2;
    bool hi = (j % 2) == 1;
    for (int k = 0; k < 32; k++) {
      uint8_t q = sc > 0.0f ? (uint8_t)clampi(nearest_int((s[k] + m) / sc), 0, 15) : 0;
      if (hi)
        out.qs[chunk * 32 + k] |= (uint8_t)(q << 4);
      else
        out.qs[chunk * 32 + k] |= q;
    }
  }
  out.d = f32_to_f16(d);
  out.dmin = f32_to_f16(dmin);
  return out;
}

// ------------------------------------------------------------- kquant.rs:715-771
BlockQ6K quantize_q6k_ref(const float* src) {
  float group_amax[16];
  for (int g = 0; g < 16; g++) {
    float m = 0.0f;
    for (int k = 0; k < 16; k++) m = rust_max(m, fabsf(src[g * 16 + k]));
    group_amax[g] = m;
  }
  float amax = 0.0f;
  for (int g = 0; g < 16; g++) amax = rust_max(amax, group_amax[g]);
  float d = amax / (127.0f * 31.0f);
  float df = f16_to_f32(f32_to_f16(d));
  BlockQ6K out;
  memset(&out, 0, sizeof(out));
  for (int g = 0; g < 16; g++)
    out.scales[g] = df > 0.0f ? (int8_t)clampi(nearest_int(group_amax[g] / (df * 31.0f)), -128, 127) : 0;
  for (int half = 0; half < 2; half++) {
    for (int l = 0; l < 32; l++) {
      // set(slot, qh_shift, ql_idx, hi) of kquant.rs:740-762
      const int slots[4] = {0, 1, 2, 3};
      const int shifts[4] = {0, 2, 4, 6};
      const int qlidx[4] = {l, l + 32, l, l + 32};
      const bool his[4] = {false, false, true, true};
      for (int s = 0; s < 4; s++) {
        int slot = slots[s];
        int g = (half * 128 + slot * 32 + l) / 16;
        float sc = df * (float)out.scales[g];
        float v = src[half * 128 + slot * 32 + l];
        uint8_t q = sc != 0.0f ? (uint8_t)clampi((int32_t)((uint32_t)nearest_int(v / sc) + 32u), 0, 63)
                               : 32;
        uint8_t lo = q & 0x0F, hib = (q >> 4) & 3;
        int qli = half * 64 + qlidx[s];
        if (his[s])
          out.ql[qli] |= (uint8_t)(lo << 4);
        else
          out.ql[qli] |= lo;
        out.qh[half * 32 + l] |= (uint8_t)(hib << shifts[s]);
      }
    }
  }
  out.d = f32_to_f16(d);
  return out;
}

// -------------------------------------------------------------- kernels.rs:72-82
float dot_q8_scalar(const BlockQ8_0* w, const BlockQ8_0* x, size_t nb) {
  float sum = 0.0f;
  for (size_t b = 0; b < nb; b++) {
    int32_t acc = 0;
    for (int i = 0; i < QK8_0; i++) acc += (int32_t)w[b].qs[i] * (int32_t)x[b].qs[i];
    sum += (float)acc * f16_to_f32(w[b].d) * f16_to_f32(x[b].d);
  }
  return sum;
}

// ------------------------------------------------------------- kernels.rs:261-286
__attribute__((target("avx2,fma"))) float dot_q8_avx2(const BlockQ8_0* w, const BlockQ8_0* x,
                                                      size_t nb) {
  __m256 acc = _mm256_setzero_ps();
  for (size_t b = 0; b < nb; b++) {
    __m256 d = _mm256_set1_ps(f16_to_f32(w[b].d) * f16_to_f32(x[b].d));
    __m256i qw = _mm256_loadu_si256((const __m256i*)w[b].qs);
    __m256i qx = _mm256_loadu_si256((const __m256i*)x[b].qs);
    __m256i abs_w = _mm256_sign_epi8(qw, qw);
    __m256i sgn_x = _mm256_sign_epi8(qx, qw);
    __m256i p16 = _mm256_maddubs_epi16(abs_w, sgn_x);
    __m256i p32 = _mm256_madd_epi16(p16, _mm256_set1_epi16(1));
    acc = _mm256_fmadd_ps(d, _mm256_cvtepi32_ps(p32), acc);
  }
  return hsum256(acc);
}

// ------------------------------------------------------------- kernels.rs:227-256
__attribute__((target("avx2,fma"))) void dot_q8_avx2_x4(const BlockQ8_0* w,
                                                        const BlockQ8_0* const xs[4], size_t nb,
                                                        float out[4]) {
  __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(),
                   _mm256_setzero_ps()};
  for (size_t bi = 0; bi < nb; bi++) {
    __m256i qw = _mm256_loadu_si256((const __m256i*)w[bi].qs);
    __m256i abs_w = _mm256_sign_epi8(qw, qw);
    float dw = f16_to_f32(w[bi].d);
    for (int lane = 0; lane < 4; lane++) {
      const BlockQ8_0* bx = xs[lane] + bi;
      __m256 d = _mm256_set1_ps(dw * f16_to_f32(bx->d));
      __m256i qx = _mm256_loadu_si256((const __m256i*)bx->qs);
      __m256i sgn_x = _mm256_sign_epi8(qx, qw);
      __m256i p16 = _mm256_maddubs_epi16(abs_w, sgn_x);
      __m256i p32 = _mm256_madd_epi16(p16, _mm256_set1_epi16(1));
      acc[lane] = _mm256_fmadd_ps(d, _mm256_cvtepi32_ps(p32), acc[lane]);
    }
  }
  for (int lane = 0; lane < 4; lane++) out[lane] = hsum256(acc[lane]);
}

// ------------------------------------------------------- kernels.rs:36-70, 91-143
namespace {
struct Q8Job {
  float* y;
  const BlockQ8_0* w;
  const BlockQ8_0* x;
  size_t rows, bpr, batch;
};
void q8_matvec_range(void* p, size_t r0, size_t r1) {
  auto* j = (Q8Job*)p;
  bool fast = g_fast_path;
  for (size_t r = r0; r < r1; r++) {
    const BlockQ8_0* row = j->w + r * j->bpr;
    j->y[r] = fast ? dot_q8_avx2(row, j->x, j->bpr) : dot_q8_scalar(row, j->x, j->bpr);
  }
}
void q8_matmul_range(void* p, size_t r0, size_t r1) {
  auto* j = (Q8Job*)p;
  bool fast = g_fast_path;
  size_t bpr = j->bpr, rows = j->rows, batch = j->batch;
  for (size_t r = r0; r < r1; r++) {
    const BlockQ8_0* row = j->w + r * bpr;
    size_t b = 0;
    while (fast && b + 4 <= batch) {
      const BlockQ8_0* xs[4] = {j->x + b * bpr, j->x + (b + 1) * bpr, j->x + (b + 2) * bpr,
                                j->x + (b + 3) * bpr};
      float o[4];
      dot_q8_avx2_x4(row, xs, bpr, o);
      for (int i = 0; i < 4; i++) j->y[(b + i) * rows + r] = o[i];
      b += 4;
    }
    while (b < batch) {
      const BlockQ8_0* x = j->x + b * bpr;
      j->y[b * rows + r] = fast ? dot_q8_avx2(row, x, bpr) : dot_q8_scalar(row, x, bpr);
      b += 1;
    }
  }
}
}  // namespace

void matvec_q8(float* y, const BlockQ8_0* w, const BlockQ8_0* x, size_t rows, size_t cols) {
  Q8Job j{y, w, x, rows, cols / QK8_0, 1};
  pool_run(rows, q8_matvec_range, &j);
}
void matmul_q8(float* y, const BlockQ8_0* w, const BlockQ8_0* xs, size_t rows, size_t cols,
               size_t batch) {
  Q8Job j{y, w, xs, rows, cols / QK8_0, batch};
  pool_run(rows, q8_matmul_range, &j);
}

// ---------------------------------------------- kernels.rs:146-220 (f16 KV helpers)
__attribute__((target("avx2,fma,f16c"))) static float dot_f16_f16c(const uint16_t* k,
                                                                   const float* q, size_t n) {
  __m256 acc = _mm256_setzero_ps();
  size_t chunks = n / 8;
  for (size_t i = 0; i < chunks; i++) {
    __m128i kh = _mm_loadu_si128((const __m128i*)(k + i * 8));
    __m256 kf = _mm256_cvtph_ps(kh);
    __m256 qf = _mm256_loadu_ps(q + i * 8);
    acc = _mm256_fmadd_ps(kf, qf, acc);
  }
  float sum = hsum256(acc);
  for (size_t i = chunks * 8; i < n; i++) sum += f16_to_f32(k[i]) * q[i];
  return sum;
}

__attribute__((target("avx2,fma,f16c"))) static void axpy_f16_f16c(float* out, float a,
                                                                   const uint16_t* v, size_t n) {
  __m256 av = _mm256_set1_ps(a);
  size_t chunks = n / 8;
  for (size_t i = 0; i < chunks; i++) {
    __m128i vh = _mm_loadu_si128((const __m128i*)(v + i * 8));
    __m256 vf = _mm256_cvtph_ps(vh);
    __m256 of = _mm256_loadu_ps(out + i * 8);
    _mm256_storeu_ps(out + i * 8, _mm256_fmadd_ps(av, vf, of));
  }
  for (size_t i = chunks * 8; i < n; i++) out[i] += a * f16_to_f32(v[i]);
}

float dot_f16(const uint16_t* k, const float* q, size_t n) {
  if (g_fast_f16) return dot_f16_f16c(k, q, n);
  float s = 0.0f;
  for (size_t i = 0; i < n; i++) s += f16_to_f32(k[i]) * q[i];
  return s;
}

void axpy_f16(float* out, float a, const uint16_t* v, size_t n) {
  if (g_fast_f16) {
    axpy_f16_f16c(out, a, v, n);
    return;
  }
  for (size_t i = 0; i < n; i++) out[i] += a * f16_to_f32(v[i]);
}

// ------------------------------------------------------------------- vec.rs:4-90
void rmsnorm(float* out, const float* x, const float* w, size_t n, float eps) {
  float ss = 0.0f;
  for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
  float scale = 1.0f / sqrtf(ss / (float)n + eps);
  for (size_t i = 0; i < n; i++) out[i] = x[i] * scale * w[i];
}

void rmsnorm_inplace(float* x, const float* w, size_t n, float eps) {
  float ss = 0.0f;
  for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
  float scale = 1.0f / sqrtf(ss / (float)n + eps);
  for (size_t i = 0; i < n; i++) x[i] *= scale * w[i];
}

void softmax(float* x, size_t n) {
  float max = -INFINITY;
  for (size_t i = 0; i < n; i++) max = rust_max(max, x[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; i++) {
    x[i] = expf_cr(x[i] - max);  // libm::expf (vec.rs:34) -> correctly rounded expf
    sum += x[i];
  }
  float inv = 1.0f / sum;
  for (size_t i = 0; i < n; i++) x[i] *= inv;
}

void swiglu(float* gate, const float* up, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float x = gate[i];
    float silu = x / (1.0f + expf_cr(-x));  // libm::expf (vec.rs:47)
    gate[i] = silu * up[i];
  }
}

float vdot(const float* a, const float* b, size_t n) {
  float s = 0.0f;
  for (size_t i = 0; i < n; i++) s += a[i] * b[i];
  return s;
}

void scale_inplace(float* x, size_t n, float s) {
  for (size_t i = 0; i < n; i++) x[i] *= s;
}

void saxpy(float* y, float a, const float* x, size_t n) {
  for (size_t i = 0; i < n; i++) y[i] += a * x[i];
}

size_t argmax(const float* x, size_t n) {
  size_t best = 0;
  float bv = -INFINITY;
  for (size_t i = 0; i < n; i++) {
    if (x[i] > bv) {
      bv = x[i];
      best = i;
    }
  }
  return best;
}

// ------------------------------------------------------------------ rope.rs:14-34
void rope_freqs(float* out, size_t head_dim, float theta, const Llama3Scaling* s) {
  size_t half = head_dim / 2;
  const float PI = 3.14159265358979323846f;
  for (size_t i = 0; i < half; i++) {
    float exponent = -2.0f * (float)i / (float)head_dim;
    float freq = powf(theta, exponent);
    if (s) {
      float wavelen = 2.0f * PI / freq;
      float low_wavelen = s->original_context / s->low_freq_factor;
      float high_wavelen = s->original_context / s->high_freq_factor;
      if (wavelen > low_wavelen) {
        freq /= s->factor;
      } else if (wavelen > high_wavelen) {
        float smooth = (s->original_context / wavelen - s->low_freq_factor) /
                       (s->high_freq_factor - s->low_freq_factor);
        freq = (1.0f - smooth) * freq / s->factor + smooth * freq;
      }
    }
    out[i] = freq;
  }
}

// ------------------------------------------------------------------ rope.rs:49-65
void rope_apply(float* x, size_t len, size_t head_dim, const float* freqs, size_t pos, int style) {
  size_t half = head_dim / 2;
  for (size_t h0 = 0; h0 + head_dim <= len; h0 += head_dim) {
    float* head = x + h0;
    for (size_t i = 0; i < half; i++) {
      float angle = (float)pos * freqs[i];
      float sn, cs;
      sincosf(angle, &sn, &cs);
      size_t ia = style == ROPE_ADJACENT ? 2 * i : i;
      size_t ib = style == ROPE_ADJACENT ? 2 * i + 1 : i + half;
      float a = head[ia], b = head[ib];
      head[ia] = a * cs - b * sn;
      head[ib] = a * sn + b * cs;
    }
  }
}

// ---------------------------------------------------------------- crc32.rs:6-79
namespace {
struct CrcTables {
  uint32_t t[8][256];
  CrcTables() {
    for (uint32_t i = 0; i < 256; i++) {
      uint32_t c = i;
      for (int k = 0; k < 8; k++) c = (c & 1) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
      t[0][i] = c;
    }
    for (int s = 1; s < 8; s++)
      for (int i = 0; i < 256; i++) t[s][i] = t[0][t[s - 1][i] & 0xff] ^ (t[s - 1][i] >> 8);
  }
};
const CrcTables& tables() {
  static CrcTables t;
  return t;
}
}  // namespace

uint32_t crc32_update(uint32_t c, const uint8_t* w, size_t n) {
  const CrcTables& T = tables();
  size_t i = 0;
  for (; i + 8 <= n; i += 8) {
    uint32_t lo = ((uint32_t)w[i] | ((uint32_t)w[i + 1] << 8) | ((uint32_t)w[i + 2] << 16) |
                   ((uint32_t)w[i + 3] << 24)) ^ c;
    c = T.t[7][lo & 0xff] ^ T.t[6][(lo >> 8) & 0xff] ^ T.t[5][(lo >> 16) & 0xff] ^
        T.t[4][lo >> 24] ^ T.t[3][w[i + 4]] ^ T.t[2][w[i + 5]] ^ T.t[1][w[i + 6]] ^ T.t[0][w[i + 7]];
  }
  for (; i < n; i++) c = T.t[0][(c ^ w[i]) & 0xff] ^ (c >> 8);
  return c;
}

uint32_t crc32(const uint8_t* data, size_t n) { return crc32_update(0xffffffffu, data, n) ^ 0xffffffffu; }

}  // namespace oracle
