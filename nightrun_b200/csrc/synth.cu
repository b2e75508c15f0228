// Seeded synthetic model weights generated directly in device memory.
//
// Recipe (shared with the CPU generator the tests use; results are
// byte-identical because only integer hashing and correctly rounded IEEE
// operations are involved):
//   key(kind, layer) = mix64(seed ^ mix64(kind << 32 | layer))
//   gauss(key, i)    = (Σ 12 24-bit uniforms of mix64(key + (6i+j)·φ), j=1..6) − 6·2^24, × 2^-24
//   linear weight    = gauss · 0.02 quantized per row with the reference quantizer of its dtype
//                      (q8.rs:27-44, kquant.rs:647-712, kquant.rs:715-771)
//   norm weight      = 1 + gauss · 0.01 (f32); rope_freqs factor = 1 + 0.5·(i mod 3)
#include "common.cuh"
#include "synth.cuh"

namespace nrc {
namespace {

NRC_DEV uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
constexpr uint64_t GOLDEN = 0x9E3779B97F4A7C15ull;

NRC_DEV float gauss(uint64_t key, uint64_t idx) {
  uint32_t s = 0;
  const uint64_t base = key + idx * 6 * GOLDEN;
#pragma unroll
  for (uint64_t j = 1; j <= 6; j++) {
    const uint64_t h = mix64(base + j * GOLDEN);
    s += (uint32_t)(h >> 40) + (uint32_t)((h >> 16) & 0xFFFFFF);
  }
  const int32_t t = (int32_t)s - 100663296;
  return __fmul_rn(__int2float_rn(t), 5.9604644775390625e-08f);
}

NRC_DEV int32_t nearest_int(float v) {
  return v >= 0.0f ? rust_f2i(__fadd_rn(v, 0.5f)) : rust_f2i(__fsub_rn(v, 0.5f));
}
NRC_DEV int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

__global__ void k_gen_f32(float* out, uint64_t n, uint64_t key, int rope_factors) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = rope_factors ? __fadd_rn(1.0f, __fmul_rn(0.5f, (float)(i % 3)))
                          : __fadd_rn(1.0f, __fmul_rn(gauss(key, i), 0.01f));
}

// One warp per Q8_0 block (q8::quantize of the row's f32 values).
__global__ void k_gen_q8_0(uint8_t* out, uint64_t nblocks, uint64_t key) {
  const int lane = threadIdx.x & 31;
  for (uint64_t b = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; b < nblocks;
       b += ((uint64_t)gridDim.x * blockDim.x) / 32) {
    const float v = __fmul_rn(gauss(key, b * 32 + lane), 0.02f);
    const float amax = warp_max(fabsf(v));
    const uint16_t dbits = f32_to_f16(__fdiv_rn(amax, 127.0f));
    const float d = f16_to_f32(dbits);
    const float inv = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float xs = __fmul_rn(v, inv);
    const float r = xs >= 0.0f ? __fadd_rn(xs, 0.5f) : __fsub_rn(xs, 0.5f);
    const int q = clampi(rust_f2i(r), -127, 127);
    uint8_t* blk = out + b * 34;
    blk[2 + lane] = (uint8_t)(int8_t)q;
    if (lane == 0) {
      blk[0] = (uint8_t)(dbits & 0xff);
      blk[1] = (uint8_t)(dbits >> 8);
    }
  }
}

// One thread per Q4_K super-block (kquant.rs:647-712, quantize_q4k_ref).
__global__ void k_gen_q4k(uint8_t* out, uint64_t nblocks, uint64_t key) {
  for (uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += (uint64_t)gridDim.x * blockDim.x) {
    float src[256];
    for (int k = 0; k < 256; k++) src[k] = __fmul_rn(gauss(key, b * 256 + k), 0.02f);
    float sub_scale[8], sub_min[8];
    for (int j = 0; j < 8; j++) {
      float mx = -3.40282347e38f, mn = 3.40282347e38f;
      for (int k = 0; k < 32; k++) {
        mx = fmaxf(mx, src[j * 32 + k]);
        mn = fminf(mn, src[j * 32 + k]);
      }
      sub_min[j] = fmaxf(-mn, 0.0f);
      sub_scale[j] = fmaxf(__fdiv_rn(__fadd_rn(mx, sub_min[j]), 15.0f), 0.0f);
    }
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; j++) {
      max_scale = fmaxf(max_scale, sub_scale[j]);
      max_min = fmaxf(max_min, sub_min[j]);
    }
    const float d = __fdiv_rn(max_scale, 63.0f);
    const float dmin = __fdiv_rn(max_min, 63.0f);
    const float df = f16_to_f32(f32_to_f16(d));
    const float dminf = f16_to_f32(f32_to_f16(dmin));
    uint32_t scales6[8], mins6[8];
    for (int j = 0; j < 8; j++) {
      scales6[j] = df > 0.0f ? (uint32_t)clampi(nearest_int(__fdiv_rn(sub_scale[j], df)), 0, 63) : 0u;
      mins6[j] = dminf > 0.0f ? (uint32_t)clampi(nearest_int(__fdiv_rn(sub_min[j], dminf)), 0, 63) : 0u;
    }
    uint8_t* o = out + b * 144;
    const uint16_t db = f32_to_f16(d), dmb = f32_to_f16(dmin);
    o[0] = (uint8_t)(db & 0xff);
    o[1] = (uint8_t)(db >> 8);
    o[2] = (uint8_t)(dmb & 0xff);
    o[3] = (uint8_t)(dmb >> 8);
    for (int j = 0; j < 4; j++) {
      o[4 + j] = (uint8_t)((scales6[j] & 63) | ((scales6[j + 4] >> 4) << 6));
      o[4 + j + 4] = (uint8_t)((mins6[j] & 63) | ((mins6[j + 4] >> 4) << 6));
      o[4 + j + 8] = (uint8_t)((scales6[j + 4] & 0x0F) | ((mins6[j + 4] & 0x0F) << 4));
    }
    uint8_t qs[128];
    for (int i = 0; i < 128; i++) qs[i] = 0;
    for (int j = 0; j < 8; j++) {
      const float sc = __fmul_rn(df, (float)scales6[j]);
      const float m = __fmul_rn(dminf, (float)mins6[j]);
      const int chunk = j / 2;
      const bool hi = (j & 1) != 0;
      for (int k = 0; k < 32; k++) {
        const uint32_t q =
            sc > 0.0f ? (uint32_t)clampi(nearest_int(__fdiv_rn(__fadd_rn(src[j * 32 + k], m), sc)), 0, 15) : 0u;
        if (hi)
          qs[chunk * 32 + k] |= (uint8_t)(q << 4);
        else
          qs[chunk * 32 + k] |= (uint8_t)q;
      }
    }
    for (int i = 0; i < 128; i++) o[16 + i] = qs[i];
  }
}

// One thread per Q6_K super-block (kquant.rs:715-771, quantize_q6k_ref).
__global__ void k_gen_q6k(uint8_t* out, uint64_t nblocks, uint64_t key) {
  for (uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += (uint64_t)gridDim.x * blockDim.x) {
    float src[256];
    for (int k = 0; k < 256; k++) src[k] = __fmul_rn(gauss(key, b * 256 + k), 0.02f);
    float ga[16];
    float amax = 0.0f;
    for (int g = 0; g < 16; g++) {
      float m = 0.0f;
      for (int k = 0; k < 16; k++) m = fmaxf(m, fabsf(src[g * 16 + k]));
      ga[g] = m;
    }
    for (int g = 0; g < 16; g++) amax = fmaxf(amax, ga[g]);
    const float d = __fdiv_rn(amax, 3937.0f);  // 127.0 * 31.0
    const float df = f16_to_f32(f32_to_f16(d));
    int8_t scales[16];
    for (int g = 0; g < 16; g++)
      scales[g] = df > 0.0f ? (int8_t)clampi(nearest_int(__fdiv_rn(ga[g], __fmul_rn(df, 31.0f))), -128, 127) : 0;
    uint8_t ql[128], qh[64];
    for (int i = 0; i < 128; i++) ql[i] = 0;
    for (int i = 0; i < 64; i++) qh[i] = 0;
    for (int half = 0; half < 2; half++) {
      for (int l = 0; l < 32; l++) {
        for (int slot = 0; slot < 4; slot++) {
          const int g = (half * 128 + slot * 32 + l) / 16;
          const float sc = __fmul_rn(df, (float)scales[g]);
          const float v = src[half * 128 + slot * 32 + l];
          const uint32_t q =
              sc != 0.0f ? (uint32_t)clampi((int)((uint32_t)nearest_int(__fdiv_rn(v, sc)) + 32u), 0, 63) : 32u;
          const uint32_t lo = q & 0x0F, hb = (q >> 4) & 3;
          const int qli = half * 64 + ((slot & 1) ? l + 32 : l);
          if (slot >= 2)
            ql[qli] |= (uint8_t)(lo << 4);
          else
            ql[qli] |= (uint8_t)lo;
          qh[half * 32 + l] |= (uint8_t)(hb << (2 * slot));
        }
      }
    }
    uint8_t* o = out + b * 210;
    for (int i = 0; i < 128; i++) o[i] = ql[i];
    for (int i = 0; i < 64; i++) o[128 + i] = qh[i];
    for (int i = 0; i < 16; i++) o[192 + i] = (uint8_t)scales[i];
    const uint16_t db = f32_to_f16(d);
    o[208] = (uint8_t)(db & 0xff);
    o[209] = (uint8_t)(db >> 8);
  }
}

uint64_t mix64_h(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

}  // namespace

uint64_t synth_tensor_key(uint64_t seed, uint32_t kind, uint32_t layer) {
  return mix64_h(seed ^ mix64_h(((uint64_t)kind << 32) | layer));
}

cudaError_t synth_fill(uint8_t* dst, int dtype, uint32_t kind, uint64_t rows, uint64_t cols, uint64_t key,
                       cudaStream_t s) {
  const uint64_t n = rows * cols;
  if (n == 0) return cudaSuccess;
  if (dtype == 0) {
    k_gen_f32<<<(unsigned)std::min<uint64_t>((n + 255) / 256, 4096), 256, 0, s>>>(reinterpret_cast<float*>(dst), n,
                                                                                   key, kind == 4 ? 1 : 0);
  } else if (dtype == 1) {
    const uint64_t nb = n / 32;
    k_gen_q8_0<<<(unsigned)std::min<uint64_t>((nb + 7) / 8, 65535), 256, 0, s>>>(dst, nb, key);
  } else if (dtype == 2) {
    const uint64_t nb = n / 256;
    k_gen_q4k<<<(unsigned)std::min<uint64_t>((nb + 127) / 128, 65535), 128, 0, s>>>(dst, nb, key);
  } else {
    const uint64_t nb = n / 256;
    k_gen_q6k<<<(unsigned)std::min<uint64_t>((nb + 127) / 128, 65535), 128, 0, s>>>(dst, nb, key);
  }
  return cudaGetLastError();
}

}  // namespace nrc
