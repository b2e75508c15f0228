// Streaming quantized GEMV for sm_100a: y = W · x over in-place Q8_0 / Q4_K /
// Q6_K weight blocks, for 1..8 activation vectors.
//
// Reference: crates/nr-tensor/src/kernels.rs:36-143 (Q8_0) and
// crates/nr-tensor/src/kquant.rs:192-250, 536-639 (Q4_K / Q6_K).
//
// Structure (persistent CTAs, up to two per SM):
//  * warp 8 (producer) streams the CTA's row tiles — contiguous byte ranges of
//    the weight matrix — into a ring of 16 KB shared-memory stages with 1-D TMA
//    bulk copies (cp.async.bulk, L2 evict-first, no cluster multicast), one
//    full/empty mbarrier pair per stage;
//  * warps 0-7 (consumers) stage the activations in shared memory once per
//    CTA (coalesced load, optional RMSNorm, quantization exactly as the
//    reference quantizes them), then split every stage into units — one Q8_0
//    block or one K-quant super-block per thread — and compute each unit's
//    exact integer dots with dp4a. For K-quants the consumers form two groups
//    that work on alternate stages, so two stages are in flight;
//  * each block's f32 term is rounded exactly as the reference's scalar dot
//    rounds it (kernels.rs:79, kquant.rs:212-215, 244-247) and parked in a
//    per-tile buffer; one thread per (row, token) then adds the terms in block
//    order — the reference's summation order — so every output is
//    bit-identical to dot_q8_scalar / dot_q4k_scalar / dot_q6k_scalar.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "expf_cr.cuh"
#include "gemv.cuh"

namespace nrc {
namespace {

constexpr int NCW = 8;             // consumer warps
constexpr int NC = NCW * 32;       // consumer threads
constexpr int NTHREADS = NC + 32;  // + producer warp
constexpr int MAX_STAGES = 8;
constexpr int STAGE_PAYLOAD = 16384;
constexpr int STAGE_BUF = STAGE_PAYLOAD + 64;
constexpr int XW = 68;  // words per 256-byte activation group (64 + 4 pad: conflict-free LDS.128)
constexpr int SMEM_RESERVE = 1024;  // static shared memory of the kernel, rounded up

struct Params {
  const uint8_t* w[3];
  float* y[3];
  int rows[3];
  int ld[3];
  int tile_start[4];
  int nseg, pair;
  int K, bpr, row_bytes;
  int RT;
  int unit_bytes, units_per_stage;
  int ntiles;
  int nt;
  int nstage, groups;
  const uint8_t* xq;
  const float* xf;
  int xf_ld;
  const float* norm_w;
  float eps;
  int epi;
  float scale;
  float* resid;
  int resid_ld;
  float rs;
  unsigned long long* argmax_key;
  unsigned* err;
  int off_x, off_xd, off_xb, off_t, t_elems;  // shared-memory layout (bytes / floats)
  int xs_floats;                              // f32 staging floats at off_t (prologue)
  int n_oct;
};

NRC_DEV int imin(int a, int b) { return a < b ? a : b; }

// Load `nw` 32-bit words starting at an arbitrary (2-byte aligned) smem address.
template <int NW>
NRC_DEV void load_words_unaligned(const uint8_t* src, uint32_t* out) {
  const uint32_t* base = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(src) & ~(uintptr_t)3);
  const uint32_t sh = (uint32_t)(reinterpret_cast<uintptr_t>(src) & 3) * 8;
  uint32_t prev = base[0];
#pragma unroll
  for (int i = 0; i < NW; i++) {
    const uint32_t nx = base[i + 1];
    out[i] = __funnelshift_r(prev, nx, sh);
    prev = nx;
  }
}

// ---------------------------------------------------------------- unit kernels
// One Q8_0 block (34 bytes, any 2-byte alignment). kernels.rs:72-82.
template <int NT>
NRC_DEV void unit_q8(const uint8_t* src, const uint32_t* xq, int xtok, const float* xd, int nt, int bpr,
                     float* t, int tstride) {
  uint32_t rw[9];
  load_words_unaligned<9>(src, rw);
  const float dw = f16_to_f32(rw[0] & 0xffffu);
  uint32_t q[8];
#pragma unroll
  for (int k = 0; k < 8; k++) q[k] = __byte_perm(rw[k], rw[k + 1], 0x5432);
#pragma unroll
  for (int tok = 0; tok < NT; tok++) {
    if (tok < nt) {
      const uint4* xv = reinterpret_cast<const uint4*>(xq + tok * xtok);
      const uint4 a = xv[0], b = xv[1];
      int acc = __dp4a((int)q[0], (int)a.x, 0);
      acc = __dp4a((int)q[1], (int)a.y, acc);
      acc = __dp4a((int)q[2], (int)a.z, acc);
      acc = __dp4a((int)q[3], (int)a.w, acc);
      acc = __dp4a((int)q[4], (int)b.x, acc);
      acc = __dp4a((int)q[5], (int)b.y, acc);
      acc = __dp4a((int)q[6], (int)b.z, acc);
      acc = __dp4a((int)q[7], (int)b.w, acc);
      // kernels.rs:79 — `acc as f32 * bw.scale() * bx.scale()`
      t[tok * tstride] = __fmul_rn(__fmul_rn(i2f(acc), dw), xd[tok * bpr]);
    }
  }
}

// One Q4_K super-block (144 bytes). kquant.rs:192-218.
template <int NT, int ALIGNED>
NRC_DEV void unit_q4k(const uint8_t* src, const uint32_t* xq, const float* xd, const int* xb, int nt, int bpr,
                      float* t, int tstride) {
  uint32_t w[36];
  if (ALIGNED) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int i = 0; i < 9; i++) {
      const uint4 v = s4[i];
      w[4 * i] = v.x;
      w[4 * i + 1] = v.y;
      w[4 * i + 2] = v.z;
      w[4 * i + 3] = v.w;
    }
  } else {
    load_words_unaligned<36>(src, w);
  }
  const float dw = f16_to_f32(w[0] & 0xffffu);
  const float dminw = f16_to_f32(w[0] >> 16);
  // 12 scale bytes in w[1..3]; q4k_scale_min (kquant.rs:83-92).
  uint32_t sb[12];
#pragma unroll
  for (int i = 0; i < 12; i++) sb[i] = (w[1 + i / 4] >> (8 * (i % 4))) & 0xffu;
  int sc[8], mn[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    if (j < 4) {
      sc[j] = (int)(sb[j] & 63);
      mn[j] = (int)(sb[j + 4] & 63);
    } else {
      sc[j] = (int)((sb[j + 4] & 0x0F) | ((sb[j - 4] >> 6) << 4));
      mn[j] = (int)((sb[j + 4] >> 4) | ((sb[j] >> 6) << 4));
    }
  }
#pragma unroll
  for (int tok = 0; tok < NT; tok++) {
    if (tok < nt) {
      const uint32_t* xw = xq + tok * bpr * XW;
      float sum_q = 0.0f;
      int sum_m = 0;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const uint4* xv = reinterpret_cast<const uint4*>(xw + j * 8);
        const uint4 a = xv[0], b = xv[1];
        const int c = 4 + (j / 2) * 8;
        const bool hi = (j & 1) != 0;
        uint32_t n[8];
#pragma unroll
        for (int m = 0; m < 8; m++) n[m] = hi ? ((w[c + m] >> 4) & 0x0F0F0F0Fu) : (w[c + m] & 0x0F0F0F0Fu);
        int sub = __dp4a((int)n[0], (int)a.x, 0);
        sub = __dp4a((int)n[1], (int)a.y, sub);
        sub = __dp4a((int)n[2], (int)a.z, sub);
        sub = __dp4a((int)n[3], (int)a.w, sub);
        sub = __dp4a((int)n[4], (int)b.x, sub);
        sub = __dp4a((int)n[5], (int)b.y, sub);
        sub = __dp4a((int)n[6], (int)b.z, sub);
        sub = __dp4a((int)n[7], (int)b.w, sub);
        sum_q = __fadd_rn(sum_q, __fmul_rn((float)sc[j], i2f(sub)));
        sum_m += mn[j] * xb[tok * bpr * 8 + j];
      }
      const float dx = xd[tok * bpr];
      const float d_all = __fmul_rn(dw, dx);
      const float dmin_all = __fmul_rn(dminw, dx);
      t[tok * tstride] = __fsub_rn(__fmul_rn(d_all, sum_q), __fmul_rn(dmin_all, i2f(sum_m)));
    }
  }
}

// One Q6_K super-block (210 bytes, 2-byte aligned). kquant.rs:220-250.
template <int NT>
NRC_DEV void unit_q6k(const uint8_t* src, const uint32_t* xq, const float* xd, int nt, int bpr, float* t,
                      int tstride) {
  uint32_t rw[53];
  load_words_unaligned<53>(src, rw);
  const float dw = f16_to_f32(rw[52] & 0xffffu);
#pragma unroll
  for (int tok = 0; tok < NT; tok++) {
    if (tok < nt) {
      const uint32_t* xw = xq + tok * bpr * XW;
      float sum = 0.0f;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        int gs[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int m = 0; m < 8; m++) {
          const uint32_t l0 = rw[h * 16 + m], l1 = rw[h * 16 + 8 + m], hh = rw[32 + h * 8 + m];
          const uint32_t q1 = (l0 & 0x0F0F0F0Fu) | ((hh & 0x03030303u) << 4);
          const uint32_t q2 = (l1 & 0x0F0F0F0Fu) | ((hh << 2) & 0x30303030u);
          const uint32_t q3 = ((l0 >> 4) & 0x0F0F0F0Fu) | (hh & 0x30303030u);
          const uint32_t q4 = ((l1 >> 4) & 0x0F0F0F0Fu) | ((hh >> 2) & 0x30303030u);
          // bytewise q - 32 (q <= 63, so q + 0x60 never carries)
          const uint32_t s1 = (q1 + 0x60606060u) ^ 0x80808080u;
          const uint32_t s2 = (q2 + 0x60606060u) ^ 0x80808080u;
          const uint32_t s3 = (q3 + 0x60606060u) ^ 0x80808080u;
          const uint32_t s4 = (q4 + 0x60606060u) ^ 0x80808080u;
          const uint32_t* x = xw + h * 32;
          gs[m / 4] = __dp4a((int)s1, (int)x[m], gs[m / 4]);
          gs[2 + m / 4] = __dp4a((int)s2, (int)x[8 + m], gs[2 + m / 4]);
          gs[4 + m / 4] = __dp4a((int)s3, (int)x[16 + m], gs[4 + m / 4]);
          gs[6 + m / 4] = __dp4a((int)s4, (int)x[24 + m], gs[6 + m / 4]);
        }
#pragma unroll
        for (int g = 0; g < 8; g++) {
          const int b = h * 8 + g;
          const int scv = (int)(int8_t)((rw[48 + b / 4] >> (8 * (b % 4))) & 0xffu);
          sum = __fadd_rn(sum, __fmul_rn((float)scv, i2f(gs[g])));
        }
      }
      const float d_all = __fmul_rn(dw, xd[tok * bpr]);
      t[tok * tstride] = __fmul_rn(d_all, sum);
    }
  }
}

// ------------------------------------------------------------ activation prologue
// Activation buffers in shared memory:
//   Q8_0: xq[(tok*n_oct + b/8)*XW + (b%8)*8 + w], xd[tok*bpr + b]
//   Q8_K: xq[(tok*bpr + b)*XW + w], xd[tok*bpr + b], xb[(tok*bpr + b)*8 + j] (bsum pairs)
NRC_DEV int xq_index(int fmt, const Params& p, int tok, int b) {
  return fmt == FMT_Q8_0 ? (tok * p.n_oct + b / 8) * XW + (b % 8) * 8 : (tok * p.bpr + b) * XW;
}

// Quantize nt f32 rows (optionally RMS-normalised) into the activation buffers,
// exactly as q8::quantize (q8.rs:27-44) / quantize_q8k (kquant.rs:157-187).
// Each row is first copied to shared memory (`xs`, aliasing the term buffer)
// with one coalesced pass; the norm's sum of squares uses one fixed order, so
// every CTA and every launch derive identical activations.
template <int FMT>
NRC_DEV void build_x_f32(const Params& p, uint8_t* smem) {
  uint32_t* xq = reinterpret_cast<uint32_t*>(smem + p.off_x);
  float* xd = reinterpret_cast<float*>(smem + p.off_xd);
  int* xb = reinterpret_cast<int*>(smem + p.off_xb);
  float* xs = reinterpret_cast<float*>(smem + p.off_t);
  __shared__ float nscale[8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = p.K;
  if (p.norm_w) {
    // vec::rmsnorm (vec.rs:4-14): `ss += v * v` in index order, then
    // scale = 1 / sqrtf(ss / n + eps). Thread `tok` runs token tok's chain
    // over chunks staged in shared memory (row stride CH + 1: no bank conflicts).
    const int CH = p.xs_floats / p.nt - 1;
    float ss = 0.0f;
    for (int c0 = 0; c0 < K; c0 += CH) {
      const int cn = K - c0 < CH ? K - c0 : CH;
      for (int i = tid; i < p.nt * cn; i += NC) {
        const int tk = i / cn, k = i - tk * cn;
        xs[tk * (CH + 1) + k] = p.xf[(size_t)tk * p.xf_ld + c0 + k];
      }
      named_sync(1, NC);
      if (tid < p.nt) {
        const float* r = xs + tid * (CH + 1);
#pragma unroll 8
        for (int k = 0; k < cn; k++) ss = __fadd_rn(ss, __fmul_rn(r[k], r[k]));
      }
      named_sync(1, NC);
    }
    if (tid < p.nt) nscale[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), p.eps)));
    named_sync(1, NC);
  }
  for (int tok = 0; tok < p.nt; tok++) {
    const float* src = p.xf + (size_t)tok * p.xf_ld;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (K & 3) == 0) {
      for (int i = tid; i < K / 4; i += NC) reinterpret_cast<float4*>(xs)[i] = reinterpret_cast<const float4*>(src)[i];
    } else {
      for (int i = tid; i < K; i += NC) xs[i] = src[i];
    }
    named_sync(1, NC);
    const float sc = p.norm_w ? nscale[tok] : 1.0f;
    if (FMT == FMT_Q8_0) {
      for (int b = warp; b < p.bpr; b += NCW) {
        float v = xs[b * 32 + lane];
        if (p.norm_w) v = __fmul_rn(__fmul_rn(v, sc), p.norm_w[b * 32 + lane]);
        const float amax = warp_max(fabsf(v));
        const uint16_t dbits = f32_to_f16(__fdiv_rn(amax, 127.0f));
        const float d = f16_to_f32(dbits);
        const float inv = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const float xsv = __fmul_rn(v, inv);
        const float r = xsv >= 0.0f ? __fadd_rn(xsv, 0.5f) : __fsub_rn(xsv, 0.5f);
        int q = rust_f2i(r);
        q = q < -127 ? -127 : (q > 127 ? 127 : q);
        reinterpret_cast<uint8_t*>(xq + xq_index(FMT_Q8_0, p, tok, b))[lane] = (uint8_t)(int8_t)q;
        if (lane == 0) xd[tok * p.bpr + b] = d;
      }
    } else {
      for (int b = warp; b < p.bpr; b += NCW) {
        const float4* s4 = reinterpret_cast<const float4*>(xs + b * 256 + lane * 8);
        const float4 va = s4[0], vb = s4[1];
        float v[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
        if (p.norm_w) {
#pragma unroll
          for (int k = 0; k < 8; k++) v[k] = __fmul_rn(__fmul_rn(v[k], sc), p.norm_w[b * 256 + lane * 8 + k]);
        }
        // First strict maximum of |v| in index order (kquant.rs:160-167).
        float amax = 0.0f, mx = 0.0f;
        int idx = 0x7fffffff;
#pragma unroll
        for (int k = 0; k < 8; k++) {
          if (fabsf(v[k]) > amax) {
            amax = fabsf(v[k]);
            mx = v[k];
            idx = lane * 8 + k;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float a2 = __shfl_xor_sync(0xffffffffu, amax, o);
          const float m2 = __shfl_xor_sync(0xffffffffu, mx, o);
          const int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
          if (a2 > amax || (a2 == amax && i2 < idx)) {
            amax = a2;
            mx = m2;
            idx = i2;
          }
        }
        uint32_t* qw = xq + xq_index(FMT, p, tok, b);
        int* bs = xb + (tok * p.bpr + b) * 8;
        if (amax == 0.0f) {
          qw[lane * 2] = 0u;
          qw[lane * 2 + 1] = 0u;
          if (lane < 8) bs[lane] = 0;
          if (lane == 0) xd[tok * p.bpr + b] = 0.0f;
          continue;
        }
        const float iscale = __fdiv_rn(-128.0f, mx);
        int part = 0;
        uint32_t pk[2] = {0u, 0u};
#pragma unroll
        for (int k = 0; k < 8; k++) {
          const float z = __fmul_rn(iscale, v[k]);
          int q = z >= 0.0f ? rust_f2i(__fadd_rn(z, 0.5f)) : rust_f2i(__fsub_rn(z, 0.5f));
          q = q > 127 ? 127 : q;
          const int8_t q8 = (int8_t)(uint8_t)(q & 0xff);
          part += q8;
          pk[k / 4] |= ((uint32_t)(uint8_t)q8) << (8 * (k % 4));
        }
        qw[lane * 2] = pk[0];
        qw[lane * 2 + 1] = pk[1];
        // The Q4_K min term uses pairs of 16-value bsums = 32 values = lanes 4j..4j+3.
        int s4s = part + __shfl_down_sync(0xffffffffu, part, 1);
        s4s += __shfl_down_sync(0xffffffffu, s4s, 2);
        if ((lane & 3) == 0) bs[lane / 4] = s4s;
        if (lane == 0) xd[tok * p.bpr + b] = __fdiv_rn(1.0f, iscale);
      }
    }
    named_sync(1, NC);  // xs is reused by the next token / the term buffer
  }
}

// Activations given as blocks in global memory (the kernel-level entry points).
template <int FMT>
NRC_DEV void build_x_blocks(const Params& p, uint8_t* smem) {
  uint32_t* xq = reinterpret_cast<uint32_t*>(smem + p.off_x);
  float* xd = reinterpret_cast<float*>(smem + p.off_xd);
  int* xb = reinterpret_cast<int*>(smem + p.off_xb);
  const int tid = threadIdx.x;
  const int nblk = p.nt * p.bpr;
  if (FMT == FMT_Q8_0) {
    for (int i = tid; i < nblk; i += NC) {
      const int tok = i / p.bpr, b = i % p.bpr;
      const uint8_t* s = p.xq + (size_t)i * 34;
      uint32_t* dst = xq + xq_index(FMT_Q8_0, p, tok, b);
#pragma unroll
      for (int k = 0; k < 8; k++)
        dst[k] = (uint32_t)s[2 + 4 * k] | ((uint32_t)s[3 + 4 * k] << 8) | ((uint32_t)s[4 + 4 * k] << 16) |
                 ((uint32_t)s[5 + 4 * k] << 24);
      xd[tok * p.bpr + b] = f16_to_f32((uint32_t)s[0] | ((uint32_t)s[1] << 8));
    }
  } else {
    for (int i = tid; i < nblk; i += NC) {
      const int tok = i / p.bpr, b = i % p.bpr;
      const uint32_t* s = reinterpret_cast<const uint32_t*>(p.xq + (size_t)i * 292);
      uint32_t* dst = xq + xq_index(FMT, p, tok, b);
#pragma unroll 8
      for (int k = 0; k < 64; k++) dst[k] = s[1 + k];
      xd[tok * p.bpr + b] = __uint_as_float(s[0]);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const uint32_t pr = s[65 + j];
        xb[(tok * p.bpr + b) * 8 + j] = (int)(int16_t)(pr & 0xffffu) + (int)(int16_t)(pr >> 16);
      }
    }
  }
}

// ------------------------------------------------------------------ the kernel
struct Span {
  const uint8_t* base;  // first byte of the span's first row
  const uint8_t* wbeg;  // weight buffer bounds (never read outside)
  const uint8_t* wend;
  int row0, nrows, seg;
};

NRC_DEV int tile_spans(const Params& p, int tile, Span* sp) {
  if (p.pair) {
    const int row0 = tile * p.RT;
    const int nr = imin(p.RT, p.rows[0] - row0);
    for (int s = 0; s < 2; s++) {
      sp[s].base = p.w[s] + (size_t)row0 * p.row_bytes;
      sp[s].wbeg = p.w[s];
      sp[s].wend = p.w[s] + (size_t)p.rows[s] * p.row_bytes;
      sp[s].row0 = row0;
      sp[s].nrows = nr;
      sp[s].seg = s;
    }
    return 2;
  }
  int s = 0;
  while (s + 1 < p.nseg && tile >= p.tile_start[s + 1]) s++;
  const int row0 = (tile - p.tile_start[s]) * p.RT;
  sp[0].base = p.w[s] + (size_t)row0 * p.row_bytes;
  sp[0].wbeg = p.w[s];
  sp[0].wend = p.w[s] + (size_t)p.rows[s] * p.row_bytes;
  sp[0].row0 = row0;
  sp[0].nrows = imin(p.RT, p.rows[s] - row0);
  sp[0].seg = s;
  return 1;
}

template <int FMT, int NT, int XMODE, int ALIGNED>
__global__ void __launch_bounds__(NTHREADS, (NT <= 2 ? 2 : 1)) gemv_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.nstage * STAGE_BUF);
  uint64_t* empty = full + MAX_STAGES;
  __shared__ volatile int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NS = p.nstage;
  const int G = p.groups;            // consumer groups (stage `it` belongs to group it % G)
  const int WPG = NCW / G;           // warps per group

  if (tid == 0) {
    for (int s = 0; s < NS; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], WPG);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == NCW) {
    // ----------------------------------------------------------- producer
    const uint64_t pol = l2_evict_first();
    int it = 0;
    Span sp[2];
    for (int tile = blockIdx.x; tile < p.ntiles && !abort_flag; tile += gridDim.x) {
      const int ns = tile_spans(p, tile, sp);
      for (int si = 0; si < ns && !abort_flag; si++) {
        const int nunits = sp[si].nrows * (p.row_bytes / p.unit_bytes);
        for (int u0 = 0; u0 < nunits; u0 += p.units_per_stage, it++) {
          const int u1 = imin(u0 + p.units_per_stage, nunits);
          const int s = it % NS;
          if (it >= NS) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&empty[s], ((it / NS) - 1) & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok || abort_flag) {
              if (lane == 0) {
                abort_flag = 1;
                atomicOr(p.err, ERR_WAIT_EMPTY);
              }
              break;
            }
          }
          // Bytes [g0, g1) land at dst + (addr - floor16(g0)). The 16-byte
          // aligned part inside the weight buffer goes by one bulk copy; the
          // (at most 2x15) ragged bytes at unaligned buffer ends by plain loads.
          const uintptr_t g0 = reinterpret_cast<uintptr_t>(sp[si].base) + (size_t)u0 * p.unit_bytes;
          const uintptr_t g1 = reinterpret_cast<uintptr_t>(sp[si].base) + (size_t)u1 * p.unit_bytes;
          const uintptr_t a0 = g0 & ~(uintptr_t)15;
          const uintptr_t wb = (reinterpret_cast<uintptr_t>(sp[si].wbeg) + 15) & ~(uintptr_t)15;
          const uintptr_t we = reinterpret_cast<uintptr_t>(sp[si].wend) & ~(uintptr_t)15;
          uintptr_t blo = a0 > wb ? a0 : wb;
          uintptr_t bhi = (g1 + 15) & ~(uintptr_t)15;
          if (bhi > we) bhi = we;
          if (bhi <= blo) blo = bhi = g0;
          uint8_t* dst = stages + s * STAGE_BUF;
          for (uintptr_t a = g0 + lane; a < blo; a += 32) dst[a - a0] = *reinterpret_cast<const uint8_t*>(a);
          for (uintptr_t a = (bhi > g0 ? bhi : g0) + lane; a < g1; a += 32)
            dst[a - a0] = *reinterpret_cast<const uint8_t*>(a);
          __syncwarp();
          if (lane == 0) {
            const uint32_t nbytes = bhi > blo ? (uint32_t)(bhi - blo) : 0u;
            mbar_arrive_expect_tx(&full[s], nbytes);
            if (nbytes) bulk_g2s(dst + (blo - a0), reinterpret_cast<const void*>(blo), nbytes, &full[s], pol);
          }
        }
      }
    }
    // Drain: wait (bounded) for the copies of the last issued stages, so the
    // CTA never exits with a bulk copy in flight.
    if (lane == 0) {
      for (int k = it - 1; k >= 0 && k >= it - NS; k--) {
        if (!mbar_wait(&full[k % NS], (k / NS) & 1)) atomicOr(p.err, ERR_DRAIN);
      }
    }
    return;
  }

  // ------------------------------------------------------------- consumers
  pdl_wait();
  if (XMODE == 1)
    build_x_f32<FMT>(p, smem);
  else
    build_x_blocks<FMT>(p, smem);
  named_sync(1, NC);

  const uint32_t* xq = reinterpret_cast<const uint32_t*>(smem + p.off_x);
  const float* xd = reinterpret_cast<const float*>(smem + p.off_xd);
  const int* xb = reinterpret_cast<const int*>(smem + p.off_xb);
  float* tbuf = reinterpret_cast<float*>(smem + p.off_t);
  const int TS = p.bpr + 1;  // odd stride: conflict-free chains
  const int grp = warp / WPG;
  const int gtid = tid - grp * WPG * 32;
  const int GN = WPG * 32;  // threads per group
  const int upr = p.row_bytes / p.unit_bytes;
  const int xtok = FMT == FMT_Q8_0 ? p.n_oct * XW : p.bpr * XW;
  int it = 0, tc = 0;
  Span sp[2];
  unsigned long long best = 0ull;
  for (int tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, tc++) {
    float* tb = tbuf + (tc & 1) * p.t_elems;
    const int ns = tile_spans(p, tile, sp);
    for (int si = 0; si < ns; si++) {
      const int nunits = sp[si].nrows * upr;
      for (int u0 = 0; u0 < nunits; u0 += p.units_per_stage, it++) {
        if (it % G != grp) continue;
        const int u1 = imin(u0 + p.units_per_stage, nunits);
        const int s = it % NS;
        const bool ok = !abort_flag && mbar_wait(&full[s], (it / NS) & 1);
        if (!ok) {
          if (lane == 0 && !abort_flag) {
            abort_flag = 1;
            atomicOr(p.err, ERR_WAIT_FULL);
          }
        } else {
          const uintptr_t g0 = reinterpret_cast<uintptr_t>(sp[si].base) + (size_t)u0 * p.unit_bytes;
          const uint8_t* sbase = stages + s * STAGE_BUF + (g0 & 15);
          for (int j = gtid; j < u1 - u0; j += GN) {
            const int u = u0 + j;
            const int r = u / upr, g = u % upr;
            const uint8_t* src = sbase + (size_t)j * p.unit_bytes;
            float* t = tb + ((si * p.RT + r) * NT) * TS + g;
            if (FMT == FMT_Q8_0)
              unit_q8<NT>(src, xq + (g / 8) * XW + (g % 8) * 8, xtok, xd + g, p.nt, p.bpr, t, TS);
            else if (FMT == FMT_Q4K)
              unit_q4k<NT, ALIGNED>(src, xq + g * XW, xd + g, xb + g * 8, p.nt, p.bpr, t, TS);
            else
              unit_q6k<NT>(src, xq + g * XW, xd + g, p.nt, p.bpr, t, TS);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
    }
    named_sync(1, NC);
    if (abort_flag) continue;
    // Ordered per-(row, token) chains + epilogue.
    const int nr = sp[0].nrows;
    const int items = nr * p.nt;
    for (int i = tid; i < items; i += NC) {
      const int r = i / p.nt, tok = i % p.nt;
      const float* tp = tb + (r * NT + tok) * TS;
      float s = 0.0f;
      for (int b = 0; b < p.bpr; b++) s = __fadd_rn(s, tp[b]);
      const int row = sp[0].row0 + r;
      const int sg = sp[0].seg;
      if (p.epi == EPI_RESID) {
        float* dst = p.resid + (size_t)tok * p.resid_ld + row;
        *dst = __fadd_rn(*dst, __fmul_rn(p.rs, s));
      } else if (p.epi == EPI_SWIGLU) {
        const float* tu = tb + ((p.RT + r) * NT + tok) * TS;
        float su = 0.0f;
        for (int b = 0; b < p.bpr; b++) su = __fadd_rn(su, tu[b]);
        // vec::swiglu: silu = x / (1 + expf(-x)); gate = silu * up
        const float silu = __fdiv_rn(s, __fadd_rn(1.0f, expf_cr(-s)));
        p.y[0][(size_t)tok * p.ld[0] + row] = __fmul_rn(silu, su);
      } else {
        if (p.scale != 1.0f) s = __fmul_rn(s, p.scale);
        p.y[sg][(size_t)tok * p.ld[sg] + row] = s;
        if (p.epi == EPI_ARGMAX && tok == 0 && argmax_candidate(s)) {
          const unsigned long long k = argmax_key(s, (uint32_t)row);
          best = k > best ? k : best;
        }
      }
    }
  }
  if (p.epi == EPI_ARGMAX) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
      best = v > best ? v : best;
    }
    if (lane == 0 && best) atomicMax(p.argmax_key, best);
  }
}

// ------------------------------------------------------------------ host side
using KernelFn = void (*)(Params);

template <int FMT, int XMODE, int AL>
KernelFn pick_nt(int NTc) {
  switch (NTc) {
    case 1: return gemv_kernel<FMT, 1, XMODE, AL>;
    case 2: return gemv_kernel<FMT, 2, XMODE, AL>;
    case 4: return gemv_kernel<FMT, 4, XMODE, AL>;
    default: return gemv_kernel<FMT, 8, XMODE, AL>;
  }
}

KernelFn pick_kernel(int fmt, int NTc, int xmode, int aligned) {
  if (fmt == FMT_Q8_0) return xmode ? pick_nt<FMT_Q8_0, 1, 0>(NTc) : pick_nt<FMT_Q8_0, 0, 0>(NTc);
  if (fmt == FMT_Q4K) {
    if (aligned) return xmode ? pick_nt<FMT_Q4K, 1, 1>(NTc) : pick_nt<FMT_Q4K, 0, 1>(NTc);
    return xmode ? pick_nt<FMT_Q4K, 1, 0>(NTc) : pick_nt<FMT_Q4K, 0, 0>(NTc);
  }
  return xmode ? pick_nt<FMT_Q6K, 1, 0>(NTc) : pick_nt<FMT_Q6K, 0, 0>(NTc);
}

struct DevInfo {
  int sms = 0;
  int smem_optin = 0;
  int smem_per_sm = 0;
};

DevInfo dev_info() {
  static std::mutex mu;
  static std::map<int, DevInfo> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  auto itc = cache.find(dev);
  if (itc != cache.end()) return itc->second;
  DevInfo d;
  cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  cache[dev] = d;
  return d;
}

int occupancy(KernelFn fn, int smem, int smem_optin) {
  static std::mutex mu;
  static std::map<std::tuple<int, void*, int>, int> cache;
  static std::map<std::pair<int, void*>, bool> attr_set;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  auto key = std::make_tuple(dev, (void*)fn, smem);
  auto itc = cache.find(key);
  if (itc != cache.end()) return itc->second;
  // The attribute is an upper bound: set it once to the largest dynamic size any launch may use.
  if (!attr_set[std::make_pair(dev, (void*)fn)]) {
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin - SMEM_RESERVE);
    attr_set[std::make_pair(dev, (void*)fn)] = true;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, NTHREADS, smem) != cudaSuccess) n = 0;
  cache[key] = n;
  return n;
}

}  // namespace

cudaError_t gemv_run(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  Params p{};
  const int blk = a.fmt == FMT_Q8_0 ? QK8_0 : QK_K;
  const int bbytes = a.fmt == FMT_Q8_0 ? Q8_0_BYTES : (a.fmt == FMT_Q4K ? Q4K_BYTES : Q6K_BYTES);
  if (a.K <= 0 || a.K % blk || a.nt < 1 || a.nt > 8 || a.nseg < 1 || a.nseg > 3) return cudaErrorInvalidValue;
  p.K = a.K;
  p.bpr = a.K / blk;
  p.row_bytes = p.bpr * bbytes;
  p.nt = a.nt;
  const int NTc = a.nt <= 1 ? 1 : (a.nt <= 2 ? 2 : (a.nt <= 4 ? 4 : 8));
  bool aligned = true;
  for (int s = 0; s < a.nseg; s++) aligned = aligned && ((reinterpret_cast<uintptr_t>(a.seg[s].w) & 15) == 0);
  p.unit_bytes = bbytes;
  p.units_per_stage = STAGE_PAYLOAD / p.unit_bytes;
  p.groups = a.fmt == FMT_Q8_0 ? 1 : 2;
  p.n_oct = (p.bpr + 7) / 8;
  p.nseg = a.nseg;
  p.pair = a.pair;
  for (int s = 0; s < a.nseg; s++) {
    p.w[s] = static_cast<const uint8_t*>(a.seg[s].w);
    p.y[s] = a.seg[s].y;
    p.rows[s] = a.seg[s].rows;
    p.ld[s] = a.seg[s].ld;
  }
  p.xq = static_cast<const uint8_t*>(a.xq);
  p.xf = a.xf;
  p.xf_ld = a.xf_ld;
  p.norm_w = a.norm_w;
  p.eps = a.eps;
  p.epi = a.epi;
  p.scale = a.scale;
  p.resid = a.resid;
  p.resid_ld = a.resid_ld;
  p.rs = a.rs;
  p.argmax_key = a.argmax_key;
  p.err = a.err;
  const int xmode = a.xq ? 0 : 1;

  // Shared memory: stages | barriers | activations | per-tile term buffers
  // (the term buffers double as the f32 staging row of the prologue).
  const DevInfo di = dev_info();
  size_t fixed = 2 * MAX_STAGES * 8;
  const size_t x_off = fixed;
  size_t off = x_off;
  if (a.fmt == FMT_Q8_0)
    off += (size_t)NTc * p.n_oct * XW * 4;
  else
    off += (size_t)NTc * p.bpr * XW * 4;
  const size_t xd_off = off;
  off += (size_t)NTc * p.bpr * 4;
  const size_t xb_off = off;
  if (a.fmt != FMT_Q8_0) off += (size_t)NTc * p.bpr * 8 * 4;
  off = (off + 15) & ~(size_t)15;
  const size_t t_off = off;
  const int span_mult = a.pair ? 2 : 1;
  auto tiles_for = [&](int rt) {
    if (a.pair) return (a.seg[0].rows + rt - 1) / rt;
    int n = 0;
    for (int s = 0; s < a.nseg; s++) n += (a.seg[s].rows + rt - 1) / rt;
    return n;
  };
  auto tbytes = [&](int rt) {
    size_t t = (size_t)2 * span_mult * rt * NTc * (p.bpr + 1) * 4;
    const size_t xs = xmode ? (size_t)a.K * 4 : 0;
    return t > xs ? t : xs;
  };
  int RT = std::max(1, 32 / NTc);
  while (RT > 1 && tiles_for(RT) < 4 * di.sms) RT /= 2;
  const size_t opt_limit = (size_t)di.smem_optin - SMEM_RESERVE;
  const size_t two_limit = (size_t)di.smem_per_sm / 2 - SMEM_RESERVE;
  // Two CTAs per SM when at least 3 stages fit in half an SM, else one CTA with up to 8 stages.
  int nstage = 0;
  for (int rt = RT; rt >= 1 && nstage == 0; rt /= 2) {
    const size_t rest = off + tbytes(rt);
    if (NTc <= 2 && rest + 3 * (size_t)STAGE_BUF <= two_limit) {
      nstage = (int)std::min<size_t>(MAX_STAGES, (two_limit - rest) / STAGE_BUF);
      RT = rt;
    } else if (rest + 3 * (size_t)STAGE_BUF <= opt_limit) {
      nstage = (int)std::min<size_t>(MAX_STAGES, (opt_limit - rest) / STAGE_BUF);
      RT = rt;
    }
    if (rt == 1) break;
  }
  if (nstage < 3) return cudaErrorInvalidValue;
  p.nstage = nstage;
  p.RT = RT;
  p.t_elems = span_mult * RT * NTc * (p.bpr + 1);
  p.xs_floats = (int)(tbytes(RT) / 4);
  const size_t stage_bytes = (size_t)nstage * STAGE_BUF;
  p.off_x = (int)(stage_bytes + x_off);
  p.off_xd = (int)(stage_bytes + xd_off);
  p.off_xb = (int)(stage_bytes + xb_off);
  p.off_t = (int)(stage_bytes + t_off);
  const size_t smem = stage_bytes + off + tbytes(RT);
  p.ntiles = 0;
  if (a.pair) {
    p.ntiles = (a.seg[0].rows + RT - 1) / RT;
    p.tile_start[0] = 0;
    p.tile_start[1] = p.ntiles;
  } else {
    for (int s = 0; s < a.nseg; s++) {
      p.tile_start[s] = p.ntiles;
      p.ntiles += (a.seg[s].rows + RT - 1) / RT;
    }
    p.tile_start[a.nseg] = p.ntiles;
  }
  if (p.ntiles == 0) return cudaSuccess;
  KernelFn fn = pick_kernel(a.fmt, NTc, xmode, aligned ? 1 : 0);
  const int occ = occupancy(fn, (int)smem, di.smem_optin);
  if (occ < 1) return cudaErrorInvalidConfiguration;
  const int grid = std::min(p.ntiles, di.sms * occ);

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, p);
}

}  // namespace nrc
