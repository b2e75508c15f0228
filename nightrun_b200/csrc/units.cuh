// Exact block-dot units shared by the streaming GEMV kernels: one Q8_0 block,
// an aligned octet of 8 Q8_0 blocks, one Q4_K or one Q6_K super-block, each
// giving the per-block f32 term(s) with the reference's scalar roundings
// (crates/nr-tensor/src/kernels.rs:72-82, crates/nr-tensor/src/kquant.rs:192-250).
//
// Activation layouts in shared memory (XW words per 256 activation bytes):
//   Q8_0: xq[(tok*n_oct + b/8)*XW + (b%8)*8 + w] (quants), xd[tok*bpr + b]
//   Q8_K: xq[(tok*bpr + b)*XW + w], xd[tok*bpr + b], xb[(tok*bpr + b)*8 + j]
//         (bsums of the 32-value sub-blocks)
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"

namespace nrc {

constexpr int XW = 68;  // words per 256-byte activation group (64 + 4 pad: conflict-free LDS.128)

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
    if (NT == 1 || tok < nt) {
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

template <int NT>
NRC_DEV void oct_load(const uint8_t* src, uint32_t* w) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int i = 0; i < 17; i++) {
    const uint4 v = s4[i];
    w[4 * i] = v.x;
    w[4 * i + 1] = v.y;
    w[4 * i + 2] = v.z;
    w[4 * i + 3] = v.w;
  }
}
// Terms of block j for token tok go to t[tok * tstride + j * JS].
template <int NT, int JS = 1>
NRC_DEV void oct_compute(const uint32_t* w, const uint32_t* xq, int xtok, const float* xd, int nt, int bpr, float* t,
                         int tstride) {
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int base = (j / 2) * 17;
    uint32_t q[8];
    uint32_t dbits;
    if ((j & 1) == 0) {
      dbits = w[base] & 0xffffu;
#pragma unroll
      for (int k = 0; k < 8; k++) q[k] = __byte_perm(w[base + k], w[base + k + 1], 0x5432);
    } else {
      dbits = w[base + 8] >> 16;
#pragma unroll
      for (int k = 0; k < 8; k++) q[k] = w[base + 9 + k];
    }
    // f16 -> f32 is exact for every f16 value; the hardware conversion is used.
    const float dw = __half2float(__ushort_as_half((unsigned short)dbits));
#pragma unroll
    for (int tok = 0; tok < NT; tok++) {
      if (NT == 1 || tok < nt) {
        const uint4* xv = reinterpret_cast<const uint4*>(xq + tok * xtok + j * 8);
        const uint4 a = xv[0], b = xv[1];
        int acc = __dp4a((int)q[0], (int)a.x, 0);
        acc = __dp4a((int)q[1], (int)a.y, acc);
        acc = __dp4a((int)q[2], (int)a.z, acc);
        acc = __dp4a((int)q[3], (int)a.w, acc);
        acc = __dp4a((int)q[4], (int)b.x, acc);
        acc = __dp4a((int)q[5], (int)b.y, acc);
        acc = __dp4a((int)q[6], (int)b.z, acc);
        acc = __dp4a((int)q[7], (int)b.w, acc);
        t[tok * tstride + j * JS] = __fmul_rn(__fmul_rn(i2f(acc), dw), xd[tok * bpr + j]);
      }
    }
  }
}
// Eight consecutive Q8_0 blocks (272 bytes, 16-byte aligned: 17 uint4).
// Block j starts at byte 34j: even j at a word boundary (scale in the low
// half, quants 2 bytes in), odd j at a half word (scale in the high half,
// quants word aligned). kernels.rs:72-82 per block.
template <int NT>
NRC_DEV void unit_q8_oct(const uint8_t* src, const uint32_t* xq, int xtok, const float* xd, int nt, int bpr,
                         float* t, int tstride) {
  uint32_t w[68];
  oct_load<NT>(src, w);
  oct_compute<NT>(w, xq, xtok, xd, nt, bpr, t, tstride);
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
    if (NT == 1 || tok < nt) {
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
    if (NT == 1 || tok < nt) {
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


}  // namespace nrc
