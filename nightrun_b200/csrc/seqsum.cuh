// Sequential f32 sums in the reference's order.
//
// The reference accumulates `ss += v * v` (vec.rs:4-14, rmsnorm) and the
// softmax denominator (vec.rs:30-41) one term at a time; every partial sum is
// rounded to f32, so the result depends on the order and must be evaluated as
// one chain of n dependent adds. The chain runs on one thread at the add
// latency: terms are fetched 16 ahead of the adds (software pipelining), so a
// shared-memory or L1 fetch never stalls the chain.
#pragma once
#include "common.cuh"

namespace nrc {

// ((init + t(0)) + t(1)) + ... + t(n-1), on the calling thread. Whole blocks of
// W terms are fetched one block ahead of their adds with no per-term
// conditions (so every fetch is issued before the adds that precede its use);
// the last n mod W terms follow one by one.
template <class Term>
NRC_DEV float seq_sum_serial(int n, const Term& term, float init = 0.0f) {
  constexpr int W = 16;
  float s = init;
  const int nfull = n - n % W;
  if (nfull > 0) {
    float cur[W];
#pragma unroll
    for (int j = 0; j < W; j++) cur[j] = term(j);
    for (int i = 0; i < nfull; i += W) {
      const int nb = i + W < nfull ? i + W : i;  // the next block (the last one again at the end)
      float nxt[W];
#pragma unroll
      for (int j = 0; j < W; j++) nxt[j] = term(nb + j);
#pragma unroll
      for (int j = 0; j < W; j++) s = __fadd_rn(s, cur[j]);
#pragma unroll
      for (int j = 0; j < W; j++) cur[j] = nxt[j];
    }
  }
  for (int i = nfull; i < n; i++) s = __fadd_rn(s, term(i));
  return s;
}

// Two independent chains over the same index range (their adds interleave).
template <class TermA, class TermB>
NRC_DEV void seq_sum_serial2(int n, const TermA& ta, const TermB& tb, float& sa, float& sb) {
  constexpr int W = 8;
  sa = 0.0f;
  sb = 0.0f;
  const int nfull = n - n % W;
  if (nfull > 0) {
    float ca[W], cb[W];
#pragma unroll
    for (int j = 0; j < W; j++) {
      ca[j] = ta(j);
      cb[j] = tb(j);
    }
    for (int i = 0; i < nfull; i += W) {
      const int nb = i + W < nfull ? i + W : i;
      float na[W], nbv[W];
#pragma unroll
      for (int j = 0; j < W; j++) {
        na[j] = ta(nb + j);
        nbv[j] = tb(nb + j);
      }
#pragma unroll
      for (int j = 0; j < W; j++) {
        sa = __fadd_rn(sa, ca[j]);
        sb = __fadd_rn(sb, cb[j]);
      }
#pragma unroll
      for (int j = 0; j < W; j++) {
        ca[j] = na[j];
        cb[j] = nbv[j];
      }
    }
  }
  for (int i = nfull; i < n; i++) {
    sa = __fadd_rn(sa, ta(i));
    sb = __fadd_rn(sb, tb(i));
  }
}

struct SeqSumShared {
  float s;
};

// The same sum for a group of NTH threads: thread 0 runs the chain, `sync`
// is the group's barrier, every thread returns the result.
template <int NTH, class Term, class Sync>
NRC_DEV float seq_sum_group(int n, const Term& term, SeqSumShared& sh, int tid, const Sync& sync) {
  static_assert(NTH % 32 == 0, "group of whole warps");
  if (tid == 0) sh.s = seq_sum_serial(n, term);
  sync();
  const float r = sh.s;
  sync();  // `sh` may be reused by the caller right after
  return r;
}

// The same left-to-right sum for terms that are all >= 0 (sums of squares,
// softmax denominators), evaluated by one warp, bit-identical to the chain.
// While the running sum s = S * 2^(E-23) (S in [2^23, 2^24)) stays in one
// binade, adding t rounds to (S + rne(t / 2^(E-23))) * 2^(E-23): every term
// rounds on its own, so a chunk of 256 terms adds as one integer sum. The
// exceptions are a tie (t / ulp ends in exactly .5: the result's parity
// decides), the sum reaching the next binade, and negative or non-finite
// terms; the first such term in order is added as a plain f32 step and the
// next chunk starts after it. The first 32 terms (where the sum still
// changes binade often) and any non-normal running sum go one at a time.
template <class Term>
NRC_DEV float seq_sum_nonneg_warp(int n, const Term& term, int lane, float init = 0.0f) {
  constexpr int ROWS = 8;  // chunk = ROWS x 32 terms; term i + k * 32 + lane in lane `lane`
  constexpr uint32_t TOP = 16777216u;  // 2^24
  int i = n < 32 ? n : 32;
  float s = seq_sum_serial(i, term, init);
  while (i < n) {
    const uint32_t b = __float_as_uint(s);
    const uint32_t be = b >> 23;  // biased exponent (>= 256 when negative)
    if (be < 27u || be > 254u) {
      s = __fadd_rn(s, term(i));
      i++;
      continue;
    }
    const uint32_t S = (b & 0x7fffffu) | 0x800000u;
    const float scale = __uint_as_float((277u - be) << 23);  // 2^(23 - E): exact scaling to ulps
    uint32_t r[ROWS];
    uint32_t fl = 0, tot = 0;
#pragma unroll
    for (int k = 0; k < ROWS; k++) {
      const int j = i + k * 32 + lane;
      uint32_t rk = 0;
      if (j < n) {
        const float t = term(j);
        const float T = __fmul_rn(t, scale);
        if (T < 16777216.0f && !(t < 0.0f)) {
          rk = __float2uint_rn(T);
          if (__fsub_rn(T, __uint2float_rz(__float2uint_rz(T))) == 0.5f) fl |= 1u << k;
        } else {
          fl |= 1u << k;
        }
      }
      r[k] = rk;
      tot += rk;
    }
    const uint32_t wtot = __reduce_add_sync(0xffffffffu, tot);
    if (!__any_sync(0xffffffffu, fl != 0) && wtot < TOP - S) {
      s = __uint_as_float((be << 23) | ((S + wtot) & 0x7fffffu));
      i += ROWS * 32;
      continue;
    }
    // The first term, in order, that is flagged or takes the sum to 2^24.
    uint32_t run = S;
    int jev = i;
    uint32_t before = S;
#pragma unroll
    for (int k = 0; k < ROWS; k++) {
      uint32_t inc = r[k];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
      }
      const unsigned m = __ballot_sync(0xffffffffu, ((fl >> k) & 1u) || inc >= TOP - run);
      if (m) {
        const int L = __ffs(m) - 1;
        before = run + __shfl_sync(0xffffffffu, inc - r[k], L);
        jev = i + k * 32 + L;
        break;
      }
      run += __shfl_sync(0xffffffffu, inc, 31);
    }
    s = __fadd_rn(__uint_as_float((be << 23) | (before & 0x7fffffu)), term(jev));
    i = jev + 1;
  }
  return s;
}

// seq_sum_nonneg_warp for a group of NTH threads: warp 0 sums, every thread
// returns the result (`sync` is the group's barrier).
template <int NTH, class Term, class Sync>
NRC_DEV float seq_sum_nonneg_group(int n, const Term& term, SeqSumShared& sh, int tid, const Sync& sync) {
  static_assert(NTH % 32 == 0, "group of whole warps");
  if (tid < 32) {
    const float v = seq_sum_nonneg_warp(n, term, tid);
    if (tid == 0) sh.s = v;
  }
  sync();
  const float r = sh.s;
  sync();
  return r;
}

}  // namespace nrc
