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

// The same left-to-right sum of a[0..n) (each a[j] squared when SQ), for
// terms that are >= 0, evaluated by one warp and bit-identical to the chain.
// While the running sum s = S * 2^(E-23) (S in [2^23, 2^24)) stays in one
// binade, adding t gives (S + rne(t / ulp)) * ulp exactly, except that a tie
// (t / ulp ending in exactly .5) rounds to the even neighbour, so it depends
// on the parity of the running sum. A chunk of 256 terms (8 consecutive per
// lane) is therefore summed as integers: each lane folds its terms into two
// sums, one per incoming parity, a warp scan composes those functions, and
// each lane re-walks its terms from its exact prefix to find the first term
// that takes the sum to 2^24 (the next binade) or is negative / non-finite.
// That term is added as a plain f32 step and the next chunk starts after it.
// The first 32 terms (where the sum changes binade often) and any non-normal
// running sum go one at a time.
template <bool SQ>
NRC_DEV float seq_sum_nonneg_warp(const float* a, int n, int lane, float init = 0.0f) {
  constexpr int PER = 8;
  constexpr uint32_t TOP = 16777216u;  // 2^24
  auto term = [&](int j) {
    const float v = a[j];
    return SQ ? __fmul_rn(v, v) : v;
  };
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
    const int j0 = i + lane * PER;
    uint32_t v[PER];  // rne(t / ulp), or floor(t / ulp) for a tie
    uint32_t tie = 0, bad = 0;
#pragma unroll
    for (int k = 0; k < PER; k++) {
      v[k] = 0;
      const int j = j0 + k;
      if (j < n) {
        const float t = term(j);
        const float T = __fmul_rn(t, scale);
        if (T < 16777216.0f && !(t < 0.0f)) {
          const uint32_t fl = __float2uint_rz(T);
          if (__fsub_rn(T, __uint2float_rz(fl)) == 0.5f) {
            tie |= 1u << k;
            v[k] = fl;
          } else {
            v[k] = __float2uint_rn(T);
          }
        } else {
          bad |= 1u << k;
        }
      }
    }
    // This lane's increment for an incoming running sum of parity 0 / 1
    // (terms before its first bad one).
    uint32_t a0 = 0, a1 = 0, q0 = 0, q1 = 1;
    bool stop = false;
#pragma unroll
    for (int k = 0; k < PER; k++) {
      stop = stop || ((bad >> k) & 1u);
      if (!stop) {
        const bool tk = (tie >> k) & 1u;
        const uint32_t d0 = tk ? v[k] + ((q0 + v[k]) & 1u) : v[k];
        const uint32_t d1 = tk ? v[k] + ((q1 + v[k]) & 1u) : v[k];
        a0 += d0;
        a1 += d1;
        q0 += d0;
        q1 += d1;
      }
    }
    // Inclusive scan of the composed functions: F(p) = L(p) + C((p + L(p)) & 1).
    uint32_t c0 = a0, c1 = a1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t l0 = __shfl_up_sync(0xffffffffu, c0, o);
      const uint32_t l1 = __shfl_up_sync(0xffffffffu, c1, o);
      if (lane >= o) {
        const uint32_t n0 = l0 + ((l0 & 1u) ? c1 : c0);
        const uint32_t n1 = l1 + (((1u + l1) & 1u) ? c1 : c0);
        c0 = n0;
        c1 = n1;
      }
    }
    uint32_t e0 = __shfl_up_sync(0xffffffffu, c0, 1), e1 = __shfl_up_sync(0xffffffffu, c1, 1);
    if (lane == 0) e0 = e1 = 0;
    const bool p0 = S & 1u;
    // Exact walk from this lane's prefix: the first crossing or bad term.
    uint32_t run = S + (p0 ? e1 : e0);
    int kev = PER;
    uint32_t before = 0;
#pragma unroll
    for (int k = 0; k < PER; k++) {
      if (kev == PER && j0 + k < n) {
        const bool tk = (tie >> k) & 1u;
        const uint32_t d = tk ? v[k] + ((run + v[k]) & 1u) : v[k];
        if (((bad >> k) & 1u) || d >= TOP - run) {
          kev = k;
          before = run;
        } else {
          run += d;
        }
      }
    }
    const unsigned evl = __ballot_sync(0xffffffffu, kev < PER);
    if (evl == 0) {
      const uint32_t tot = __shfl_sync(0xffffffffu, p0 ? c1 : c0, 31);
      s = __uint_as_float((be << 23) | ((S + tot) & 0x7fffffu));
      i += 32 * PER;
      continue;
    }
    const int L = __ffs(evl) - 1;
    const uint32_t sb = __shfl_sync(0xffffffffu, before, L);
    const int jev = i + L * PER + __shfl_sync(0xffffffffu, kev, L);
    s = __fadd_rn(__uint_as_float((be << 23) | (sb & 0x7fffffu)), term(jev));
    i = jev + 1;
  }
  return s;
}

// seq_sum_nonneg_warp for a group of NTH threads: warp 0 sums, every thread
// returns the result (`sync` is the group's barrier).
template <bool SQ, int NTH, class Sync>
NRC_DEV float seq_sum_nonneg_group(const float* a, int n, SeqSumShared& sh, int tid, const Sync& sync) {
  static_assert(NTH % 32 == 0, "group of whole warps");
  if (tid < 32) {
    const float r = seq_sum_nonneg_warp<SQ>(a, n, tid);
    if (tid == 0) sh.s = r;
  }
  sync();
  const float r = sh.s;
  sync();
  return r;
}

}  // namespace nrc
