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

// ((init + a0*a0) + a1*a1) + ... for a 16-byte aligned array: the squares of
// whole 16-term blocks are loaded with 16-byte loads two blocks ahead of their
// adds, so shared-memory latency stays off the chain (rmsnorm's `ss`).
NRC_DEV float seq_sum_squares_serial(const float* a, int n, float init = 0.0f) {
  constexpr int W = 16;
  float s = init;
  const int nfull = n - n % W;
  const float4* a4 = reinterpret_cast<const float4*>(a);
  if (nfull > 0) {
    float4 c0[4], c1[4];
#pragma unroll
    for (int j = 0; j < 4; j++) c0[j] = a4[j];
#pragma unroll
    for (int j = 0; j < 4; j++) c1[j] = W < nfull ? a4[4 + j] : c0[j];
    for (int i = 0; i < nfull; i += W) {
      const int nb = i + 2 * W < nfull ? i + 2 * W : i;  // two blocks ahead (any block at the end)
      float4 c2[4];
#pragma unroll
      for (int j = 0; j < 4; j++) c2[j] = a4[nb / 4 + j];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        s = __fadd_rn(s, __fmul_rn(c0[j].x, c0[j].x));
        s = __fadd_rn(s, __fmul_rn(c0[j].y, c0[j].y));
        s = __fadd_rn(s, __fmul_rn(c0[j].z, c0[j].z));
        s = __fadd_rn(s, __fmul_rn(c0[j].w, c0[j].w));
      }
#pragma unroll
      for (int j = 0; j < 4; j++) {
        c0[j] = c1[j];
        c1[j] = c2[j];
      }
    }
  }
  for (int i = nfull; i < n; i++) s = __fadd_rn(s, __fmul_rn(a[i], a[i]));
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
  float w[32];  // per-warp partials of the tree sums
};

// seq_sum_squares_serial for a group of NTH threads (thread 0 runs it).
template <int NTH, class Sync>
NRC_DEV float seq_sum_squares_group(const float* a, int n, SeqSumShared& sh, int tid, const Sync& sync) {
  static_assert(NTH % 32 == 0, "group of whole warps");
  if (tid == 0) sh.s = seq_sum_squares_serial(a, n);
  sync();
  const float r = sh.s;
  sync();
  return r;
}

// Tolerance mode: sum of a[i]^2 for a 16-byte aligned array as a tree (each
// thread a strided partial, warp shuffles, the warps' partials in a fixed
// order): deterministic, not the reference's sequential order.
template <int NTH, class Sync>
NRC_DEV float tree_sum_squares_group(const float* a, int n, SeqSumShared& sh, int tid, const Sync& sync) {
  static_assert(NTH % 32 == 0 && NTH <= 1024, "group of whole warps");
  float part = 0.0f;
  const float4* a4 = reinterpret_cast<const float4*>(a);
  for (int i = tid; i < n / 4; i += NTH) {
    const float4 v = a4[i];
    part = fmaf(v.x, v.x, part);
    part = fmaf(v.y, v.y, part);
    part = fmaf(v.z, v.z, part);
    part = fmaf(v.w, v.w, part);
  }
  for (int i = (n & ~3) + tid; i < n; i += NTH) part = fmaf(a[i], a[i], part);
  part = warp_sum(part);
  if ((tid & 31) == 0) sh.w[tid >> 5] = part;
  sync();
  float r = 0.0f;
#pragma unroll
  for (int w = 0; w < NTH / 32; w++) r += sh.w[w];
  sync();
  return r;
}

// Tolerance mode: sum of term(i) for i < n as a tree (see above).
template <int NTH, class Term, class Sync>
NRC_DEV float tree_sum_group(int n, const Term& term, SeqSumShared& sh, int tid, const Sync& sync) {
  float part = 0.0f;
  for (int i = tid; i < n; i += NTH) part += term(i);
  part = warp_sum(part);
  if ((tid & 31) == 0) sh.w[tid >> 5] = part;
  sync();
  float r = 0.0f;
#pragma unroll
  for (int w = 0; w < NTH / 32; w++) r += sh.w[w];
  sync();
  return r;
}

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

}  // namespace nrc
