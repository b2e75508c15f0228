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

// ((0 + t(0)) + t(1)) + ... + t(n-1), on the calling thread.
template <class Term>
NRC_DEV float seq_sum_serial(int n, const Term& term) {
  constexpr int W = 16;
  float s = 0.0f;
  float cur[W];
#pragma unroll
  for (int j = 0; j < W; j++) cur[j] = j < n ? term(j) : 0.0f;
  for (int i = 0; i < n; i += W) {
    float nxt[W];
#pragma unroll
    for (int j = 0; j < W; j++) nxt[j] = i + W + j < n ? term(i + W + j) : 0.0f;
#pragma unroll
    for (int j = 0; j < W; j++)
      if (i + j < n) s = __fadd_rn(s, cur[j]);
#pragma unroll
    for (int j = 0; j < W; j++) cur[j] = nxt[j];
  }
  return s;
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

}  // namespace nrc
