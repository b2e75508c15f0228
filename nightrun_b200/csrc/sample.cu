// Sampler::sample with temperature > 0 (crates/nr-model/src/sample.rs:32-96):
// top-64 prefilter, softmax with temperature over the candidates in
// descending order, nucleus cut at top_p, one xorshift64 draw.
//
// The reference keeps a 64-slot min-heap initialised to (-inf, 0) and inserts
// logit v when v > the heap minimum (sample.rs:41-63). Its final content is
// every logit strictly above the final minimum T plus as many logits equal to
// T as fill the heap; which of several equal-to-T logits survive depends on
// the heap's history. So:
//   1. candidate pass (one CTA per 1,024 logits): each CTA sorts its keys
//      (ordered value, then lower index first; NaN and -inf never enter, as
//      in the reference) and writes its top 64 plus the 65th as a sentinel;
//   2. finish pass (one CTA): merges the candidates, takes the top 64. When
//      the 65th merged key or any CTA's sentinel equals T, more logits equal
//      T than the heap holds: warp 0 then replays the reference's heap over
//      all logits exactly (rare: ties at the boundary only), otherwise the
//      top 64 are the heap's content;
//   3. one thread evaluates the candidates in descending order, equal logits
//      by ascending index (the reference sorts with sort_unstable_by, whose
//      order among equal logits is unspecified): probs = expf((v - max) / T),
//      sum in order, cut = top_p * sum, the first prefix whose running sum
//      reaches cut, r = next_f32() * cum, the first candidate with r <= acc.
// All f32 arithmetic is explicit round-to-nearest, expf is the library's
// correctly rounded one.
#include "common.cuh"
#include "expf_cr.cuh"
#include "sample.cuh"

namespace nrc {
namespace {

constexpr int KEEP = SAMPLE_TOPK + 1;  // per-CTA candidates written (+ the tie sentinel)
constexpr int T1 = 256;                // threads of the candidate pass
constexpr int T2 = 1024;               // threads of the finish pass

// Larger key = larger logit; equal logits: lower index first; 0 = no candidate.
// -0.0 and +0.0 compare equal in the reference, so they share one key value.
NRC_DEV unsigned long long cand_key(float v, uint32_t idx) {
  if (v != v || v == -INFINITY) return 0ull;
  return argmax_key(v == 0.0f ? 0.0f : v, idx);
}
NRC_DEV float key_value(unsigned long long k) {
  const uint32_t o = (uint32_t)(k >> 32);
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

// Descending bitonic sort of n (a power of two) keys in shared memory by the
// whole CTA.
NRC_DEV void bitonic_desc(unsigned long long* k, int n) {
  for (int size = 2; size <= n; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const unsigned long long a = k[lo], b = k[hi];
        if ((a < b) == desc) {
          k[lo] = b;
          k[hi] = a;
        }
      }
      __syncthreads();
    }
}

__global__ void __launch_bounds__(T1) k_sample_candidates(const float* __restrict__ x, int n,
                                                          unsigned long long* __restrict__ cand) {
  pdl_wait();
  pdl_trigger();
  __shared__ unsigned long long k[SAMPLE_CHUNK];
  const int base = blockIdx.x * SAMPLE_CHUNK;
  for (int i = threadIdx.x; i < SAMPLE_CHUNK; i += T1) {
    const int g = base + i;
    k[i] = g < n ? cand_key(x[g], (uint32_t)g) : 0ull;
  }
  __syncthreads();
  bitonic_desc(k, SAMPLE_CHUNK);
  for (int i = threadIdx.x; i < KEEP; i += T1) cand[(size_t)blockIdx.x * KEEP + i] = k[i];
}

// The reference's heap (sample.rs:41-63) over all n logits, by warp 0: lanes
// test 32 consecutive logits against the heap minimum, the insertions happen
// one at a time in index order on lane 0.
NRC_DEV void exact_heap(const float* x, int n, float* hv, uint32_t* hi) {
  const int lane = threadIdx.x & 31;
  if (lane == 0)
    for (int i = 0; i < SAMPLE_TOPK; i++) {
      hv[i] = -INFINITY;
      hi[i] = 0;
    }
  __syncwarp();
  for (int b = 0; b < n; b += 32) {
    const int g = b + lane;
    const float v = g < n ? x[g] : -INFINITY;
    unsigned m = __ballot_sync(0xffffffffu, v > hv[0]);
    while (m) {
      const int l = __ffs(m) - 1;
      if (lane == l) {
        hv[0] = v;
        hi[0] = (uint32_t)g;
        int k = 0;
        for (;;) {
          const int lc = 2 * k + 1, rc = 2 * k + 2;
          int small = k;
          if (lc < SAMPLE_TOPK && hv[lc] < hv[small]) small = lc;
          if (rc < SAMPLE_TOPK && hv[rc] < hv[small]) small = rc;
          if (small == k) break;
          const float tv = hv[k];
          hv[k] = hv[small];
          hv[small] = tv;
          const uint32_t ti = hi[k];
          hi[k] = hi[small];
          hi[small] = ti;
          k = small;
        }
      }
      __syncwarp();
      m = __ballot_sync(0xffffffffu, lane > l && v > hv[0]);
    }
  }
}

struct FinishParams {
  const float* x;
  int n, nchunks, npad;
  float temperature, top_p;
  unsigned long long* rng;
  const unsigned long long* cand;
  uint32_t* out_idx;
  unsigned long long* out_key;
};

__global__ void __launch_bounds__(T2) k_sample_finish(const FinishParams p) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ unsigned long long keys[];  // [npad]
  __shared__ float hv[SAMPLE_TOPK];
  __shared__ uint32_t hi[SAMPLE_TOPK];
  __shared__ unsigned long long top[SAMPLE_TOPK];
  __shared__ int excess;
  const int tid = threadIdx.x;
  const int m = p.nchunks * SAMPLE_TOPK;
  for (int i = tid; i < p.npad; i += T2) keys[i] = i < m ? p.cand[(size_t)(i / SAMPLE_TOPK) * KEEP + i % SAMPLE_TOPK] : 0ull;
  if (tid == 0) excess = 0;
  __syncthreads();
  bitonic_desc(keys, p.npad);
  const unsigned long long kT = keys[SAMPLE_TOPK - 1];
  if (kT != 0ull) {
    const uint32_t vT = (uint32_t)(kT >> 32);
    if (tid == 0 && p.npad > SAMPLE_TOPK && keys[SAMPLE_TOPK] != 0ull && (uint32_t)(keys[SAMPLE_TOPK] >> 32) == vT)
      excess = 1;
    for (int c = tid; c < p.nchunks; c += T2) {
      const unsigned long long s = p.cand[(size_t)c * KEEP + SAMPLE_TOPK];
      if (s != 0ull && (uint32_t)(s >> 32) == vT) excess = 1;
    }
  }
  __syncthreads();
  if (excess) {
    // More logits equal the 64th largest than the heap holds: the reference's
    // heap decides which of them survive.
    if (tid < 32) exact_heap(p.x, p.n, hv, hi);
    __syncthreads();
    if (tid < SAMPLE_TOPK) keys[tid] = cand_key(hv[tid], hi[tid]);
    __syncthreads();
    if (tid < SAMPLE_TOPK) {
      // rank among the 64 (all keys distinct: distinct indices)
      const unsigned long long me = keys[tid];
      int r = 0;
      for (int j = 0; j < SAMPLE_TOPK; j++) r += keys[j] > me;
      top[r] = me;
    }
  } else if (tid < SAMPLE_TOPK) {
    top[tid] = keys[tid];
  }
  __syncthreads();
  if (tid != 0) return;
  float cv[SAMPLE_TOPK];
  uint32_t ci[SAMPLE_TOPK];
  for (int i = 0; i < SAMPLE_TOPK; i++) {
    const unsigned long long k = top[i];
    cv[i] = k ? key_value(k) : -INFINITY;  // unfilled heap slots stay (-inf, 0)
    ci[i] = k ? argmax_index(k) : 0u;
  }
  const float mx = cv[0];
  float probs[SAMPLE_TOPK];
  float sum = 0.0f;
  for (int i = 0; i < SAMPLE_TOPK; i++) {
    probs[i] = expf_cr(__fdiv_rn(__fsub_rn(cv[i], mx), p.temperature));
    sum = __fadd_rn(sum, probs[i]);
  }
  const float cut = __fmul_rn(p.top_p, sum);
  float cum = 0.0f;
  int nk = SAMPLE_TOPK;
  for (int i = 0; i < SAMPLE_TOPK; i++) {
    cum = __fadd_rn(cum, probs[i]);
    if (cum >= cut) {
      nk = i + 1;
      break;
    }
  }
  unsigned long long s = *p.rng;
  s ^= s << 13;
  s ^= s >> 7;
  s ^= s << 17;
  *p.rng = s;
  const float u = __fdiv_rn((float)(uint32_t)(s >> 40), 16777216.0f);  // exact: (s >> 40) < 2^24
  const float r = __fmul_rn(u, cum);
  float acc = 0.0f;
  uint32_t pick = ci[nk - 1];
  for (int i = 0; i < nk; i++) {
    acc = __fadd_rn(acc, probs[i]);
    if (r <= acc) {
      pick = ci[i];
      break;
    }
  }
  if (p.out_idx) *p.out_idx = pick;
  if (p.out_key) *p.out_key = (1ull << 32) | (unsigned long long)(0xffffffffu - pick);
}

int pow2_at_least(int v) {
  int p = SAMPLE_TOPK;
  while (p < v) p <<= 1;
  return p;
}

cudaError_t launch_ex(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, void** args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

size_t sample_scratch_bytes(int n) {
  const int nchunks = (n + SAMPLE_CHUNK - 1) / SAMPLE_CHUNK;
  return (size_t)(nchunks > 0 ? nchunks : 1) * KEEP * sizeof(unsigned long long);
}

cudaError_t sample_run(const SampleArgs& a, cudaStream_t s, bool pdl) {
  if (a.n < 1 || a.n > SAMPLE_MAX_N || !a.rng || !a.cand || (!a.out_idx && !a.out_key)) return cudaErrorInvalidValue;
  const int nchunks = (a.n + SAMPLE_CHUNK - 1) / SAMPLE_CHUNK;
  {
    const float* x = a.logits;
    int n = a.n;
    unsigned long long* cand = a.cand;
    void* args[] = {&x, &n, &cand};
    cudaError_t e = launch_ex((const void*)k_sample_candidates, dim3(nchunks), dim3(T1), 0, s, pdl, args);
    if (e != cudaSuccess) return e;
  }
  FinishParams p{a.logits, a.n, nchunks, pow2_at_least(nchunks * SAMPLE_TOPK), a.temperature, a.top_p,
                 a.rng, a.cand, a.out_idx, a.out_key};
  const size_t smem = (size_t)p.npad * sizeof(unsigned long long);
  if (cudaError_t e = ensure_smem_attr((const void*)k_sample_finish, (int)(SAMPLE_MAX_N / SAMPLE_CHUNK * SAMPLE_TOPK * 8)))
    return e;
  void* args[] = {&p};
  return launch_ex((const void*)k_sample_finish, dim3(1), dim3(T2), smem, s, pdl, args);
}

}  // namespace nrc
