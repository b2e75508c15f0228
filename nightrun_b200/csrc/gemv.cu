// Streaming quantized GEMV for sm_100a: y = W · x over in-place Q8_0 / Q4_K /
// Q6_K weight blocks, for 1..8 activation vectors.
//
// Reference: crates/nr-tensor/src/kernels.rs:36-143 (Q8_0) and
// crates/nr-tensor/src/kquant.rs:192-250, 536-639 (Q4_K / Q6_K).
//
// Structure (persistent, one CTA per SM, 12 consumer warps + 1 producer warp):
//  * a tile is R consecutive weight rows (whole rows; gate and up are two
//    spans of one tile in the SwiGLU pair), i.e. one or two contiguous byte
//    ranges. The producer warp copies each tile HBM -> shared memory with one
//    1-D TMA bulk copy per span (cp.async.bulk, L2 evict-first, no cluster
//    multicast) into a ring of stage buffers, one full/empty mbarrier pair
//    per stage; weights never depend on the previous kernel, so streaming
//    starts before the programmatic-dependency wait;
//  * the consumers stage the activations in shared memory once per CTA
//    (optional RMSNorm, quantization exactly as the reference quantizes them,
//    one thread per 32-value block);
//  * tile k belongs to warp k mod ncw and every ring slot to one warp (the
//    ring holds ncw or 2 ncw stages), so the warps run independently. The
//    owning warp's lanes compute the tile's units — an aligned octet of 8
//    Q8_0 blocks, one Q8_0 block, or one K-quant super-block — as exact
//    integer dp4a dots, round each block's f32 term exactly as the
//    reference's scalar dot rounds it (kernels.rs:79, kquant.rs:212-215,
//    244-247) and park it in the warp's term buffer; then one lane per
//    (row, token) adds the row's terms in block order, the reference's
//    summation order, and applies the fused epilogue.
#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "expf_cr.cuh"
#include "gemv.cuh"
#include "seqsum.cuh"
#include "tma.cuh"
#include "units.cuh"

namespace nrc {
namespace {

constexpr int NCW = 12;            // consumer warps (a stage's units are latency-bound: more warps, more stages in flight)
constexpr int NC = NCW * 32;       // consumer threads
constexpr int NTHREADS = NC + 32;  // + producer warp
constexpr int MAX_STAGES = 24;
constexpr int SMEM_RESERVE = 1024;  // static shared memory of the kernel, rounded up

struct Params {
  const uint8_t* w[3];
  float* y[3];
  int rows[3];
  int ld[3];
  int tile_start[4];
  int nseg, pair;
  int K, bpr, row_bytes;
  int R;            // rows per tile (= per stage)
  int unit_bytes;   // bytes per unit (272: Q8_0 octet, 34: Q8_0 block, 144 / 210: super-block)
  int upr;          // units per row
  int span_stride;  // stage bytes reserved per span (16-byte multiple)
  int stage_bytes;
  int ntiles;
  int nt;
  int nstage;       // a multiple of ncw: every slot belongs to one warp
  int ncw;          // consumer warps that own tiles (the others only help with the prologue)
  const uint8_t* xq;
  uint8_t* xq_out;
  uint8_t* yq_out;  // EPI_SWIGLU output as Q8_0 blocks (lane-per-row kernel, 32-row groups), or null
  const float* xf;
  int xf_ld;
  const float* norm_w;
  float eps;
  int fast_norm;
  int epi;
  float scale;
  float* resid;
  int resid_ld;
  float rs;
  unsigned long long* argmax_key;
  int argmax_base;
  unsigned* err;
  const uint8_t* pf;  // next kernel's weights to prefetch into L2 (16-byte aligned), or null
  size_t pf_bytes;
  int off_x, off_xd, off_xb, off_t;  // shared-memory layout (bytes)
  int tb_warp;                       // floats of one warp's term buffer
  int xs_floats;                     // f32 staging floats at off_t (prologue)
  int n_oct;
  int off_nw;                        // norm weights staged in shared memory (bytes), or -1
};

NRC_DEV int imin(int a, int b) { return a < b ? a : b; }

// ------------------------------------------------------------ activation prologue
// Activation buffers in shared memory:
//   Q8_0: xq[(tok*n_oct + b/8)*XW + (b%8)*8 + w], xd[tok*bpr + b]
//   Q8_K: xq[(tok*bpr + b)*XW + w], xd[tok*bpr + b], xb[(tok*bpr + b)*8 + j] (bsum pairs)
NRC_DEV int xq_index(int fmt, const Params& p, int tok, int b) {
  return fmt == FMT_Q8_0 ? (tok * p.n_oct + b / 8) * XW + (b % 8) * 8 : (tok * p.bpr + b) * XW;
}

// q8::quantize (q8.rs:27-44) of the row's 32-value blocks after the optional
// RMSNorm scaling, G lanes per block (lane g of a group holds values
// [g * 32 / G, (g + 1) * 32 / G)). The block maximum |v| is a max-reduction
// (order-free); a NaN value counts as 0, as in the reference's running fmax
// from 0. Every lane of a warp runs the same rounds (the shuffles are
// warp-wide).
template <int G, int NCT>
NRC_DEV void quant_q8_groups(const Params& p, const float* xs, const float* nw, float sc, uint32_t* xq, float* xd,
                             int tok) {
  constexpr int P = 32 / G;
  const int tid = threadIdx.x, gid = tid / G, gl = tid % G;
  for (int base = 0; base < p.bpr; base += NCT / G) {
    const int b = base + gid;
    const bool on = b < p.bpr;
    float v[P];
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < P; k++) {
      const int idx = b * 32 + gl * P + k;
      v[k] = on ? xs[idx] : 0.0f;
      if (on && p.norm_w) v[k] = __fmul_rn(__fmul_rn(v[k], sc), nw[idx]);
      amax = fmaxf(amax, fabsf(v[k]));
    }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (!on) continue;
    const uint16_t dbits = f32_to_f16(__fdiv_rn(amax, 127.0f));
    const float d = f16_to_f32(dbits);
    const float inv = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int8_t* dst = reinterpret_cast<int8_t*>(xq + xq_index(FMT_Q8_0, p, tok, b)) + gl * P;
#pragma unroll
    for (int k = 0; k < P; k++) {
      const float xsv = __fmul_rn(v[k], inv);
      const float r = xsv >= 0.0f ? __fadd_rn(xsv, 0.5f) : __fsub_rn(xsv, 0.5f);
      int q = rust_f2i(r);
      q = q < -127 ? -127 : (q > 127 ? 127 : q);
      dst[k] = (int8_t)q;
    }
    if (gl == 0) xd[tok * p.bpr + b] = d;
  }
}

// Quantize nt f32 rows (optionally RMS-normalised) into the activation buffers,
// exactly as q8::quantize (q8.rs:27-44) / quantize_q8k (kquant.rs:157-187).
// Each row is first copied to shared memory (`xs`, aliasing the term buffer)
// with one coalesced pass; the norm's sum of squares uses one fixed order, so
// every CTA and every launch derive identical activations.
template <int FMT, int NCT = NC>
NRC_DEV void build_x_f32(const Params& p, uint8_t* smem) {
  uint32_t* xq = reinterpret_cast<uint32_t*>(smem + p.off_x);
  float* xd = reinterpret_cast<float*>(smem + p.off_xd);
  int* xb = reinterpret_cast<int*>(smem + p.off_xb);
  float* xs = reinterpret_cast<float*>(smem + p.off_t);
  __shared__ SeqSumShared ssh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = p.K;
  for (int tok = 0; tok < p.nt; tok++) {
    const float* src = p.xf + (size_t)tok * p.xf_ld;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (K & 3) == 0) {
      for (int i = tid; i < K / 4; i += NCT) reinterpret_cast<float4*>(xs)[i] = reinterpret_cast<const float4*>(src)[i];
    } else {
      for (int i = tid; i < K; i += NCT) xs[i] = src[i];
    }
    named_sync(1, NCT);
    float sc = 1.0f;
    if (p.norm_w) {
      // vec::rmsnorm (vec.rs:4-14): `ss += v * v` in index order (one chain,
      // seqsum.cuh), then scale = 1 / sqrtf(ss / n + eps).
      const float ss = p.fast_norm ? tree_sum_squares_group<NCT>(xs, K, ssh, tid, [] { named_sync(1, NCT); })
                                   : seq_sum_squares_group<NCT>(xs, K, ssh, tid, [] { named_sync(1, NCT); });
      sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), p.eps)));
    }
    if (FMT == FMT_Q8_0) {
      // q8::quantize (q8.rs:27-44): G lanes per 32-value block, as many as
      // lets every block of the row go in one round.
      // Norm weights: staged in shared memory before the dependency wait when
      // the launch reserved room for them, else read through the cache.
      const float* nw = p.off_nw >= 0 ? reinterpret_cast<const float*>(smem + p.off_nw) : p.norm_w;
      if (p.bpr <= NCT / 8)
        quant_q8_groups<8, NCT>(p, xs, nw, sc, xq, xd, tok);
      else if (p.bpr <= NCT / 4)
        quant_q8_groups<4, NCT>(p, xs, nw, sc, xq, xd, tok);
      else if (p.bpr <= NCT / 2)
        quant_q8_groups<2, NCT>(p, xs, nw, sc, xq, xd, tok);
      else
        quant_q8_groups<1, NCT>(p, xs, nw, sc, xq, xd, tok);
    } else {
      for (int b = warp; b < p.bpr; b += NCT / 32) {
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
    named_sync(1, NCT);  // xs is reused by the next token / the term buffer
  }
  if (p.xq_out && blockIdx.x == 0) {
    // The activations as blocks for a following launch (XMODE 0 reads them back).
    for (int i = tid; i < p.nt * p.bpr; i += NCT) {
      const int tok = i / p.bpr, b = i % p.bpr;
      const uint32_t* src = xq + xq_index(FMT, p, tok, b);
      if (FMT == FMT_Q8_0) {
        uint8_t* d = p.xq_out + (size_t)i * Q8_0_BYTES;
        const uint16_t hb = f32_to_f16(xd[tok * p.bpr + b]);  // exact: the scale is an f16 value
        d[0] = (uint8_t)(hb & 0xff);
        d[1] = (uint8_t)(hb >> 8);
        for (int k = 0; k < 8; k++) {
          const uint32_t w = src[k];
          d[2 + 4 * k] = (uint8_t)w;
          d[3 + 4 * k] = (uint8_t)(w >> 8);
          d[4 + 4 * k] = (uint8_t)(w >> 16);
          d[5 + 4 * k] = (uint8_t)(w >> 24);
        }
      } else {
        uint32_t* d = reinterpret_cast<uint32_t*>(p.xq_out + (size_t)i * Q8K_BYTES);
        d[0] = __float_as_uint(xd[tok * p.bpr + b]);
        for (int k = 0; k < 64; k++) d[1 + k] = src[k];
        for (int j = 0; j < 8; j++) d[65 + j] = (uint32_t)(uint16_t)(int16_t)xb[(tok * p.bpr + b) * 8 + j];
      }
    }
  }
}

// Activations given as blocks in global memory (the kernel-level entry points).
template <int FMT, int NCT = NC>
NRC_DEV void build_x_blocks(const Params& p, uint8_t* smem) {
  uint32_t* xq = reinterpret_cast<uint32_t*>(smem + p.off_x);
  float* xd = reinterpret_cast<float*>(smem + p.off_xd);
  int* xb = reinterpret_cast<int*>(smem + p.off_xb);
  const int tid = threadIdx.x;
  const int nblk = p.nt * p.bpr;
  if (FMT == FMT_Q8_0) {
    for (int i = tid; i < nblk; i += NCT) {
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
    for (int i = tid; i < nblk; i += NCT) {
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

// The tile's spans: span 0 (the tile's segment), span 1 (up rows in pair mode).
NRC_DEV void tile_spans(const Params& p, int tile, Span& s0, Span& s1) {
  int s = 0;
  if (!p.pair)
    while (s + 1 < p.nseg && tile >= p.tile_start[s + 1]) s++;
  const int row0 = (tile - p.tile_start[s]) * p.R;
  const int nr = imin(p.R, p.rows[s] - row0);
  s0.base = p.w[s] + (size_t)row0 * p.row_bytes;
  s0.wbeg = p.w[s];
  s0.wend = p.w[s] + (size_t)p.rows[s] * p.row_bytes;
  s0.row0 = row0;
  s0.nrows = nr;
  s0.seg = s;
  s1 = s0;
  if (p.pair) {
    s1.base = p.w[1] + (size_t)row0 * p.row_bytes;
    s1.wbeg = p.w[1];
    s1.wend = p.w[1] + (size_t)p.rows[1] * p.row_bytes;
    s1.seg = 1;
  }
}

// Byte range [g0, g1) of a span lands at slot + (addr - a0), a0 = floor16(g0).
// The 16-byte aligned part inside the weight buffer goes by one bulk copy
// [blo, bhi); the (at most 2x15) ragged bytes at unaligned buffer ends by
// plain loads.
struct SegRange {
  uintptr_t g0, g1, a0, blo, bhi;
};
NRC_DEV SegRange seg_range(const Span& sp, int row_bytes) {
  SegRange q;
  q.g0 = reinterpret_cast<uintptr_t>(sp.base);
  q.g1 = q.g0 + (size_t)sp.nrows * row_bytes;
  q.a0 = q.g0 & ~(uintptr_t)15;
  const uintptr_t wb = (reinterpret_cast<uintptr_t>(sp.wbeg) + 15) & ~(uintptr_t)15;
  const uintptr_t we = reinterpret_cast<uintptr_t>(sp.wend) & ~(uintptr_t)15;
  q.blo = q.a0 > wb ? q.a0 : wb;
  q.bhi = (q.g1 + 15) & ~(uintptr_t)15;
  if (q.bhi > we) q.bhi = we;
  if (q.bhi <= q.blo) q.blo = q.bhi = q.g0;
  return q;
}

template <int FMT, int NT, int XMODE, int ALIGNED>
__global__ void __launch_bounds__(NTHREADS, 1) gemv_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)p.nstage * p.stage_bytes);
  uint64_t* empty = full + MAX_STAGES;
  __shared__ volatile int abort_flag;
  __shared__ uint64_t pf_go;  // completes once: the ring's first stages are issued
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NS = p.nstage;
  const int nspan = p.pair ? 2 : 1;

  if (tid == 0) {
    for (int s = 0; s < NS; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&pf_go, NS % 4 == 0 ? 4 : (NS % 2 == 0 ? 2 : 1));  // one arrival per issuing lane
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == NCW) {
    // ----------------------------------------------------------- producer
    // Lanes [0, nprod) issue the tiles (tile k by lane k mod nprod, which
    // therefore owns the ring slots k mod NS); more issuing threads keep more
    // copies in flight. The other lanes prefetch the next kernel's weights.
    const int nprod = NS % 4 == 0 ? 4 : (NS % 2 == 0 ? 2 : 1);
    if (lane < nprod) {
      const uint64_t pol = l2_evict_first();
      int last = -1;
      int it = lane;
      bool go = false;
      Span sp0, sp1;
      for (int tile = blockIdx.x + lane * gridDim.x; tile < p.ntiles; tile += nprod * gridDim.x, it += nprod) {
        const int s = it % NS;
        if (!go && it >= NS) {
          mbar_arrive(&pf_go);
          go = true;
        }
        if (it >= NS && (abort_flag || !mbar_wait(&empty[s], ((it / NS) - 1) & 1))) {
          abort_flag = 1;
          atomicOr(p.err, ERR_WAIT_EMPTY);
          break;
        }
        tile_spans(p, tile, sp0, sp1);
        uint8_t* sbuf = stages + (size_t)s * p.stage_bytes;
        const SegRange g0 = seg_range(sp0, p.row_bytes);
        const SegRange g1 = seg_range(sp1, p.row_bytes);
        uint32_t total = 0;
        bool ragged = false;
        for (int si = 0; si < nspan; si++) {
          const SegRange g = si ? g1 : g0;
          uint8_t* dst = sbuf + (size_t)si * p.span_stride;
          for (uintptr_t a = g.g0; a < g.blo; a++) dst[a - g.a0] = *reinterpret_cast<const uint8_t*>(a);
          for (uintptr_t a = (g.bhi > g.g0 ? g.bhi : g.g0); a < g.g1; a++)
            dst[a - g.a0] = *reinterpret_cast<const uint8_t*>(a);
          ragged |= g.g0 < g.blo || g.bhi < g.g1;
          total += (uint32_t)(g.bhi - g.blo);
        }
        // Order these byte stores before this thread's later bulk copies into
        // the same slot.
        if (ragged) fence_proxy_async_smem();
        mbar_arrive_expect_tx(&full[s], total);
        for (int si = 0; si < nspan; si++) {
          const SegRange g = si ? g1 : g0;
          if (g.bhi > g.blo)
            bulk_g2s(sbuf + (size_t)si * p.span_stride + (g.blo - g.a0), reinterpret_cast<const void*>(g.blo),
                     (uint32_t)(g.bhi - g.blo), &full[s], pol);
        }
        last = it;
      }
      if (!go) mbar_arrive(&pf_go);
      // Drain: wait (bounded) for this lane's copies still in flight, so the
      // CTA never exits with a bulk copy pending.
      for (int k = last; k >= 0 && k > last - NS; k -= nprod)
        if (!mbar_wait(&full[k % NS], (k / NS) & 1)) atomicOr(p.err, ERR_DRAIN);
    } else if (p.pf != nullptr && p.pf_bytes >= 16 && blockIdx.x < p.ntiles) {
      // Once the issuing lanes have filled the ring, prefetch this CTA's share
      // of the next kernel's weights into L2 (a hint; nothing waits for it).
      if (mbar_wait(&pf_go, 0)) {
        const int nl = 32 - nprod, l = lane - nprod;
        const size_t share = ((p.pf_bytes / gridDim.x) + (size_t)nl * 16 - 1) / ((size_t)nl * 16) * ((size_t)nl * 16);
        const size_t lo = (size_t)blockIdx.x * share + (size_t)l * (share / nl);
        const size_t end = p.pf_bytes & ~(size_t)15;
        const size_t hi = lo + share / nl < end ? lo + share / nl : end;
        for (size_t a = lo; a < hi; a += 65536) {
          const size_t n = hi - a < 65536 ? hi - a : 65536;
          bulk_prefetch_l2(p.pf + a, (uint32_t)n);
        }
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
  float* tbw = reinterpret_cast<float*>(smem + p.off_t) + (size_t)warp * p.tb_warp;
  const int bpr = p.bpr;
  const int TS = bpr + 1;  // odd stride: conflict-free chains
  const bool oct = FMT == FMT_Q8_0 && p.unit_bytes == 8 * Q8_0_BYTES;
  const int bpu = oct ? 8 : 1;  // blocks per unit
  const int xtok = FMT == FMT_Q8_0 ? p.n_oct * XW : bpr * XW;
  const int R = p.R;
  // This lane's (row, token) chain within a tile.
  const int c_r = lane / NT, c_tok = lane % NT;
  unsigned long long best = 0ull;
  Span sp0, sp1;
  int k = 0;
  for (int tile = blockIdx.x; tile < p.ntiles && warp < p.ncw; tile += gridDim.x, k++) {
    if ((k % p.ncw) != warp) continue;
    const int s = k % NS;
    // Every lane waits (each acquires the stage); the decision is warp-uniform.
    const bool ok = __all_sync(0xffffffffu, !abort_flag && mbar_wait(&full[s], (k / NS) & 1));
    if (!ok) {
      if (lane == 0 && !abort_flag) {
        abort_flag = 1;
        atomicOr(p.err, ERR_WAIT_FULL);
      }
      break;
    }
    tile_spans(p, tile, sp0, sp1);
    const int nr = sp0.nrows;
    const uint8_t* sbuf = stages + (size_t)s * p.stage_bytes;
    const uint8_t* sb0 = sbuf + (reinterpret_cast<uintptr_t>(sp0.base) & 15);
    const uint8_t* sb1 = sbuf + p.span_stride + (reinterpret_cast<uintptr_t>(sp1.base) & 15);
    const int upr = p.upr;
    const int nunits = nspan * nr * upr;
    // Unit u = (span, row, unit-in-row), walked with counters (no divisions).
    int uo = lane % upr, r = lane / upr, si = 0;
    while (r >= nr && si < nspan) {
      r -= nr;
      si++;
    }
    bool released = false;
    if (oct && nunits <= 32) {
      // One octet per lane: copy it to registers and hand the stage back to
      // the producer before the dot products, so the slot refills while this
      // warp computes.
      const bool has = lane < nunits;
      uint32_t w[68];
      const uint8_t* src = (si ? sb1 : sb0) + (size_t)r * p.row_bytes + (size_t)uo * p.unit_bytes;
      if (has) oct_load<NT>(src, w);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      released = true;
      if (has)
        oct_compute<NT>(w, xq + uo * XW, xtok, xd + 8 * uo, p.nt, bpr,
                        tbw + (size_t)((si * R + r) * NT) * TS + uo * 8, TS);
    }
    for (int u = released ? nunits : lane; u < nunits; u += 32) {
      const uint8_t* src = (si ? sb1 : sb0) + (size_t)r * p.row_bytes + (size_t)uo * p.unit_bytes;
      float* t = tbw + (size_t)((si * R + r) * NT) * TS + uo * bpu;
      if (FMT == FMT_Q8_0) {
        if (oct)
          unit_q8_oct<NT>(src, xq + uo * XW, xtok, xd + 8 * uo, p.nt, bpr, t, TS);
        else
          unit_q8<NT>(src, xq + (uo / 8) * XW + (uo % 8) * 8, xtok, xd + uo, p.nt, bpr, t, TS);
      } else if (FMT == FMT_Q4K) {
        unit_q4k<NT, ALIGNED>(src, xq + uo * XW, xd + uo, xb + uo * 8, p.nt, bpr, t, TS);
      } else {
        unit_q6k<NT>(src, xq + uo * XW, xd + uo, p.nt, bpr, t, TS);
      }
      uo += 32;
      while (uo >= upr) {
        uo -= upr;
        if (++r == nr) {
          r = 0;
          si++;
        }
      }
    }
    __syncwarp();
    if (!released && lane == 0) mbar_arrive(&empty[s]);
    // Ordered chains: lane (r, tok) sums its row's terms in block order.
    const bool chain = lane < nr * NT && c_tok < p.nt;
    float acc = 0.0f, acc_u = 0.0f;
    if (chain) {
      const float* tp = tbw + (size_t)(c_r * NT + c_tok) * TS;
      if (nspan == 2) {
        const float* tu = tbw + (size_t)((R + c_r) * NT + c_tok) * TS;
        seq_sum_serial2(bpr, [&](int b) { return tp[b]; }, [&](int b) { return tu[b]; }, acc, acc_u);
      } else {
        acc = seq_sum_serial(bpr, [&](int b) { return tp[b]; });
      }
      const int row = sp0.row0 + c_r;
      if (p.epi == EPI_SWIGLU) {
        // vec::swiglu: silu = x / (1 + expf(-x)); gate = silu * up
        const float silu = __fdiv_rn(acc, __fadd_rn(1.0f, expf_cr(-acc)));
        p.y[0][(size_t)c_tok * p.ld[0] + row] = __fmul_rn(silu, acc_u);
      } else if (p.epi == EPI_RESID) {
        float* dst = p.resid + (size_t)c_tok * p.resid_ld + row;
        *dst = __fadd_rn(*dst, __fmul_rn(p.rs, acc));
      } else {
        float sv = acc;
        if (p.scale != 1.0f) sv = __fmul_rn(sv, p.scale);
        const int sg = sp0.seg;
        p.y[sg][(size_t)c_tok * p.ld[sg] + row] = sv;
        if (p.epi == EPI_ARGMAX && c_tok == 0 && argmax_candidate(sv)) {
          const unsigned long long key = argmax_key(sv, (uint32_t)(row + p.argmax_base));
          best = key > best ? key : best;
        }
      }
    }
    __syncwarp();  // the term buffer is rewritten by the warp's next tile
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

// ============================================================ lane-per-row GEMV
// Q8_0 weights whose rows are whole 16-byte aligned octets (K a multiple of
// 256, 16-byte aligned matrices): the common case of every model here.
//
//  * a group is 32 consecutive rows, one per lane; a stage is one octet column
//    of the group (32 rows x 272 bytes), fetched by one 2-D TMA tensor copy
//    (no swizzle, no multicast). In shared memory a stage is 32 rows of 272
//    bytes: 17 x 16 bytes, an odd number of 16-byte words, so the 32 lanes'
//    16-byte loads of their own rows never share a bank;
//  * stage i of the CTA goes to consumer warp i mod 16, which owns ring slot
//    and term slot i mod 16: its lanes load their rows' octets to registers,
//    hand the slot straight back (so every slot is in flight while its warp
//    computes), form the 8 block terms per token exactly as the reference
//    rounds them (kernels.rs:79) and park them in the term slot;
//  * one chain warp takes the term slots in stage order and adds each row's
//    terms to its running sum (lane = row), block by block, the reference's
//    summation order (kernels.rs:72-82); after a group's last octet it runs
//    the fused epilogue. Gate and up (SwiGLU pair) alternate stage by stage
//    with one running sum each.
constexpr int LR_CW = 16;                     // consumer warps (one ring slot each)
constexpr int LR_NCH = 2;                     // chain warps (alternate row groups)
constexpr int LR_THREADS = (LR_CW + LR_NCH + 1) * 32;  // + chain warps + producer warp
constexpr int LR_STAGE = 32 * 8 * Q8_0_BYTES;  // 32 octets = 8704 bytes, a multiple of 128

struct LrParams {
  CUtensorMap tmap[3];  // one per weight matrix: dims {row_bytes / 4, rows}, box {68, 32}
  Params p;             // activations, prologue layout, epilogue (shared with gemv_kernel)
  int group_start[4];   // first group of each matrix (pair: gate and up share groups)
  int ngroups;
  int spg;       // stages per group: n_oct (x 2 in pair mode)
  int off_tr;    // term ring: LR_CW slots of NT x 8 x 32 floats (bytes from the dynamic base)
  int off_bar;   // full / empty barriers of the ring, term-slot free barriers
  int rg;        // rows per group: 32 / OPS
};

// 2-D tiled TMA load of one box into shared memory, completion counted on
// `bar`. dst 128-byte aligned; x * 4 bytes a multiple of 16. No multicast.
// The group's matrix and first row.
NRC_DEV void lr_group(const LrParams& lp, int g, int& seg, int& row0) {
  seg = 0;
  if (!lp.p.pair)
    while (seg + 1 < lp.p.nseg && g >= lp.group_start[seg + 1]) seg++;
  row0 = (g - lp.group_start[seg]) * lp.rg;
}

template <int NT, int XMODE, int OPS>
__global__ void __launch_bounds__(LR_THREADS, 1) gemv_lr_kernel(const __grid_constant__ LrParams lp) {
  const Params& p = lp.p;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* stages = smem;
  constexpr int NS = LR_CW;  // ring slots = term slots = consumer warps
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + lp.off_bar);
  uint64_t* empty = full + NS;
  uint64_t* tfree = empty + NS;  // term slot s read by the chain warp (consumers sleep on it)
  float* tring = reinterpret_cast<float*>(smem + lp.off_tr);
  constexpr int TSF = NT * 8 * 32;  // floats per term slot
  __shared__ volatile int abort_flag;
  __shared__ uint64_t pf_go;     // completes once: the ring's first stages are issued
  __shared__ uint32_t tflag[NS];  // stage i's terms are in slot i mod NS: tflag = i + 1
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int spg = lp.spg;
  // This CTA's groups: blockIdx.x, + gridDim.x, ...; its stages: group-major.
  const int my_groups = lp.ngroups > (int)blockIdx.x ? (lp.ngroups - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int nstages = my_groups * spg;
  // Tensor copies need a 128-byte aligned destination: refuse to run otherwise.
  if (smem_u32(smem) & 127u) {
    if (tid == 0) atomicOr(p.err, ERR_DRAIN);
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < NS; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&tfree[s], 1);
      tflag[s] = 0;
    }
    mbar_init(&pf_go, 4);  // one arrival per issuing lane
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == LR_CW + LR_NCH) {
    // ----------------------------------------------------------- producer
    // Lanes 0..3 issue (stage i by lane i mod 4, which therefore owns the ring
    // slots i mod NS): a tensor copy takes a while to issue, so several
    // issuing threads keep more copies in flight. The other lanes prefetch
    // the next kernel's weights into L2 once the ring is filled.
    constexpr int NPROD = 4;
    if (lane < NPROD) {
      const uint64_t pol = l2_evict_first();
      int last = -1;
      bool go = false;
      for (int i = lane; i < nstages; i += NPROD) {
        const int s = i % NS;
        if (!go && i >= NS) {
          mbar_arrive(&pf_go);
          go = true;
        }
        if (i >= NS && (abort_flag || !mbar_wait(&empty[s], ((i / NS) - 1) & 1))) {
          abort_flag = 1;
          atomicOr(p.err, ERR_WAIT_EMPTY);
          break;
        }
        const int gl = i / spg, q = i - gl * spg;
        int seg, row0;
        lr_group(lp, (int)blockIdx.x + gl * (int)gridDim.x, seg, row0);
        const int og = p.pair ? q >> 1 : q;  // octet column group of this stage
        const int m = p.pair ? (q & 1) : seg;
        mbar_arrive_expect_tx(&full[s], (uint32_t)LR_STAGE);
        tma_load_2d(stages + (size_t)s * LR_STAGE, &lp.tmap[m], og * OPS * (8 * Q8_0_BYTES / 8), row0, &full[s], pol);
        last = i;
      }
      if (!go) mbar_arrive(&pf_go);
      // Drain: wait (bounded) for this lane's copies still in flight.
      for (int k = last; k >= 0 && k > last - NS; k -= NPROD)
        if (!mbar_wait(&full[k % NS], (k / NS) & 1)) atomicOr(p.err, ERR_DRAIN);
    } else if (p.pf != nullptr && p.pf_bytes >= 16) {
      if (mbar_wait(&pf_go, 0)) {
        const int nl = 32 - NPROD, l = lane - NPROD;
        const size_t share = ((p.pf_bytes / gridDim.x) + (size_t)nl * 16 - 1) / ((size_t)nl * 16) * ((size_t)nl * 16);
        const size_t lo = (size_t)blockIdx.x * share + (size_t)l * (share / nl);
        const size_t end = p.pf_bytes & ~(size_t)15;
        const size_t hi = lo + share / nl < end ? lo + share / nl : end;
        for (size_t a = lo; a < hi; a += 65536) {
          const size_t n = hi - a < 65536 ? hi - a : 65536;
          bulk_prefetch_l2(p.pf + a, (uint32_t)n);
        }
      }
    }
    return;
  }

  if (warp >= LR_CW) {
    // ------------------------------------------------------- chain warps
    // Chain warp c takes the CTA's row groups c, c + LR_NCH, ...: each group's
    // stages in order (so every row's terms are added in block order), CB
    // stages (64 terms per lane) per flag round. Hand-offs: acquire flags in,
    // mbarriers out.
    const int c = warp - LR_CW;
    constexpr int CB = NT * OPS >= 8 ? 1 : 8 / (NT * OPS);
    // Sleep through the consumers' prologue (no polling beside its chain).
    named_sync(2, (LR_CW + LR_NCH) * 32);
    // The SwiGLU epilogue's expf table, brought into L1 while the sums run.
    if (p.epi == EPI_SWIGLU && lane < (int)(sizeof(EXPCR_T_DEV) / 128))
      asm volatile("prefetch.global.L1 [%0];" ::"l"(__cvta_generic_to_global(EXPCR_T_DEV) + (size_t)lane * 128));
    unsigned long long best = 0ull;
    bool stop = false;
    for (int gl = c; gl < my_groups && !stop; gl += LR_NCH) {
      float acc[NT], accu[NT];
#pragma unroll
      for (int t = 0; t < NT; t++) acc[t] = accu[t] = 0.0f;
      int seg, row0;
      lr_group(lp, (int)blockIdx.x + gl * (int)gridDim.x, seg, row0);
      const int row = row0 + lane;
      const bool own = lane < lp.rg && row < p.rows[seg];
      // Residual epilogue: the lane's residual values are final (every earlier
      // launch completed before the consumers' dependency wait, and only this
      // lane writes them), so they are read now, off the end of the chain.
      float rold[NT];
#pragma unroll
      for (int t = 0; t < NT; t++) rold[t] = 0.0f;
      if (p.epi == EPI_RESID && own) {
#pragma unroll
        for (int t = 0; t < NT; t++)
          if (NT == 1 || t < p.nt) rold[t] = p.resid[(size_t)t * p.resid_ld + row];
      }
      for (int q0 = 0; q0 < spg; q0 += CB) {
        const int i0 = gl * spg + q0;
        const int nb = spg - q0 < CB ? spg - q0 : CB;
        // Lane l < nb waits for stage i0 + l.
        const bool ok = __all_sync(0xffffffffu, lane >= nb || flag_wait_geq(&tflag[(i0 + lane) & (NS - 1)],
                                                                               (uint32_t)(i0 + lane) + 1));
        if (!ok || abort_flag) {
          if (lane == 0 && !abort_flag) {
            abort_flag = 1;
            atomicOr(p.err, ERR_WAIT_FULL);
          }
          stop = true;
          break;
        }
        // Row `lane` (< 32 / OPS): octets lane * OPS .. + OPS - 1 of the stage, in order.
        float v[CB][NT][8 * OPS];
#pragma unroll
        for (int b = 0; b < CB; b++) {
          const float* tp = tring + ((i0 + b) & (NS - 1)) * TSF + lane * OPS;
#pragma unroll
          for (int t = 0; t < NT; t++)
#pragma unroll
            for (int o = 0; o < OPS; o++)
#pragma unroll
              for (int j = 0; j < 8; j++)
                v[b][t][o * 8 + j] = b < nb && lane * OPS < 32 ? tp[(t * 8 + j) * 32 + o] : 0.0f;
        }
        __syncwarp();
        if (lane < nb) mbar_arrive(&tfree[(i0 + lane) & (NS - 1)]);
#pragma unroll
        for (int b = 0; b < CB; b++) {
          if (b >= nb) break;
          if (p.pair && ((q0 + b) & 1)) {
#pragma unroll
            for (int t = 0; t < NT; t++)
#pragma unroll
              for (int j = 0; j < 8 * OPS; j++) accu[t] = __fadd_rn(accu[t], v[b][t][j]);
          } else {
#pragma unroll
            for (int t = 0; t < NT; t++)
#pragma unroll
              for (int j = 0; j < 8 * OPS; j++) acc[t] = __fadd_rn(acc[t], v[b][t][j]);
          }
        }
      }
      if (stop) break;
      float hv[NT] = {};
      if (own) {
#pragma unroll
        for (int t = 0; t < NT; t++) {
          if (NT > 1 && t >= p.nt) break;
          if (p.epi == EPI_SWIGLU) {
            // vec::swiglu: silu = x / (1 + expf(-x)); gate = silu * up
            const float silu = __fdiv_rn(acc[t], __fadd_rn(1.0f, expf_cr(-acc[t])));
            hv[t] = __fmul_rn(silu, accu[t]);
            p.y[0][(size_t)t * p.ld[0] + row] = hv[t];
          } else if (p.epi == EPI_RESID) {
            p.resid[(size_t)t * p.resid_ld + row] = __fadd_rn(rold[t], __fmul_rn(p.rs, acc[t]));
          } else {
            float sv = acc[t];
            if (p.scale != 1.0f) sv = __fmul_rn(sv, p.scale);
            p.y[seg][(size_t)t * p.ld[seg] + row] = sv;
            if (p.epi == EPI_ARGMAX && t == 0 && argmax_candidate(sv)) {
              const unsigned long long key = argmax_key(sv, (uint32_t)(row + p.argmax_base));
              best = key > best ? key : best;
            }
          }
        }
      }
      if (p.yq_out) {
        // The host sets yq_out only for 32-row groups of a row count that is a
        // multiple of 32: every lane holds one row, row0 starts a block.
#pragma unroll
        for (int t = 0; t < NT; t++) {
          if (NT > 1 && t >= p.nt) break;
          warp_quant_q8_block(hv[t], lane, p.yq_out + ((size_t)t * (p.rows[0] / 32) + row0 / 32) * Q8_0_BYTES);
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
    return;
  }

  // ------------------------------------------------------------- consumers
  if (XMODE == 1 && p.off_nw >= 0) {
    // The norm weights do not depend on the previous kernel: stage them now.
    float4* dst = reinterpret_cast<float4*>(smem + p.off_nw);
    const float4* src = reinterpret_cast<const float4*>(p.norm_w);
    for (int i = tid; i < p.K / 4; i += LR_CW * 32) dst[i] = src[i];
  }
  pdl_wait();
  if (XMODE == 1)
    build_x_f32<FMT_Q8_0, LR_CW * 32>(p, smem);
  else
    build_x_blocks<FMT_Q8_0, LR_CW * 32>(p, smem);
  named_sync(1, LR_CW * 32);
  named_arrive(2, (LR_CW + LR_NCH) * 32);  // wakes the chain warps

  const uint32_t* xq = reinterpret_cast<const uint32_t*>(smem + p.off_x);
  const float* xd = reinterpret_cast<const float*>(smem + p.off_xd);
  const int xtok = p.n_oct * XW;
  // Lane = (row lane / OPS, octet lane % OPS) of the stage's box.
  const int lo = lane % OPS;
  // Stage i = warp + k * NS: ring slot and term slot `warp`, parity k & 1.
  int q = warp % spg;
  const int qstep = NS % spg;
  for (int i = warp, k = 0; i < nstages; i += NS, k++) {
    const bool ok = __all_sync(0xffffffffu, !abort_flag && mbar_wait(&full[warp], k & 1));
    if (!ok) {
      if (lane == 0 && !abort_flag) {
        abort_flag = 1;
        atomicOr(p.err, ERR_WAIT_FULL);
      }
      break;
    }
    uint32_t w[68];
    oct_load<NT>(stages + (size_t)warp * LR_STAGE + (size_t)lane * (8 * Q8_0_BYTES), w);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[warp]);
    // The term slot is free once the chain warp has read its previous stage
    // (an mbarrier: waiting warps sleep instead of polling).
    if (k > 0) {
      const bool ok2 = __all_sync(0xffffffffu, !abort_flag && mbar_wait(&tfree[warp], (k - 1) & 1));
      if (!ok2) {
        if (lane == 0 && !abort_flag) {
          abort_flag = 1;
          atomicOr(p.err, ERR_WAIT_EMPTY);
        }
        break;
      }
    }
    const int o = (p.pair ? q >> 1 : q) * OPS + lo;
    oct_compute<NT, 32>(w, xq + o * XW, xtok, xd + 8 * o, p.nt, p.bpr, tring + warp * TSF + lane, 8 * 32);
    __syncwarp();
    if (lane == 0) st_release_smem(&tflag[warp], (uint32_t)i + 1);
    q += qstep;
    if (q >= spg) q -= spg;
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
  int dev = 0;
  cudaGetDevice(&dev);
  // The attribute is an upper bound: set it once to the largest dynamic size any launch may use.
  if (ensure_smem_attr((const void*)fn, smem_optin - SMEM_RESERVE) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> g(mu);
  auto key = std::make_tuple(dev, (void*)fn, smem);
  auto itc = cache.find(key);
  if (itc != cache.end()) return itc->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, NTHREADS, smem) != cudaSuccess) n = 0;
  cache[key] = n;
  return n;
}

// ------------------------------------------------------------- lane-per-row host
// rows x (row_bytes / 8) u64 view of a Q8_0 matrix; box = `ops` octet columns
// of 32 / ops rows (8704 bytes, the rows' octets back to back).
bool encode_rows_map(CUtensorMap* m, const void* w, int rows, int row_bytes, int ops) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)(ops * 8 * Q8_0_BYTES / 8), (cuuint32_t)(32 / ops)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(w), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

using LrFn = void (*)(LrParams);
// Instances with NT x OPS <= 4 (the chain warp keeps NT x 8 x OPS terms in registers).
template <int NT, int OPS>
LrFn pick_lr_x(int xmode) {
  return xmode ? gemv_lr_kernel<NT, 1, OPS> : gemv_lr_kernel<NT, 0, OPS>;
}
LrFn pick_lr(int NTc, int xmode, int ops) {
  if (NTc == 1) return ops == 4 ? pick_lr_x<1, 4>(xmode) : (ops == 2 ? pick_lr_x<1, 2>(xmode) : pick_lr_x<1, 1>(xmode));
  if (NTc == 2) return ops == 2 ? pick_lr_x<2, 2>(xmode) : pick_lr_x<2, 1>(xmode);
  return pick_lr_x<4, 1>(xmode);
}

// Launch the lane-per-row kernel if the shape allows it. Returns false (and
// launches nothing) when it does not; `*err` holds a launch error otherwise.
bool gemv_lr_try(const GemvArgs& a, const Params& base, int NTc, int xmode, cudaStream_t stream, bool pdl,
                 cudaError_t* err) {
  *err = cudaSuccess;
  if (a.fmt != FMT_Q8_0 || base.bpr % 8 != 0 || NTc > 4) return false;
  for (int s = 0; s < a.nseg; s++)
    if ((reinterpret_cast<uintptr_t>(a.seg[s].w) & 15) != 0) return false;
  const DevInfo di = dev_info();
  LrParams lp;
  memset(&lp, 0, sizeof(lp));
  lp.p = base;
  Params& p = lp.p;
  const int n_oct = p.bpr / 8;
  const int nspan = a.pair ? 2 : 1;
  // A stage is 32 octets: OPS octet columns of 32 / OPS rows. One column of
  // 32 rows keeps the chain warps' per-stage work short; matrices whose
  // 32-row groups would leave SMs idle take up to 4 columns of 8 rows instead
  // (more, smaller groups), as far as the row length and NT allow.
  int groups32 = 0;
  if (a.pair)
    groups32 = (a.seg[0].rows + 31) / 32;
  else
    for (int s = 0; s < a.nseg; s++) groups32 += (a.seg[s].rows + 31) / 32;
  int ops = 1;
  if (groups32 < di.sms)
    while (ops < 4 && n_oct % (2 * ops) == 0 && NTc * 2 * ops <= 4) ops *= 2;
  lp.rg = 32 / ops;
  lp.spg = n_oct / ops * nspan;
  const size_t ts_floats = (size_t)NTc * 8 * 32;
  // Shared memory: ring | barriers | activations | term ring (doubles as the
  // prologue's f32 staging row).
  const size_t opt_limit = (size_t)di.smem_optin - SMEM_RESERVE;
  const size_t x_bytes = (size_t)NTc * n_oct * XW * 4, xd_bytes = (size_t)NTc * p.bpr * 4;
  // Every ring slot and term slot belongs to one consumer warp (LR_CW of each).
  const size_t off_bar = (size_t)LR_CW * LR_STAGE;
  const size_t off_x = off_bar + 3 * LR_CW * 8;
  const size_t off_xd = off_x + x_bytes;
  const size_t off_tr = (off_xd + xd_bytes + 127) & ~(size_t)127;
  size_t tr = (size_t)LR_CW * ts_floats * 4;
  if (xmode && (size_t)a.K * 4 > tr) tr = (size_t)a.K * 4;
  size_t total = off_tr + tr;
  if (total > opt_limit) return false;
  // Norm weights staged in shared memory when they are 16-byte aligned and fit.
  p.off_nw = -1;
  if (xmode && a.norm_w && (reinterpret_cast<uintptr_t>(a.norm_w) & 15) == 0 && total + (size_t)a.K * 4 <= opt_limit) {
    p.off_nw = (int)total;
    total += (size_t)a.K * 4;
  }
  int ng = 0;
  if (a.pair) {
    ng = (a.seg[0].rows + lp.rg - 1) / lp.rg;
    lp.group_start[0] = 0;
    lp.group_start[1] = ng;
  } else {
    for (int s = 0; s < a.nseg; s++) {
      lp.group_start[s] = ng;
      ng += (a.seg[s].rows + lp.rg - 1) / lp.rg;
    }
    lp.group_start[a.nseg] = ng;
  }
  if (ng == 0) return true;
  for (int s = 0; s < a.nseg; s++)
    if (!encode_rows_map(&lp.tmap[s], a.seg[s].w, a.seg[s].rows, p.row_bytes, ops)) {
      *err = cudaErrorNotSupported;
      return true;
    }
  lp.ngroups = ng;
  if (a.yq_out && a.pair && a.epi == EPI_SWIGLU && lp.rg == 32 && a.seg[0].rows % 32 == 0) {
    p.yq_out = a.yq_out;
    if (a.yq_done) *a.yq_done = 1;
  }
  lp.off_tr = (int)off_tr;
  lp.off_bar = (int)off_bar;
  p.nstage = LR_CW;
  p.n_oct = n_oct;
  p.off_x = (int)off_x;
  p.off_xd = (int)off_xd;
  p.off_xb = (int)off_xd;
  p.off_t = (int)off_tr;
  p.xs_floats = (int)((total - off_tr) / 4);
  LrFn fn = pick_lr(NTc, xmode, ops);
  if ((*err = ensure_smem_attr((const void*)fn, (int)opt_limit)) != cudaSuccess) return true;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(std::min(ng, di.sms));
  cfg.blockDim = dim3(LR_THREADS);
  cfg.dynamicSmemBytes = total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  *err = cudaLaunchKernelEx(&cfg, fn, lp);
  return true;
}

}  // namespace

cudaError_t gemv_run(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  Params p{};
  const int blk = a.fmt == FMT_Q8_0 ? QK8_0 : QK_K;
  const int bbytes = a.fmt == FMT_Q8_0 ? Q8_0_BYTES : (a.fmt == FMT_Q4K ? Q4K_BYTES : Q6K_BYTES);
  if (a.K <= 0 || a.K % blk || a.nt < 1 || a.nt > 8 || a.nseg < 1 || a.nseg > 3) return cudaErrorInvalidValue;
  if (a.pair && (a.nseg != 2 || a.seg[0].rows != a.seg[1].rows)) return cudaErrorInvalidValue;
  if (a.yq_done) *a.yq_done = 0;
  p.K = a.K;
  p.bpr = a.K / blk;
  p.row_bytes = p.bpr * bbytes;
  p.nt = a.nt;
  const int NTc = a.nt <= 1 ? 1 : (a.nt <= 2 ? 2 : (a.nt <= 4 ? 4 : 8));
  bool aligned = true;
  for (int s = 0; s < a.nseg; s++) aligned = aligned && ((reinterpret_cast<uintptr_t>(a.seg[s].w) & 15) == 0);
  p.n_oct = (p.bpr + 7) / 8;
  p.nseg = a.nseg;
  p.pair = a.pair;
  for (int s = 0; s < a.nseg; s++) {
    p.w[s] = static_cast<const uint8_t*>(a.seg[s].w);
    p.y[s] = a.seg[s].y;
    p.rows[s] = a.seg[s].rows;
    p.ld[s] = a.seg[s].ld;
  }
  p.off_nw = -1;
  p.xq = static_cast<const uint8_t*>(a.xq);
  p.xq_out = a.xf ? static_cast<uint8_t*>(a.xq_out) : nullptr;
  p.xf = a.xf;
  p.xf_ld = a.xf_ld;
  p.norm_w = a.norm_w;
  p.eps = a.eps;
  p.fast_norm = a.fast_norm;
  p.epi = a.epi;
  p.scale = a.scale;
  p.resid = a.resid;
  p.resid_ld = a.resid_ld;
  p.rs = a.rs;
  p.argmax_key = a.argmax_key;
  p.argmax_base = a.argmax_base;
  p.err = a.err;
  if (a.pf && (reinterpret_cast<uintptr_t>(a.pf) & 15) == 0) {
    p.pf = static_cast<const uint8_t*>(a.pf);
    p.pf_bytes = a.pf_bytes & ~(size_t)15;
  }
  const int xmode = a.xq ? 0 : 1;
  {
    cudaError_t lr_err;
    if (gemv_lr_try(a, p, NTc, xmode, stream, pdl, &lr_err)) return lr_err;
  }
  const int nspan = a.pair ? 2 : 1;
  const DevInfo di = dev_info();
  // Units: aligned octets of Q8_0 blocks when every row starts 16-byte aligned.
  const bool oct = a.fmt == FMT_Q8_0 && p.bpr % 8 == 0 && aligned;
  p.unit_bytes = oct ? 8 * bbytes : bbytes;
  p.upr = oct ? p.bpr / 8 : p.bpr;
  auto tiles_for = [&](int r) {
    if (a.pair) return (a.seg[0].rows + r - 1) / r;
    int n = 0;
    for (int s = 0; s < a.nseg; s++) n += (a.seg[s].rows + r - 1) / r;
    return n;
  };
  // Shared memory before the stage ring: barriers | activations | term buffers
  // (which double as the f32 staging row of the prologue).
  size_t off = 2 * MAX_STAGES * 8;
  const size_t x_off = off;
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
  const size_t opt_limit = (size_t)di.smem_optin - SMEM_RESERVE;
  // Rows per tile: one unit per lane (one round) when rows are short, at
  // least one row; at most 32 (row, token) chains per warp. Then fewer rows
  // while tiles do not cover every SM, then fewer rows and owning warps until
  // the term buffers and the ring fit.
  int R = std::max(1, std::min(32 / NTc, 32 / (nspan * p.upr)));
  while (R > 1 && tiles_for(R) < di.sms) R--;
  int nstage = 0;
  size_t tbytes = 0;
  for (int ncw = NCW; ncw >= 1 && nstage == 0; ncw--) {
    for (int r = R; r >= 1; r--) {
      p.R = r;
      p.ncw = ncw;
      p.span_stride = (int)(((size_t)r * p.row_bytes + 32 + 15) & ~(size_t)15);
      p.stage_bytes = nspan * p.span_stride;
      p.tb_warp = nspan * r * NTc * (p.bpr + 1);
      tbytes = (size_t)ncw * p.tb_warp * 4;
      if (xmode && (size_t)a.K * 4 > tbytes) tbytes = (size_t)a.K * 4;  // the prologue's f32 row
      const size_t rest = off + tbytes;
      if (2 * ncw <= MAX_STAGES && rest + (size_t)2 * ncw * p.stage_bytes <= opt_limit) {
        nstage = 2 * ncw;
        break;
      }
      if (rest + (size_t)ncw * p.stage_bytes <= opt_limit) {
        nstage = ncw;
        break;
      }
    }
  }
  if (nstage == 0) return cudaErrorInvalidValue;
  p.nstage = nstage;
  p.xs_floats = (int)(tbytes / 4);
  const size_t stage_total = (size_t)nstage * p.stage_bytes;
  p.off_x = (int)(stage_total + x_off);
  p.off_xd = (int)(stage_total + xd_off);
  p.off_xb = (int)(stage_total + xb_off);
  p.off_t = (int)(stage_total + t_off);
  const size_t smem = stage_total + off + tbytes;
  const int RT = p.R;
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
  const int grid = std::min(p.ntiles, di.sms);

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
