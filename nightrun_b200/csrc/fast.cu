// Decode GEMV of the tolerance mode (one token, f32 activations in, every
// epilogue of the exact GEMV): y = W · quantize(rmsnorm?(x)).
//
// Same arithmetic per block as the exact kernels (the block units of
// units.cuh: integer dots, the reference's per-block f32 roundings, the
// reference's activation quantization), but the row's block terms are added
// by a warp tree instead of one sequential chain, and the RMSNorm sum of
// squares is a CTA tree (kernels.rs:72-82 and vec.rs:4-14 up to summation
// order).
//
// Built for latency inside a chain of dependent launches:
//  * persistent CTAs, one per SM at most, each owning a contiguous range of
//    output rows ("units"; a SwiGLU unit is a gate row and its up row);
//  * about 106 KB of shared memory, so a CTA of the next kernel fits beside
//    one of this kernel on every SM: its producer warp streams the next
//    matrix into its own ring while this kernel still runs;
//  * the producer warp (warp 7) copies the CTA's rows HBM -> shared memory
//    with 1-D bulk copies (cp.async.bulk, no multicast, L2 evict-first) into
//    a 4-stage ring before the programmatic-dependency wait (weights never
//    depend on the previous kernel); its other lanes prefetch the next
//    kernel's weights into L2;
//  * 7 consumer warps wait for the previous kernel, stage the quantized
//    activations, then take the rows of each stage round-robin: a warp per
//    row, lanes over the row's blocks, a shuffle tree, the epilogue on lane 0.
// Every wait is bounded by %globaltimer; on expiry the kernel sets the error
// word, drains its own copies and returns.
#include <algorithm>

#include "common.cuh"
#include "expf_cr.cuh"
#include "fast.cuh"
#include "units.cuh"

namespace nrc {
namespace {

constexpr int FW = 8;          // warps
constexpr int FCW = FW - 1;    // consumer warps
constexpr int FT = FW * 32;
constexpr int FNS = 4;         // ring stages
constexpr int FSTAGE = 24 * 1024;
constexpr int FMAXP = 3;       // copies per stage at most (a stage spans <= 3 matrices, or gate + up)

struct FParams {
  const uint8_t* w[3];
  float* y[3];
  int ld0;
  int ustart[4];  // first unit of each matrix (pair: gate and up share units)
  int nseg, pair, fmt;
  int K, bpr, row_bytes, n_oct;
  int units;  // rows (pair: gate rows)
  int R;      // units per stage
  const float* x;
  const float* norm_w;
  float eps;
  int epi;
  float scale;
  float* resid;
  float rs;
  unsigned long long* argmax_key;
  unsigned* err;
  const uint8_t* pf;
  size_t pf_bytes;
  int off_bar, off_xq, off_xd, off_xb;
};

struct Piece {
  const uint8_t* lo;  // 16-byte aligned source
  uint32_t bytes;     // 16-byte multiple
  uint32_t dst;       // offset in the stage
  uint32_t skew;      // first row's offset from dst
  int seg, row0, n;
};

// The copies of stage units [a, b): one per matrix piece (pair: gate rows,
// then up rows), each a 16-byte aligned superset of its rows.
NRC_DEV int stage_pieces(const FParams& p, int a, int b, Piece* pc) {
  int np = 0;
  uint32_t off = 0;
  auto add = [&](int seg, int r0, int n) {
    const uintptr_t s = reinterpret_cast<uintptr_t>(p.w[seg]) + (size_t)r0 * p.row_bytes;
    const uintptr_t e = s + (size_t)n * p.row_bytes;
    const uintptr_t lo = s & ~(uintptr_t)15, hi = (e + 15) & ~(uintptr_t)15;
    pc[np].lo = reinterpret_cast<const uint8_t*>(lo);
    pc[np].bytes = (uint32_t)(hi - lo);
    pc[np].dst = off;
    pc[np].skew = (uint32_t)(s - lo);
    pc[np].seg = seg;
    pc[np].row0 = r0;
    pc[np].n = n;
    off += (uint32_t)(hi - lo);
    np++;
  };
  if (p.pair) {
    add(0, a, b - a);
    add(1, a, b - a);
  } else {
    for (int sg = 0; sg < p.nseg; sg++) {
      const int s0 = max(a, p.ustart[sg]), s1 = min(b, p.ustart[sg + 1]);
      if (s1 > s0) add(sg, s0 - p.ustart[sg], s1 - s0);
    }
  }
  return np;
}

// Dot of one row held in shared memory with the staged activations: lanes
// over the row's blocks (Q8_0) or super-blocks (K-quants), exact per-block
// terms, a shuffle tree. Every lane returns the sum.
template <int FMT>
NRC_DEV float row_dot(const uint8_t* row, const uint32_t* xq, const float* xd, const int* xb, int bpr, int lane) {
  float acc = 0.0f;
  for (int b = lane; b < bpr; b += 32) {
    float t;
    if (FMT == FMT_Q8_0)
      unit_q8<1>(row + (size_t)b * Q8_0_BYTES, xq + (b / 8) * XW + (b % 8) * 8, 0, xd + b, 1, bpr, &t, 0);
    else if (FMT == FMT_Q4K)
      unit_q4k<1, 1>(row + (size_t)b * Q4K_BYTES, xq + b * XW, xd + b, xb + b * 8, 1, bpr, &t, 0);
    else
      unit_q6k<1>(row + (size_t)b * Q6K_BYTES, xq + b * XW, xd + b, 1, bpr, &t, 0);
    acc = __fadd_rn(acc, t);
  }
  return warp_sum(acc);
}

// Activations: optional RMSNorm (CTA tree for the sum of squares), then the
// reference's quantization (q8::quantize, q8.rs:27-44, or quantize_q8k,
// kquant.rs:157-187) into shared memory. Consumer threads only.
template <int FMT>
NRC_DEV void fast_prologue(const FParams& p, uint8_t* smem, float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NCT = FCW * 32;
  uint32_t* xq = reinterpret_cast<uint32_t*>(smem + p.off_xq);
  float* xd = reinterpret_cast<float*>(smem + p.off_xd);
  int* xb = reinterpret_cast<int*>(smem + p.off_xb);
  const float* x = p.x;
  float sc = 1.0f;
  if (p.norm_w) {
    float part = 0.0f;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int i = tid; i < p.K / 4; i += NCT) {
      const float4 v = x4[i];
      part = __fadd_rn(part, __fadd_rn(__fadd_rn(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y)),
                                       __fadd_rn(__fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w))));
    }
    part = warp_sum(part);
    if (lane == 0) red[warp] = part;
    named_sync(1, NCT);
    float ss = 0.0f;
#pragma unroll
    for (int w = 0; w < FCW; w++) ss = __fadd_rn(ss, red[w]);
    sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)p.K), p.eps)));
  }
  if (FMT == FMT_Q8_0) {
    // 8 lanes per 32-value block, 4 values each; 4 blocks per warp pass.
    const int g = lane & 7, sub = lane >> 3;
    for (int b0 = warp * 4; b0 < p.bpr; b0 += FCW * 4) {
      const int b = b0 + sub;
      const bool on = b < p.bpr;
      float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (on) {
        const float4 q = reinterpret_cast<const float4*>(x + b * 32 + g * 4)[0];
        v[0] = q.x;
        v[1] = q.y;
        v[2] = q.z;
        v[3] = q.w;
        if (p.norm_w) {
          const float4 w4 = reinterpret_cast<const float4*>(p.norm_w + b * 32 + g * 4)[0];
          v[0] = __fmul_rn(__fmul_rn(v[0], sc), w4.x);
          v[1] = __fmul_rn(__fmul_rn(v[1], sc), w4.y);
          v[2] = __fmul_rn(__fmul_rn(v[2], sc), w4.z);
          v[3] = __fmul_rn(__fmul_rn(v[3], sc), w4.w);
        }
      }
      float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (!on) continue;
      const float d = f16_to_f32(f32_to_f16(__fdiv_rn(amax, 127.0f)));
      const float inv = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
      uint32_t wv = 0;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const float xs = __fmul_rn(v[k], inv);
        const float r = xs >= 0.0f ? __fadd_rn(xs, 0.5f) : __fsub_rn(xs, 0.5f);
        int q = rust_f2i(r);
        q = q < -127 ? -127 : (q > 127 ? 127 : q);
        wv |= (uint32_t)(uint8_t)(int8_t)q << (8 * k);
      }
      xq[(b / 8) * XW + (b % 8) * 8 + g] = wv;
      if (g == 0) xd[b] = d;
    }
  } else {
    // One warp per 256-value super-block, 8 values per lane (quantize_q8k).
    for (int b = warp; b < p.bpr; b += FCW) {
      const float4* s4 = reinterpret_cast<const float4*>(x + b * 256 + lane * 8);
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
      for (int k = 0; k < 8; k++)
        if (fabsf(v[k]) > amax) {
          amax = fabsf(v[k]);
          mx = v[k];
          idx = lane * 8 + k;
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
      uint32_t* qw = xq + b * XW;
      int* bs = xb + b * 8;
      if (amax == 0.0f) {
        qw[lane * 2] = 0u;
        qw[lane * 2 + 1] = 0u;
        if (lane < 8) bs[lane] = 0;
        if (lane == 0) xd[b] = 0.0f;
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
      int s4s = part + __shfl_down_sync(0xffffffffu, part, 1);
      s4s += __shfl_down_sync(0xffffffffu, s4s, 2);
      if ((lane & 3) == 0) bs[lane / 4] = s4s;
      if (lane == 0) xd[b] = __fdiv_rn(1.0f, iscale);
    }
  }
  named_sync(1, NCT);
}

template <int FMT>
__global__ void __launch_bounds__(FT, 2) k_fast_gemv(const __grid_constant__ FParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* empty = full + FNS;
  __shared__ volatile int abort_flag;
  __shared__ float red[FCW];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // This CTA's units [u0, u1), stages of R units.
  const int G = gridDim.x;
  const int u0 = (int)(((long long)p.units * blockIdx.x) / G), u1 = (int)(((long long)p.units * (blockIdx.x + 1)) / G);
  const int nst = (u1 - u0 + p.R - 1) / p.R;
  if (tid == 0) {
    for (int s = 0; s < FNS; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], FCW);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == FCW) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first();
      int i = 0;
      for (; i < nst; i++) {
        const int s = i % FNS;
        if (i >= FNS && (abort_flag || !mbar_wait(&empty[s], ((i / FNS) - 1) & 1))) {
          abort_flag = 1;
          atomicOr(p.err, ERR_WAIT_EMPTY);
          break;
        }
        Piece pc[FMAXP];
        const int a = u0 + i * p.R, b = min(u1, a + p.R);
        const int np = stage_pieces(p, a, b, pc);
        uint32_t total = 0;
        for (int k = 0; k < np; k++) total += pc[k].bytes;
        mbar_arrive_expect_tx(&full[s], total);
        uint8_t* st = smem + (size_t)s * FSTAGE;
        for (int k = 0; k < np; k++) bulk_g2s(st + pc[k].dst, pc[k].lo, pc[k].bytes, &full[s], pol);
      }
      // Drain this CTA's copies still in flight before exit.
      for (int k = i - 1; k >= 0 && k >= i - FNS; k--)
        if (!mbar_wait(&full[k % FNS], (k / FNS) & 1)) atomicOr(p.err, ERR_DRAIN);
    } else if (p.pf != nullptr && p.pf_bytes >= 16) {
      // Prefetch this CTA's share of the next kernel's weights into L2 (a
      // hint: nothing waits for it).
      const int nl = 31, l = lane - 1;
      const size_t share = ((p.pf_bytes / G) + (size_t)nl * 16 - 1) / ((size_t)nl * 16) * ((size_t)nl * 16);
      const size_t lo = (size_t)blockIdx.x * share + (size_t)l * (share / nl);
      const size_t end = p.pf_bytes & ~(size_t)15;
      const size_t hi = lo + share / nl < end ? lo + share / nl : end;
      for (size_t a = lo; a < hi; a += 65536) {
        const size_t n = hi - a < 65536 ? hi - a : 65536;
        bulk_prefetch_l2(p.pf + a, (uint32_t)n);
      }
    }
    return;
  }

  // ------------------------------------------------------------- consumers
  pdl_wait();
  fast_prologue<FMT>(p, smem, red);
  const uint32_t* xq = reinterpret_cast<const uint32_t*>(smem + p.off_xq);
  const float* xd = reinterpret_cast<const float*>(smem + p.off_xd);
  const int* xb = reinterpret_cast<const int*>(smem + p.off_xb);
  unsigned long long best = 0ull;
  for (int i = 0; i < nst; i++) {
    const int s = i % FNS;
    const bool ok = __all_sync(0xffffffffu, !abort_flag && mbar_wait(&full[s], (i / FNS) & 1));
    if (!ok) {
      if (lane == 0 && !abort_flag) {
        abort_flag = 1;
        atomicOr(p.err, ERR_WAIT_FULL);
      }
      break;
    }
    Piece pc[FMAXP];
    const int a = u0 + i * p.R, b = min(u1, a + p.R);
    const int np = stage_pieces(p, a, b, pc);
    const uint8_t* st = smem + (size_t)s * FSTAGE;
    for (int u = a + warp; u < b; u += FCW) {
      // The unit's piece (and, in pair mode, its up row in piece 1).
      int k = 0;
      if (!p.pair)
        while (k + 1 < np && u >= p.ustart[pc[k].seg] + pc[k].row0 + pc[k].n) k++;
      const int r = u - (p.pair ? 0 : p.ustart[pc[k].seg]);
      const uint8_t* row = st + pc[k].dst + pc[k].skew + (size_t)(r - pc[k].row0) * p.row_bytes;
      const float acc = row_dot<FMT>(row, xq, xd, xb, p.bpr, lane);
      if (p.pair) {
        const uint8_t* urow = st + pc[1].dst + pc[1].skew + (size_t)(r - pc[1].row0) * p.row_bytes;
        const float accu = row_dot<FMT>(urow, xq, xd, xb, p.bpr, lane);
        if (lane == 0) {
          // vec::swiglu: silu = x / (1 + expf(-x)); gate = silu * up
          const float silu = __fdiv_rn(acc, __fadd_rn(1.0f, expf_cr(-acc)));
          p.y[0][r] = __fmul_rn(silu, accu);
        }
      } else if (lane == 0) {
        if (p.epi == EPI_RESID) {
          p.resid[r] = __fadd_rn(p.resid[r], __fmul_rn(p.rs, acc));
        } else {
          float sv = acc;
          if (p.scale != 1.0f) sv = __fmul_rn(sv, p.scale);
          p.y[pc[k].seg][r] = sv;
          if (p.epi == EPI_ARGMAX && argmax_candidate(sv)) {
            const unsigned long long key = argmax_key(sv, (uint32_t)r);
            best = key > best ? key : best;
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (p.epi == EPI_ARGMAX && lane == 0 && best) atomicMax(p.argmax_key, best);
}

cudaError_t launch_fast(const void* fn, int grid, size_t smem, const FParams& p, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(FT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FParams pp = p;
  void* args[] = {&pp};
  return cudaLaunchKernelExC(&cfg, fn, args);
}

int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev] > 0 ? n[dev] : 148;
}

}  // namespace

cudaError_t fast_gemv_run(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  const int blk = a.fmt == FMT_Q8_0 ? QK8_0 : QK_K;
  const int bbytes = a.fmt == FMT_Q8_0 ? Q8_0_BYTES : (a.fmt == FMT_Q4K ? Q4K_BYTES : Q6K_BYTES);
  if (a.K <= 0 || a.K % blk || a.nt != 1 || !a.xf || a.xq || a.nseg < 1 || a.nseg > 3 || (a.K % 256))
    return cudaErrorInvalidValue;
  if (a.pair && (a.nseg != 2 || a.seg[0].rows != a.seg[1].rows)) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.xf) & 15) || (a.norm_w && (reinterpret_cast<uintptr_t>(a.norm_w) & 15)))
    return cudaErrorInvalidValue;
  FParams p{};
  p.fmt = a.fmt;
  p.K = a.K;
  p.bpr = a.K / blk;
  p.row_bytes = p.bpr * bbytes;
  p.n_oct = (p.bpr + 7) / 8;
  p.nseg = a.nseg;
  p.pair = a.pair;
  int units = 0;
  for (int s = 0; s < a.nseg; s++) {
    if (reinterpret_cast<uintptr_t>(a.seg[s].w) & 15) return cudaErrorInvalidValue;
    p.w[s] = static_cast<const uint8_t*>(a.seg[s].w);
    p.y[s] = a.seg[s].y;
    p.ustart[s] = a.pair ? 0 : units;
    if (!a.pair) units += a.seg[s].rows;
  }
  if (a.pair) units = a.seg[0].rows;
  p.ustart[a.nseg] = units;
  p.units = units;
  if (units == 0) return cudaSuccess;
  // Units per stage: the stage holds R rows (x 2 in pair mode) plus the
  // alignment slack of each copy (at most 15 bytes before and 15 after each
  // of up to FMAXP copies; the row loads read at most 6 bytes past a row).
  const int per_unit = p.row_bytes * (a.pair ? 2 : 1);
  p.R = (FSTAGE - 32 * FMAXP - 16) / per_unit;
  if (p.R < 1) return cudaErrorInvalidValue;  // a row larger than a stage
  p.x = a.xf;
  p.norm_w = a.norm_w;
  p.eps = a.eps;
  p.epi = a.epi;
  p.scale = a.scale;
  p.resid = a.resid;
  p.rs = a.rs;
  p.argmax_key = a.argmax_key;
  p.err = a.err;
  if (a.pf && (reinterpret_cast<uintptr_t>(a.pf) & 15) == 0) {
    p.pf = static_cast<const uint8_t*>(a.pf);
    p.pf_bytes = a.pf_bytes & ~(size_t)15;
  }
  // Shared memory: ring | barriers | activations.
  size_t o = (size_t)FNS * FSTAGE;
  p.off_bar = (int)o;
  o += 2 * FNS * 8;
  o = (o + 15) & ~(size_t)15;
  p.off_xq = (int)o;
  o += (size_t)(a.fmt == FMT_Q8_0 ? p.n_oct : p.bpr) * XW * 4;
  p.off_xd = (int)o;
  o += (size_t)p.bpr * 4;
  p.off_xb = (int)o;
  if (a.fmt != FMT_Q8_0) o += (size_t)p.bpr * 8 * 4;
  const size_t smem = (o + 15) & ~(size_t)15;
  const void* fn = a.fmt == FMT_Q8_0 ? (const void*)k_fast_gemv<FMT_Q8_0>
                                     : (a.fmt == FMT_Q4K ? (const void*)k_fast_gemv<FMT_Q4K> : (const void*)k_fast_gemv<FMT_Q6K>);
  if (cudaError_t e = ensure_smem_attr(fn, (int)smem)) return e;
  const int grid = std::min(units, sm_count());
  return launch_fast(fn, grid, smem, p, stream, pdl);
}

}  // namespace nrc
