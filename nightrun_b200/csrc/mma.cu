// Batched Q8_0 GEMM (prefill, up to 64 tokens per pass) on sm_100a tensor
// cores: tcgen05.mma kind::i8 with TMEM accumulators.
//
// Reference: kernels::matmul_q8 (crates/nr-tensor/src/kernels.rs:91-143) with the
// scalar dot order of dot_q8_scalar (kernels.rs:72-82): for every (row, token)
//   sum = 0; for each block b: sum += (i32 dot_b as f32 * d_w[b]) * d_x[b]
// The tensor core produces each block's exact i32 dot (one K=32 MMA per block,
// written to its own TMEM slot, never accumulated across blocks); the epilogue
// warps apply the per-block scales with the reference's two roundings and add
// the terms in block order, so outputs are bit-identical to the scalar path.
//
// CTA = 128 weight rows x NS tokens, 14 warps:
//   warps 0-7  epilogue: TMEM lane quarter warp % 4 = weight rows, token half
//              warp / 4; per block tcgen05.ld of its half of the slot, exact
//              scaling, running f32 sums in registers; the slot's cells are
//              preset to the bits of 1.5 * 2^23 before the MMA adds onto them;
//   warps 8-11 repack: raw Q8_0 rows (TMA-staged) -> UMMA K-major canonical
//              int8 tiles + f32 row scales;
//   warp 12    producer: per stage one 2-D tensor copy of the tile's raw
//              weight rows (128 rows x 8 blocks) and bulk copies of the
//              activation tiles and scales, into a 2-stage ring (no multicast);
//   warp 13    TMEM allocator and single-thread MMA issuer.
// Every mbarrier wait is bounded (error word + clean exit, never a trap).
#include <algorithm>

#include "common.cuh"
#include "gemv.cuh"
#include "mma.cuh"
#include "seqsum.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace nrc {
namespace {

constexpr int TM = 128;      // weight rows per tile (MMA M)
constexpr int KB = 8;        // Q8_0 blocks per stage (K = 256; 272-byte row chunks are 16-byte aligned)
constexpr int NST = 2;       // pipeline stages
constexpr int NSLOT = 4;     // TMEM accumulator slots
constexpr int NTHR = 448;
constexpr int WP = 12, WM = 13;
constexpr int EPI_WARPS = 8, REP_WARPS = 4;
constexpr uint32_t MAGIC_BITS = 0x4B400000u;  // 12582912.0f = 1.5 * 2^23
constexpr float MAGIC_F = 12582912.0f;

struct Params {
  const uint8_t* w[3];
  float* yseg[3];
  int rows[3];
  int ldseg[3];
  int tile_start[4];
  int nseg;
  int bpr, row_bytes;
  const uint8_t* xq;
  const float* xd;
  int nt, NS, ntg;
  int epi;
  float scale;
  float* resid;
  int resid_ld;
  float rs;
  unsigned* err;
  int off_raw, off_a, off_b, off_dw, off_dx, off_bar, stage_bytes;
  uint32_t tmem_cols;
  CUtensorMap tmap[3];  // per matrix: dims {row_bytes / 2, rows} (u16), box {KB * 34 / 2, TM}
};

template <int NS>
__global__ void __launch_bounds__(NTHR, 1) k_mma_q8(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* full = bars;               // producer -> repack / epilogue (tx bytes)
  uint64_t* aready = bars + NST;       // repack -> MMA (canonical A + row scales written)
  uint64_t* empty = bars + 2 * NST;    // MMA commit + epilogue warps -> producer
  uint64_t* mdone = bars + 3 * NST;    // MMA commit -> epilogue (slot written)
  uint64_t* tfree = bars + 3 * NST + NSLOT;  // epilogue warps -> MMA (slot drained)
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x / p.ntg, tg = blockIdx.x % p.ntg;
  int sg = 0;
  while (sg + 1 < p.nseg && tile >= p.tile_start[sg + 1]) sg++;
  const int row0 = (tile - p.tile_start[sg]) * TM;
  const int nrows = min(TM, p.rows[sg] - row0);
  const int nstages = p.bpr / KB;

  if (tid == 0) {
    for (int s = 0; s < NST; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&aready[s], REP_WARPS);
      mbar_init(&empty[s], 1 + EPI_WARPS);
    }
    for (int k = 0; k < NSLOT; k++) {
      mbar_init(&mdone[k], 1);
      mbar_init(&tfree[k], EPI_WARPS);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == WM) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                 "r"(p.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  pdl_wait();  // activations (B) and the residual stream come from the previous kernel
  const uint32_t tbase = tmem_base_sh;

  auto st_raw = [&](int s) { return smem + p.off_raw + s * p.stage_bytes; };
  auto st_a = [&](int s) { return smem + p.off_a + s * p.stage_bytes; };
  auto st_b = [&](int s) { return smem + p.off_b + s * p.stage_bytes; };
  auto st_dw = [&](int s) { return reinterpret_cast<float*>(smem + p.off_dw + s * p.stage_bytes); };
  auto st_dx = [&](int s) { return reinterpret_cast<float*>(smem + p.off_dx + s * p.stage_bytes); };
  auto fail = [&](unsigned bit) {
    if (!abort_flag) {
      abort_flag = 1;
      atomicOr(p.err, bit);
    }
  };

  if (warp == WP) {
    // ------------------------------------------------------------ producer
    const uint64_t pol = l2_evict_first();
    const uint32_t raw_bytes = (uint32_t)TM * KB * 34;  // whole box: rows past the matrix read as zero
    const uint32_t b_bytes = (uint32_t)KB * NS * 32;
    const uint32_t dx_bytes = (uint32_t)KB * NS * 4;
    int st = 0;
    for (; st < nstages; st++) {
      const int s = st % NST, u = st / NST;
      if (u >= 1) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait(&empty[s], (u - 1) & 1);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) fail(ERR_WAIT_EMPTY);
      }
      if (__any_sync(0xffffffffu, abort_flag)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], raw_bytes + b_bytes + dx_bytes);
        // x = st * 272 bytes: a multiple of 16, as a tensor copy needs.
        tma_load_2d(st_raw(s), &p.tmap[sg], st * (KB * 34 / 2), row0, &full[s], pol);
        const size_t tile = ((size_t)tg * p.bpr + (size_t)st * KB);
        bulk_g2s(st_b(s), p.xq + tile * NS * 32, b_bytes, &full[s], 0ull);
        bulk_g2s(st_dx(s), p.xd + tile * NS, dx_bytes, &full[s], 0ull);
      }
    }
    // Drain the copies of the last issued stages before exit.
    if (lane == 0)
      for (int k = st - 1; k >= 0 && k >= st - NST; k--)
        if (!mbar_wait(&full[k % NST], (k / NST) & 1)) atomicOr(p.err, ERR_DRAIN);
  } else if (warp >= EPI_WARPS && warp < EPI_WARPS + REP_WARPS) {
    // -------------------------------------------------------------- repack
    const int r = tid - EPI_WARPS * 32;  // weight row of this thread
    for (int st = 0; st < nstages; st++) {
      const int s = st % NST, u = st / NST;
      const bool ok = !abort_flag && mbar_wait(&full[s], u & 1);
      if (!ok) {
        fail(ERR_WAIT_FULL);
        break;
      }
      uint8_t* a = st_a(s);
      float* dw = st_dw(s);
      if (r < nrows) {
        const uint8_t* src = st_raw(s) + r * KB * 34;
#pragma unroll
        for (int blk = 0; blk < KB; blk++) {
          // Block blk of this row: d (2 bytes) + 32 int8 quants, 2-byte aligned.
          const uint32_t* base = reinterpret_cast<const uint32_t*>(src + blk * 34 - ((blk & 1) ? 2 : 0));
          uint32_t wv[9];
#pragma unroll
          for (int i = 0; i < 9; i++) wv[i] = base[i];
          uint32_t q[8];
          uint32_t dbits;
          if ((blk & 1) == 0) {
            dbits = wv[0] & 0xffffu;
#pragma unroll
            for (int k = 0; k < 8; k++) q[k] = __byte_perm(wv[k], wv[k + 1], 0x5432);
          } else {
            dbits = wv[0] >> 16;
#pragma unroll
            for (int k = 0; k < 8; k++) q[k] = wv[k + 1];
          }
          uint8_t* ab = a + blk * (TM * 32);
          *reinterpret_cast<uint4*>(ab + canon_off(r, 0)) = make_uint4(q[0], q[1], q[2], q[3]);
          *reinterpret_cast<uint4*>(ab + canon_off(r, 1)) = make_uint4(q[4], q[5], q[6], q[7]);
          dw[blk * TM + r] = f16_to_f32(dbits);
        }
      } else {
#pragma unroll
        for (int blk = 0; blk < KB; blk++) {
          uint8_t* ab = a + blk * (TM * 32);
          *reinterpret_cast<uint4*>(ab + canon_off(r, 0)) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(ab + canon_off(r, 1)) = make_uint4(0, 0, 0, 0);
          dw[blk * TM + r] = 0.0f;
        }
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&aready[s]);
    }
  } else if (warp == WM) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(NS);
      int issued = 0;  // blocks whose MMA was issued
      for (int st = 0; st < nstages && !abort_flag; st++) {
        const int s = st % NST, u = st / NST;
        if (!mbar_wait(&aready[s], u & 1)) {
          fail(ERR_WAIT_FULL);
          break;
        }
        tc_fence_after();
        for (int blk = 0; blk < KB; blk++) {
          const int b = st * KB + blk;
          const int slot = b % NSLOT;
          // The slot drained and preset by the epilogue (first use: preset only).
          if (!mbar_wait(&tfree[slot], (b / NSLOT) & 1)) {
            fail(ERR_WAIT_EMPTY);
            break;
          }
          tc_fence_after();
          const uint64_t ad = smem_desc(st_a(s) + blk * (TM * 32), 128, 256);
          const uint64_t bd = smem_desc(st_b(s) + blk * (NS * 32), 128, 256);
          tc_mma_i8(tbase + (uint32_t)(slot * NS), ad, bd, idesc, 1u);  // onto the preset cells
          tc_commit(&mdone[slot]);
          issued = b + 1;
        }
        tc_commit(&empty[s]);  // stage's smem free once these MMAs completed
      }
      // Never release TMEM with an MMA in flight: wait (bounded) for the last commit.
      if (issued > 0) {
        const int b = issued - 1;
        if (!mbar_wait(&mdone[b % NSLOT], (b / NSLOT) & 1)) atomicOr(p.err, ERR_DRAIN);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    constexpr int NH = NS / 2;  // tokens of this warp
    const int q = warp & 3, half = warp >> 2;
    const int r = q * 32 + lane;  // TMEM lane = weight row
    const int n0 = half * NH;
    float acc[NH];
#pragma unroll
    for (int i = 0; i < NH; i++) acc[i] = 0.0f;
    const uint32_t lane_base = tbase + ((uint32_t)(q * 32) << 16);
    auto preset_slot = [&](int slot) {
#pragma unroll
      for (int c = 0; c < NH; c += 8) tc_st8_fill(lane_base + (uint32_t)(slot * NS + n0 + c), MAGIC_BITS);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tfree[slot]);
    };
    for (int k = 0; k < NSLOT; k++) preset_slot(k);
    for (int st = 0; st < nstages && !abort_flag; st++) {
      const int s = st % NST, u = st / NST;
      if (!mbar_wait(&full[s], u & 1) || !mbar_wait(&aready[s], u & 1)) {
        fail(ERR_WAIT_FULL);
        break;
      }
      const float* dw = st_dw(s);
      const float* dx = st_dx(s);
      bool bad = false;
      for (int blk = 0; blk < KB; blk++) {
        const int b = st * KB + blk;
        const int slot = b % NSLOT;
        if (!mbar_wait(&mdone[slot], (b / NSLOT) & 1)) {
          fail(ERR_WAIT_FULL);
          bad = true;
          break;
        }
        tc_fence_after();
        // Each cell holds the bits of 1.5 * 2^23 + acc (|acc| < 2^22).
        uint32_t v[NH];
#pragma unroll
        for (int c = 0; c < NH; c += 8) tc_ld8(lane_base + (uint32_t)(slot * NS + n0 + c), v + c);
        tc_wait_ld_regs<NH>(v);
        preset_slot(slot);  // values in registers: the slot goes back to the MMA issuer
        const float d = dw[blk * TM + r];
        const float negmd = -MAGIC_F * d;  // exact: d has <= 11 significant bits
        const bool fin = isfinite(d);
        const float* dxb = dx + blk * NS + n0;
#pragma unroll
        for (int j = 0; j < NH; j += 2) {
          // (acc as f32 * d_w) * d_x, then sum += term (kernels.rs:79).
          // M + acc is exact, and fma(M + acc, d, -M*d) rounds acc*d once,
          // exactly like the reference's multiply.
          float2 t1;
          if (fin) {
            t1 = __ffma2_rn(make_float2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])), make_float2(d, d),
                            make_float2(negmd, negmd));
          } else {
            t1 = make_float2(__fmul_rn(i2f((int)(v[j] - MAGIC_BITS)), d), __fmul_rn(i2f((int)(v[j + 1] - MAGIC_BITS)), d));
          }
          // The product and the sum stay two roundings (scalar _rn operations,
          // never contracted; a packed multiply feeding a packed add would be).
          const float2 x2 = *reinterpret_cast<const float2*>(dxb + j);
          acc[j] = __fadd_rn(acc[j], __fmul_rn(t1.x, x2.x));
          acc[j + 1] = __fadd_rn(acc[j + 1], __fmul_rn(t1.y, x2.y));
        }
      }
      if (bad) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!abort_flag && r < nrows) {
      const int row = row0 + r;
#pragma unroll
      for (int n = 0; n < NH; n++) {
        const int tok = tg * NS + n0 + n;
        if (tok >= p.nt) break;
        float sv = acc[n];
        if (p.epi == EPI_RESID) {
          float* dst = p.resid + (size_t)tok * p.resid_ld + row;
          *dst = __fadd_rn(*dst, __fmul_rn(p.rs, sv));
        } else {
          if (p.scale != 1.0f) sv = __fmul_rn(sv, p.scale);
          p.yseg[sg][(size_t)tok * p.ldseg[sg] + row] = sv;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == WM) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(p.tmem_cols) : "memory");
  }
}

// ------------------------------------------------------------ activation quantization
// One CTA (256 threads) per token: optional RMSNorm (the same reduction order
// as the GEMV prologue, so both paths derive identical activations), then
// q8::quantize, one thread per 32-value block, into the canonical tiles.
__global__ void __launch_bounds__(256) k_mma_quant_act(const MmaActArgs a) {
  pdl_wait();
  pdl_trigger();
  const int n = blockIdx.x;  // token slot (0 .. ntg*NS - 1)
  const int tid = threadIdx.x;
  const int bpr = a.K / 32;
  const int tg = n / a.NS, nn = n % a.NS;
  __shared__ SeqSumShared ssh;
  if (n >= a.nt) {
    for (int b = tid; b < bpr; b += 256) {
      uint8_t* t = a.xq + ((size_t)tg * bpr + b) * a.NS * 32;
      *reinterpret_cast<uint4*>(t + canon_off(nn, 0)) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(t + canon_off(nn, 1)) = make_uint4(0, 0, 0, 0);
      a.xd[((size_t)tg * bpr + b) * a.NS + nn] = 0.0f;
    }
    return;
  }
  extern __shared__ float xrow[];  // the token's K values
  const float* x = a.x + (size_t)n * a.x_ld;
  for (int i = tid; i < a.K; i += 256) xrow[i] = x[i];
  __syncthreads();
  float sc = 1.0f;
  if (a.norm_w) {
    // vec::rmsnorm (vec.rs:4-14): `ss += v * v` in index order (one chain, seqsum.cuh).
    const float ss = seq_sum_squares_group<256>(xrow, a.K, ssh, tid, [] { __syncthreads(); });
    sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)a.K), a.eps)));
  }
  // q8::quantize (q8.rs:27-44), one thread per 32-value block.
  for (int b = tid; b < bpr; b += 256) {
    float v[32];
#pragma unroll
    for (int k = 0; k < 32; k++) {
      v[k] = xrow[b * 32 + k];
      if (a.norm_w) v[k] = __fmul_rn(__fmul_rn(v[k], sc), __ldg(a.norm_w + b * 32 + k));
    }
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 32; k++) amax = fmaxf(amax, fabsf(v[k]));
    const uint16_t dbits = f32_to_f16(__fdiv_rn(amax, 127.0f));
    const float d = f16_to_f32(dbits);
    const float inv = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t pk[8];
#pragma unroll
    for (int c = 0; c < 8; c++) {
      uint32_t wv = 0;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const float xsv = __fmul_rn(v[4 * c + k], inv);
        const float r = xsv >= 0.0f ? __fadd_rn(xsv, 0.5f) : __fsub_rn(xsv, 0.5f);
        int q = rust_f2i(r);
        q = q < -127 ? -127 : (q > 127 ? 127 : q);
        wv |= (uint32_t)(uint8_t)(int8_t)q << (8 * k);
      }
      pk[c] = wv;
    }
    uint8_t* t = a.xq + ((size_t)tg * bpr + b) * a.NS * 32;
    *reinterpret_cast<uint4*>(t + canon_off(nn, 0)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    *reinterpret_cast<uint4*>(t + canon_off(nn, 1)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    a.xd[((size_t)tg * bpr + b) * a.NS + nn] = d;
  }
}

// Pre-quantized Q8_0 activation blocks [nt][bpr] -> canonical per-block tiles.
__global__ void k_mma_pack_q8(const uint8_t* __restrict__ x, int nt, int bpr, int NS, int ntg, uint8_t* xq,
                              float* xd) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // (token slot, block)
  if (i >= NS * ntg * bpr) return;
  const int n = i / bpr, b = i % bpr;
  const int tg = n / NS, nn = n % NS;
  uint8_t* t = xq + ((size_t)tg * bpr + b) * NS * 32;
  uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float d = 0.0f;
  if (n < nt) {
    const uint8_t* s = x + ((size_t)n * bpr + b) * 34;
#pragma unroll
    for (int k = 0; k < 8; k++)
      w[k] = (uint32_t)s[2 + 4 * k] | ((uint32_t)s[3 + 4 * k] << 8) | ((uint32_t)s[4 + 4 * k] << 16) |
             ((uint32_t)s[5 + 4 * k] << 24);
    d = f16_to_f32((uint32_t)s[0] | ((uint32_t)s[1] << 8));
  }
  *reinterpret_cast<uint4*>(t + canon_off(nn, 0)) = make_uint4(w[0], w[1], w[2], w[3]);
  *reinterpret_cast<uint4*>(t + canon_off(nn, 1)) = make_uint4(w[4], w[5], w[6], w[7]);
  xd[((size_t)tg * bpr + b) * NS + nn] = d;
}

cudaError_t launch(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, void** args) {
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

cudaError_t mma_quant_act_run(const MmaActArgs& a, cudaStream_t s, bool pdl) {
  if (a.K % 256 || (a.NS != 16 && a.NS != 32 && a.NS != 64) || a.nt > a.NS * a.ntg) return cudaErrorInvalidValue;
  MmaActArgs aa = a;
  void* args[] = {&aa};
  const size_t smem = (size_t)a.K * 4;
  if (cudaError_t e = ensure_smem_attr((const void*)k_mma_quant_act, 64 * 1024)) return e;
  if (smem > 64 * 1024) return cudaErrorInvalidValue;
  return launch((const void*)k_mma_quant_act, dim3(a.NS * a.ntg), dim3(256), smem, s, pdl, args);
}

cudaError_t mma_pack_q8_run(const uint8_t* x, int nt, int K, int NS, int ntg, uint8_t* xq, float* xd, cudaStream_t s) {
  if (K % 256 || nt > NS * ntg) return cudaErrorInvalidValue;
  const int bpr = K / 32;
  const int total = NS * ntg * bpr;
  k_mma_pack_q8<<<(total + 255) / 256, 256, 0, s>>>(x, nt, bpr, NS, ntg, xq, xd);
  return cudaGetLastError();
}

cudaError_t mma_q8_run(const MmaArgs& a, cudaStream_t s, bool pdl) {
  if (a.K % 256 || (a.NS != 16 && a.NS != 32 && a.NS != 64) || a.nseg < 1 || a.nseg > 3)
    return cudaErrorInvalidValue;
  Params p{};
  int tiles = 0;
  for (int i = 0; i < a.nseg; i++) {
    if (reinterpret_cast<uintptr_t>(a.seg[i].w) & 15) return cudaErrorInvalidValue;
    p.w[i] = static_cast<const uint8_t*>(a.seg[i].w);
    p.yseg[i] = a.seg[i].y;
    p.rows[i] = a.seg[i].rows;
    p.ldseg[i] = a.seg[i].ld > 0 ? a.seg[i].ld : a.seg[i].rows;
    p.tile_start[i] = tiles;
    tiles += (a.seg[i].rows + TM - 1) / TM;
  }
  p.tile_start[a.nseg] = tiles;
  p.nseg = a.nseg;
  p.bpr = a.K / 32;
  p.row_bytes = p.bpr * 34;
  p.xq = a.xq;
  p.xd = a.xd;
  p.nt = a.nt;
  p.NS = a.NS;
  p.ntg = a.ntg;
  p.epi = a.epi;
  p.scale = a.scale;
  p.resid = a.resid;
  p.resid_ld = a.resid_ld;
  p.rs = a.rs;
  p.err = a.err;
  auto enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  for (int i = 0; i < a.nseg; i++) {
    // rows x (row_bytes / 2) u16 view (row_bytes = 272 * K / 256, a multiple of 16).
    const cuuint64_t dims[2] = {(cuuint64_t)(p.row_bytes / 2), (cuuint64_t)a.seg[i].rows};
    const cuuint64_t strides[1] = {(cuuint64_t)p.row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(KB * 34 / 2), (cuuint32_t)TM};
    const cuuint32_t estr[2] = {1, 1};
    if (a.seg[i].rows > 0 &&
        enc(&p.tmap[i], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(a.seg[i].w), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  // Stage layout: A canonical (1024-aligned) | raw rows (128-aligned) | B | dw | dx.
  size_t o = 0;
  p.off_a = (int)o;
  o += (size_t)KB * TM * 32;
  p.off_raw = (int)o;
  o += (size_t)TM * KB * 34;
  o = (o + 127) & ~(size_t)127;
  p.off_b = (int)o;
  o += (size_t)KB * a.NS * 32;
  p.off_dw = (int)o;
  o += (size_t)KB * TM * 4;
  p.off_dx = (int)o;
  o += (size_t)KB * a.NS * 4;
  o = (o + 1023) & ~(size_t)1023;
  p.stage_bytes = (int)o;
  p.off_bar = (int)(o * NST);
  const size_t smem = o * NST + (3 * NST + 2 * NSLOT) * 8;
  uint32_t cols = 32;
  while (cols < (uint32_t)(NSLOT * a.NS)) cols <<= 1;
  p.tmem_cols = cols;
  const void* fn = a.NS == 16 ? (const void*)k_mma_q8<16> : (a.NS == 32 ? (const void*)k_mma_q8<32> : (const void*)k_mma_q8<64>);
  if (cudaError_t e = ensure_smem_attr(fn, 225 * 1024)) return e;
  if (smem > 225 * 1024) return cudaErrorInvalidValue;
  if (tiles == 0) return cudaSuccess;
  void* args[] = {&p};
  return launch(fn, dim3(tiles * a.ntg), dim3(NTHR), smem, s, pdl, args);
}

}  // namespace nrc
