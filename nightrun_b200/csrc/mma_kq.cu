// Batched K-quant GEMM (Q4_K / Q6_K weights x Q8_K activations, 9+ tokens:
// prefill chunks and multi-sequence decode) on sm_100a tensor cores:
// tcgen05.mma kind::i8 with TMEM accumulators.
//
// Reference: kquant::matmul_q4k / matmul_q6k (crates/nr-tensor/src/kquant.rs:
// 566-639) with the scalar dot order of dot_q4k_scalar / dot_q6k_scalar
// (kquant.rs:192-250). Per (row, token, super-block):
//   Q4_K: sum_q = sum over 32-value sub-blocks j of f32(sc_j) * f32(dot_j), in
//         order; sum_m = sum_j m_j * (bsum_2j + bsum_2j+1) (integer);
//         term = (d*dx) * sum_q - (dmin*dx) * f32(sum_m)
//   Q6_K: sum = sum over 16-value groups g of f32(sc_g) * f32(dot_g), in order;
//         term = (d*dx) * sum
// and the row's terms are added over super-blocks in order. The tensor core
// produces every dot exactly: one K=32 MMA per Q4_K sub-block, and for Q6_K
// two per 32-value chunk whose A tiles keep one 16-value half each (the other
// half zero), each into its own TMEM slot; the epilogue applies the scales
// with the reference's roundings in the reference's order, so outputs are
// bit-identical to the scalar path.
//
// CTA = 128 weight rows x 32 tokens, one super-block per stage (Q4_K three
// shared-memory stages, Q6_K two), 14 warps:
//   warps 0-7   epilogue: TMEM lane quarter warp % 4 (rows), token half warp / 4;
//   warps 8-11  repack: raw rows -> canonical int8 A tiles + row scales;
//   warp 12     producer: eight 2-D tensor copies per super-block (the
//               matrix as rows of 8-row groups; box = one super-block window
//               of 16 groups), the last rows % 8 by cp.async, the activation
//               tiles and their scales / chunk sums by bulk copies (no multicast);
//   warp 13     TMEM allocator and single-thread MMA issuer.
// TMEM: two units of 8 slots x 32 columns; a Q4_K super-block fills one unit
// (two super-blocks in flight), a Q6_K one fills both in turn (the MMA fills
// one unit while the epilogue drains the other).
// Every mbarrier wait is bounded (error word + clean exit, never a trap).
#include <algorithm>

#include "common.cuh"
#include "gemv.cuh"
#include "mma.cuh"
#include "seqsum.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"
#include "units.cuh"

namespace nrc {
namespace {

constexpr int KNS = 32;      // tokens per CTA
constexpr int KTHR = 448;
constexpr int WREP = 8, WPROD = 12, WMMA = 13;
constexpr int EPI_WARPS = 8, REP_WARPS = 4;
constexpr int NMR = 4;       // row / token scale ring (repack -> epilogue)
constexpr int RMETA = 24;    // bytes per row in a scale slot: d, dmin (f32) + sc[8], m[8] (Q6_K: d + sc[16])

struct KqParams {
  const uint8_t* w[3];
  float* yseg[3];
  int rows[3];
  int ldseg[3];
  int tile_start[4];
  int nseg;
  int fmt, nsb, row_bytes;  // super-blocks per row
  const uint8_t* xq;        // canonical activation tiles [ntg][nsb][NBT][KNS x 32]
  const float* xd;          // [ntg][nsb][KNS]
  const int* xb;            // [ntg][nsb][KNS][8] sums of each 32-value chunk (Q4_K)
  int nt, ntg;
  int epi;
  float scale;
  float* resid;
  int resid_ld;
  float rs;
  unsigned* err;
  int rfull[3];  // rows of each matrix covered by its tensor map (a multiple of 8)
  int off_a, off_raw, off_tail, off_b, off_xd, off_xb, stage_bytes, off_meta, off_bar;
  CUtensorMap tmap[3];  // per matrix: dims {8 * row_bytes, rows / 8} (u8), box {BW, 16}
};

// Per format: MMAs (TMEM slots) per super-block, A tiles, B tiles, TMEM
// buffers, pipeline stages, the width of a tensor-map box (a 16-byte aligned
// window holding one super-block of a row: Q4_K super-blocks are 16-byte
// aligned, a Q6_K one starts at an even offset; both widths are an odd
// number of 16-byte units, so rows 8 apart land in different bank groups)
// and of a raw slot for rows copied by cp.async (up to 240 bytes for Q6_K).
template <int FMT> struct KqShape {
  static constexpr int NA = FMT == FMT_Q4K ? 8 : 16;   // MMAs = TMEM slots per super-block
  static constexpr int NAT = 8;                        // A tiles: the 8 chunks of 32 values
  static constexpr int NBT = FMT == FMT_Q4K ? 8 : 16;  // B tiles (Q6_K: each chunk's two masked halves)
  static constexpr int UPS = NA / 8;                   // TMEM units (8 slots, 256 columns) per super-block
  static constexpr int NST = FMT == FMT_Q4K ? 3 : 2;   // smem stages
  static constexpr int BW = FMT == FMT_Q4K ? Q4K_BYTES : 240;
  static constexpr int RAW = FMT == FMT_Q4K ? Q4K_BYTES : 240;
};

// Byte q in [0, 63] -> int8 q - 32, four lanes at once (no borrow between bytes).
NRC_DEV uint32_t q6_minus32(uint32_t q) { return ((q | 0x80808080u) - 0x20202020u) ^ 0x80808080u; }

template <int FMT>
__global__ void __launch_bounds__(KTHR, 1) k_mma_kq(const __grid_constant__ KqParams p) {
  using SH = KqShape<FMT>;
  constexpr int UPS = SH::UPS, NST = SH::NST, RAW = SH::RAW, BW = SH::BW;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* full = bars;                  // producer -> repack (32 lane arrivals + tx bytes)
  uint64_t* aready = full + NST;          // repack -> MMA (A tiles, scales written)
  uint64_t* empty = aready + NST;         // MMA commit -> producer (stage consumed)
  // TMEM holds two units of 8 slots (32 columns each); fill f (f = st * UPS + h,
  // unit f % 2) is the h-th unit of super-block st: Q4_K a super-block per
  // unit (double-buffered), Q6_K two units per super-block (the MMA fills one
  // unit while the epilogue drains the other).
  uint64_t* mdone = empty + NST;          // MMA commit -> epilogue (a unit's slots written), per unit
  uint64_t* tfree = mdone + 2;            // epilogue warps -> MMA (unit drained and preset), per unit
  uint64_t* mfree = tfree + 2;            // epilogue warps -> repack (scale slot read)
  uint64_t* mready = mfree + NMR;         // repack warps -> epilogue (scale slot written)
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x / p.ntg, tg = blockIdx.x % p.ntg;
  int sg = 0;
  while (sg + 1 < p.nseg && tile >= p.tile_start[sg + 1]) sg++;
  const int row0 = (tile - p.tile_start[sg]) * TC_M;
  const int nrows = min(TC_M, p.rows[sg] - row0);
  const uint8_t* wseg = p.w[sg];
  const uint8_t* wend = wseg + (size_t)p.rows[sg] * p.row_bytes;
  const int nsb = p.nsb;
  const int bpb = FMT == FMT_Q4K ? Q4K_BYTES : Q6K_BYTES;
  // Rows [row0, row0 + tma_rows) come through the tensor map: eight 2-D
  // copies per super-block, copy j bringing rows j, j + 8, ... of the tile
  // (consecutive 8-row groups are contiguous, 16-byte aligned spans, so any
  // row length works). The matrix's last rows % 8 rows are copied by cp.async.
  const int tma_rows = max(0, min(nrows, p.rfull[sg] - row0));
  const int tail0 = row0 + tma_rows;  // first row (absolute) of the cp.async tail

  if (tid == 0) {
    for (int s = 0; s < NST; s++) {
      mbar_init(&full[s], 32 + 1);
      mbar_init(&aready[s], REP_WARPS);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&mdone[b], 1);
      mbar_init(&tfree[b], EPI_WARPS);
    }
    for (int m = 0; m < NMR; m++) {
      mbar_init(&mfree[m], EPI_WARPS);
      mbar_init(&mready[m], REP_WARPS);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == WMMA) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_trigger();
  pdl_wait();  // activations and the residual stream come from the previous kernel
  const uint32_t tbase = tmem_base_sh;
  auto st_base = [&](int s) { return smem + (size_t)s * p.stage_bytes; };
  auto meta = [&](int m) { return smem + p.off_meta + (size_t)m * (TC_M * RMETA + KNS * 36); };
  auto fail = [&](unsigned bit) {
    if (!abort_flag) {
      abort_flag = 1;
      atomicOr(p.err, bit);
    }
  };

  if (warp == WPROD) {
    // ------------------------------------------------------------ producer
    // Per super-block: the eight tensor-map copies of the tile's rows (lane 0,
    // one request per 16 rows), the tail rows as 16-byte cp.async copies
    // (their ragged last bytes by plain loads), each lane's arrival on `full`
    // once its copies landed, and the super-block's activation tiles, token
    // scales and chunk sums as bulk copies. No multicast anywhere. A stage is
    // refilled as soon as its MMAs completed (the epilogue reads its scales
    // from the scale ring).
    const uint64_t pol = l2_evict_first();
    const uintptr_t wend_al = reinterpret_cast<uintptr_t>(wend) & ~(uintptr_t)15;
    const uint32_t b_bytes = (uint32_t)SH::NBT * KNS * 32;
    const uint32_t tx_bytes = (tma_rows ? 8u * 16u * BW : 0u) + b_bytes + KNS * 4 + (FMT == FMT_Q4K ? KNS * 32 : 0);
    constexpr int CH = RAW / 16;  // 16-byte chunks per tail slot
    const int ntail = nrows - tma_rows;
    int st = 0;
    for (; st < nsb; st++) {
      const int s = st % NST, u = st / NST;
      if (u >= 1) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait(&empty[s], (u - 1) & 1);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) fail(ERR_WAIT_EMPTY);
      }
      if (__any_sync(0xffffffffu, abort_flag)) break;
      const size_t sb_off = (size_t)st * bpb;
      if (ntail) {
        uint8_t* tail = st_base(s) + p.off_tail;
        if (lane == 0) {
          // Only the matrix's last row can end past its last 16-byte boundary.
          const int t = ntail - 1;
          const uintptr_t a = reinterpret_cast<uintptr_t>(wseg + (size_t)(tail0 + t) * p.row_bytes + sb_off);
          const uintptr_t lo = a & ~(uintptr_t)15;
          for (uintptr_t b = wend_al > a ? wend_al : a; b < a + bpb; b++)
            tail[t * RAW + (b - lo)] = *reinterpret_cast<const uint8_t*>(b);
        }
        for (int i = lane; i < ntail * CH; i += 32) {
          const int t = i / CH, c = i - t * CH;
          const uintptr_t a = reinterpret_cast<uintptr_t>(wseg + (size_t)(tail0 + t) * p.row_bytes + sb_off);
          const uintptr_t g = (a & ~(uintptr_t)15) + 16u * c;
          if (g < a + bpb && g < wend_al) cp_async16(tail + t * RAW + 16 * c, reinterpret_cast<const void*>(g), pol);
        }
      }
      __syncwarp();  // the plain byte stores before lane 0's release arrive
      if (lane == 0) {
        const size_t tix = (size_t)tg * nsb + st;
        mbar_arrive_expect_tx(&full[s], tx_bytes);
        if (tma_rows) {
          uint8_t* raw = st_base(s) + p.off_raw;
#pragma unroll 1
          for (int j = 0; j < 8; j++) {
            const int x = (int)(((size_t)j * p.row_bytes + sb_off) & ~(size_t)15);
            tma_load_2d(raw + j * (16 * BW), &p.tmap[sg], x, row0 / 8, &full[s], pol);
          }
        }
        bulk_g2s(st_base(s) + p.off_b, p.xq + tix * b_bytes, b_bytes, &full[s], 0ull);
        bulk_g2s(st_base(s) + p.off_xd, p.xd + tix * KNS, KNS * 4, &full[s], 0ull);
        if (FMT == FMT_Q4K) bulk_g2s(st_base(s) + p.off_xb, p.xb + tix * KNS * 8, KNS * 32, &full[s], 0ull);
      }
      cp_async_arrive_noinc(&full[s]);
    }
    cp_async_wait_all();
    if (lane == 0)
      for (int k = st - 1; k >= 0 && k >= st - NST; k--)
        if (!mbar_wait(&full[k % NST], (k / NST) & 1)) atomicOr(p.err, ERR_DRAIN);
  } else if (warp >= WREP && warp < WREP + REP_WARPS) {
    // -------------------------------------------------------------- repack
    // Weight row of this thread: r = 8g + j with, in every 8 consecutive lanes,
    // eight different 8-row groups g (their box rows sit in different bank
    // groups) and eight different j (their canonical-tile rows do too).
    const int rw = warp - WREP, ri = lane & 7, rq = lane >> 3;
    const int r = 8 * (ri + 8 * (rw & 1)) + ((ri + rq + 4 * (rw >> 1)) & 7);
    for (int st = 0; st < nsb; st++) {
      const int s = st % NST, u = st / NST, m = st % NMR;
      if (abort_flag || !mbar_wait(&full[s], u & 1) || (st >= NMR && !mbar_wait(&mfree[m], ((st / NMR) - 1) & 1))) {
        fail(ERR_WAIT_FULL);
        break;
      }
      uint8_t* a = st_base(s) + p.off_a;
      uint8_t* rm = meta(m) + r * RMETA;
      if (r < nrows) {
        const uint8_t* b;
        if (r < tma_rows) {
          // Copy j = r % 8, box row r / 8; the super-block at its offset in the box.
          const size_t off = (size_t)(r & 7) * p.row_bytes + (size_t)st * bpb;
          b = st_base(s) + p.off_raw + ((r & 7) * 16 + (r >> 3)) * BW + (off & 15);
        } else {
          const uintptr_t ga = reinterpret_cast<uintptr_t>(wseg + (size_t)(row0 + r) * p.row_bytes + (size_t)st * bpb);
          b = st_base(s) + p.off_tail + (r - tma_rows) * RAW + (ga & 15);
        }
        if (FMT == FMT_Q4K) {
          // d, dmin (f16), 12 scale bytes s[0..11] (q4k_scale_min, kquant.rs:83-92),
          // 128 bytes of nibbles. One 16-byte load; the 6-bit (sc, m) pairs are
          // unpacked four bytes at a time: sc[j] = s[j] & 63 and m[j] = s[j+4] & 63
          // for j < 4; sc[j] = (s[j+4] & 15) | (s[j-4] >> 6) << 4 and
          // m[j] = (s[j+4] >> 4) | (s[j] >> 6) << 4 for j >= 4.
          const uint4 hd = *reinterpret_cast<const uint4*>(b);
          float* fm = reinterpret_cast<float*>(rm);
          fm[0] = f16_to_f32(hd.x & 0xffffu);
          fm[1] = f16_to_f32(hd.x >> 16);
          const uint32_t s0 = hd.y, s4 = hd.z, s8 = hd.w;
          *reinterpret_cast<uint2*>(rm + 8) =
              make_uint2(s0 & 0x3F3F3F3Fu, (s8 & 0x0F0F0F0Fu) | (((s0 >> 6) & 0x03030303u) << 4));
          *reinterpret_cast<uint2*>(rm + 16) =
              make_uint2(s4 & 0x3F3F3F3Fu, ((s8 >> 4) & 0x0F0F0F0Fu) | (((s4 >> 6) & 0x03030303u) << 4));
          // 16-byte loads: the rows sit 144 bytes (9 x 16) apart, so eight threads'
          // loads never share a bank group.
          const uint4* qs = reinterpret_cast<const uint4*>(b + 16);
#pragma unroll
          for (int c = 0; c < 4; c++) {
            const uint4 q0 = qs[2 * c], q1 = qs[2 * c + 1];
            const uint32_t wv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            uint8_t* lo = a + (2 * c) * (TC_M * 32);
            uint8_t* hi = a + (2 * c + 1) * (TC_M * 32);
            *reinterpret_cast<uint4*>(lo + canon_off(r, 0)) =
                make_uint4(wv[0] & 0x0F0F0F0Fu, wv[1] & 0x0F0F0F0Fu, wv[2] & 0x0F0F0F0Fu, wv[3] & 0x0F0F0F0Fu);
            *reinterpret_cast<uint4*>(lo + canon_off(r, 1)) =
                make_uint4(wv[4] & 0x0F0F0F0Fu, wv[5] & 0x0F0F0F0Fu, wv[6] & 0x0F0F0F0Fu, wv[7] & 0x0F0F0F0Fu);
            *reinterpret_cast<uint4*>(hi + canon_off(r, 0)) = make_uint4(
                (wv[0] >> 4) & 0x0F0F0F0Fu, (wv[1] >> 4) & 0x0F0F0F0Fu, (wv[2] >> 4) & 0x0F0F0F0Fu, (wv[3] >> 4) & 0x0F0F0F0Fu);
            *reinterpret_cast<uint4*>(hi + canon_off(r, 1)) = make_uint4(
                (wv[4] >> 4) & 0x0F0F0F0Fu, (wv[5] >> 4) & 0x0F0F0F0Fu, (wv[6] >> 4) & 0x0F0F0F0Fu, (wv[7] >> 4) & 0x0F0F0F0Fu);
          }
        } else {
          // ql[128], qh[64], scales[16] (int8), d (f16): value v = q - 32 in natural
          // order (kquant.rs:112-142). The super-block sits at an even offset: whole
          // words are loaded and realigned by funnel shifts, four values per word.
          uint32_t tl[5];
          load_words_unaligned<5>(b + 192, tl);
          float* fm = reinterpret_cast<float*>(rm);
          fm[0] = f16_to_f32(tl[4] & 0xffffu);
          uint32_t* scw = reinterpret_cast<uint32_t*>(rm + 4);
#pragma unroll
          for (int k = 0; k < 4; k++) scw[k] = tl[k];
#pragma unroll
          for (int h = 0; h < 2; h++) {
            uint32_t ql[16], qh[8];
            load_words_unaligned<16>(b + 64 * h, ql);
            load_words_unaligned<8>(b + 128 + 32 * h, qh);
            // Values 128h + 32qd + l (l = 4k .. 4k+3): chunk 4h + qd, word k;
            // words 0-3 of each chunk, then words 4-7 (one 16-byte half each).
#pragma unroll
            for (int c = 0; c < 2; c++) {
              uint32_t o[4][4];
#pragma unroll
              for (int kk = 0; kk < 4; kk++) {
                const int k = 4 * c + kk;
                const uint32_t wl = ql[k], wl2 = ql[k + 8], wh = qh[k];
                o[0][kk] = q6_minus32((wl & 0x0F0F0F0Fu) | ((wh & 0x03030303u) << 4));
                o[1][kk] = q6_minus32((wl2 & 0x0F0F0F0Fu) | (((wh >> 2) & 0x03030303u) << 4));
                o[2][kk] = q6_minus32(((wl >> 4) & 0x0F0F0F0Fu) | (((wh >> 4) & 0x03030303u) << 4));
                o[3][kk] = q6_minus32(((wl2 >> 4) & 0x0F0F0F0Fu) | (((wh >> 6) & 0x03030303u) << 4));
              }
#pragma unroll
              for (int qd = 0; qd < 4; qd++)
                *reinterpret_cast<uint4*>(a + (4 * h + qd) * (TC_M * 32) + canon_off(r, c)) =
                    make_uint4(o[qd][0], o[qd][1], o[qd][2], o[qd][3]);
            }
          }
        }
      } else {
#pragma unroll 1
        for (int k = 0; k < SH::NAT; k++) {
          *reinterpret_cast<uint4*>(a + k * (TC_M * 32) + canon_off(r, 0)) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(a + k * (TC_M * 32) + canon_off(r, 1)) = make_uint4(0, 0, 0, 0);
        }
      }
      // The super-block's token scales (and Q4_K chunk sums), copied with the
      // stage, into the scale slot. A chunk sum s (|s| <= 4096) is kept as the
      // bytes lo = s & 255 (unsigned) and hi = s >> 8 (signed), s = lo + 256 hi,
      // so the epilogue forms sum_j m_j * s_j with four dp4a.
      if (r < KNS) {
        float* dxs = reinterpret_cast<float*>(meta(m) + TC_M * RMETA);
        dxs[r] = reinterpret_cast<const float*>(st_base(s) + p.off_xd)[r];
        if (FMT == FMT_Q4K) {
          const int4* xs = reinterpret_cast<const int4*>(st_base(s) + p.off_xb) + 2 * r;
          const int4 a0 = xs[0], a1 = xs[1];
          const int v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          uint32_t lo[2] = {0, 0}, hi[2] = {0, 0};
#pragma unroll
          for (int j = 0; j < 8; j++) {
            lo[j >> 2] |= (uint32_t)(v[j] & 255) << (8 * (j & 3));
            hi[j >> 2] |= (uint32_t)((v[j] >> 8) & 255) << (8 * (j & 3));
          }
          reinterpret_cast<uint4*>(dxs + KNS)[r] = make_uint4(lo[0], lo[1], hi[0], hi[1]);
        }
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&aready[s]);
        mbar_arrive(&mready[m]);
      }
    }
  } else if (warp == WMMA) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(KNS);
      int last = -1;  // last unit fill whose MMAs were issued
      bool bad = false;
      for (int st = 0; st < nsb && !abort_flag && !bad; st++) {
        const int s = st % NST, u = st / NST;
        if (!mbar_wait(&aready[s], u & 1)) {
          fail(ERR_WAIT_FULL);
          break;
        }
        const uint8_t* a = st_base(s) + p.off_a;
        const uint8_t* bt = st_base(s) + p.off_b;
#pragma unroll 1
        for (int h = 0; h < UPS; h++) {
          const int f = st * UPS + h, unit = f & 1;
          // The unit drained and preset by the epilogue (first use: preset only).
          if (!mbar_wait(&tfree[unit], (f >> 1) & 1)) {
            fail(ERR_WAIT_EMPTY);
            bad = true;
            break;
          }
          tc_fence_after();
          const uint32_t dbase = tbase + (uint32_t)(unit * 8 * KNS);
#pragma unroll 1
          for (int kk = 0; kk < 8; kk++) {
            const int k = 8 * h + kk;
            const int at = FMT == FMT_Q4K ? k : k / 2;  // Q6_K: group k = half (k % 2) of chunk k / 2
            const uint64_t ad = smem_desc(a + at * (TC_M * 32), 128, 256);
            const uint64_t bd = smem_desc(bt + k * (KNS * 32), 128, 256);
            tc_mma_i8(dbase + (uint32_t)(kk * KNS), ad, bd, idesc, 1u);  // onto the preset cell
          }
          tc_commit(&mdone[unit]);
          last = f;
        }
        if (!bad) tc_commit(&empty[s]);
      }
      // Never release TMEM with an MMA in flight: wait (bounded) for the last commit.
      if (last >= 0 && !mbar_wait(&mdone[last & 1], (last >> 1) & 1)) atomicOr(p.err, ERR_DRAIN);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // Every TMEM cell is preset to the bits of 1.5 * 2^23 before its MMA adds
    // the dot onto it, so a cell holds the float 1.5 * 2^23 + dot exactly
    // (|dot| < 2^17) and one subtraction recovers f32(dot). Every dot is an
    // integer below 2^17 in magnitude and every scale an integer below 2^7
    // (Q4_K: |dot| <= 32*15*128, sc <= 63; Q6_K: |dot| <= 16*32*128, |sc| <=
    // 128), so f32(sc) * f32(dot) is exact (< 2^24) and fma(f32(dot), f32(sc),
    // sum) rounds exactly like the reference's `sum += sc as f32 * dot as f32`;
    // two tokens per packed operation throughout.
    const int q = warp & 3, half = warp >> 2;
    const int r = q * 32 + lane;  // TMEM lane = weight row
    const int n0 = half * 16;     // this warp's 16 tokens
    const uint32_t lane_base = tbase + ((uint32_t)(q * 32) << 16);
    const float2 mneg = make_float2(-TC_MAGIC_F, -TC_MAGIC_F);
    auto preset_unit = [&](int unit) {
#pragma unroll
      for (int k = 0; k < 8; k++) tc_st16_fill(lane_base + (uint32_t)(unit * 8 * KNS + k * KNS + n0), TC_MAGIC_BITS);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tfree[unit]);
    };
    preset_unit(0);
    preset_unit(1);
    float2 acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = make_float2(0.0f, 0.0f);
    for (int st = 0; st < nsb && !abort_flag; st++) {
      const int m = st % NMR;
      // mready and each unit's mdone complete at most one phase ahead of this
      // warp: their next phases need this super-block's mfree / the unit's tfree.
      if (!mbar_wait(&mready[m], (st / NMR) & 1)) {
        fail(ERR_WAIT_FULL);
        break;
      }
      const uint8_t* rm = meta(m) + r * RMETA;
      const float* dxs = reinterpret_cast<const float*>(meta(m) + TC_M * RMETA);
      const uint4* lohi = reinterpret_cast<const uint4*>(dxs + KNS);
      // Row scales: Q4_K d, dmin, sc[8] (u8), m[8] (u8); Q6_K d, sc[16] (i8),
      // kept packed and widened per slot.
      float d, dmin = 0.0f;
      uint2 mw = make_uint2(0, 0);
      uint32_t sws[4];
      if (FMT == FMT_Q4K) {
        const float* fm = reinterpret_cast<const float*>(rm);
        d = fm[0];
        dmin = fm[1];
        const uint2 sw = *reinterpret_cast<const uint2*>(rm + 8);
        mw = *reinterpret_cast<const uint2*>(rm + 16);
        sws[0] = sw.x;
        sws[1] = sw.y;
      } else {
        d = reinterpret_cast<const float*>(rm)[0];
        const uint32_t* sw = reinterpret_cast<const uint32_t*>(rm + 4);  // 4-byte aligned
#pragma unroll
        for (int k = 0; k < 4; k++) sws[k] = sw[k];
      }
      auto scale_of = [&](int k) {
        const uint32_t b = (sws[k >> 2] >> (8 * (k & 3))) & 0xffu;
        return FMT == FMT_Q4K ? (float)b : (float)(int)(int8_t)b;
      };
      float2 sq[8];
#pragma unroll
      for (int i = 0; i < 8; i++) sq[i] = make_float2(0.0f, 0.0f);
      bool bad = false;
#pragma unroll
      for (int h = 0; h < UPS; h++) {
        const int f = st * UPS + h, unit = f & 1;
        if (!mbar_wait(&mdone[unit], (f >> 1) & 1)) {
          fail(ERR_WAIT_FULL);
          bad = true;
          break;
        }
        tc_fence_after();
        const uint32_t slot0 = lane_base + (uint32_t)(unit * 8 * KNS + n0);
        uint32_t va[32], vb[32];
        tc_ld16(slot0, va);
        tc_ld16(slot0 + (uint32_t)KNS, va + 16);
        tc_wait_ld_regs<32>(va);
        // Two slots per TMEM round trip, the next pair's loads in flight while
        // this pair is scaled; each slot's dots in slot order.
#pragma unroll
        for (int kk = 0; kk < 8; kk += 2) {
          const int k = 8 * h + kk;
          uint32_t* cur = ((kk >> 1) & 1) ? vb : va;
          uint32_t* nxt = ((kk >> 1) & 1) ? va : vb;
          if (kk + 2 < 8) {
            tc_ld16(slot0 + (uint32_t)((kk + 2) * KNS), nxt);
            tc_ld16(slot0 + (uint32_t)((kk + 3) * KNS), nxt + 16);
          }
          const float sc0 = scale_of(k), sc1 = scale_of(k + 1);
          const float2 s0 = make_float2(sc0, sc0), s1 = make_float2(sc1, sc1);
#pragma unroll
          for (int i = 0; i < 8; i++)
            sq[i] = __ffma2_rn(add2_rn(make_float2(__uint_as_float(cur[2 * i]), __uint_as_float(cur[2 * i + 1])), mneg),
                               s0, sq[i]);
#pragma unroll
          for (int i = 0; i < 8; i++)
            sq[i] = __ffma2_rn(
                add2_rn(make_float2(__uint_as_float(cur[16 + 2 * i]), __uint_as_float(cur[16 + 2 * i + 1])), mneg), s1,
                sq[i]);
          if (kk + 2 < 8) tc_wait_ld_regs<32>(nxt);
        }
        // Unit drained: preset its cells again and hand it back.
        preset_unit(unit);
      }
      if (bad) break;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const int n = n0 + 2 * i;
        const float2 dx2 = *reinterpret_cast<const float2*>(dxs + n);
        const float2 dd = mul2_rn(make_float2(d, d), dx2);  // feeds products only
        if (FMT == FMT_Q4K) {
          const uint4 l0 = lohi[n], l1 = lohi[n + 1];
          const int sm0 = (int)(__dp4a(mw.x, l0.x, 0u) + __dp4a(mw.y, l0.y, 0u)) +
                          256 * (__dp4a((int)mw.x, (int)l0.z, 0) + __dp4a((int)mw.y, (int)l0.w, 0));
          const int sm1 = (int)(__dp4a(mw.x, l1.x, 0u) + __dp4a(mw.y, l1.y, 0u)) +
                          256 * (__dp4a((int)mw.x, (int)l1.z, 0) + __dp4a((int)mw.y, (int)l1.w, 0));
          // |sm| <= 8 * 63 * 4096 < 2^22: exact through the magic constant.
          const float2 fsm = add2_rn(make_float2(__uint_as_float((uint32_t)sm0 + TC_MAGIC_BITS),
                                                 __uint_as_float((uint32_t)sm1 + TC_MAGIC_BITS)),
                                     mneg);
          const float2 dm = mul2_rn(make_float2(dmin, dmin), dx2);
          const float tx = __fsub_rn(__fmul_rn(dd.x, sq[i].x), __fmul_rn(dm.x, fsm.x));
          const float ty = __fsub_rn(__fmul_rn(dd.y, sq[i].y), __fmul_rn(dm.y, fsm.y));
          acc[i] = add2_rn(acc[i], make_float2(tx, ty));  // fed by subtractions
        } else {
          acc[i].x = __fadd_rn(acc[i].x, __fmul_rn(dd.x, sq[i].x));
          acc[i].y = __fadd_rn(acc[i].y, __fmul_rn(dd.y, sq[i].y));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&mfree[m]);
    }
    if (!abort_flag && r < nrows) {
      const int row = row0 + r;
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const int tok = tg * KNS + n0 + i;
        if (tok >= p.nt) break;
        float sv = (i & 1) ? acc[i >> 1].y : acc[i >> 1].x;
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
  if (warp == WMMA) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(512) : "memory");
  }
}

// Activations of the K-quant GEMM: one CTA (256 threads) per token slot:
// optional exact RMSNorm (the GEMV prologue's order), then quantize_q8k
// (kquant.rs:157-187) of every 256-value block, one warp per block, into the
// canonical tiles of 32-value chunks, the block scale and the chunk sums.
__global__ void __launch_bounds__(256) k_mma_kq_act(const MmaKqActArgs a) {
  pdl_wait();
  pdl_trigger();
  const int n = blockIdx.x;  // token slot (0 .. ntg*NS - 1)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nsb = a.K / 256;
  const int tg = n / a.NS, nn = n % a.NS;
  const int nbt = a.masked ? 16 : 8;  // tiles per super-block
  __shared__ SeqSumShared ssh;
  auto tile = [&](int sb, int c) { return a.xq + (((size_t)tg * nsb + sb) * nbt + c) * a.NS * 32; };
  if (n >= a.nt) {
    for (int i = tid; i < nsb * nbt; i += 256) {
      uint8_t* t = tile(i / nbt, i % nbt);
      *reinterpret_cast<uint4*>(t + canon_off(nn, 0)) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(t + canon_off(nn, 1)) = make_uint4(0, 0, 0, 0);
    }
    for (int i = tid; i < nsb * 8; i += 256) a.xb[(((size_t)tg * nsb + i / 8) * a.NS + nn) * 8 + i % 8] = 0;
    for (int sb = tid; sb < nsb; sb += 256) a.xd[((size_t)tg * nsb + sb) * a.NS + nn] = 0.0f;
    return;
  }
  extern __shared__ __align__(16) float xrow[];  // the token's K values
  const float* x = a.x + (size_t)n * a.x_ld;
  for (int i = tid; i < a.K; i += 256) xrow[i] = x[i];
  __syncthreads();
  float sc = 1.0f;
  if (a.norm_w) {
    // vec::rmsnorm (vec.rs:4-14): `ss += v * v` in index order (one chain, seqsum.cuh).
    const float ss = seq_sum_squares_group<256>(xrow, a.K, ssh, tid, [] { __syncthreads(); });
    sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)a.K), a.eps)));
  }
  for (int b = warp; b < nsb; b += 8) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      v[k] = xrow[b * 256 + lane * 8 + k];
      if (a.norm_w) v[k] = __fmul_rn(__fmul_rn(v[k], sc), a.norm_w[b * 256 + lane * 8 + k]);
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
    uint32_t pk[2] = {0u, 0u};
    int part = 0;
    float dval = 0.0f;
    if (amax != 0.0f) {
      const float iscale = __fdiv_rn(-128.0f, mx);
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const float z = __fmul_rn(iscale, v[k]);
        int q = z >= 0.0f ? rust_f2i(__fadd_rn(z, 0.5f)) : rust_f2i(__fsub_rn(z, 0.5f));
        q = q > 127 ? 127 : q;
        const int8_t q8 = (int8_t)(uint8_t)(q & 0xff);
        part += q8;
        pk[k / 4] |= ((uint32_t)(uint8_t)q8) << (8 * (k % 4));
      }
      dval = __fdiv_rn(1.0f, iscale);
    }
    // Lane holds values 8*lane .. +7 of the block: chunk lane / 4, bytes 8*(lane % 4).
    const int byte = 8 * (lane % 4), hf = byte / 16;
    if (a.masked) {
      // Two tiles per chunk, each keeping one 16-value half (the other half zero).
      *reinterpret_cast<uint2*>(tile(b, 2 * (lane / 4) + hf) + canon_off(nn, hf) + byte % 16) = make_uint2(pk[0], pk[1]);
      *reinterpret_cast<uint2*>(tile(b, 2 * (lane / 4) + 1 - hf) + canon_off(nn, hf) + byte % 16) = make_uint2(0u, 0u);
    } else {
      *reinterpret_cast<uint2*>(tile(b, lane / 4) + canon_off(nn, hf) + byte % 16) = make_uint2(pk[0], pk[1]);
    }
    int s4 = part + __shfl_down_sync(0xffffffffu, part, 1);
    s4 += __shfl_down_sync(0xffffffffu, s4, 2);
    if ((lane & 3) == 0) a.xb[(((size_t)tg * nsb + b) * a.NS + nn) * 8 + lane / 4] = s4;
    if (lane == 0) a.xd[((size_t)tg * nsb + b) * a.NS + nn] = dval;
  }
}

// Pre-quantized Q8_K activation blocks [nt][nsb] (292 bytes: d f32, 256 int8,
// 16 int16 bsums; kquant.rs:46-52) -> the canonical tiles, scales and chunk sums.
__global__ void k_mma_kq_pack(const uint8_t* __restrict__ x, int nt, int nsb, int NS, int ntg, int masked,
                              uint8_t* xq, float* xd, int* xb) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // (token slot, block, chunk)
  if (i >= NS * ntg * nsb * 8) return;
  const int c = i % 8, b = (i / 8) % nsb, n = i / (8 * nsb);
  const int tg = n / NS, nn = n % NS;
  const int nbt = masked ? 16 : 8;
  uint8_t* t = xq + (((size_t)tg * nsb + b) * nbt + (masked ? 2 * c : c)) * NS * 32;
  uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int pair = 0;
  float d = 0.0f;
  if (n < nt) {
    const uint8_t* s = x + ((size_t)n * nsb + b) * Q8K_BYTES;
#pragma unroll
    for (int k = 0; k < 8; k++)
      w[k] = (uint32_t)s[4 + 32 * c + 4 * k] | ((uint32_t)s[5 + 32 * c + 4 * k] << 8) |
             ((uint32_t)s[6 + 32 * c + 4 * k] << 16) | ((uint32_t)s[7 + 32 * c + 4 * k] << 24);
    const int16_t b0 = (int16_t)((uint32_t)s[260 + 4 * c] | ((uint32_t)s[261 + 4 * c] << 8));
    const int16_t b1 = (int16_t)((uint32_t)s[262 + 4 * c] | ((uint32_t)s[263 + 4 * c] << 8));
    pair = (int)b0 + (int)b1;
    uint32_t db = (uint32_t)s[0] | ((uint32_t)s[1] << 8) | ((uint32_t)s[2] << 16) | ((uint32_t)s[3] << 24);
    d = __uint_as_float(db);
  }
  if (masked) {
    uint8_t* t1 = t + NS * 32;  // the chunk's second tile: values 16..31
    *reinterpret_cast<uint4*>(t + canon_off(nn, 0)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(t + canon_off(nn, 1)) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(t1 + canon_off(nn, 0)) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(t1 + canon_off(nn, 1)) = make_uint4(w[4], w[5], w[6], w[7]);
  } else {
    *reinterpret_cast<uint4*>(t + canon_off(nn, 0)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(t + canon_off(nn, 1)) = make_uint4(w[4], w[5], w[6], w[7]);
  }
  xb[(((size_t)tg * nsb + b) * NS + nn) * 8 + c] = pair;
  if (c == 0) xd[((size_t)tg * nsb + b) * NS + nn] = d;
}

cudaError_t launch_kq(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, void** args) {
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

int mma_kq_ns(int fmt) {
  (void)fmt;
  return KNS;
}

cudaError_t mma_kq_act_run(const MmaKqActArgs& a, cudaStream_t s, bool pdl) {
  if (a.K % 256 || a.NS != KNS || a.nt > a.NS * a.ntg) return cudaErrorInvalidValue;
  if ((size_t)a.K * 4 > 64 * 1024) return cudaErrorInvalidValue;
  if (cudaError_t e = ensure_smem_attr((const void*)k_mma_kq_act, 64 * 1024)) return e;
  MmaKqActArgs aa = a;
  void* args[] = {&aa};
  return launch_kq((const void*)k_mma_kq_act, dim3(a.NS * a.ntg), dim3(256), (size_t)a.K * 4, s, pdl, args);
}

cudaError_t mma_kq_pack_run(const uint8_t* x, int nt, int K, int NS, int ntg, int masked, uint8_t* xq, float* xd,
                            int* xb, cudaStream_t s) {
  if (K % 256 || nt > NS * ntg || NS != KNS) return cudaErrorInvalidValue;
  const int nsb = K / 256;
  const int total = NS * ntg * nsb * 8;
  k_mma_kq_pack<<<(total + 255) / 256, 256, 0, s>>>(x, nt, nsb, NS, ntg, masked, xq, xd, xb);
  return cudaGetLastError();
}

cudaError_t mma_kq_run(const MmaKqArgs& a, cudaStream_t s, bool pdl) {
  if ((a.fmt != FMT_Q4K && a.fmt != FMT_Q6K) || a.K % 256 || a.NS != KNS || a.nseg < 1 || a.nseg > 3)
    return cudaErrorInvalidValue;
  KqParams p{};
  int tiles = 0;
  for (int i = 0; i < a.nseg; i++) {
    // 16-byte aligned matrices: a row's aligned superset never starts before the matrix.
    if (reinterpret_cast<uintptr_t>(a.seg[i].w) & 15) return cudaErrorInvalidValue;
    p.w[i] = static_cast<const uint8_t*>(a.seg[i].w);
    p.yseg[i] = a.seg[i].y;
    p.rows[i] = a.seg[i].rows;
    p.ldseg[i] = a.seg[i].ld > 0 ? a.seg[i].ld : a.seg[i].rows;
    p.tile_start[i] = tiles;
    tiles += (a.seg[i].rows + TC_M - 1) / TC_M;
  }
  p.tile_start[a.nseg] = tiles;
  p.nseg = a.nseg;
  p.fmt = a.fmt;
  p.nsb = a.K / 256;
  p.row_bytes = p.nsb * (a.fmt == FMT_Q4K ? Q4K_BYTES : Q6K_BYTES);
  p.xq = a.xq;
  p.xd = a.xd;
  p.xb = a.xb;
  p.nt = a.nt;
  p.ntg = a.ntg;
  p.epi = a.epi;
  p.scale = a.scale;
  p.resid = a.resid;
  p.resid_ld = a.resid_ld;
  p.rs = a.rs;
  p.err = a.err;
  const bool q4 = a.fmt == FMT_Q4K;
  for (int i = 0; i < a.nseg; i++) {
    // 8-row groups of the matrix as rows of a 2-D u8 tensor (stride 8 * row_bytes,
    // a multiple of 16 for both formats); a box is one super-block window of 16 groups.
    p.rfull[i] = a.seg[i].rows / 8 * 8;
    if (p.rfull[i] == 0) continue;
    auto enc = tensor_map_encoder();
    if (!enc) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)8 * p.row_bytes, (cuuint64_t)(a.seg[i].rows / 8)};
    const cuuint64_t strides[1] = {(cuuint64_t)8 * p.row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(q4 ? KqShape<FMT_Q4K>::BW : KqShape<FMT_Q6K>::BW), 16};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&p.tmap[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(a.seg[i].w), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  const int nst = q4 ? KqShape<FMT_Q4K>::NST : KqShape<FMT_Q6K>::NST;
  const int nbt = q4 ? KqShape<FMT_Q4K>::NBT : KqShape<FMT_Q6K>::NBT;
  // Stage: A tiles (1024-aligned) | raw rows | B tiles | token scales | chunk
  // sums. Then the scale ring and the barriers.
  const int raw_slot = q4 ? KqShape<FMT_Q4K>::RAW : KqShape<FMT_Q6K>::RAW;
  const int bw = q4 ? KqShape<FMT_Q4K>::BW : KqShape<FMT_Q6K>::BW;
  size_t o = 0;
  p.off_a = 0;
  o += (size_t)8 * TC_M * 32;
  p.off_raw = (int)o;  // 128-byte aligned, as every box (16 x bw bytes, bw * 16 % 128 == 0)
  o += (size_t)8 * 16 * bw;
  p.off_tail = (int)o;
  o += (size_t)8 * raw_slot;
  o = (o + 127) & ~(size_t)127;
  p.off_b = (int)o;
  o += (size_t)nbt * KNS * 32;
  p.off_xd = (int)o;
  o += (size_t)KNS * 4;
  p.off_xb = (int)o;
  o += (size_t)KNS * 32;
  o = (o + 1023) & ~(size_t)1023;
  p.stage_bytes = (int)o;
  p.off_meta = (int)(o * nst);
  const size_t meta_bytes = (size_t)NMR * (TC_M * RMETA + KNS * 36);
  p.off_bar = (int)((p.off_meta + meta_bytes + 15) & ~(size_t)15);
  const size_t smem = p.off_bar + (size_t)(3 * nst + 4 + 2 * NMR) * 8;
  const void* fn = q4 ? (const void*)k_mma_kq<FMT_Q4K> : (const void*)k_mma_kq<FMT_Q6K>;
  if (smem > 225 * 1024) return cudaErrorInvalidValue;
  if (cudaError_t e = ensure_smem_attr(fn, 225 * 1024)) return e;
  if (tiles == 0) return cudaSuccess;
  void* args[] = {&p};
  return launch_kq(fn, dim3(tiles * a.ntg), dim3(KTHR), smem, s, pdl, args);
}

}  // namespace nrc
