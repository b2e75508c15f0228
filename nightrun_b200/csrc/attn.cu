// Position-dependent kernels of the forward pass:
//  * rope_append: Qwen3 per-head q/k RMSNorm (vec.rs:17-27), RoPE (rope.rs:49-65,
//    from host-built cos/sin tables) and the f16 KV-cache append
//    (crates/nr-model/src/infer.rs:533-551, 639-659);
//  * attention: GQA attention over the f16 cache (infer.rs:553-572, 661-685);
//  * embed: token-embedding row dequantization (infer.rs:37-56, 516-521);
//  * step_finish: position advance and greedy-token decode.
// Every reduction keeps the reference's sequential order (index order for
// sums of squares and softmax sums, position order for the V accumulation),
// so results are bit-identical to the scalar reference, and every per-token
// result depends only on that token's position: batched prefill and
// token-by-token decode agree bit for bit.
#include <cuda_fp16.h>

#include "common.cuh"
#include "expf_cr.cuh"
#include "ops.cuh"
#include "seqsum.cuh"

namespace nrc {
namespace {

constexpr int ATT_THREADS = 128;  // >= head_dim: one V output chain per thread
// V rows staged per pass: 128 for single-token decode (few CTAs, deep
// staging), 32 when many tokens run (more CTAs resident per SM).
constexpr int ATT_VCH_DECODE = 128, ATT_VCH_MANY = 32;

NRC_DEV float h2f(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)bits)); }  // exact

// One warp: a head vector src[hd] -> optional per-head RMSNorm
// (rmsnorm_inplace, vec.rs:17-27: ss in index order, x *= scale * w) -> RoPE
// at the position whose cos/sin rows are ct/st (rope.rs:49-65: Adjacent pairs
// (2i, 2i+1) or Neox halves (i, i + hd/2)). Lane holds elements lane + 32 i.
// hb is hd floats of shared scratch for the warp.
NRC_DEV void warp_rope_head(const float* src, const float* nw, float eps, const float* ct, const float* st,
                            int style, int hd, float* hb, int lane, float* outv) {
  const int per = hd / 32, half = hd / 2;
  float vals[4];
#pragma unroll
  for (int i = 0; i < 4; i++)
    if (i < per) {
      vals[i] = src[lane + 32 * i];
      hb[lane + 32 * i] = vals[i];
    }
  __syncwarp();
  if (nw) {
    float scale = 0.0f;
    if (lane == 0) {
      float ss = 0.0f;
      for (int i = 0; i < hd; i++) ss = __fadd_rn(ss, __fmul_rn(hb[i], hb[i]));
      scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), eps)));
    }
    scale = __shfl_sync(0xffffffffu, scale, 0);
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (i < per) vals[i] = __fmul_rn(vals[i], __fmul_rn(scale, nw[lane + 32 * i]));
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (i < per) hb[lane + 32 * i] = vals[i];
    __syncwarp();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    if (i < per) {
      const int e = lane + 32 * i;
      int pi, ia, ib;
      if (style == 0) {
        pi = e / 2;
        ia = 2 * pi;
        ib = ia + 1;
      } else {
        pi = e % half;
        ia = pi;
        ib = pi + half;
      }
      const float c = ct[pi], sn = st[pi];
      const float av = hb[ia], bv = hb[ib];
      // head[ia] = a*cos - b*sin; head[ib] = a*sin + b*cos
      outv[i] = (e == ia) ? __fsub_rn(__fmul_rn(av, c), __fmul_rn(bv, sn)) : __fadd_rn(__fmul_rn(av, sn), __fmul_rn(bv, c));
    }
  }
  __syncwarp();  // hb is free again
}

// Prefill (nt tokens): one warp per (token, head).
__global__ void k_rope_append(const RopeArgs a) {
  pdl_wait();
  pdl_trigger();
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x & 31;
  const int nh = a.n_heads + a.n_kv_heads;
  const int hd = a.head_dim, half = hd / 2;
  const int att_dim = a.n_heads * hd, kv_dim = a.n_kv_heads * hd;
  const int item = blockIdx.x * warps + threadIdx.x / 32;  // (token, head)
  if (item >= a.nt * nh) return;
  const int tok = item / nh, h = item % nh;
  const uint32_t pos = a.pos_tok ? a.pos_tok[tok] : a.pos_dev[0] + (uint32_t)tok;
  const size_t cache_off = a.pos_tok ? (size_t)a.seq_tok[tok] * a.seq_stride : 0;
  const bool is_q = h < a.n_heads;
  const int kvh = h - a.n_heads;
  __shared__ float buf[8][128];
  const int per = hd / 32;
  float outv[4];
  const float* src = is_q ? a.q + (size_t)tok * att_dim + h * hd : a.k + (size_t)tok * kv_dim + kvh * hd;
  warp_rope_head(src, is_q ? a.q_norm : a.k_norm, a.eps, a.cos_tab + (size_t)pos * half,
                 a.sin_tab + (size_t)pos * half, a.style, hd, buf[threadIdx.x / 32], lane, outv);
  if (is_q) {
    float* dst = a.q + (size_t)tok * att_dim + h * hd;
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (i < per) dst[lane + 32 * i] = outv[i];
  } else {
    uint16_t* kd = a.kcache + cache_off + (size_t)pos * kv_dim + kvh * hd;
    uint16_t* vd = a.vcache + cache_off + (size_t)pos * kv_dim + kvh * hd;
    const float* vs = a.v + (size_t)tok * kv_dim + kvh * hd;
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (i < per) {
        kd[lane + 32 * i] = f32_to_f16(outv[i]);
        vd[lane + 32 * i] = f32_to_f16(vs[lane + 32 * i]);
      }
  }
}

// cp.async 16-byte global -> shared copies (L2 only), grouped by commit.
NRC_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
NRC_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
NRC_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One CTA per (query head, token) over every position 0..=pos
// (infer.rs:553-572 decode, 661-685 prefill):
//  0. decode only (fused): warp 0 normalizes and rotates this query head,
//     warp 1 the new k row, warp 2 converts the new v row of the head's KV
//     group to f16; the first query head of the group stores both in the
//     cache. Every head of the group reads the new position from shared
//     memory (the cache row is being written concurrently);
//  1. scores: one thread per position, the whole K row loaded before the
//     dot_f16 chain in the scalar order (kernels.rs:146-157), times the scale;
//  2. softmax (vec.rs:30-41): max, expf, the sum in position order (one
//     chain), then p_t = e_t * (1 / sum);
//  3. out[d] = sum over positions, in position order, of p_t * v_t[d]
//     (axpy_f16, kernels.rs:160-169): one thread per d, V rows staged in
//     shared memory by cp.async, double-buffered, the first chunk issued
//     before the scores so its latency overlaps them.
// f16 -> f32 uses the hardware conversion, exact for every f16 value.
// FAST (tolerance mode): the same structure with fused multiply-adds in the
// dot products, the softmax sum as a CTA tree and the V sums split over
// ATT_THREADS / head_dim position groups combined in a fixed order.
// HD: head_dim as a constant (32, 64 or 128), so a thread's K row lives in
// HD / 8 registers of 16 bytes; the register bound keeps three (HD 128) or
// four CTAs resident per SM when many (token, head) CTAs run.
template <bool FAST, int HD>
__global__ void __launch_bounds__(ATT_THREADS, HD >= 128 ? 3 : 4) k_attention(const AttnArgs a) {
  const bool fused = a.fused != 0;
  // Single-token decode with the KV append fused: the position and the cached
  // rows [0, pos) were final before the previous attention (or embedding)
  // kernel returned from its own dependency wait, and every kernel between
  // them lets its dependents start only once it is running, so they are read
  // before this kernel's wait, overlapping the QKV launch's tail. Everything
  // the previous kernel writes (q, k, v; rows appended by a separate kernel)
  // is read after it.
  if (!fused) pdl_wait();
  const int h = blockIdx.x, tok = blockIdx.y;
  const int hd = a.head_dim, half = hd / 2;
  const int gqa = a.n_heads / a.n_kv_heads;
  const int g = h / gqa;
  const int att_dim = a.n_heads * hd, kv_dim = a.n_kv_heads * hd;
  const uint32_t pos = a.pos_tok ? a.pos_tok[tok] : a.pos_dev[0] + (uint32_t)tok;
  const int npos = (int)pos + 1;
  const size_t cache_off = a.pos_tok ? (size_t)a.seq_tok[tok] * a.seq_stride : 0;
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                                               // [hd]
  float* hbuf = qs + hd;                                        // [3][hd] rope scratch (fused)
  uint16_t* knew = reinterpret_cast<uint16_t*>(hbuf + 3 * hd);  // [hd] new k (f16, fused)
  uint16_t* vnew = knew + hd;                                   // [hd] new v (f16, fused)
  float* sc = reinterpret_cast<float*>(vnew + hd);              // [ctx] scores, then probabilities
  const int sc_len = ((a.ctx + 3) & ~3) > ATT_THREADS ? ((a.ctx + 3) & ~3) : ATT_THREADS;
  uint16_t* vs = reinterpret_cast<uint16_t*>(sc + sc_len);      // [2][vch][hd]
  const int vch = a.nt > 1 ? ATT_VCH_MANY : ATT_VCH_DECODE;
  __shared__ float red[ATT_THREADS / 32];
  __shared__ SeqSumShared ssh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint16_t* kbase = a.kcache + cache_off + (size_t)g * hd;
  uint16_t* vbase = a.vcache + cache_off + (size_t)g * hd;
  const int cpr = hd / 8;  // 16-byte chunks per K/V row
  // Rows [0, cached) come from the cache; with the append fused, row `pos`
  // comes from shared memory.
  const int cached = fused ? (int)pos : npos;
  auto stage_v = [&](int t0, int buf) {
    const int tn = min(vch, cached - t0);
    uint16_t* dst = vs + (size_t)buf * vch * hd;
    for (int i = tid; i < tn * cpr; i += ATT_THREADS) {
      const int r = i / cpr, c = i - r * cpr;
      cp_async16(dst + r * hd + c * 8, vbase + (size_t)(t0 + r) * kv_dim + c * 8);
    }
    cp_async_commit();
  };
  stage_v(0, 0);
  // The K row of this thread's first position, loaded now so its latency
  // overlaps the RoPE work below.
  uint4 k0[HD / 8];
  if (tid < cached) {
    const uint4* kr = reinterpret_cast<const uint4*>(kbase + (size_t)tid * kv_dim);
#pragma unroll
    for (int c = 0; c < HD / 8; c++) k0[c] = kr[c];
  }
  if (fused) pdl_wait();
  pdl_trigger();
  if (fused) {
    const float* ct = a.cos_tab + (size_t)pos * half;
    const float* st = a.sin_tab + (size_t)pos * half;
    const int per = hd / 32;
    float outv[4];
    if (warp == 0) {
      warp_rope_head(a.q + (size_t)h * hd, a.q_norm, a.eps, ct, st, a.style, hd, hbuf, lane, outv);
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (i < per) qs[lane + 32 * i] = outv[i];
    } else if (warp == 1) {
      warp_rope_head(a.k + (size_t)g * hd, a.k_norm, a.eps, ct, st, a.style, hd, hbuf + hd, lane, outv);
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (i < per) {
          const uint16_t kb = f32_to_f16(outv[i]);
          knew[lane + 32 * i] = kb;
          if (h % gqa == 0) kbase[(size_t)pos * kv_dim + lane + 32 * i] = kb;
        }
    } else if (warp == 2) {
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (i < per) {
          const uint16_t vb = f32_to_f16(a.v[(size_t)g * hd + lane + 32 * i]);
          vnew[lane + 32 * i] = vb;
          if (h % gqa == 0) vbase[(size_t)pos * kv_dim + lane + 32 * i] = vb;
        }
    }
  } else {
    for (int i = tid; i < hd; i += ATT_THREADS) qs[i] = a.q[(size_t)tok * att_dim + (size_t)h * hd + i];
  }
  __syncthreads();

  float mloc = -INFINITY;
  for (int t = tid; t < npos; t += ATT_THREADS) {
    float s = 0.0f;
    if (t == tid && t < cached) {
#pragma unroll
      for (int c = 0; c < HD / 8; c++) {
        {
          const uint32_t w[4] = {k0[c].x, k0[c].y, k0[c].z, k0[c].w};
          const float* qd = qs + c * 8;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            if (FAST) {
              s = fmaf(h2f(w[j] & 0xffffu), qd[2 * j], s);
              s = fmaf(h2f(w[j] >> 16), qd[2 * j + 1], s);
            } else {
              s = __fadd_rn(s, __fmul_rn(h2f(w[j] & 0xffffu), qd[2 * j]));
              s = __fadd_rn(s, __fmul_rn(h2f(w[j] >> 16), qd[2 * j + 1]));
            }
          }
        }
      }
    } else if (t < cached) {
      const uint4* kr = reinterpret_cast<const uint4*>(kbase + (size_t)t * kv_dim);
      for (int c0 = 0; c0 < cpr; c0 += 8) {
        uint4 k8[8];
#pragma unroll
        for (int c = 0; c < 8; c++)
          if (c0 + c < cpr) k8[c] = kr[c0 + c];
#pragma unroll
        for (int c = 0; c < 8; c++) {
          if (c0 + c < cpr) {
            const uint32_t w[4] = {k8[c].x, k8[c].y, k8[c].z, k8[c].w};
            const float* qd = qs + (c0 + c) * 8;
#pragma unroll
            for (int j = 0; j < 4; j++) {
              if (FAST) {
                s = fmaf(h2f(w[j] & 0xffffu), qd[2 * j], s);
                s = fmaf(h2f(w[j] >> 16), qd[2 * j + 1], s);
              } else {
                s = __fadd_rn(s, __fmul_rn(h2f(w[j] & 0xffffu), qd[2 * j]));
                s = __fadd_rn(s, __fmul_rn(h2f(w[j] >> 16), qd[2 * j + 1]));
              }
            }
          }
        }
      }
    } else {
      for (int d = 0; d < hd; d++) s = __fadd_rn(s, __fmul_rn(h2f(knew[d]), qs[d]));
    }
    s = __fmul_rn(s, a.scale);
    sc[t] = s;
    mloc = fmaxf(mloc, s);
  }
  mloc = warp_max(mloc);
  if (lane == 0) red[warp] = mloc;
  __syncthreads();
  float mx = red[0];
#pragma unroll
  for (int w = 1; w < ATT_THREADS / 32; w++) mx = fmaxf(mx, red[w]);
  for (int t = tid; t < npos; t += ATT_THREADS) sc[t] = expf_cr(__fsub_rn(sc[t], mx));
  __syncthreads();
  // The sum in position order (vec.rs:35-36), one chain (seqsum.cuh); a tree in the tolerance mode.
  const float sum = FAST ? tree_sum_group<ATT_THREADS>(npos, [&](int t) { return sc[t]; }, ssh, tid, [] { __syncthreads(); })
                         : seq_sum_group<ATT_THREADS>(npos, [&](int t) { return sc[t]; }, ssh, tid, [] { __syncthreads(); });
  const float inv = __fdiv_rn(1.0f, sum);
  for (int t = tid; t < npos; t += ATT_THREADS) sc[t] = __fmul_rn(sc[t], inv);

  float acc = 0.0f;
  // Exact: thread d chains every position. FAST: H position groups per dim.
  const int H = FAST ? ATT_THREADS / hd : 1;
  const int d = FAST ? tid % hd : tid, grp = FAST ? tid / hd : 0;
  int buf = 0;
  for (int t0 = 0; t0 < npos; t0 += vch, buf ^= 1) {
    const int tn = min(vch, npos - t0);
    if (t0 + vch < cached) {
      stage_v(t0 + vch, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    uint16_t* vb = vs + (size_t)buf * vch * hd;
    if (fused && (int)pos < t0 + tn)
      for (int i = tid; i < hd; i += ATT_THREADS) vb[((int)pos - t0) * hd + i] = vnew[i];
    __syncthreads();
    if (FAST) {
      const uint16_t* vr = vb + d;
      const float* p = sc + t0;
#pragma unroll 4
      for (int t = grp; t < tn; t += H) acc = fmaf(p[t], h2f(vr[(size_t)t * hd]), acc);
    } else if (d < hd) {
      const uint16_t* vr = vb + d;
      const float* p = sc + t0;
      acc = seq_sum_serial(tn, [&](int t) { return __fmul_rn(p[t], h2f(vr[(size_t)t * hd])); }, acc);
    }
    __syncthreads();  // the buffer is restaged two chunks later
  }
  if (FAST) {
    // Combine the position groups in a fixed order (the scores buffer is free now).
    sc[tid] = acc;
    __syncthreads();
    if (tid < hd) {
      float o = 0.0f;
      for (int g2 = 0; g2 < H; g2++) o += sc[g2 * hd + tid];
      a.out[(size_t)tok * att_dim + (size_t)h * hd + tid] = o;
      if (a.xq_out) warp_quant_q8_block(o, lane, a.xq_out + (size_t)((h * hd + tid) >> 5) * Q8_0_BYTES);
    }
    return;
  }
  if (d < hd) {
    a.out[(size_t)tok * att_dim + (size_t)h * hd + d] = acc;
    // hd is a multiple of 32: whole warps, one 32-value block each.
    if (a.xq_out) warp_quant_q8_block(acc, lane, a.xq_out + (size_t)((h * hd + d) >> 5) * Q8_0_BYTES);
  }
}

// Multi-token attention (prefill chunks, batched sequences; never fused with
// the KV append): one CTA per (KV head, token) serving the query heads of its
// GQA group, so each K and V row is read once per group instead of once per
// head. Per head the arithmetic is k_attention<false>'s exactly: the dot in
// dimension order, the scale, the max, expf, the sum in position order, the
// reciprocal, and each output dimension chained over positions in order.
// Threads: gqa x HD (thread = (head, dim) in the V phase, = position in the
// score phase).
constexpr int ATT_GROUP_MAX = 8;  // query heads per KV head served by one CTA
constexpr int ATT_VCH_GROUP = 64;

template <int HD>
__global__ void __launch_bounds__(1024) k_attention_group(const AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int g = blockIdx.x, tok = blockIdx.y;
  const int gqa = a.n_heads / a.n_kv_heads;
  const int nth = gqa * HD;
  const int att_dim = a.n_heads * HD, kv_dim = a.n_kv_heads * HD;
  const uint32_t pos = a.pos_tok ? a.pos_tok[tok] : a.pos_dev[0] + (uint32_t)tok;
  const int npos = (int)pos + 1;
  const size_t cache_off = a.pos_tok ? (size_t)a.seq_tok[tok] * a.seq_stride : 0;
  const int sc_len = (a.ctx + 3) & ~3;
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                                                   // [gqa][HD]
  float* sc = qs + gqa * HD;                                        // [gqa][sc_len] scores, then probabilities
  uint16_t* vs = reinterpret_cast<uint16_t*>(sc + gqa * sc_len);   // [2][ATT_VCH_GROUP][HD]
  __shared__ float red[32][ATT_GROUP_MAX];
  __shared__ float hval[ATT_GROUP_MAX];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarp = nth >> 5;
  const uint16_t* kbase = a.kcache + cache_off + (size_t)g * HD;
  const uint16_t* vbase = a.vcache + cache_off + (size_t)g * HD;
  constexpr int CPR = HD / 8;  // 16-byte chunks per K/V row
  auto stage_v = [&](int t0, int buf) {
    const int tn = min(ATT_VCH_GROUP, npos - t0);
    uint16_t* dst = vs + (size_t)buf * ATT_VCH_GROUP * HD;
    for (int i = tid; i < tn * CPR; i += nth) {
      const int r = i / CPR, c = i - r * CPR;
      cp_async16(dst + r * HD + c * 8, vbase + (size_t)(t0 + r) * kv_dim + c * 8);
    }
    cp_async_commit();
  };
  stage_v(0, 0);
  for (int i = tid; i < gqa * HD; i += nth) qs[i] = a.q[(size_t)tok * att_dim + (size_t)g * gqa * HD + i];
  __syncthreads();

  // Scores: one position per thread, its K row loaded once for every head.
  float mloc[ATT_GROUP_MAX];
#pragma unroll
  for (int hh = 0; hh < ATT_GROUP_MAX; hh++) mloc[hh] = -INFINITY;
  for (int t = tid; t < npos; t += nth) {
    const uint4* kr = reinterpret_cast<const uint4*>(kbase + (size_t)t * kv_dim);
    uint4 kk[CPR];
#pragma unroll
    for (int c = 0; c < CPR; c++) kk[c] = kr[c];
    float s[ATT_GROUP_MAX];
#pragma unroll
    for (int hh = 0; hh < ATT_GROUP_MAX; hh++) s[hh] = 0.0f;
#pragma unroll
    for (int c = 0; c < CPR; c++) {
      const uint32_t w[4] = {kk[c].x, kk[c].y, kk[c].z, kk[c].w};
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const float kv = h2f((w[e >> 1] >> (16 * (e & 1))) & 0xffffu);
#pragma unroll
        for (int hh = 0; hh < ATT_GROUP_MAX; hh++)
          if (hh < gqa) s[hh] = __fadd_rn(s[hh], __fmul_rn(kv, qs[hh * HD + c * 8 + e]));
      }
    }
#pragma unroll
    for (int hh = 0; hh < ATT_GROUP_MAX; hh++)
      if (hh < gqa) {
        const float v = __fmul_rn(s[hh], a.scale);
        sc[hh * sc_len + t] = v;
        mloc[hh] = fmaxf(mloc[hh], v);
      }
  }
#pragma unroll
  for (int hh = 0; hh < ATT_GROUP_MAX; hh++)
    if (hh < gqa) {
      const float m = warp_max(mloc[hh]);
      if (lane == 0) red[warp][hh] = m;
    }
  __syncthreads();
  if (tid < gqa) {
    float mx = red[0][tid];
    for (int w = 1; w < nwarp; w++) mx = fmaxf(mx, red[w][tid]);
    hval[tid] = mx;
  }
  __syncthreads();
  for (int i = tid; i < gqa * npos; i += nth) {
    const int hh = i / npos, t = i - hh * npos;
    sc[hh * sc_len + t] = expf_cr(__fsub_rn(sc[hh * sc_len + t], hval[hh]));
  }
  __syncthreads();
  // Each head's sum in position order (vec.rs:35-36), one chain per head,
  // the heads' chains on different warps.
  if (lane == 0 && warp < gqa) {
    const float* p = sc + warp * sc_len;
    hval[warp] = __fdiv_rn(1.0f, seq_sum_serial(npos, [&](int t) { return p[t]; }));
  }
  __syncthreads();
  for (int i = tid; i < gqa * npos; i += nth) {
    const int hh = i / npos, t = i - hh * npos;
    sc[hh * sc_len + t] = __fmul_rn(sc[hh * sc_len + t], hval[hh]);
  }

  const int hh = tid / HD, d = tid - hh * HD;
  const float* ph = sc + hh * sc_len;
  float acc = 0.0f;
  int buf = 0;
  for (int t0 = 0; t0 < npos; t0 += ATT_VCH_GROUP, buf ^= 1) {
    const int tn = min(ATT_VCH_GROUP, npos - t0);
    if (t0 + ATT_VCH_GROUP < npos) {
      stage_v(t0 + ATT_VCH_GROUP, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // the chunk (and, the first time, the probabilities) visible to all
    const uint16_t* vr = vs + (size_t)buf * ATT_VCH_GROUP * HD + d;
    const float* p = ph + t0;
    acc = seq_sum_serial(tn, [&](int t) { return __fmul_rn(p[t], h2f(vr[(size_t)t * HD])); }, acc);
    __syncthreads();  // the buffer is restaged two chunks later
  }
  a.out[(size_t)tok * att_dim + (size_t)(g * gqa + hh) * HD + d] = acc;
}

__global__ void k_embed(const EmbedArgs a) {
  pdl_wait();
  pdl_trigger();
  const int tok = blockIdx.y;
  const uint32_t id = a.tok_dev[tok];
  if (blockIdx.x == 0 && threadIdx.x == 0 && tok == 0 && a.argmax_key) *a.argmax_key = 0ull;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.dim; i += gridDim.x * blockDim.x) {
    float v;
    if (a.fmt == FMT_Q8_0) {
      const uint8_t* blk = a.embed + ((size_t)id * (a.dim / 32) + i / 32) * 34;
      const float d = f16_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
      v = __fmul_rn((float)(int8_t)blk[2 + i % 32], d);
    } else if (a.fmt == FMT_Q4K) {
      const uint8_t* b = a.embed + ((size_t)id * (a.dim / 256) + i / 256) * 144;
      const int e = i % 256, chunk = e / 64, within = e % 64, j = chunk * 2 + (within >= 32 ? 1 : 0);
      const uint8_t* sc = b + 4;
      int s, m;
      if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
      } else {
        s = (sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
      }
      const float d = f16_to_f32((uint32_t)b[0] | ((uint32_t)b[1] << 8));
      const float dmin = f16_to_f32((uint32_t)b[2] | ((uint32_t)b[3] << 8));
      const uint8_t qq = b[16 + chunk * 32 + within % 32];
      const int q = within >= 32 ? (qq >> 4) : (qq & 0x0F);
      v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s), (float)q), __fmul_rn(dmin, (float)m));
    } else {
      const uint8_t* b = a.embed + ((size_t)id * (a.dim / 256) + i / 256) * 210;
      const int e = i % 256, half = e / 128, r = e % 128, slot = r / 32, l = r % 32;
      const uint8_t* ql = b + half * 64;
      const uint8_t* qh = b + 128 + half * 32;
      const int8_t* scv = reinterpret_cast<const int8_t*>(b + 192) + half * 8;
      int q;
      if (slot == 0)
        q = (int)((ql[l] & 0x0F) | ((qh[l] & 3) << 4)) - 32;
      else if (slot == 1)
        q = (int)((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
      else if (slot == 2)
        q = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
      else
        q = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
      const float d = f16_to_f32((uint32_t)b[208] | ((uint32_t)b[209] << 8));
      v = __fmul_rn(__fmul_rn(d, (float)scv[l / 16 + 2 * slot]), (float)q);
    }
    if (a.embed_scale != 1.0f) v = __fmul_rn(v, a.embed_scale);
    a.x[(size_t)tok * a.dim + i] = v;
  }
}

// Rows of x selected for the classifier of a multi-sequence pass.
__global__ void k_gather_rows(const float* __restrict__ x, int dim, const uint32_t* __restrict__ rows,
                              float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const float* src = x + (size_t)rows[blockIdx.x] * dim;
  float* dst = out + (size_t)blockIdx.x * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) dst[i] = src[i];
}

// Greedy choice of each classifier row (vec::argmax, vec.rs:80-90: first
// maximum) and the bookkeeping of its sequence: next token, next input,
// position after the row's token, history.
__global__ void k_rows_argmax(const float* __restrict__ logits, int vocab, const uint32_t* __restrict__ rows,
                              const uint32_t* __restrict__ seq, const uint32_t* __restrict__ pos, uint32_t* bpos,
                              uint32_t* btok, uint32_t* bnext, uint32_t* bhist, int ctx) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const float* lr = logits + (size_t)r * vocab;
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = lr[i];
    if (argmax_candidate(v)) {
      const unsigned long long k = argmax_key(v, (uint32_t)i);
      best = k > best ? k : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
    best = v > best ? v : best;
  }
  __shared__ unsigned long long wb[32];
  if ((threadIdx.x & 31) == 0) wb[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) best = wb[w] > best ? wb[w] : best;
  const uint32_t t = rows[r], sq = seq[t], p = pos[t];
  const uint32_t nt = argmax_index(best);
  bnext[sq] = nt;
  btok[sq] = nt;
  if ((int)p < ctx) bhist[(size_t)sq * ctx + p] = nt;
  bpos[sq] = p + 1;
}

__global__ void k_step_finish(uint32_t* pos, uint32_t n, const unsigned long long* key, uint32_t* next_tok,
                              uint32_t* tok_in, uint32_t* hist) {
  pdl_wait();
  const uint32_t nt = argmax_index(*key);
  const uint32_t p = *pos + n;
  *next_tok = nt;
  if (tok_in) *tok_in = nt;
  if (hist) hist[p - 1] = nt;
  *pos = p;
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

cudaError_t rope_append_run(const RopeArgs& a, cudaStream_t s, bool pdl) {
  if (a.head_dim % 32 || a.head_dim > 128) return cudaErrorInvalidValue;
  const int items = a.nt * (a.n_heads + a.n_kv_heads);
  const int wpb = 8;
  RopeArgs aa = a;
  void* args[] = {&aa};
  return launch((const void*)k_rope_append, dim3((items + wpb - 1) / wpb), dim3(32 * wpb), 0, s, pdl, args);
}

size_t attention_smem_bytes(int n_heads, int n_kv_heads, int head_dim, int ctx, int nt) {
  (void)n_heads;
  (void)n_kv_heads;
  // q + rope scratch (4 hd floats) | new k, v (2 hd f16) | scores (at least one float per thread: the
  // tolerance mode combines its V partial sums there) | 2 V chunks
  const int sc = ((ctx + 3) & ~3) > ATT_THREADS ? ((ctx + 3) & ~3) : ATT_THREADS;
  const int vch = nt > 1 ? ATT_VCH_MANY : ATT_VCH_DECODE;
  return (size_t)head_dim * 4 * 4 + (size_t)head_dim * 2 * 2 + (size_t)sc * 4 + (size_t)2 * vch * head_dim * 2;
}

size_t attention_group_smem_bytes(int n_heads, int n_kv_heads, int head_dim, int ctx) {
  const int gqa = n_heads / n_kv_heads;
  return (size_t)gqa * head_dim * 4 + (size_t)gqa * ((ctx + 3) & ~3) * 4 + (size_t)2 * ATT_VCH_GROUP * head_dim * 2;
}

cudaError_t attention_run(const AttnArgs& a, cudaStream_t s, bool pdl, bool fast) {
  if (a.n_kv_heads < 1 || a.n_heads % a.n_kv_heads || a.head_dim % 32 || a.head_dim > ATT_THREADS ||
      (a.fused && (a.nt != 1 || a.pos_tok)))
    return cudaErrorInvalidValue;
  const int gqa = a.n_heads / a.n_kv_heads;
  if (!a.fused && !fast && a.nt > 1 && gqa <= ATT_GROUP_MAX && gqa * a.head_dim <= 1024) {
    const size_t gsmem = attention_group_smem_bytes(a.n_heads, a.n_kv_heads, a.head_dim, a.ctx);
    if (gsmem <= ATTN_MAX_SMEM) {
      const void* gfn = a.head_dim == 32 ? (const void*)k_attention_group<32>
                        : a.head_dim == 64 ? (const void*)k_attention_group<64>
                                           : (const void*)k_attention_group<128>;
      if (cudaError_t e = ensure_smem_attr(gfn, ATTN_MAX_SMEM)) return e;
      AttnArgs aa = a;
      void* args[] = {&aa};
      return launch(gfn, dim3(a.n_kv_heads, a.nt), dim3(gqa * a.head_dim), gsmem, s, pdl, args);
    }
  }
  const size_t smem = attention_smem_bytes(a.n_heads, a.n_kv_heads, a.head_dim, a.ctx, a.nt);
  if (smem > ATTN_MAX_SMEM) return cudaErrorInvalidValue;
  const void* fn = nullptr;
  switch (a.head_dim) {
    case 32: fn = fast ? (const void*)k_attention<true, 32> : (const void*)k_attention<false, 32>; break;
    case 64: fn = fast ? (const void*)k_attention<true, 64> : (const void*)k_attention<false, 64>; break;
    case 128: fn = fast ? (const void*)k_attention<true, 128> : (const void*)k_attention<false, 128>; break;
    default: return cudaErrorInvalidValue;
  }
  if (cudaError_t e = ensure_smem_attr(fn, ATTN_MAX_SMEM)) return e;
  AttnArgs aa = a;
  void* args[] = {&aa};
  return launch(fn, dim3(a.n_heads, a.nt), dim3(ATT_THREADS), smem, s, pdl, args);
}

cudaError_t embed_run(const EmbedArgs& a, cudaStream_t s, bool pdl) {
  EmbedArgs aa = a;
  void* args[] = {&aa};
  const int bx = (a.dim + 255) / 256;
  return launch((const void*)k_embed, dim3(bx < 16 ? bx : 16, a.nt), dim3(256), 0, s, pdl, args);
}

cudaError_t gather_rows_run(const float* x, int dim, const uint32_t* rows, int nrows, float* out, cudaStream_t s,
                            bool pdl) {
  if (nrows <= 0) return cudaSuccess;
  void* args[] = {&x, &dim, &rows, &out};
  return launch((const void*)k_gather_rows, dim3(nrows), dim3(256), 0, s, pdl, args);
}

cudaError_t rows_argmax_run(const float* logits, int vocab, int nrows, const uint32_t* rows, const uint32_t* seq,
                            const uint32_t* pos, uint32_t* bpos, uint32_t* btok, uint32_t* bnext, uint32_t* bhist,
                            int ctx, cudaStream_t s, bool pdl) {
  if (nrows <= 0) return cudaSuccess;
  void* args[] = {&logits, &vocab, &rows, &seq, &pos, &bpos, &btok, &bnext, &bhist, &ctx};
  return launch((const void*)k_rows_argmax, dim3(nrows), dim3(512), 0, s, pdl, args);
}

cudaError_t step_finish_run(uint32_t* pos_dev, uint32_t n, const unsigned long long* key, uint32_t* next_tok,
                            uint32_t* tok_in, uint32_t* hist, cudaStream_t s, bool pdl) {
  void* args[] = {&pos_dev, &n, &key, &next_tok, &tok_in, &hist};
  return launch((const void*)k_step_finish, dim3(1), dim3(1), 0, s, pdl, args);
}

}  // namespace nrc
