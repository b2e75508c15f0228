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
constexpr int ATT_VCH = 128;      // V rows staged per pass

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
  const uint32_t pos = a.pos_dev[0] + (uint32_t)tok;
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
    uint16_t* kd = a.kcache + (size_t)pos * kv_dim + kvh * hd;
    uint16_t* vd = a.vcache + (size_t)pos * kv_dim + kvh * hd;
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
__global__ void __launch_bounds__(ATT_THREADS) k_attention(const AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x, tok = blockIdx.y;
  const int hd = a.head_dim, half = hd / 2;
  const int gqa = a.n_heads / a.n_kv_heads;
  const int g = h / gqa;
  const int att_dim = a.n_heads * hd, kv_dim = a.n_kv_heads * hd;
  const uint32_t pos = a.pos_dev[0] + (uint32_t)tok;
  const int npos = (int)pos + 1;
  const bool fused = a.fused != 0;
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                                               // [hd]
  float* hbuf = qs + hd;                                        // [3][hd] rope scratch (fused)
  uint16_t* knew = reinterpret_cast<uint16_t*>(hbuf + 3 * hd);  // [hd] new k (f16, fused)
  uint16_t* vnew = knew + hd;                                   // [hd] new v (f16, fused)
  float* sc = reinterpret_cast<float*>(vnew + hd);              // [ctx] scores, then probabilities
  uint16_t* vs = reinterpret_cast<uint16_t*>(sc + ((a.ctx + 3) & ~3));  // [2][ATT_VCH][hd]
  __shared__ float red[ATT_THREADS / 32];
  __shared__ SeqSumShared ssh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint16_t* kbase = a.kcache + (size_t)g * hd;
  uint16_t* vbase = a.vcache + (size_t)g * hd;
  const int cpr = hd / 8;  // 16-byte chunks per K/V row
  // Rows [0, cached) come from the cache; with the append fused, row `pos`
  // comes from shared memory.
  const int cached = fused ? (int)pos : npos;
  auto stage_v = [&](int t0, int buf) {
    const int tn = min(ATT_VCH, cached - t0);
    uint16_t* dst = vs + (size_t)buf * ATT_VCH * hd;
    for (int i = tid; i < tn * cpr; i += ATT_THREADS) {
      const int r = i / cpr, c = i - r * cpr;
      cp_async16(dst + r * hd + c * 8, vbase + (size_t)(t0 + r) * kv_dim + c * 8);
    }
    cp_async_commit();
  };
  stage_v(0, 0);
  // The K row of this thread's first position, loaded now so its latency
  // overlaps the RoPE work below.
  uint4 k0[16];
  if (tid < cached) {
    const uint4* kr = reinterpret_cast<const uint4*>(kbase + (size_t)tid * kv_dim);
#pragma unroll
    for (int c = 0; c < 16; c++)
      if (c < cpr) k0[c] = kr[c];
  }
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
      for (int c = 0; c < 16; c++) {
        if (c < cpr) {
          const uint32_t w[4] = {k0[c].x, k0[c].y, k0[c].z, k0[c].w};
          const float* qd = qs + c * 8;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            s = __fadd_rn(s, __fmul_rn(h2f(w[j] & 0xffffu), qd[2 * j]));
            s = __fadd_rn(s, __fmul_rn(h2f(w[j] >> 16), qd[2 * j + 1]));
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
              s = __fadd_rn(s, __fmul_rn(h2f(w[j] & 0xffffu), qd[2 * j]));
              s = __fadd_rn(s, __fmul_rn(h2f(w[j] >> 16), qd[2 * j + 1]));
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
  // The sum in position order (vec.rs:35-36), one chain (seqsum.cuh).
  const float sum = seq_sum_group<ATT_THREADS>(npos, [&](int t) { return sc[t]; }, ssh, tid, [] { __syncthreads(); });
  const float inv = __fdiv_rn(1.0f, sum);
  for (int t = tid; t < npos; t += ATT_THREADS) sc[t] = __fmul_rn(sc[t], inv);

  float acc = 0.0f;
  const int d = tid;
  int buf = 0;
  for (int t0 = 0; t0 < npos; t0 += ATT_VCH, buf ^= 1) {
    const int tn = min(ATT_VCH, npos - t0);
    if (t0 + ATT_VCH < cached) {
      stage_v(t0 + ATT_VCH, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    uint16_t* vb = vs + (size_t)buf * ATT_VCH * hd;
    if (fused && (int)pos < t0 + tn)
      for (int i = tid; i < hd; i += ATT_THREADS) vb[((int)pos - t0) * hd + i] = vnew[i];
    __syncthreads();
    if (d < hd) {
      const uint16_t* vr = vb + d;
      const float* p = sc + t0;
      acc = seq_sum_serial(tn, [&](int t) { return __fmul_rn(p[t], h2f(vr[(size_t)t * hd])); }, acc);
    }
    __syncthreads();  // the buffer is restaged two chunks later
  }
  if (d < hd) a.out[(size_t)tok * att_dim + (size_t)h * hd + d] = acc;
}

// Decode attention of the tolerance mode (infer.rs:553-572 up to summation
// order): grid (query head, position split). The fused per-head norms, RoPE
// and KV append are those of k_attention. Scores: one thread per position
// (fused multiply-adds); softmax max and sum as CTA trees; V: hd/8 threads
// per cached row, 16-byte loads, 8 accumulators each, the position groups
// combined in a fixed order. With several splits each CTA writes (max, sum,
// unnormalised output) and the last CTA of the head (an arrival counter, no
// waiting) merges the splits in split order and resets the counter.
constexpr int AF_THREADS = 128;

__global__ void __launch_bounds__(AF_THREADS) k_attention_fast(const AttnArgs a, float* part, unsigned* count,
                                                               int nsplit, int max_per) {
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x, sp = blockIdx.y;
  const int hd = a.head_dim, half = hd / 2;
  const int gqa = a.n_heads / a.n_kv_heads;
  const int g = h / gqa;
  const int kv_dim = a.n_kv_heads * hd;
  const uint32_t pos = a.pos_dev[0];
  const int npos = (int)pos + 1;
  const int per = (npos + nsplit - 1) / nsplit;
  const int t0 = min(npos, sp * per), t1 = min(npos, t0 + per);
  const bool mine = (int)pos >= t0 && (int)pos < t1;  // this split holds the new position
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                                               // [hd]
  float* hbuf = qs + hd;                                        // [3][hd]
  uint16_t* knew = reinterpret_cast<uint16_t*>(hbuf + 3 * hd);  // [hd]
  uint16_t* vnew = knew + hd;                                   // [hd]
  float* sc = reinterpret_cast<float*>(vnew + hd);              // [max_per]
  float* vpart = sc + ((max_per + 3) & ~3);                     // [16][hd]
  __shared__ float red[AF_THREADS / 32];
  __shared__ unsigned last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint16_t* kbase = a.kcache + (size_t)g * hd;
  const uint16_t* vbase = a.vcache + (size_t)g * hd;
  {
    const float* ct = a.cos_tab + (size_t)pos * half;
    const float* st = a.sin_tab + (size_t)pos * half;
    const int pr = hd / 32;
    float outv[4];
    if (warp == 0) {
      warp_rope_head(a.q + (size_t)h * hd, a.q_norm, a.eps, ct, st, a.style, hd, hbuf, lane, outv);
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (i < pr) qs[lane + 32 * i] = outv[i];
    } else if (warp == 1 && mine) {
      warp_rope_head(a.k + (size_t)g * hd, a.k_norm, a.eps, ct, st, a.style, hd, hbuf + hd, lane, outv);
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (i < pr) {
          const uint16_t kb = f32_to_f16(outv[i]);
          knew[lane + 32 * i] = kb;
          if (h % gqa == 0) a.kcache[(size_t)pos * kv_dim + (size_t)g * hd + lane + 32 * i] = kb;
        }
    } else if (warp == 2 && mine) {
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (i < pr) {
          const uint16_t vb = f32_to_f16(a.v[(size_t)g * hd + lane + 32 * i]);
          vnew[lane + 32 * i] = vb;
          if (h % gqa == 0) a.vcache[(size_t)pos * kv_dim + (size_t)g * hd + lane + 32 * i] = vb;
        }
    }
  }
  __syncthreads();
  // Scores.
  const int cpr = hd / 8;
  float mloc = -INFINITY;
  for (int t = t0 + tid; t < t1; t += AF_THREADS) {
    float s = 0.0f;
    if (t == (int)pos) {
      for (int d = 0; d < hd; d++) s = fmaf(h2f(knew[d]), qs[d], s);
    } else {
      const uint4* kr = reinterpret_cast<const uint4*>(kbase + (size_t)t * kv_dim);
      for (int c0 = 0; c0 < cpr; c0 += 8) {
        uint4 k8[8];
#pragma unroll
        for (int c = 0; c < 8; c++)
          if (c0 + c < cpr) k8[c] = kr[c0 + c];
#pragma unroll
        for (int c = 0; c < 8; c++)
          if (c0 + c < cpr) {
            const uint32_t w[4] = {k8[c].x, k8[c].y, k8[c].z, k8[c].w};
            const float* qd = qs + (c0 + c) * 8;
#pragma unroll
            for (int j = 0; j < 4; j++) {
              s = fmaf(h2f(w[j] & 0xffffu), qd[2 * j], s);
              s = fmaf(h2f(w[j] >> 16), qd[2 * j + 1], s);
            }
          }
      }
    }
    s = s * a.scale;
    sc[t - t0] = s;
    mloc = fmaxf(mloc, s);
  }
  mloc = warp_max(mloc);
  if (lane == 0) red[warp] = mloc;
  __syncthreads();
  float mx = red[0];
#pragma unroll
  for (int w = 1; w < AF_THREADS / 32; w++) mx = fmaxf(mx, red[w]);
  __syncthreads();  // red is reused below
  float lsum = 0.0f;
  for (int t = t0 + tid; t < t1; t += AF_THREADS) {
    const float e = expf_cr(sc[t - t0] - mx);
    sc[t - t0] = e;
    lsum += e;
  }
  lsum = warp_sum(lsum);
  if (lane == 0) red[warp] = lsum;
  __syncthreads();
  float l = 0.0f;
#pragma unroll
  for (int w = 0; w < AF_THREADS / 32; w++) l += red[w];
  // V: thread (c, grp) accumulates dims c*8 .. c*8+7 over positions t0 + grp, + P, ...
  const int P = AF_THREADS / cpr;
  const int c = tid % cpr, grp = tid / cpr;
  float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
  for (int t = t0 + grp; t < t1; t += P) {
    const float e = sc[t - t0];
    uint4 vv;
    if (t == (int)pos)
      vv = reinterpret_cast<const uint4*>(vnew)[c];
    else
      vv = reinterpret_cast<const uint4*>(vbase + (size_t)t * kv_dim)[c];
    const uint32_t w[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      acc[2 * j] = fmaf(e, h2f(w[j] & 0xffffu), acc[2 * j]);
      acc[2 * j + 1] = fmaf(e, h2f(w[j] >> 16), acc[2 * j + 1]);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; j++) vpart[grp * hd + c * 8 + j] = acc[j];
  __syncthreads();
  float o = 0.0f;
  if (tid < hd)
    for (int q = 0; q < P; q++) o += vpart[q * hd + tid];
  float* out = a.out + (size_t)h * hd;
  if (nsplit == 1) {
    if (tid < hd) out[tid] = o / l;
    return;
  }
  float* pp = part + ((size_t)h * nsplit + sp) * (hd + 2);
  if (tid < hd) pp[2 + tid] = o;
  if (tid == 0) {
    pp[0] = mx;
    pp[1] = l;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&count[h], 1u);
  __syncthreads();
  if (last != (unsigned)nsplit - 1) return;
  __threadfence();
  const float* ph = part + (size_t)h * nsplit * (hd + 2);
  float M = -INFINITY;
  for (int k = 0; k < nsplit; k++) M = fmaxf(M, ph[k * (hd + 2)]);
  float L = 0.0f, O = 0.0f;
  for (int k = 0; k < nsplit; k++) {
    const float* q = ph + k * (hd + 2);
    const float f = q[1] > 0.0f ? expf_cr(q[0] - M) : 0.0f;
    L += q[1] * f;
    if (tid < hd) O += q[2 + tid] * f;
  }
  if (tid < hd) out[tid] = O / L;
  if (tid == 0) count[h] = 0u;
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

size_t attention_smem_bytes(int n_heads, int n_kv_heads, int head_dim, int ctx) {
  (void)n_heads;
  (void)n_kv_heads;
  // q + rope scratch (4 hd floats) | new k, v (2 hd f16) | scores | 2 V chunks
  return (size_t)head_dim * 4 * 4 + (size_t)head_dim * 2 * 2 + (size_t)((ctx + 3) & ~3) * 4 +
         (size_t)2 * ATT_VCH * head_dim * 2;
}

cudaError_t attention_run(const AttnArgs& a, cudaStream_t s, bool pdl) {
  if (a.n_kv_heads < 1 || a.n_heads % a.n_kv_heads || a.head_dim % 32 || a.head_dim > ATT_THREADS ||
      (a.fused && a.nt != 1))
    return cudaErrorInvalidValue;
  const size_t smem = attention_smem_bytes(a.n_heads, a.n_kv_heads, a.head_dim, a.ctx);
  if (smem > ATTN_MAX_SMEM) return cudaErrorInvalidValue;
  if (cudaError_t e = ensure_smem_attr((const void*)k_attention, ATTN_MAX_SMEM)) return e;
  AttnArgs aa = a;
  void* args[] = {&aa};
  return launch((const void*)k_attention, dim3(a.n_heads, a.nt), dim3(ATT_THREADS), smem, s, pdl, args);
}

int attention_fast_splits(int ctx) {
  const int n = (ctx + 255) / 256;
  return n < 1 ? 1 : (n > 32 ? 32 : n);
}
size_t attention_fast_scratch_floats(int n_heads, int head_dim, int nsplit) {
  return (size_t)n_heads * nsplit * (head_dim + 2);
}
size_t attention_fast_smem_bytes(int head_dim, int ctx, int nsplit) {
  const int max_per = (ctx + nsplit - 1) / nsplit;
  return (size_t)head_dim * 4 * 4 + (size_t)head_dim * 2 * 2 + (size_t)((max_per + 3) & ~3) * 4 +
         (size_t)16 * head_dim * 4;
}

cudaError_t attention_fast_run(const AttnArgs& a, float* part, unsigned* count, int nsplit, cudaStream_t s,
                               bool pdl) {
  if (a.n_kv_heads < 1 || a.n_heads % a.n_kv_heads || a.head_dim % 32 || a.head_dim < 64 || a.head_dim > 128 ||
      a.nt != 1 || nsplit < 1 || (nsplit > 1 && (!part || !count)))
    return cudaErrorInvalidValue;
  const int max_per = (a.ctx + nsplit - 1) / nsplit;
  const size_t smem = attention_fast_smem_bytes(a.head_dim, a.ctx, nsplit);
  if (smem > ATTN_MAX_SMEM) return cudaErrorInvalidValue;
  if (cudaError_t e = ensure_smem_attr((const void*)k_attention_fast, (int)ATTN_MAX_SMEM)) return e;
  AttnArgs aa = a;
  void* args[] = {&aa, &part, &count, &nsplit, (void*)&max_per};
  return launch((const void*)k_attention_fast, dim3(a.n_heads, nsplit), dim3(AF_THREADS), smem, s, pdl, args);
}

cudaError_t embed_run(const EmbedArgs& a, cudaStream_t s, bool pdl) {
  EmbedArgs aa = a;
  void* args[] = {&aa};
  const int bx = (a.dim + 255) / 256;
  return launch((const void*)k_embed, dim3(bx < 16 ? bx : 16, a.nt), dim3(256), 0, s, pdl, args);
}

cudaError_t step_finish_run(uint32_t* pos_dev, uint32_t n, const unsigned long long* key, uint32_t* next_tok,
                            uint32_t* tok_in, uint32_t* hist, cudaStream_t s, bool pdl) {
  void* args[] = {&pos_dev, &n, &key, &next_tok, &tok_in, &hist};
  return launch((const void*)k_step_finish, dim3(1), dim3(1), 0, s, pdl, args);
}

}  // namespace nrc
