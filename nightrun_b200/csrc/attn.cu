// Position-dependent kernels of the forward pass:
//  * rope_append: Qwen3 per-head q/k RMSNorm (vec.rs:17-27), RoPE (rope.rs:49-65,
//    from host-built cos/sin tables) and the f16 KV-cache append
//    (crates/nr-model/src/infer.rs:533-551, 639-659);
//  * attention: GQA attention over the f16 cache (infer.rs:553-572, 661-685),
//    split over positions in chunks of ATTN_SPLIT, partial softmax states
//    combined by the last CTA of each (token, kv head);
//  * embed: token-embedding row dequantization (infer.rs:37-56, 516-521);
//  * step_finish: position advance and greedy-token decode.
// Every per-token result depends only on that token's position, so batched
// prefill and token-by-token decode produce bit-identical outputs.
#include "common.cuh"
#include "ops.cuh"

namespace nrc {
namespace {

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
  float vals[4];  // head_dim <= 128: 4 values per lane
  const float* src = is_q ? a.q + (size_t)tok * att_dim + h * hd : a.k + (size_t)tok * kv_dim + kvh * hd;
  const int per = hd / 32;
#pragma unroll
  for (int i = 0; i < 4; i++)
    if (i < per) vals[i] = src[lane + 32 * i];
  const float* nw = is_q ? a.q_norm : a.k_norm;
  if (nw) {
    // rmsnorm_inplace: x *= scale * w, scale = 1 / sqrtf(ss / n + eps)
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (i < per) ss = __fadd_rn(ss, __fmul_rn(vals[i], vals[i]));
    ss = warp_sum(ss);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), a.eps)));
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (i < per) vals[i] = __fmul_rn(vals[i], __fmul_rn(scale, nw[lane + 32 * i]));
  }
  // Rotation: each lane owns elements lane + 32*i; partners are exchanged via smem.
  __shared__ float buf[8][128];
  float* hb = buf[threadIdx.x / 32];
#pragma unroll
  for (int i = 0; i < 4; i++)
    if (i < per) hb[lane + 32 * i] = vals[i];
  __syncwarp();
  const float* ct = a.cos_tab + (size_t)pos * half;
  const float* st = a.sin_tab + (size_t)pos * half;
  float outv[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    if (i < per) {
      const int e = lane + 32 * i;
      int pi, ia, ib;
      if (a.style == 0) {
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
      outv[i] = (e == ia) ? __fsub_rn(__fmul_rn(av, c), __fmul_rn(bv, sn))
                          : __fadd_rn(__fmul_rn(av, sn), __fmul_rn(bv, c));
    }
  }
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

// One CTA per (kv head, position split, token); ATTN_SPLIT threads, one per position.
__global__ void __launch_bounds__(ATTN_SPLIT) k_attention(const AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int g = blockIdx.x, split = blockIdx.y, tok = blockIdx.z;
  const uint32_t pos = a.pos_dev[0] + (uint32_t)tok;
  const int npos = (int)pos + 1;
  const int nsplit = (npos + ATTN_SPLIT - 1) / ATTN_SPLIT;
  if (split >= nsplit) return;
  const int hd = a.head_dim;
  const int gqa = a.n_heads / a.n_kv_heads;
  const int att_dim = a.n_heads * hd, kv_dim = a.n_kv_heads * hd;
  const int max_splits = (a.ctx + ATTN_SPLIT - 1) / ATTN_SPLIT;
  const int t0 = split * ATTN_SPLIT;
  const int tn = min(ATTN_SPLIT, npos - t0);
  extern __shared__ float sm[];
  float* qs = sm;                      // [gqa][hd]
  float* sc = qs + gqa * hd;           // [gqa][ATTN_SPLIT]
  __shared__ float red[ATTN_SPLIT / 32];
  __shared__ float mh[8], lh[8];
  __shared__ int is_last;
  const int tid = threadIdx.x;
  for (int i = tid; i < gqa * hd; i += blockDim.x) qs[i] = a.q[(size_t)tok * att_dim + g * gqa * hd + i];
  __syncthreads();
  // Scores: dot_f16 in the scalar order (kernels.rs:146-157), times the score scale.
  if (tid < tn) {
    const uint16_t* kr = a.kcache + (size_t)(t0 + tid) * kv_dim + g * hd;
    for (int h = 0; h < gqa; h++) {
      float s = 0.0f;
      const float* qh = qs + h * hd;
      for (int d0 = 0; d0 < hd; d0 += 8) {
        const uint4 kv8 = *reinterpret_cast<const uint4*>(kr + d0);
        const uint32_t w[4] = {kv8.x, kv8.y, kv8.z, kv8.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          s = __fadd_rn(s, __fmul_rn(f16_to_f32(w[j] & 0xffffu), qh[d0 + 2 * j]));
          s = __fadd_rn(s, __fmul_rn(f16_to_f32(w[j] >> 16), qh[d0 + 2 * j + 1]));
        }
      }
      sc[h * ATTN_SPLIT + tid] = __fmul_rn(s, a.scale);
    }
  }
  __syncthreads();
  // Per-head max and exp-sum over this split.
  for (int h = 0; h < gqa; h++) {
    float m = tid < tn ? sc[h * ATTN_SPLIT + tid] : -INFINITY;
    m = warp_max(m);
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
      float mm = -INFINITY;
      for (int w = 0; w < ATTN_SPLIT / 32; w++) mm = fmaxf(mm, red[w]);
      mh[h] = mm;
    }
    __syncthreads();
    float e = 0.0f;
    if (tid < tn) {
      e = expf(__fsub_rn(sc[h * ATTN_SPLIT + tid], mh[h]));
      sc[h * ATTN_SPLIT + tid] = e;
    }
    e = warp_sum(e);
    if ((tid & 31) == 0) red[tid >> 5] = e;
    __syncthreads();
    if (tid == 0) {
      float ll = 0.0f;
      for (int w = 0; w < ATTN_SPLIT / 32; w++) ll = __fadd_rn(ll, red[w]);
      lh[h] = ll;
    }
    __syncthreads();
  }
  const int nout = gqa * hd;
  if (nsplit == 1) {
    // softmax normalisation then axpy_f16 in position order (infer.rs:565-571).
    for (int o = tid; o < nout; o += blockDim.x) {
      const int h = o / hd, d = o % hd;
      const float inv = __fdiv_rn(1.0f, lh[h]);
      float acc = 0.0f;
      const uint16_t* vr = a.vcache + g * hd + d;
      for (int t = 0; t < tn; t++) {
        const float p = __fmul_rn(sc[h * ATTN_SPLIT + t], inv);
        acc = __fadd_rn(acc, __fmul_rn(p, f16_to_f32(vr[(size_t)(t0 + t) * kv_dim])));
      }
      a.out[(size_t)tok * att_dim + g * gqa * hd + o] = acc;
    }
    return;
  }
  // Multi-split: unnormalised partial state, combined by the last CTA.
  float* part = a.partial + ((size_t)tok * a.n_heads + g * gqa) * max_splits * (hd + 2);
  for (int o = tid; o < nout; o += blockDim.x) {
    const int h = o / hd, d = o % hd;
    float acc = 0.0f;
    const uint16_t* vr = a.vcache + g * hd + d;
    for (int t = 0; t < tn; t++)
      acc = __fadd_rn(acc, __fmul_rn(sc[h * ATTN_SPLIT + t], f16_to_f32(vr[(size_t)(t0 + t) * kv_dim])));
    part[((size_t)h * max_splits + split) * (hd + 2) + d] = acc;
  }
  if (tid < gqa) {
    part[((size_t)tid * max_splits + split) * (hd + 2) + hd] = mh[tid];
    part[((size_t)tid * max_splits + split) * (hd + 2) + hd + 1] = lh[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    unsigned* ctr = a.counters + (size_t)tok * a.n_kv_heads + g;
    const unsigned prev = atomicAdd(ctr, 1u);
    is_last = (prev == (unsigned)nsplit - 1);
    if (is_last) *ctr = 0u;  // ready for the next launch
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int o = tid; o < nout; o += blockDim.x) {
    const int h = o / hd, d = o % hd;
    const float* ph = part + (size_t)h * max_splits * (hd + 2);
    float M = -INFINITY;
    for (int s = 0; s < nsplit; s++) M = fmaxf(M, __ldcg(ph + (size_t)s * (hd + 2) + hd));
    float L = 0.0f, O = 0.0f;
    for (int s = 0; s < nsplit; s++) {
      const float* ps = ph + (size_t)s * (hd + 2);
      const float f = expf(__fsub_rn(__ldcg(ps + hd), M));
      L = __fadd_rn(L, __fmul_rn(__ldcg(ps + hd + 1), f));
      O = __fadd_rn(O, __fmul_rn(__ldcg(ps + d), f));
    }
    a.out[(size_t)tok * att_dim + g * gqa * hd + o] = __fdiv_rn(O, L);
  }
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

cudaError_t attention_run(const AttnArgs& a, cudaStream_t s, bool pdl) {
  const int gqa = a.n_heads / a.n_kv_heads;
  if (gqa > 8 || a.head_dim % 8) return cudaErrorInvalidValue;
  const int max_splits = (a.ctx + ATTN_SPLIT - 1) / ATTN_SPLIT;
  const size_t smem = (size_t)gqa * a.head_dim * 4 + (size_t)gqa * ATTN_SPLIT * 4;
  AttnArgs aa = a;
  void* args[] = {&aa};
  return launch((const void*)k_attention, dim3(a.n_kv_heads, max_splits, a.nt), dim3(ATTN_SPLIT), smem, s, pdl,
                args);
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
