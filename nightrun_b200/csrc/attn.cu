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
#include "common.cuh"
#include "expf_cr.cuh"
#include "ops.cuh"

namespace nrc {
namespace {

constexpr int ATT_THREADS = 256;
constexpr int VCHUNK = 128;  // V rows staged per pass

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
  float* hb = buf[threadIdx.x / 32];
  const float* src = is_q ? a.q + (size_t)tok * att_dim + h * hd : a.k + (size_t)tok * kv_dim + kvh * hd;
  const int per = hd / 32;
  float vals[4];
#pragma unroll
  for (int i = 0; i < 4; i++)
    if (i < per) {
      vals[i] = src[lane + 32 * i];
      hb[lane + 32 * i] = vals[i];
    }
  __syncwarp();
  const float* nw = is_q ? a.q_norm : a.k_norm;
  if (nw) {
    // rmsnorm_inplace (vec.rs:17-27): ss in index order, then x *= scale * w.
    float scale = 0.0f;
    if (lane == 0) {
      float ss = 0.0f;
      for (int i = 0; i < hd; i++) ss = __fadd_rn(ss, __fmul_rn(hb[i], hb[i]));
      scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), a.eps)));
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

// One CTA per (kv head, token) over every position 0..=pos:
//  1. scores: one thread per position, dot_f16 in the scalar order
//     (kernels.rs:146-157) times the score scale, for each query head of the group;
//  2. softmax per head (vec.rs:30-41): max, expf, the sum in position order
//     (one thread per head), normalisation;
//  3. out[h][d] = sum over positions, in position order, of p_t * v_t[d]
//     (axpy_f16, kernels.rs:160-169), V rows staged in shared memory.
__global__ void __launch_bounds__(ATT_THREADS) k_attention(const AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int g = blockIdx.x, tok = blockIdx.z;
  const uint32_t pos = a.pos_dev[0] + (uint32_t)tok;
  const int npos = (int)pos + 1;
  const int hd = a.head_dim;
  const int gqa = a.n_heads / a.n_kv_heads;
  const int att_dim = a.n_heads * hd, kv_dim = a.n_kv_heads * hd;
  const int cap = a.ctx;  // score row capacity
  extern __shared__ __align__(16) float sm[];
  float* qs = sm;                    // [gqa][hd]
  float* sc = qs + gqa * hd;         // [gqa][cap]
  uint16_t* vs = reinterpret_cast<uint16_t*>(sc + gqa * cap);  // [VCHUNK][hd]
  __shared__ float red[ATT_THREADS / 32];
  __shared__ float mh[8], inv_h[8];
  const int tid = threadIdx.x;
  for (int i = tid; i < gqa * hd; i += ATT_THREADS) qs[i] = a.q[(size_t)tok * att_dim + g * gqa * hd + i];
  __syncthreads();
  for (int t = tid; t < npos; t += ATT_THREADS) {
    const uint16_t* kr = a.kcache + (size_t)t * kv_dim + g * hd;
    for (int h = 0; h < gqa; h++) {
      const float* qh = qs + h * hd;
      float s = 0.0f;
      for (int d0 = 0; d0 < hd; d0 += 8) {
        const uint4 kv8 = *reinterpret_cast<const uint4*>(kr + d0);
        const uint32_t w[4] = {kv8.x, kv8.y, kv8.z, kv8.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          s = __fadd_rn(s, __fmul_rn(f16_to_f32(w[j] & 0xffffu), qh[d0 + 2 * j]));
          s = __fadd_rn(s, __fmul_rn(f16_to_f32(w[j] >> 16), qh[d0 + 2 * j + 1]));
        }
      }
      sc[h * cap + t] = __fmul_rn(s, a.scale);
    }
  }
  __syncthreads();
  for (int h = 0; h < gqa; h++) {
    float m = -INFINITY;
    for (int t = tid; t < npos; t += ATT_THREADS) m = fmaxf(m, sc[h * cap + t]);
    m = warp_max(m);
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
      float mm = -INFINITY;
      for (int w = 0; w < ATT_THREADS / 32; w++) mm = fmaxf(mm, red[w]);
      mh[h] = mm;
    }
    __syncthreads();
    const float mx = mh[h];
    for (int t = tid; t < npos; t += ATT_THREADS) sc[h * cap + t] = expf_cr(__fsub_rn(sc[h * cap + t], mx));
  }
  __syncthreads();
  if (tid < gqa) {
    const float* e = sc + tid * cap;
    float s = 0.0f;
    for (int t = 0; t < npos; t++) s = __fadd_rn(s, e[t]);
    inv_h[tid] = __fdiv_rn(1.0f, s);
  }
  __syncthreads();
  for (int h = 0; h < gqa; h++) {
    const float inv = inv_h[h];
    for (int t = tid; t < npos; t += ATT_THREADS) sc[h * cap + t] = __fmul_rn(sc[h * cap + t], inv);
  }
  // Output chains: thread owns outputs o = tid + i*ATT_THREADS (i < 4), o = h*hd + d.
  const int nout = gqa * hd;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  const int cpr = hd / 8;  // 16-byte chunks per V row
  for (int t0 = 0; t0 < npos; t0 += VCHUNK) {
    const int tn = npos - t0 < VCHUNK ? npos - t0 : VCHUNK;
    __syncthreads();
    for (int i = tid; i < tn * cpr; i += ATT_THREADS) {
      const int r = i / cpr, c = i - r * cpr;
      *reinterpret_cast<uint4*>(vs + r * hd + c * 8) =
          *reinterpret_cast<const uint4*>(a.vcache + (size_t)(t0 + r) * kv_dim + g * hd + c * 8);
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int o = tid + i * ATT_THREADS;
      if (o < nout) {
        const int h = o / hd, d = o - h * hd;
        const float* p = sc + h * cap + t0;
        float ac = acc[i];
        for (int t = 0; t < tn; t++) ac = __fadd_rn(ac, __fmul_rn(p[t], f16_to_f32(vs[t * hd + d])));
        acc[i] = ac;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int o = tid + i * ATT_THREADS;
    if (o < nout) a.out[(size_t)tok * att_dim + g * gqa * hd + o] = acc[i];
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

size_t attention_smem_bytes(int n_heads, int n_kv_heads, int head_dim, int ctx) {
  const int gqa = n_heads / n_kv_heads;
  return (size_t)gqa * head_dim * 4 + (size_t)gqa * ctx * 4 + (size_t)VCHUNK * head_dim * 2 + 16;
}

cudaError_t attention_run(const AttnArgs& a, cudaStream_t s, bool pdl) {
  const int gqa = a.n_heads / a.n_kv_heads;
  if (gqa > 8 || a.head_dim % 8 || a.head_dim > 128) return cudaErrorInvalidValue;
  const size_t smem = attention_smem_bytes(a.n_heads, a.n_kv_heads, a.head_dim, a.ctx);
  if (smem > ATTN_MAX_SMEM) return cudaErrorInvalidValue;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaFuncSetAttribute((const void*)k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, ATTN_MAX_SMEM);
    attr_done[dev] = true;
  }
  AttnArgs aa = a;
  void* args[] = {&aa};
  return launch((const void*)k_attention, dim3(a.n_kv_heads, 1, a.nt), dim3(ATT_THREADS), smem, s, pdl, args);
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
