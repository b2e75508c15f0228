// Element-wise and reduction kernels of the kernel-level C ABI
// (crates/nr-tensor/src/{q8,kquant,f16,vec,rope}.rs). The fused forward path
// uses the same arithmetic inside its GEMV prologues/epilogues and attention.
#include "common.cuh"
#include "expf_cr.cuh"
#include "seqsum.cuh"
#include "ops.cuh"

namespace nrc {
namespace {

// q8::quantize (q8.rs:27-44): one warp per 32-value block.
__global__ void k_quantize_q8_0(const float* __restrict__ x, uint8_t* __restrict__ out, size_t nblk) {
  const size_t b = (size_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (b >= nblk) return;
  const float v = x[b * 32 + lane];
  const float amax = warp_max(fabsf(v));
  const uint16_t dbits = f32_to_f16(__fdiv_rn(amax, 127.0f));
  const float d = f16_to_f32(dbits);
  const float inv = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  const float xs = __fmul_rn(v, inv);
  const float r = xs >= 0.0f ? __fadd_rn(xs, 0.5f) : __fsub_rn(xs, 0.5f);
  int q = rust_f2i(r);
  q = q < -127 ? -127 : (q > 127 ? 127 : q);
  uint8_t* blk = out + b * 34;
  blk[2 + lane] = (uint8_t)(int8_t)q;
  if (lane == 0) {
    blk[0] = (uint8_t)(dbits & 0xff);
    blk[1] = (uint8_t)(dbits >> 8);
  }
}

// q8::dequantize (q8.rs:47-55).
__global__ void k_dequantize_q8_0(const uint8_t* __restrict__ in, float* __restrict__ out, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t* blk = in + (i / 32) * 34;
  const float d = f16_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
  out[i] = __fmul_rn((float)(int8_t)blk[2 + (i % 32)], d);
}

// kquant::quantize_q8k (kquant.rs:157-187): one warp per 256-value block,
// eight consecutive values per lane.
__global__ void k_quantize_q8k(const float* __restrict__ x, uint8_t* __restrict__ out, size_t nblk) {
  const size_t b = (size_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (b >= nblk) return;
  float v[8];
#pragma unroll
  for (int k = 0; k < 8; k++) v[k] = x[b * 256 + lane * 8 + k];
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
  uint8_t* blk = out + b * 292;
  uint32_t* qw = reinterpret_cast<uint32_t*>(blk + 4);
  int16_t* bs = reinterpret_cast<int16_t*>(blk + 260);
  if (amax == 0.0f) {
    qw[lane * 2] = 0u;
    qw[lane * 2 + 1] = 0u;
    if (lane < 16) bs[lane] = 0;
    if (lane == 0) *reinterpret_cast<float*>(blk) = 0.0f;
    return;
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
  const int s16 = part + __shfl_down_sync(0xffffffffu, part, 1);
  if ((lane & 1) == 0) bs[lane / 2] = (int16_t)s16;
  if (lane == 0) *reinterpret_cast<float*>(blk) = __fdiv_rn(1.0f, iscale);
}

// kquant::dequant_q4k (kquant.rs:95-118): one thread per output value.
__global__ void k_dequant_q4k(const uint8_t* __restrict__ in, float* __restrict__ out, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t* b = in + (i / 256) * 144;
  const int e = (int)(i % 256);
  const int chunk = e / 64, within = e % 64, j = chunk * 2 + (within >= 32 ? 1 : 0), k = within % 32;
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
  const uint8_t qq = b[16 + chunk * 32 + k];
  const int q = (within >= 32) ? (qq >> 4) : (qq & 0x0F);
  out[i] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s), (float)q), __fmul_rn(dmin, (float)m));
}

// kquant::dequant_q6k (kquant.rs:121-142).
__global__ void k_dequant_q6k(const uint8_t* __restrict__ in, float* __restrict__ out, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t* b = in + (i / 256) * 210;
  const int e = (int)(i % 256);
  const int half = e / 128, r = e % 128, slot = r / 32, l = r % 32;
  const uint8_t* ql = b + half * 64;
  const uint8_t* qh = b + 128 + half * 32;
  const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192) + half * 8;
  const int is = l / 16;
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
  out[i] = __fmul_rn(__fmul_rn(d, (float)sc[is + 2 * slot]), (float)q);
}

__global__ void k_f32_to_f16(const float* __restrict__ x, uint16_t* __restrict__ o, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) o[i] = f32_to_f16(x[i]);
}
__global__ void k_f16_to_f32(const uint16_t* __restrict__ x, float* __restrict__ o, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) o[i] = f16_to_f32(x[i]);
}

NRC_DEV float block_max(float m, float* red) {
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float t = -INFINITY;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) t = fmaxf(t, red[w]);
  __syncthreads();
  return t;
}

// vec::rmsnorm (vec.rs:4-14), one CTA per row: the sum of squares in index
// order (one chain, seqsum.cuh) over the row staged in shared memory when it
// fits, the scaling in parallel.
__global__ void k_rmsnorm(float* __restrict__ out, const float* __restrict__ x, const float* __restrict__ w,
                          int n, float eps, int staged) {
  __shared__ SeqSumShared sh;
  extern __shared__ float row[];
  const float* xr = x + (size_t)blockIdx.x * n;
  float* orow = out + (size_t)blockIdx.x * n;
  const float* src = xr;
  if (staged) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) row[i] = xr[i];
    __syncthreads();
    src = row;
  }
  const float ss = seq_sum_group<256>(
      n, [&](int i) { return __fmul_rn(src[i], src[i]); }, sh, (int)threadIdx.x, [] { __syncthreads(); });
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
  for (int i = threadIdx.x; i < n; i += blockDim.x) orow[i] = __fmul_rn(__fmul_rn(src[i], scale), w[i]);
}

// vec::softmax (vec.rs:30-41), one CTA per row, in place: max (order-free),
// exponentials in parallel, their sum in index order (one chain), then the scaling.
__global__ void k_softmax(float* __restrict__ x, int n, int staged) {
  __shared__ float red[32];
  __shared__ SeqSumShared sh;
  extern __shared__ float row[];
  float* xr = x + (size_t)blockIdx.x * n;
  float* e = staged ? row : xr;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, xr[i]);
  m = block_max(m, red);
  for (int i = threadIdx.x; i < n; i += blockDim.x) e[i] = expf_cr(__fsub_rn(xr[i], m));
  __syncthreads();
  const float sum = seq_sum_group<256>(n, [&](int i) { return e[i]; }, sh, (int)threadIdx.x, [] { __syncthreads(); });
  const float inv = __fdiv_rn(1.0f, sum);
  for (int i = threadIdx.x; i < n; i += blockDim.x) xr[i] = __fmul_rn(e[i], inv);
}

// vec::swiglu (vec.rs:44-50).
__global__ void k_swiglu(float* __restrict__ g, const float* __restrict__ u, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = g[i];
  g[i] = __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, expf_cr(-x))), u[i]);
}

// Self-test of the bounded waits every pipelined kernel uses: one thread
// waits on something nobody completes (kind 0: an mbarrier expecting two
// arrivals that gets one; kind 1: a shared-memory flag nobody raises). The
// wait gives up after limit_ns, the kernel records the bit its production
// callers record and returns; nothing traps, the context stays usable.
__global__ void k_wait_selftest(unsigned* err, unsigned long long limit_ns, int kind) {
  __shared__ uint64_t bar;
  __shared__ uint32_t flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 2);
    flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_arrive(&bar);  // the second arrival is withheld
  __syncwarp();
  if (threadIdx.x == 1) {
    const bool ok = kind == 0 ? mbar_wait(&bar, 0, limit_ns) : flag_wait_geq(&flag, 1, limit_ns);
    if (!ok) atomicOr(err, kind == 0 ? ERR_WAIT_FULL : ERR_WAIT_EMPTY);
  }
}

// Elementwise correctly rounded expf (checked against the CPU oracle bit for bit).
__global__ void k_expf(const float* __restrict__ x, float* __restrict__ y, size_t n) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = expf_cr(x[i]);
}

// Hash of expf_cr over every binary32 input, 2^20 inputs per chunk (same
// mixing as the oracle's exhaustive check), one thread per chunk, one warp
// per CTA so the chunks spread over every SM.
__global__ void k_expf_hash(unsigned long long* out, int chunk0, int nchunks) {
  const int c = chunk0 + blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= chunk0 + nchunks) return;
  unsigned long long h = 0;
  for (uint32_t i = 0; i < (1u << 20); i++) {
    const uint32_t bits = ((uint32_t)c << 20) | i;
    const uint32_t y = __float_as_uint(expf_cr(__uint_as_float(bits)));
    h ^= y + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
    h *= 0xBF58476D1CE4E5B9ull;
  }
  out[c - chunk0] = h;
}

// vec::argmax (vec.rs:80-90): packed (value, index) keys, max over the grid.
__global__ void k_argmax_init(unsigned long long* key) { *key = 0ull; }
__global__ void k_argmax(const float* __restrict__ x, size_t n, unsigned long long* key) {
  unsigned long long best = 0ull;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float v = x[i];
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
  if ((threadIdx.x & 31) == 0 && best) atomicMax(key, best);
}
__global__ void k_argmax_finish(const unsigned long long* key, uint32_t* out) { *out = argmax_index(*key); }

}  // namespace

static inline unsigned blocks_for(size_t n, unsigned per) { return (unsigned)((n + per - 1) / per); }

cudaError_t op_quantize_q8_0(const float* x, void* out, size_t n, cudaStream_t s) {
  const size_t nb = n / 32;
  if (nb) k_quantize_q8_0<<<blocks_for(nb, 8), 256, 0, s>>>(x, static_cast<uint8_t*>(out), nb);
  return cudaGetLastError();
}
cudaError_t op_dequantize_q8_0(const void* b, float* out, size_t n, cudaStream_t s) {
  if (n) k_dequantize_q8_0<<<blocks_for(n, 256), 256, 0, s>>>(static_cast<const uint8_t*>(b), out, n);
  return cudaGetLastError();
}
cudaError_t op_quantize_q8k(const float* x, void* out, size_t n, cudaStream_t s) {
  const size_t nb = n / 256;
  if (nb) k_quantize_q8k<<<blocks_for(nb, 8), 256, 0, s>>>(x, static_cast<uint8_t*>(out), nb);
  return cudaGetLastError();
}
cudaError_t op_dequant_q4k(const void* b, float* out, size_t nblocks, cudaStream_t s) {
  const size_t n = nblocks * 256;
  if (n) k_dequant_q4k<<<blocks_for(n, 256), 256, 0, s>>>(static_cast<const uint8_t*>(b), out, n);
  return cudaGetLastError();
}
cudaError_t op_dequant_q6k(const void* b, float* out, size_t nblocks, cudaStream_t s) {
  const size_t n = nblocks * 256;
  if (n) k_dequant_q6k<<<blocks_for(n, 256), 256, 0, s>>>(static_cast<const uint8_t*>(b), out, n);
  return cudaGetLastError();
}
cudaError_t op_f32_to_f16(const float* x, uint16_t* o, size_t n, cudaStream_t s) {
  if (n) k_f32_to_f16<<<blocks_for(n, 256), 256, 0, s>>>(x, o, n);
  return cudaGetLastError();
}
cudaError_t op_f16_to_f32(const uint16_t* x, float* o, size_t n, cudaStream_t s) {
  if (n) k_f16_to_f32<<<blocks_for(n, 256), 256, 0, s>>>(x, o, n);
  return cudaGetLastError();
}
cudaError_t op_rmsnorm(float* out, const float* x, const float* w, size_t n, size_t rows, float eps,
                       cudaStream_t s) {
  const int staged = n <= 12288;  // the row fits the default 48 KB of dynamic shared memory
  if (rows && n) k_rmsnorm<<<(unsigned)rows, 256, staged ? n * 4 : 0, s>>>(out, x, w, (int)n, eps, staged);
  return cudaGetLastError();
}
cudaError_t op_softmax(float* x, size_t n, size_t rows, cudaStream_t s) {
  const int staged = n <= 12288;
  if (rows && n) k_softmax<<<(unsigned)rows, 256, staged ? n * 4 : 0, s>>>(x, (int)n, staged);
  return cudaGetLastError();
}
cudaError_t op_swiglu(float* g, const float* u, size_t n, cudaStream_t s) {
  if (n) k_swiglu<<<blocks_for(n, 256), 256, 0, s>>>(g, u, n);
  return cudaGetLastError();
}
cudaError_t op_wait_selftest(unsigned* err, unsigned long long limit_ns, int kind, cudaStream_t s) {
  k_wait_selftest<<<1, 32, 0, s>>>(err, limit_ns, kind);
  return cudaGetLastError();
}
cudaError_t op_expf(const float* x, float* y, size_t n, cudaStream_t s) {
  if (n) k_expf<<<blocks_for(n, 256), 256, 0, s>>>(x, y, n);
  return cudaGetLastError();
}
cudaError_t op_expf_hash(unsigned long long* out, int chunk0, int nchunks, cudaStream_t s) {
  if (nchunks > 0) k_expf_hash<<<(nchunks + 31) / 32, 32, 0, s>>>(out, chunk0, nchunks);
  return cudaGetLastError();
}
cudaError_t op_argmax(const float* x, size_t n, unsigned long long* key_scratch, uint32_t* out, cudaStream_t s) {
  k_argmax_init<<<1, 1, 0, s>>>(key_scratch);
  if (n) {
    unsigned g = blocks_for(n, 256);
    if (g > 1184) g = 1184;
    k_argmax<<<g, 256, 0, s>>>(x, n, key_scratch);
  }
  k_argmax_finish<<<1, 1, 0, s>>>(key_scratch, out);
  return cudaGetLastError();
}

}  // namespace nrc
