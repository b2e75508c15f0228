// Kernel-level C ABI (include/nrcuda.h, "nr-tensor" section): the reference's
// crates/nr-tensor entry points over device buffers.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>

#include <map>
#include <mutex>
#include <string>

#include "common.cuh"
#include "gemv.cuh"
#include "mma.cuh"
#include "nrcuda.h"
#include "ops.cuh"
#include "sample.cuh"

using namespace nrc;

int nrc_fail_api(int code, const char* fmt, ...);  // engine-side error slot

namespace {

// Per-device scratch: the kernel error word and the argmax key.
struct DevScratch {
  unsigned* err = nullptr;
  unsigned long long* key = nullptr;
  unsigned long long* cand = nullptr;  // sampler candidates (SAMPLE_MAX_N logits)
};

int dev_scratch(DevScratch* out) {
  static std::mutex mu;
  static std::map<int, DevScratch> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nrc_fail_api(NRC_ERR_CUDA, "no CUDA device");
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) {
    *out = it->second;
    return NRC_OK;
  }
  DevScratch s;
  void* p = nullptr;
  const size_t bytes = 256 + sample_scratch_bytes(SAMPLE_MAX_N);
  if (cudaMalloc(&p, bytes) != cudaSuccess) return nrc_fail_api(NRC_ERR_ALLOC, "scratch allocation failed");
  cudaMemset(p, 0, 256);
  s.err = static_cast<unsigned*>(p);
  s.key = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(p) + 64);
  s.cand = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(p) + 256);
  cache[dev] = s;
  *out = s;
  return NRC_OK;
}

int cuda_rc(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return NRC_OK;
  return nrc_fail_api(NRC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

int matvec_common(int fmt, float* y, const void* w, const void* x, size_t rows, size_t cols, size_t batch,
                  void* stream) {
  const size_t blk = fmt == FMT_Q8_0 ? 32 : 256;
  if (!y || (!w && rows) || (!x && batch)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  if (cols % blk) return nrc_fail_api(NRC_ERR_INVALID, "cols %zu not a multiple of %zu", cols, blk);
  if (rows > 0x7fffffff || cols > 0x7fffffff || batch > 0x7fffffff)
    return nrc_fail_api(NRC_ERR_INVALID, "shape too large");
  if (fmt != FMT_Q8_0 && (reinterpret_cast<uintptr_t>(x) & 3))
    return nrc_fail_api(NRC_ERR_INVALID, "Q8_K activations must be 4-byte aligned");
  if (rows == 0 || batch == 0) return NRC_OK;
  if (cols == 0) return cuda_rc(cudaMemsetAsync(y, 0, rows * batch * 4, S(stream)), "memset");
  DevScratch sc;
  int rc = dev_scratch(&sc);
  if (rc) return rc;
  const size_t xblk = fmt == FMT_Q8_0 ? 34 : 292;
  if (fmt == FMT_Q8_0 && batch > 8 && cols % 256 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
    // Tensor-core path (tcgen05 kind::i8), 64 tokens per pass.
    const int tiles = (int)((rows + 127) / 128);
    for (size_t t0 = 0; t0 < batch; t0 += 64) {
      const int nt = (int)(batch - t0 < 64 ? batch - t0 : 64);
      int NS, ntg;
      mma_choose(tiles, nt, &NS, &ntg);
      const size_t bpr = cols / 32;
      uint8_t* xq = nullptr;
      float* xd = nullptr;
      if (cudaMallocAsync((void**)&xq, (size_t)ntg * NS * cols, S(stream)) != cudaSuccess)
        return nrc_fail_api(NRC_ERR_ALLOC, "activation tile allocation failed");
      if (cudaMallocAsync((void**)&xd, (size_t)ntg * NS * bpr * 4, S(stream)) != cudaSuccess) {
        cudaFreeAsync(xq, S(stream));
        return nrc_fail_api(NRC_ERR_ALLOC, "activation scale allocation failed");
      }
      rc = cuda_rc(mma_pack_q8_run(static_cast<const uint8_t*>(x) + t0 * bpr * 34, nt, (int)cols, NS, ntg, xq, xd,
                                   S(stream)),
                   "mma pack");
      MmaArgs m{};
      m.seg[0] = MmaSeg{w, y + t0 * rows, (int)rows, (int)rows};
      m.nseg = 1;
      m.K = (int)cols;
      m.xq = xq;
      m.xd = xd;
      m.nt = nt;
      m.NS = NS;
      m.ntg = ntg;
      m.epi = EPI_STORE;
      m.scale = 1.0f;
      m.err = sc.err;
      if (!rc) rc = cuda_rc(mma_q8_run(m, S(stream), false), "mma launch");
      cudaFreeAsync(xq, S(stream));
      cudaFreeAsync(xd, S(stream));
      if (rc) return rc;
    }
    return NRC_OK;
  }
  if (fmt != FMT_Q8_0 && batch > 8 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
    // Tensor-core path (tcgen05 kind::i8 per sub-block), one pass per NS x ntg tokens.
    const int NS = mma_kq_ns(fmt);
    const size_t nsb = cols / 256;
    const size_t per = (size_t)NS * 8;  // tokens per pass: eight token groups
    for (size_t t0 = 0; t0 < batch; t0 += per) {
      const int nt = (int)(batch - t0 < per ? batch - t0 : per);
      const int ntg = (nt + NS - 1) / NS;
      uint8_t* xq = nullptr;
      float* xd = nullptr;
      int* xb = nullptr;
      const int masked = fmt == FMT_Q6K ? 1 : 0;
      if (cudaMallocAsync((void**)&xq, (size_t)ntg * NS * cols * (masked ? 2 : 1), S(stream)) != cudaSuccess)
        return nrc_fail_api(NRC_ERR_ALLOC, "activation tile allocation failed");
      if (cudaMallocAsync((void**)&xd, (size_t)ntg * NS * nsb * 4, S(stream)) != cudaSuccess) {
        cudaFreeAsync(xq, S(stream));
        return nrc_fail_api(NRC_ERR_ALLOC, "activation scale allocation failed");
      }
      if (cudaMallocAsync((void**)&xb, (size_t)ntg * NS * nsb * 32, S(stream)) != cudaSuccess) {
        cudaFreeAsync(xq, S(stream));
        cudaFreeAsync(xd, S(stream));
        return nrc_fail_api(NRC_ERR_ALLOC, "activation sum allocation failed");
      }
      rc = cuda_rc(mma_kq_pack_run(static_cast<const uint8_t*>(x) + t0 * nsb * 292, nt, (int)cols, NS, ntg, masked, xq,
                                   xd, xb, S(stream)),
                   "kq pack");
      MmaKqArgs m{};
      m.fmt = fmt;
      m.seg[0] = MmaSeg{w, y + t0 * rows, (int)rows, (int)rows};
      m.nseg = 1;
      m.K = (int)cols;
      m.xq = xq;
      m.xd = xd;
      m.xb = xb;
      m.nt = nt;
      m.NS = NS;
      m.ntg = ntg;
      m.epi = EPI_STORE;
      m.scale = 1.0f;
      m.err = sc.err;
      if (!rc) rc = cuda_rc(mma_kq_run(m, S(stream), false), "kq launch");
      cudaFreeAsync(xq, S(stream));
      cudaFreeAsync(xd, S(stream));
      cudaFreeAsync(xb, S(stream));
      if (rc) return rc;
    }
    return NRC_OK;
  }
  for (size_t t0 = 0; t0 < batch; t0 += 8) {
    GemvArgs a{};
    a.fmt = fmt;
    a.K = (int)cols;
    a.nt = (int)(batch - t0 < 8 ? batch - t0 : 8);
    a.seg[0] = GemvSegArg{w, y + t0 * rows, (int)rows, (int)rows};
    a.nseg = 1;
    a.xq = static_cast<const uint8_t*>(x) + t0 * (cols / blk) * xblk;
    a.epi = EPI_STORE;
    a.scale = 1.0f;
    a.err = sc.err;
    rc = cuda_rc(gemv_run(a, S(stream), false), "gemv launch");
    if (rc) return rc;
  }
  return NRC_OK;
}

struct RopeCS {
  float v[128];
};
__global__ void k_rope_one_param(float* x, int len, int hd, int style, const RopeCS cs) {
  const int half = hd / 2;
  const int npairs = (len / hd) * half;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < npairs; i += gridDim.x * blockDim.x) {
    const int h = i / half, p = i % half;
    float* head = x + (size_t)h * hd;
    const int ia = style == 0 ? 2 * p : p, ib = style == 0 ? 2 * p + 1 : p + half;
    const float a = head[ia], b = head[ib], c = cs.v[p], s = cs.v[half + p];
    head[ia] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    head[ib] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
  }
}

}  // namespace

extern "C" {

int nrc_quantize_q8_0(const float* x, void* out, size_t n, void* stream) {
  if (n % 32) return nrc_fail_api(NRC_ERR_INVALID, "n %zu not a multiple of 32", n);
  if (n && (!x || !out)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  return cuda_rc(op_quantize_q8_0(x, out, n, S(stream)), "quantize_q8_0");
}
int nrc_dequantize_q8_0(const void* b, float* out, size_t n, void* stream) {
  if (n % 32) return nrc_fail_api(NRC_ERR_INVALID, "n %zu not a multiple of 32", n);
  if (n && (!b || !out)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  return cuda_rc(op_dequantize_q8_0(b, out, n, S(stream)), "dequantize_q8_0");
}
int nrc_quantize_q8k(const float* x, void* out, size_t n, void* stream) {
  if (n % 256) return nrc_fail_api(NRC_ERR_INVALID, "n %zu not a multiple of 256", n);
  if (n && (!x || !out)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  if (reinterpret_cast<uintptr_t>(out) & 3) return nrc_fail_api(NRC_ERR_INVALID, "Q8_K output must be 4-byte aligned");
  return cuda_rc(op_quantize_q8k(x, out, n, S(stream)), "quantize_q8k");
}
int nrc_dequant_q4k(const void* b, float* out, size_t nb, void* stream) {
  if (nb && (!b || !out)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  return cuda_rc(op_dequant_q4k(b, out, nb, S(stream)), "dequant_q4k");
}
int nrc_dequant_q6k(const void* b, float* out, size_t nb, void* stream) {
  if (nb && (!b || !out)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  return cuda_rc(op_dequant_q6k(b, out, nb, S(stream)), "dequant_q6k");
}
int nrc_matvec_q8_0(float* y, const void* w, const void* x, size_t rows, size_t cols, void* stream) {
  return matvec_common(FMT_Q8_0, y, w, x, rows, cols, 1, stream);
}
int nrc_matmul_q8_0(float* y, const void* w, const void* xs, size_t rows, size_t cols, size_t batch, void* stream) {
  return matvec_common(FMT_Q8_0, y, w, xs, rows, cols, batch, stream);
}
int nrc_matvec_q4k(float* y, const void* w, const void* x, size_t rows, size_t cols, void* stream) {
  return matvec_common(FMT_Q4K, y, w, x, rows, cols, 1, stream);
}
int nrc_matvec_q6k(float* y, const void* w, const void* x, size_t rows, size_t cols, void* stream) {
  return matvec_common(FMT_Q6K, y, w, x, rows, cols, 1, stream);
}
int nrc_matmul_q4k(float* y, const void* w, const void* xs, size_t rows, size_t cols, size_t batch, void* stream) {
  return matvec_common(FMT_Q4K, y, w, xs, rows, cols, batch, stream);
}
int nrc_matmul_q6k(float* y, const void* w, const void* xs, size_t rows, size_t cols, size_t batch, void* stream) {
  return matvec_common(FMT_Q6K, y, w, xs, rows, cols, batch, stream);
}
int nrc_f32_to_f16(const float* x, uint16_t* out, size_t n, void* stream) {
  if (n && (!x || !out)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  return cuda_rc(op_f32_to_f16(x, out, n, S(stream)), "f32_to_f16");
}
int nrc_f16_to_f32(const uint16_t* x, float* out, size_t n, void* stream) {
  if (n && (!x || !out)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  return cuda_rc(op_f16_to_f32(x, out, n, S(stream)), "f16_to_f32");
}
int nrc_rmsnorm(float* out, const float* x, const float* w, size_t n, size_t rows, float eps, void* stream) {
  if (rows && n && (!out || !x || !w)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  return cuda_rc(op_rmsnorm(out, x, w, n, rows, eps, S(stream)), "rmsnorm");
}
int nrc_softmax(float* x, size_t n, size_t rows, void* stream) {
  if (rows && n && !x) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  return cuda_rc(op_softmax(x, n, rows, S(stream)), "softmax");
}
int nrc_swiglu(float* g, const float* u, size_t n, void* stream) {
  if (n && (!g || !u)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  return cuda_rc(op_swiglu(g, u, n, S(stream)), "swiglu");
}
int nrc_argmax(const float* x, size_t n, uint32_t* out_dev, void* stream) {
  if (!out_dev || (n && !x)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  DevScratch sc;
  int rc = dev_scratch(&sc);
  if (rc) return rc;
  return cuda_rc(op_argmax(x, n, sc.key, out_dev, S(stream)), "argmax");
}

int nrc_sample(const float* logits, size_t n, float temperature, float top_p, uint64_t* rng_dev, uint32_t* out_dev,
               void* stream) {
  if (!out_dev || !rng_dev || (n && !logits)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  if (n == 0 || n > (size_t)SAMPLE_MAX_N)
    return nrc_fail_api(NRC_ERR_INVALID, "sampler over %zu logits (1..%d supported)", n, SAMPLE_MAX_N);
  DevScratch sc;
  int rc = dev_scratch(&sc);
  if (rc) return rc;
  if (temperature <= 0.0f) return cuda_rc(op_argmax(logits, n, sc.key, out_dev, S(stream)), "argmax");
  SampleArgs a{logits, (int)n, temperature, top_p, reinterpret_cast<unsigned long long*>(rng_dev), sc.cand, out_dev,
               nullptr};
  return cuda_rc(sample_run(a, S(stream), false), "sample");
}

int nrc_rope_freqs(float* out, size_t head_dim, float theta, float factor, float low, float high, float orig) {
  if (!out || head_dim % 2) return nrc_fail_api(NRC_ERR_INVALID, "bad rope_freqs arguments");
  const size_t half = head_dim / 2;
  const float PI = 3.14159265358979323846f;
  for (size_t i = 0; i < half; i++) {
    volatile float exponent = -2.0f * (float)i / (float)head_dim;
    float freq = powf(theta, exponent);
    if (factor > 0.0f) {
      const float wavelen = 2.0f * PI / freq;
      if (wavelen > orig / low) {
        freq /= factor;
      } else if (wavelen > orig / high) {
        volatile float smooth = (orig / wavelen - low) / (high - low);
        volatile float a = (1.0f - smooth) * freq;
        volatile float b = a / factor;
        volatile float c = smooth * freq;
        freq = b + c;
      }
    }
    out[i] = freq;
  }
  return NRC_OK;
}

int nrc_rope_apply(float* x, size_t len, size_t head_dim, const float* freqs, size_t pos, int style, void* stream) {
  if (!x || !freqs || head_dim == 0 || head_dim % 2 || head_dim > 128 || (style != 0 && style != 1))
    return nrc_fail_api(NRC_ERR_INVALID, "bad rope_apply arguments");
  const size_t half = head_dim / 2;
  RopeCS cs;
  for (size_t i = 0; i < half; i++) {
    volatile float angle = (float)pos * freqs[i];
    sincosf(angle, &cs.v[half + i], &cs.v[i]);
  }
  const int npairs = (int)((len / head_dim) * half);
  if (npairs == 0) return NRC_OK;
  k_rope_one_param<<<(npairs + 255) / 256, 256, 0, S(stream)>>>(x, (int)len, (int)head_dim, style, cs);
  return cuda_rc(cudaGetLastError(), "rope_apply");
}

int nrc_expf(const float* x, float* y, size_t n, void* stream) {
  if (n && (!x || !y)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  return cuda_rc(op_expf(x, y, n, S(stream)), "expf");
}

int nrc_expf_hash(uint64_t* out_dev, int chunk0, int nchunks, void* stream) {
  if (!out_dev || chunk0 < 0 || nchunks < 0 || chunk0 + nchunks > 4096)
    return nrc_fail_api(NRC_ERR_INVALID, "bad expf_hash range");
  return cuda_rc(op_expf_hash(reinterpret_cast<unsigned long long*>(out_dev), chunk0, nchunks, S(stream)),
                 "expf_hash");
}

int nrc_wait_selftest(int kind, uint64_t limit_ns, void* stream) {
  if (kind != 0 && kind != 1) return nrc_fail_api(NRC_ERR_INVALID, "kind must be 0 or 1");
  if (limit_ns == 0 || limit_ns > 10000000000ull) return nrc_fail_api(NRC_ERR_INVALID, "limit outside 1 ns .. 10 s");
  DevScratch sc;
  int rc = dev_scratch(&sc);
  if (rc) return rc;
  if ((rc = cuda_rc(op_wait_selftest(sc.err, limit_ns, kind, S(stream)), "wait self-test"))) return rc;
  return nrc_sync_check(stream);
}

int nrc_sync_check(void* stream) {
  if (cudaStreamSynchronize(S(stream)) != cudaSuccess) return nrc_fail_api(NRC_ERR_CUDA, "stream synchronize failed");
  DevScratch sc;
  int rc = dev_scratch(&sc);
  if (rc) return rc;
  unsigned err = 0;
  if (cudaMemcpy(&err, sc.err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return nrc_fail_api(NRC_ERR_CUDA, "read error word");
  if (err) {
    cudaMemset(sc.err, 0, 4);
    return nrc_fail_api(NRC_ERR_DEVICE, "kernel wait expired (error bits 0x%x)", err);
  }
  return NRC_OK;
}

}  // extern "C"
