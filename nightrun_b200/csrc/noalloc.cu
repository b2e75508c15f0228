// nrc_matmul_q8_0_noalloc: kernels::matmul_q8 (crates/nr-tensor/src/kernels.rs:91-143)
// with the same results as nrc_matmul_q8_0, allocating nothing. Every byte of
// working memory it needs lives in one file-scope device array:
//
//   [0, 256)                       error word (uint32 at 0) of the bounded waits
//   [256, 256 + 64·MAX_COLS)       tensor-core activation tiles of one 64-token pass
//   [.., + 64·(MAX_COLS/32)·4)     their f32 block scales
//
// Only the error word must start at zero: static device storage is zeroed
// when the module loads, and each call clears it again (stream-ordered
// memset) before its kernels run. The tiles and scales are fully rewritten
// by every pass before they are read.
//
// The device address of the array is resolved once per device with
// cudaGetSymbolAddress. Calls that overlap in time on one device (different
// streams or host threads) share the array and race; the caller serializes
// them. Every call blocks the host until its kernels have finished (it reads
// the error word back and synchronizes the stream, so an expired bounded wait
// is reported by the same call); it therefore cannot be made inside a stream
// capture.
#include <mutex>

#include "common.cuh"
#include "gemv.cuh"
#include "mma.cuh"
#include "nrcuda.h"

using namespace nrc;

int nrc_fail_api(int code, const char* fmt, ...);  // engine-side error slot

namespace {

constexpr size_t ERR_BYTES = 256;
constexpr size_t MAX_TOK = 64;  // tokens per tensor-core pass
constexpr size_t XQ_BYTES = MAX_TOK * NRC_NOALLOC_MAX_COLS;
constexpr size_t XD_BYTES = MAX_TOK * (NRC_NOALLOC_MAX_COLS / 32) * 4;
static_assert(ERR_BYTES + XQ_BYTES + XD_BYTES == NRC_NOALLOC_SCRATCH_BYTES, "scratch layout");

static __device__ __align__(256) uint8_t g_noalloc_scratch[NRC_NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEV = 64;

int scratch_addr(uint8_t** out) {
  static std::mutex mu;
  static uint8_t* addr[MAX_DEV] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEV)
    return nrc_fail_api(NRC_ERR_CUDA, "no usable CUDA device");
  std::lock_guard<std::mutex> g(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return nrc_fail_api(NRC_ERR_CUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    addr[dev] = static_cast<uint8_t*>(p);
  }
  *out = addr[dev];
  return NRC_OK;
}

int rc_of(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return NRC_OK;
  return nrc_fail_api(NRC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace

extern "C" int nrc_matmul_q8_0_noalloc(float* y, const void* w, const void* xs, size_t rows, size_t cols,
                                       size_t batch, void* stream) {
  if (!y || (!w && rows) || (!xs && batch)) return nrc_fail_api(NRC_ERR_INVALID, "null pointer");
  if (cols % 32) return nrc_fail_api(NRC_ERR_INVALID, "cols %zu not a multiple of 32", cols);
  if (cols > NRC_NOALLOC_MAX_COLS)
    return nrc_fail_api(NRC_ERR_INVALID, "cols %zu exceeds the static scratch limit of %d columns", cols,
                        NRC_NOALLOC_MAX_COLS);
  if (rows > 0x7fffffff || batch > 0x7fffffff) return nrc_fail_api(NRC_ERR_INVALID, "shape too large");
  if (rows == 0 || batch == 0) return NRC_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cols == 0) return rc_of(cudaMemsetAsync(y, 0, rows * batch * 4, s), "memset");
  uint8_t* base = nullptr;
  int rc = scratch_addr(&base);
  if (rc) return rc;
  unsigned* err = reinterpret_cast<unsigned*>(base);
  uint8_t* xq = base + ERR_BYTES;
  float* xd = reinterpret_cast<float*>(base + ERR_BYTES + XQ_BYTES);
  if ((rc = rc_of(cudaMemsetAsync(err, 0, 4, s), "clear error word"))) return rc;
  const size_t bpr = cols / 32;
  if (batch > 8 && cols % 256 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
    // Tensor-core path: 64 tokens per pass through the static tiles.
    const int tiles = (int)((rows + 127) / 128);
    for (size_t t0 = 0; t0 < batch && !rc; t0 += MAX_TOK) {
      const int nt = (int)(batch - t0 < MAX_TOK ? batch - t0 : MAX_TOK);
      int NS, ntg;
      mma_choose(tiles, nt, &NS, &ntg);
      rc = rc_of(mma_pack_q8_run(static_cast<const uint8_t*>(xs) + t0 * bpr * 34, nt, (int)cols, NS, ntg, xq, xd, s),
                 "mma pack");
      if (rc) break;
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
      m.err = err;
      rc = rc_of(mma_q8_run(m, s, false), "mma launch");
    }
  } else {
    for (size_t t0 = 0; t0 < batch && !rc; t0 += 8) {
      GemvArgs a{};
      a.fmt = FMT_Q8_0;
      a.K = (int)cols;
      a.nt = (int)(batch - t0 < 8 ? batch - t0 : 8);
      a.seg[0] = GemvSegArg{w, y + t0 * rows, (int)rows, (int)rows};
      a.nseg = 1;
      a.xq = static_cast<const uint8_t*>(xs) + t0 * bpr * 34;
      a.epi = EPI_STORE;
      a.scale = 1.0f;
      a.err = err;
      rc = rc_of(gemv_run(a, s, false), "gemv launch");
    }
  }
  if (rc) return rc;
  unsigned word = 0;
  if ((rc = rc_of(cudaMemcpyAsync(&word, err, 4, cudaMemcpyDeviceToHost, s), "read error word"))) return rc;
  if ((rc = rc_of(cudaStreamSynchronize(s), "synchronize"))) return rc;
  if (word) return nrc_fail_api(NRC_ERR_DEVICE, "kernel wait expired (error bits 0x%x)", word);
  return NRC_OK;
}
