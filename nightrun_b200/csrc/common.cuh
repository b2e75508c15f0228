// Shared device helpers of the nrcuda library (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <set>
#include <tuple>

#define NRC_HD __host__ __device__ __forceinline__
#define NRC_DEV __device__ __forceinline__

namespace nrc {

// Raise kernel `fn`'s dynamic shared-memory limit to `bytes` once per
// (device, kernel, size). The setting is recorded only when the call
// succeeds, so a failed first attempt is retried by the next launch; the
// record is guarded for callers on several host threads.
inline cudaError_t ensure_smem_attr(const void* fn, int bytes) {
  static std::mutex mu;
  static std::set<std::tuple<int, const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> g(mu);
  const auto key = std::make_tuple(dev, fn, bytes);
  if (done.count(key)) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.insert(key);
  return e;
}

// ---------------------------------------------------------------- constants
constexpr int QK8_0 = 32;
constexpr int QK_K = 256;
constexpr int Q8_0_BYTES = 34;
constexpr int Q4K_BYTES = 144;
constexpr int Q6K_BYTES = 210;
constexpr int Q8K_BYTES = 292;
enum Fmt { FMT_Q8_0 = 1, FMT_Q4K = 2, FMT_Q6K = 3 };

// Error bits written to the per-device error word by kernels whose bounded
// waits expired (the kernel then returns without touching its outputs).
enum : unsigned { ERR_WAIT_FULL = 1u, ERR_WAIT_EMPTY = 2u, ERR_DRAIN = 4u };

// ------------------------------------------------------------ f16 (f16.rs)
// Exact reference conversions (crates/nr-tensor/src/f16.rs:3-56): RNE for
// normals, round-half-UP for subnormals, NaN keeps its payload on widening
// and becomes 0x7e00|sign on narrowing.
NRC_HD float f16_to_f32(uint32_t h) {
  uint32_t sign = (h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t frac = h & 0x3ffu;
  uint32_t out;
  if (exp == 0) {
    if (frac == 0) {
      out = sign;
    } else {
#ifdef __CUDA_ARCH__
      uint32_t msb = 31 - __clz(frac);
#else
      uint32_t msb = 31 - __builtin_clz(frac);
#endif
      out = sign | ((127 - 24 + msb) << 23) | ((frac << (23 - msb)) & 0x7fffffu);
    }
  } else if (exp == 0x1f) {
    out = sign | 0x7f800000u | (frac << 13);
  } else {
    out = sign | ((exp + 112) << 23) | (frac << 13);
  }
#ifdef __CUDA_ARCH__
  return __uint_as_float(out);
#else
  float f;
  __builtin_memcpy(&f, &out, 4);
  return f;
#endif
}

NRC_HD uint16_t f32_to_f16(float v) {
#ifdef __CUDA_ARCH__
  uint32_t bits = __float_as_uint(v);
#else
  uint32_t bits;
  __builtin_memcpy(&bits, &v, 4);
#endif
  uint32_t sign = (bits >> 16) & 0x8000u;
  int32_t exp = (int32_t)((bits >> 23) & 0xff);
  uint32_t frac = bits & 0x7fffffu;
  if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (frac ? 0x200u : 0u));
  int32_t e = exp - 112;
  if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    uint32_t f = frac | 0x800000u;
    uint32_t shift = (uint32_t)(14 - e);
    return (uint16_t)(sign | ((f + (1u << (shift - 1))) >> shift));
  }
  uint32_t out = sign | ((uint32_t)e << 10) | (frac >> 13);
  uint32_t round = frac & 0x1fffu;
  if (round > 0x1000u || (round == 0x1000u && (out & 1u))) out += 1;
  return (uint16_t)out;
}

// Rust `f as i32`: truncate toward zero, saturate, NaN -> 0 (cvt.rzi.s32.f32
// has exactly these semantics).
NRC_DEV int32_t rust_f2i(float f) { return __float2int_rz(f); }

// Exact int -> float for |v| < 2^24 is cvt.rn; used where the reference casts.
NRC_DEV float i2f(int32_t v) { return __int2float_rn(v); }

// q8::quantize (q8.rs:27-44) of one 32-value block held one value per lane
// of a full warp: d = f16(amax / 127) (amax folded from 0, NaN ignored like
// f32::max), q = v / d rounded half away from zero, saturated to +-127.
NRC_DEV void warp_quant_q8_block(float v, int lane, uint8_t* blk) {
  float amax = fmaxf(0.0f, fabsf(v));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const uint16_t dbits = f32_to_f16(__fdiv_rn(amax, 127.0f));
  const float d = f16_to_f32(dbits);
  const float inv = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  const float xsv = __fmul_rn(v, inv);
  const float r = xsv >= 0.0f ? __fadd_rn(xsv, 0.5f) : __fsub_rn(xsv, 0.5f);
  int q = rust_f2i(r);
  q = q < -127 ? -127 : (q > 127 ? 127 : q);
  blk[2 + lane] = (uint8_t)(int8_t)q;
  if (lane == 0) {
    blk[0] = (uint8_t)(dbits & 0xffu);
    blk[1] = (uint8_t)(dbits >> 8);
  }
}

// ------------------------------------------------------------ misc device
NRC_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

NRC_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch: wait for the upstream grid's memory, and let
// the downstream grid start its (weight-prefetch) prologue early.
NRC_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
NRC_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------ mbarriers + bulk copies
NRC_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
NRC_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
NRC_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
NRC_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
NRC_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
NRC_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `limit_ns` of global time and returns false.
NRC_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > limit_ns) return false;
  }
  return true;
}
// Shared-memory flags with acquire / release ordering at CTA scope: a
// cheaper hand-off than an mbarrier when one warp publishes data to another.
NRC_DEV uint32_t ld_acquire_smem(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
NRC_DEV void st_release_smem(uint32_t* p, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
// Bounded wait until the flag reaches `target` (flags only grow): gives up
// after `limit_ns` of global time (the clock is read every 1024 polls).
NRC_DEV bool flag_wait_geq(const uint32_t* p, uint32_t target, uint64_t limit_ns = 2000000000ull) {
  if (ld_acquire_smem(p) >= target) return true;
  uint64_t t0 = 0;
  for (uint32_t k = 1;; k++) {
    if (ld_acquire_smem(p) >= target) return true;
    if ((k & 1023u) == 0) {
      const uint64_t t = globaltimer();
      if (t0 == 0)
        t0 = t;
      else if (t - t0 > limit_ns)
        return false;
    }
  }
}

// 1-D TMA bulk copy global -> shared, completion counted on `bar` (tx bytes).
// dst, src 16-byte aligned; bytes a multiple of 16. No cluster multicast.
NRC_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// 16-byte asynchronous copy global -> shared through L2 (both addresses
// 16-byte aligned). Many small copies per stage cost one LSU request each,
// where one bulk copy per small span would queue behind the TMA unit.
NRC_DEV void cp_async16(void* dst, const void* src, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "l"(policy)
               : "memory");
}
// One arrival on `bar` once all of this thread's earlier cp.async copies
// have landed (.noinc: the arrival is part of the barrier's expected count).
NRC_DEV void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
NRC_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Fire-and-forget prefetch of [src, src + bytes) into L2 (both 16-byte
// multiples); nothing waits for it.
NRC_DEV void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// L2 policy for weights that are streamed once per step: evict first, so the
// activations and KV rows stay resident.
NRC_DEV uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Named barrier among the first `nthreads` threads (consumer warps only).
NRC_DEV void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Arrive at named barrier `id` without waiting (the waiting side uses
// named_sync with the same total thread count).
NRC_DEV void named_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------ reductions
NRC_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
NRC_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Orderable key for a float (NaN and -inf excluded by the caller): larger key =
// larger value; ties broken toward the lower index (vec::argmax keeps the
// first maximum, crates/nr-tensor/src/vec.rs:80-90). -0.0 and +0.0 compare
// equal there, so both map to the key of +0.0.
NRC_DEV unsigned long long argmax_key(float v, uint32_t idx) {
  uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
  uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)o << 32) | (unsigned long long)(0xffffffffu - idx);
}
NRC_DEV bool argmax_candidate(float v) { return !(v != v) && v != -INFINITY; }
NRC_HD uint32_t argmax_index(unsigned long long key) {
  return key == 0ull ? 0u : (uint32_t)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
}

}  // namespace nrc
