// Shared device helpers for the AxiomLM-B200 kernels (sm_100a only).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/axb.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "AxiomLM-B200 kernels are written for sm_100a only"
#endif

namespace axb {

// ---------------------------------------------------------------- host side
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);
int launch_status(const char* what);
int num_sms();

// Per-device "set-up done" flags: bit d is set once device d has been prepared
// (function attributes raised, symbol addresses looked up).  Concurrent first
// calls on one device may both run the set-up, which is idempotent.
struct DeviceOnce {
  std::atomic<unsigned long long> mask{0};
  bool done(int dev) const {
    return dev >= 0 && dev < 64 && ((mask.load(std::memory_order_acquire) >> dev) & 1ull) != 0;
  }
  void set(int dev) {
    if (dev >= 0 && dev < 64) mask.fetch_or(1ull << dev, std::memory_order_acq_rel);
  }
};

#define AXB_CHECK_ARG(cond, ...)            \
  do {                                      \
    if (!(cond)) {                          \
      ::axb::set_error(__VA_ARGS__);        \
      return AXB_EINVAL;                    \
    }                                       \
  } while (0)

// Launch with programmatic dependent launch (PDL) enabled, so the kernel may
// start its weight prefetch while the previous kernel on the stream drains.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------- device side
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm volatile("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                          const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---- mbarrier + bulk async copy (TMA, non-tensor form) -------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// global -> shared bulk copy; dst/src 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// L2 policy for data read once per pass (weights, cached K/V rows): evict
// first, so the stream does not push out what is reused (the kernel's own
// instructions, activations, counters).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// bulk copy as bulk_g2s, with an L2 cache policy
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Bring [src, src + bytes) into L2 without a destination (bulk prefetch):
// src 16-byte aligned, bytes a multiple of 16
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 16-byte global -> shared copy through L2 (Ampere-style async copy), for
// scattered or padded destinations; completes per thread with cp_async_wait_all
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Bounded wait on an mbarrier phase: returns false if it did not complete
// within `limit` polls (the caller records an error instead of hanging).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, uint32_t limit) {
  uint32_t done = 0;
  for (uint32_t it = 0; it < limit; ++it) {
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    if (done) return true;
    __nanosleep(64);  // a waiting warp yields its issue slots to the SM's working warps
  }
  return false;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// e4m3fn byte -> float (exact), via the hardware pair conversion.
__device__ __forceinline__ float2 e4m3x2_to_float2(uint16_t two) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two), __NV_E4M3);
  return __half22float2(*reinterpret_cast<__half2*>(&h));
}
// float -> e4m3fn byte with round-half-even and no saturation: magnitudes
// above 464 (that would round to 480) and NaN/inf encode as NaN (0x7F | sign),
// the rule of torch's Tensor.to(float8_e4m3fn) used by the reference.
__device__ __forceinline__ uint8_t float_to_e4m3(float f) {
  const uint32_t bits = __float_as_uint(f);
  const uint32_t sign = (bits >> 24) & 0x80u;
  const float a = fabsf(f);
  if (!(a < 480.0f)) return (uint8_t)(sign | 0x7Fu);  // NaN, inf, >= 480
  if (a < 0.015625f) {                                  // subnormal range: quantum 2^-9
    return (uint8_t)(sign | (uint32_t)rintf(a * 512.0f));  // 0..8 (8 == min normal)
  }
  int e = (int)((__float_as_uint(a) >> 23) & 0xFF) - 127;  // [-6, 8]
  float m = rintf(ldexpf(a, 3 - e));                         // [8, 16]
  if (m >= 16.0f) {
    m = 8.0f;
    ++e;
  }
  uint32_t code = ((uint32_t)(e + 7) << 3) | ((uint32_t)m - 8u);
  if (code > 0x7Fu) code = 0x7Fu;
  return (uint8_t)(sign | code);
}

// Reference SiLU on fp32: x / (1 + exp(-x)).
__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }
// SwiGLU of fp16 gate / up values as the reference's fp16 tensors compute
// F.silu(g) * u (transformer.py:1187-1188): the silu rounded to fp16, then the
// product rounded to fp16
__device__ __forceinline__ __half swiglu_h(float g, float u) {
  return __float2half_rn(__fmul_rn(__half2float(__float2half_rn(silu_f(g))), u));
}

}  // namespace axb
