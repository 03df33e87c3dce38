// Status handling, device checks and the small row kernels (RMSNorm, argmax).
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "axb_common.cuh"

namespace axb {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return AXB_OK;
  set_error("%s: %s", what, cudaGetErrorString(e));
  return AXB_ECUDA;
}

int launch_status(const char* what) { return cuda_status(cudaGetLastError(), what); }

int num_sms() {
  static std::atomic<int> cached[64];  // zero-initialized (static storage)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// modules.py:41-43 with an fp32 weight: rms = 1 / sqrt(mean(x^2) + eps),
// out = fp16((x * rms) * w), every op rounded in fp32.
__global__ void rmsnorm_kernel(const __half* __restrict__ x, const float* __restrict__ w, int K, float eps,
                               __half* __restrict__ out) {
  const int row = blockIdx.x;
  const __half* xr = x + (size_t)row * K;
  float ss = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    float v = __half2float(xr[k]);
    ss = __fmaf_rn(v, v, ss);
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(red[0], (float)K), eps)));
  for (int k = threadIdx.x; k < K; k += blockDim.x)
    out[(size_t)row * K + k] = __float2half_rn(__fmul_rn(__fmul_rn(__half2float(xr[k]), rms), w[k]));
}

// torch.argmax semantics: the first index of the maximum.
__global__ void argmax_kernel(const __half* __restrict__ x, int n, int ld, int32_t* __restrict__ out) {
  const int row = blockIdx.x;
  const __half* xr = x + (size_t)row * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int k = threadIdx.x; k < n; k += blockDim.x) {
    float v = __half2float(xr[k]);
    if (v > best || (v == best && k < bi)) {
      best = v;
      bi = k;
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    out[row] = bi == 0x7fffffff ? 0 : bi;
  }
}

int rmsnorm(const __half* x, const float* w, int M, int K, float eps, __half* out, cudaStream_t s) {
  AXB_CHECK_ARG(x && w && out && M >= 0 && K > 0, "rmsnorm: bad args");
  if (M == 0) return AXB_OK;
  rmsnorm_kernel<<<M, 256, 0, s>>>(x, w, K, eps, out);
  return launch_status("rmsnorm");
}

int argmax(const __half* x, int rows, int n, int ld, int32_t* out, cudaStream_t s) {
  AXB_CHECK_ARG(x && out && rows >= 0 && n > 0 && ld >= n, "argmax: bad args");
  if (rows == 0) return AXB_OK;
  argmax_kernel<<<rows, 1024, 0, s>>>(x, n, ld, out);
  return launch_status("argmax");
}

}  // namespace axb

extern "C" {

const char* axb_last_error(void) { return axb::g_err; }
int axb_version(void) { return 100; }

int axb_check_device(void) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return axb::cuda_status(e, "cudaGetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) {
    axb::set_error("device %d is sm_%d%d; this library is built for sm_100a (B200)", dev, major, minor);
    return AXB_EUNSUPPORTED;
  }
  return AXB_OK;
}

int axb_rmsnorm(const uint16_t* x, const float* w, int M, int K, float eps, uint16_t* out, void* stream) {
  return axb::rmsnorm((const __half*)x, w, M, K, eps, (__half*)out, (cudaStream_t)stream);
}

int axb_argmax(const uint16_t* x, int rows, int n, int ld, int32_t* out, void* stream) {
  return axb::argmax((const __half*)x, rows, n, ld, out, (cudaStream_t)stream);
}

}  // extern "C"
