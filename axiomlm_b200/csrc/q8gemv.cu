// Q8_G64 GEMV / small-M GEMM: y = x W^T with the reference's 8-bit affine
// weights, for the tied lm_head (the reference default: the token embedding
// matrix, packed Q8_G64, doubles as the output projection) and other Q8
// projections.
//
// Replaces qmv_q8_g64 / qmm_q8_g64 (axiomlm/kernels/quant.py:201-233; Metal
// qmv_q8_g64_half_kernel :1941).  The weights stay in the reference's own
// layout: w_packed (N, K/4) int32 with code k of a row in byte k % 4 of word
// k / 4, scales_biases (N, K/64, 2) fp16.  Each weight is dequantized exactly
// as dequantize_q8_g64 does (quant.py:132-147): fp16(fp32(q) * fp32(s) +
// fp32(b)), the product exact in fp32 and the sum rounded to fp32, then to
// fp16; the products with the fp16 activations accumulate in fp32 and the
// output is rounded to fp16 once, as F.linear in fp16 does.  An optional
// bias is added to that fp16 output and rounded again, as _qlin does for Q8
// projections (transformer.py:1026-1029: y = qmv_q8_g64(x) + bias, in fp16).
//
// One warp per output row at a time: lane l reads 16 codes (one 16-byte load)
// at k = 16 (l + 32 i), the four lanes of a 64-wide group share its scale and
// bias, and the warp's partial sums meet in a shuffle tree.  The activations
// of up to 8 tokens at a time are staged in shared memory.  8-bit weights are
// read once, in 512-byte coalesced warp requests.
#include <algorithm>

#include "axb_common.cuh"

namespace axb {

constexpr int kQ8Warps = 8;
constexpr int kQ8MaxMb = 8;  // tokens per pass over the weights

__device__ __forceinline__ float q8_weight(uint32_t word, int byte, float s, float b) {
  const float q = (float)((word >> (8 * byte)) & 0xFFu);
  return __half2float(__float2half_rn(__fadd_rn(__fmul_rn(q, s), b)));
}

// x: (M, ldx) fp16 rows, w: (N, K/4) int32, sb: (N, K/64) half2, y: (M, ldy) fp16,
// bias: (N) fp16 or null
__global__ void __launch_bounds__(kQ8Warps * 32) q8_gemv_kernel(const __half* __restrict__ x, int ldx, int m0,
                                                                   int Mb, int K, const uint32_t* __restrict__ w,
                                                                   const __half2* __restrict__ sb, int N,
                                                                   __half* __restrict__ y, int ldy,
                                                                   const __half* __restrict__ bias) {
  extern __shared__ __align__(16) __half xs[];  // (Mb, K)
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < Mb * K / 8; i += blockDim.x) {
    const int m = i / (K / 8), c = i % (K / 8);
    reinterpret_cast<uint4*>(xs)[i] = __ldg(reinterpret_cast<const uint4*>(x + (size_t)(m0 + m) * ldx) + c);
  }
  __syncthreads();
  const int K16 = K / 16;  // 16-code chunks per row
  for (int row = blockIdx.x * kQ8Warps + wid; row < N; row += gridDim.x * kQ8Warps) {
    const uint4* wr = reinterpret_cast<const uint4*>(w + (size_t)row * (K / 4));
    const __half2* sr = sb + (size_t)row * (K / 64);
    float acc[kQ8MaxMb];
#pragma unroll
    for (int m = 0; m < kQ8MaxMb; ++m) acc[m] = 0.f;
    for (int c = lane; c < K16; c += 32) {
      const uint4 wv = __ldg(wr + c);
      const float2 s_b = __half22float2(__ldg(sr + (c >> 2)));
      float wf[16];
      const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) wf[4 * j + e] = q8_weight(words[j], e, s_b.x, s_b.y);
#pragma unroll
      for (int m = 0; m < kQ8MaxMb; ++m) {
        if (m >= Mb) break;
        const uint4* xr = reinterpret_cast<const uint4*>(xs + (size_t)m * K + 16 * c);
        const uint4 xv[2] = {xr[0], xr[1]};
        const __half2* xh = reinterpret_cast<const __half2*>(xv);
        float a = acc[m];
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const float2 xf = __half22float2(xh[p]);
          a = __fmaf_rn(wf[2 * p], xf.x, a);
          a = __fmaf_rn(wf[2 * p + 1], xf.y, a);
        }
        acc[m] = a;
      }
    }
#pragma unroll
    for (int m = 0; m < kQ8MaxMb; ++m) {
      if (m >= Mb) break;
      const float v = warp_sum(acc[m]);
      if (lane == 0) {
        __half o = __float2half_rn(v);
        if (bias) o = __float2half_rn(__fadd_rn(__half2float(o), __half2float(bias[row])));
        y[(size_t)(m0 + m) * ldy + row] = o;
      }
    }
  }
}

int q8_gemv(const __half* x, int ldx, int M, int K, const uint32_t* w, const __half2* sb, int N, __half* y, int ldy,
            cudaStream_t st, const __half* bias) {
  AXB_CHECK_ARG(x && w && sb && y, "q8_gemv: null pointer");
  AXB_CHECK_ARG(M >= 1 && N >= 1 && K >= 64 && K % 64 == 0 && ldx >= K && ldy >= N && ldx % 8 == 0,
                "q8_gemv: bad shape (M %d, N %d, K %d, ldx %d, ldy %d)", M, N, K, ldx, ldy);
  AXB_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0,
                "q8_gemv: x and w must be 16-byte aligned");
  const size_t smem = (size_t)std::min(M, kQ8MaxMb) * K * sizeof(__half);
  AXB_CHECK_ARG(smem <= 200 * 1024, "q8_gemv: K %d too large for the staged activations", K);
  static DeviceOnce once;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!once.done(dev)) {
    cudaError_t e = cudaFuncSetAttribute(q8_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return cuda_status(e, "q8_gemv attribute");
    once.set(dev);
  }
  const int blocks = (int)std::min<long long>((N + kQ8Warps - 1) / kQ8Warps, (long long)num_sms() * 4);
  for (int m0 = 0; m0 < M; m0 += kQ8MaxMb) {
    const int Mb = std::min(kQ8MaxMb, M - m0);
    q8_gemv_kernel<<<blocks, kQ8Warps * 32, (size_t)Mb * K * sizeof(__half), st>>>(x, ldx, m0, Mb, K, w, sb, N, y,
                                                                                     ldy, bias);
    if (int rc = cuda_status(cudaGetLastError(), "q8_gemv launch")) return rc;
  }
  return AXB_OK;
}

}  // namespace axb

extern "C" int axb_q8g64_gemv(const void* x, int ldx, int M, int K, const int32_t* w_packed,
                              const uint16_t* scales_biases, int N, void* y, int ldy, void* stream) {
  return axb::q8_gemv(static_cast<const __half*>(x), ldx, M, K, reinterpret_cast<const uint32_t*>(w_packed),
                      reinterpret_cast<const __half2*>(scales_biases), N, static_cast<__half*>(y), ldy,
                      static_cast<cudaStream_t>(stream), nullptr);
}
