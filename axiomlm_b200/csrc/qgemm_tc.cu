// W4A16 GEMM on the 5th-generation tensor cores (tcgen05) for the token
// counts where the projection becomes a dense contraction: tree verification
// with many candidates, chunked prefill, decode batches of 16-64.
//
// Replaces qmm_q4_marlin (axiomlm/kernels/quant.py:664-684; Metal
// qmm_q4_marlin_apple_kernel :2404, BM=32 x BN=16 simdgroup tiles) for
// M > 16.  At 64 tokens a Q4 weight byte feeds 256 flops, the B200's ridge:
// the legacy warp-level mma path cannot keep up with HBM there.
//
// One CTA computes a 128-row x 64-token tile of y over a K range (split-K
// across CTAs when the rows alone do not fill the GPU):
//  * 4 warps dequantize the q4t weights of the CTA's 8 row tiles (one
//    64-wide k-block per stage, loaded straight from HBM with 128-bit loads)
//    into fp16 in shared memory -- the dequantized value is the reference's
//    (fp16((q - 8) s) symmetric, fp16(q s + b) affine) -- and stage the
//    activations; both in the canonical K-major no-swizzle layout (8-row x
//    16-byte core matrices).
//  * one thread issues tcgen05.mma (M = 128, N = 64, K = 16, fp16 in, fp32
//    accumulate in tensor memory) and commits each stage to an mbarrier, so
//    the warps fill the other stage while the tensor core works.
//  * the epilogue reads the accumulator with tcgen05.ld (warp w: lanes 32w..),
//    adds the bias and stores fp16 (or, split-K, fp32 partials that the last
//    CTA of the row block sums in split order).
// Every mbarrier wait is bounded; a wait that runs out records AXB_ETIMEOUT,
// waits (bounded) for the tensor core, frees the tensor memory and returns.
#include <algorithm>

#include "axb_common.cuh"
#include "q4t.cuh"

namespace axb {

constexpr int kTcRows = 128;  // weight rows per CTA (MMA M)
constexpr int kTcTok = 64;    // tokens per CTA (MMA N)
constexpr int kTcKC = 64;     // k per stage (one q4t k-block)
constexpr int kTcStages = 2;  // dequantized weight (A) stages
constexpr int kTcAhead = 3;   // chunks whose raw weights and activations are in flight ahead
constexpr int kTcSlots = kTcAhead + kTcStages;  // raw / activation slots (a slot is held until its MMA is done)
constexpr int kTcThreads = 256;  // 8 warps: warp w dequantizes row tile w of the CTA
constexpr int kTcA = kTcRows * kTcKC * 2;  // 16 KB of fp16 weights per stage
constexpr int kTcB = kTcTok * kTcKC * 2;   // 8 KB of fp16 activations per slot
constexpr int kTcRawW = 8 * 512;           // q4t words of the CTA's 8 tiles per chunk
constexpr int kTcRawS = 8 * 8 * 8;         // their scales (affine: 8 x (s, b, s, b) per tile)
constexpr int kTcRaw = kTcRawW + kTcRawS;
constexpr int kTcSmem = kTcStages * kTcA + kTcSlots * (kTcB + kTcRaw) + 128;
constexpr int kTcCols = 64;  // tensor-memory columns: 64 fp32 tokens x 128 lanes
constexpr uint32_t kTcWaitLimit = 1u << 24;
// instruction descriptor (kind::f16): D fp32, A and B fp16, both K-major,
// N = 64 (bits 17-22: N / 8), M = 128 (bits 24-28: M / 16)
constexpr uint32_t kTcIdesc = (1u << 4) | ((uint32_t)(kTcTok >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);

struct TcArgs {
  const uint32_t* words;
  const __half* scales;
  const __half* x;
  const __half* bias;
  __half* y;
  float* part;  // split-K partials [S][M][N] (summed by tc_reduce_kernel), or null
  int* err;
  int N, K, M, ldx, ldy, G;
};

// byte offset of element (r, k) of a stage tile: core matrices of 8 rows x
// 16 bytes; the two core matrices of one 16-wide k step are 128 B apart
// (leading byte offset), 8-row groups 1024 B apart (stride byte offset)
__device__ __forceinline__ uint32_t tc_off(int r, int k) {
  return (uint32_t)((r >> 3) * 1024 + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

// shared-memory matrix descriptor: start >> 4, LBO 128 B, SBO 1024 B,
// descriptor version 1 (bits 46-47), no swizzle
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(kTcIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
// 16-byte asynchronous copy global -> shared; src_bytes 0 writes zeros
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <bool SYM, int GB>
__global__ void __launch_bounds__(kTcThreads) qgemm_tc_kernel(const TcArgs a) {
  extern __shared__ __align__(1024) char smem[];
  char* stA = smem;                                    // [stage][kTcA] dequantized weights
  char* stB = smem + kTcStages * kTcA;                 // [slot][kTcB] activations (operand layout)
  char* raw = stB + kTcSlots * kTcB;                   // [slot][kTcRaw] q4t words + scales
  uint64_t* bars = reinterpret_cast<uint64_t*>(raw + kTcSlots * kTcRaw);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kTcStages);
  const int tid = threadIdx.x, wid = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int KB = a.K / kTcKC, Nt = (a.N + 15) / 16;
  const int rb = blockIdx.x, S = gridDim.y, sp = blockIdx.y;
  const int kb0 = (int)((long long)sp * KB / S), kb1 = (int)((long long)(sp + 1) * KB / S);
  const int nch = kb1 - kb0;
  constexpr int SB = SYM ? 32 : 64;  // scale bytes per (tile, group)

  if (wid == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTcCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < kTcStages; ++s) mbar_init(bars + s, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  // one chunk's asynchronous copies into slot `sl`: the 8 tiles' words
  // (8 x 512 B) and scales, and the 64 x 64 activation tile straight into the
  // operand layout (zeros beyond M); one commit group per chunk, empty past the end
  auto issue = [&](int c) {
    if (c < nch) {
      const int kb = kb0 + c, sl = c % kTcSlots;
      char* rw = raw + sl * kTcRaw;
      char* bm = stB + sl * kTcB;
      const int grp = (kb * kTcKC) / a.G;
      for (int i = tid; i < 8 * 32; i += kTcThreads) {  // words: tile i / 32, 16-byte piece i % 32
        const int tl = i >> 5, tile = rb * 8 + tl;
        const bool v = tile < Nt;
        const char* src = reinterpret_cast<const char*>(a.words) +
                          (((size_t)(v ? tile : 0) * KB + kb) * 512 + (i & 31) * 16);
        cp_async16(rw + i * 16, src, v ? 16u : 0u);
      }
      for (int i = tid; i < 8 * (SB / 16); i += kTcThreads) {  // scales of the chunk's group
        const int tl = i / (SB / 16), tile = rb * 8 + tl;
        const bool v = tile < Nt;
        const char* src = reinterpret_cast<const char*>(a.scales) +
                          ((size_t)(v ? tile : 0) * (a.K / a.G) + grp) * SB + (i % (SB / 16)) * 16;
        cp_async16(rw + kTcRawW + i * 16, src, v ? 16u : 0u);
      }
      for (int i = tid; i < kTcTok * (kTcKC / 8); i += kTcThreads) {
        const int n = i >> 3, kc = i & 7;
        const bool v = n < a.M;
        cp_async16(bm + tc_off(n, kc * 8), a.x + (size_t)(v ? n : 0) * a.ldx + kb * kTcKC + kc * 8, v ? 16u : 0u);
      }
    }
    cp_async_commit();
  };
  for (int c = 0; c < kTcAhead; ++c) issue(c);

  for (int c = 0; c < nch; ++c) {
    const int st = c & 1, sl = c % kTcSlots;
    cp_async_wait<kTcAhead - 1>();  // this thread's copies of chunk c have landed
    if (c >= kTcStages) {           // MMA c - 2 is done: A stage st and slot (c - 2) % kTcSlots are free
      const bool got = mbar_wait(bars + st, (uint32_t)(((c - kTcStages) >> 1) & 1), kTcWaitLimit);
      if (__syncthreads_or(!got)) {
        ok = false;
        break;
      }
    } else {
      __syncthreads();
    }
    issue(c + kTcAhead);  // slot (c + 3) % 5 == (c - 2) % 5: freed above
    char* A = stA + st * kTcA;
    const char* rw = raw + sl * kTcRaw;
    // ---- dequantize: row tile wid, this lane's fragments
    {
      const int tl = wid;
      const uint4 wv = *reinterpret_cast<const uint4*>(rw + tl * 512 + lane * 16);
      uint2 sc;
      if (SYM) sc.x = reinterpret_cast<const uint32_t*>(rw + kTcRawW + tl * SB)[g];
      else sc = reinterpret_cast<const uint2*>(rw + kTcRawW + tl * SB)[g];
      const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t f[4];
        if (SYM) {
          unpack_word<8>(w4[j], f);  // exact (q - 8) as fp16
          const __half2 s01 = u32_as_h2(sc.x);
          const __half2 sg = __half2half2(__low2half(s01)), sg8 = __half2half2(__high2half(s01));
          f[0] = h2_as_u32(__hmul2(u32_as_h2(f[0]), sg));
          f[1] = h2_as_u32(__hmul2(u32_as_h2(f[1]), sg8));
          f[2] = h2_as_u32(__hmul2(u32_as_h2(f[2]), sg));
          f[3] = h2_as_u32(__hmul2(u32_as_h2(f[3]), sg8));
        } else {
          unpack_word<0>(w4[j], f);  // q as fp16
          const __half2 p0 = u32_as_h2(sc.x), p1 = u32_as_h2(sc.y);  // (s[g], b[g]), (s[g+8], b[g+8])
          const __half2 sg = __half2half2(__low2half(p0)), bg = __half2half2(__high2half(p0));
          const __half2 sg8 = __half2half2(__low2half(p1)), bg8 = __half2half2(__high2half(p1));
          f[0] = h2_as_u32(__hfma2(u32_as_h2(f[0]), sg, bg));
          f[1] = h2_as_u32(__hfma2(u32_as_h2(f[1]), sg8, bg8));
          f[2] = h2_as_u32(__hfma2(u32_as_h2(f[2]), sg, bg));
          f[3] = h2_as_u32(__hfma2(u32_as_h2(f[3]), sg8, bg8));
        }
        // f0 / f2: row g, k = 16 t4 + 4 j + {0, 1} / {2, 3}; f1 / f3: row g + 8
        const int r = tl * 16 + g, k = 16 * t4 + 4 * j;
        *reinterpret_cast<uint2*>(A + tc_off(r, k)) = make_uint2(f[0], f[2]);
        *reinterpret_cast<uint2*>(A + tc_off(r + 8, k)) = make_uint2(f[1], f[3]);
      }
    }
    fence_proxy_async();  // the tensor core reads A (and the copied B) through the async proxy
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t sa = smem_u32(A), sb = smem_u32(stB + sl * kTcB);
#pragma unroll
      for (int ks = 0; ks < kTcKC / 16; ++ks)
        tc_mma(tmem, tc_desc(sa + 256 * ks), tc_desc(sb + 256 * ks), (c > 0 || ks > 0) ? 1u : 0u);
      tc_commit(bars + st);
    }
  }
  cp_async_wait<0>();  // no copy may still be landing when the CTA exits

  // ---- the last commit covers every MMA of this CTA
  if (nch > 0) {
    const int cl = nch - 1;
    const bool got = mbar_wait(bars + (cl & 1), (uint32_t)((cl >> 1) & 1), kTcWaitLimit);
    if (__syncthreads_or(!got)) ok = false;
  }
  if (!ok) {
    if (tid == 0) atomicExch(a.err, AXB_ETIMEOUT);
    // give the tensor core a last bounded chance to finish before the memory is freed
    if (nch > 0) mbar_wait(bars + ((nch - 1) & 1), (uint32_t)(((nch - 1) >> 1) & 1), kTcWaitLimit);
  }
  tc_fence_after();
  // warps w and w + 4 share accumulator lanes 32 (w % 4) ..: w < 4 reads tokens 0..31, w >= 4 tokens 32..63
  constexpr int kHalf = kTcTok / 2;
  const int quarter = wid & 3, n0 = (wid >> 2) * kHalf;
  float v[kHalf];
  if (ok && nch > 0) {
    uint32_t r[kHalf];
    const uint32_t taddr = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)n0;
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int n = 0; n < kHalf; ++n) v[n] = __uint_as_float(r[n]);
  } else {
#pragma unroll
    for (int n = 0; n < kHalf; ++n) v[n] = 0.f;
  }
  // ---- tensor memory is no longer needed
  tc_fence_before();
  __syncthreads();
  if (wid == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcCols) : "memory");
  if (!ok) return;

  // ---- epilogue: row = this thread's accumulator lane; fp16 (+ bias), or the split's fp32 partial
  const int row = rb * kTcRows + 32 * quarter + lane;
  if (row >= a.N) return;
  if (S == 1) {
    const float bsum = a.bias ? __half2float(a.bias[row]) : 0.f;
#pragma unroll
    for (int n = 0; n < kHalf; ++n)
      if (n0 + n < a.M) a.y[(size_t)(n0 + n) * a.ldy + row] = __float2half_rn(v[n] + bsum);
    return;
  }
#pragma unroll
  for (int n = 0; n < kHalf; ++n)
    if (n0 + n < a.M) a.part[((size_t)sp * a.M + n0 + n) * a.N + row] = v[n];
}

// split-K: y[m][n] = fp16(sum over splits in order + bias)
__global__ void tc_reduce_kernel(const float* __restrict__ part, int S, int M, int N, const __half* __restrict__ bias,
                                 __half* __restrict__ y, int ldy) {
  const size_t total = (size_t)M * N;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / N), n = (int)(i % N);
    float o = 0.f;
    for (int q = 0; q < S; ++q) o += __ldcg(part + (size_t)q * total + i);
    if (bias) o += __half2float(bias[n]);
    y[(size_t)m * ldy + n] = __float2half_rn(o);
  }
}

int tc_splits(int N, int K) {
  const int rbs = (N + kTcRows - 1) / kTcRows, KB = K / kTcKC;
  int S = (2 * num_sms() + rbs - 1) / rbs;
  S = std::max(1, std::min(S, std::min(16, KB / 2)));
  return S;
}

}  // namespace axb

using namespace axb;

extern "C" {

size_t axb_qgemm_tc_workspace_bytes(int N, int K, int M) {
  (void)M;
  if (N <= 0 || K <= 0 || K % kTcKC) return 0;
  const int S = tc_splits(N, K);
  const size_t part = S > 1 ? (size_t)S * kTcTok * N * sizeof(float) : 0;
  return 256 + part;  // error word, split-K partials
}

int axb_qgemm_tc(const axb_qgemm_desc* d, void* stream) {
  AXB_CHECK_ARG(d, "qgemm_tc: null descriptor");
  AXB_CHECK_ARG(d->fmt == AXB_W_Q4T_SYM || d->fmt == AXB_W_Q4T_AFFINE, "qgemm_tc: unsupported fmt %d", d->fmt);
  AXB_CHECK_ARG((d->fmt == AXB_W_Q4T_SYM && d->group == 128) || (d->fmt == AXB_W_Q4T_AFFINE && d->group == 64),
                "qgemm_tc: (fmt %d, group %d) not built", d->fmt, d->group);
  AXB_CHECK_ARG(d->N > 0 && d->K > 0 && d->K % d->group == 0 && d->K % kTcKC == 0, "qgemm_tc: bad N/K (%d, %d)",
                d->N, d->K);
  AXB_CHECK_ARG(d->M >= 1 && d->M <= kTcTok, "qgemm_tc: M=%d out of [1, %d]", d->M, kTcTok);
  AXB_CHECK_ARG(d->epilogue == AXB_EPI_STORE && d->norm_w == nullptr && !d->gate_up_interleave,
                "qgemm_tc: only the plain store epilogue (+bias) is built");
  AXB_CHECK_ARG(d->words && d->scales && d->x && d->y && d->ldx >= d->K && d->ldy >= d->N,
                "qgemm_tc: bad pointers / strides");
  AXB_CHECK_ARG((reinterpret_cast<uintptr_t>(d->x) & 15) == 0 && d->ldx % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(d->words) & 15) == 0,
                "qgemm_tc: x and words must be 16-byte aligned, ldx a multiple of 8");
  const size_t need = axb_qgemm_tc_workspace_bytes(d->N, d->K, d->M);
  AXB_CHECK_ARG(d->workspace && d->workspace_bytes >= need, "qgemm_tc: workspace %zu < %zu bytes",
                d->workspace_bytes, need);
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(qgemm_tc_kernel<true, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kTcSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(qgemm_tc_kernel<false, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    if (e != cudaSuccess) return cuda_status(e, "qgemm_tc attribute");
    attr_dev = dev;
  }
  const int S = tc_splits(d->N, d->K);
  const int rbs = (d->N + kTcRows - 1) / kTcRows;
  char* ws = (char*)d->workspace;
  TcArgs a;
  a.words = (const uint32_t*)d->words;
  a.scales = (const __half*)d->scales;
  a.x = (const __half*)d->x;
  a.bias = (const __half*)d->bias;
  a.y = (__half*)d->y;
  a.err = (int*)ws;
  a.part = S > 1 ? (float*)(ws + 256) : nullptr;
  a.N = d->N;
  a.K = d->K;
  a.M = d->M;
  a.ldx = d->ldx;
  a.ldy = d->ldy;
  a.G = d->group;
  dim3 grid(rbs, S);
  if (d->fmt == AXB_W_Q4T_SYM)
    qgemm_tc_kernel<true, 2><<<grid, kTcThreads, kTcSmem, (cudaStream_t)stream>>>(a);
  else
    qgemm_tc_kernel<false, 1><<<grid, kTcThreads, kTcSmem, (cudaStream_t)stream>>>(a);
  if (int rc = launch_status("qgemm_tc")) return rc;
  if (S > 1) {
    const size_t total = (size_t)d->M * d->N;
    const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)num_sms() * 8);
    tc_reduce_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(a.part, S, d->M, d->N, a.bias, a.y, d->ldy);
    return launch_status("qgemm_tc reduce");
  }
  return AXB_OK;
}

/* Synchronizes `stream`; AXB_ETIMEOUT (and clears it) when a bounded wait of
 * an earlier axb_qgemm_tc on this workspace ran out. */
int axb_qgemm_tc_status(void* workspace, void* stream) {
  AXB_CHECK_ARG(workspace, "qgemm_tc_status: null workspace");
  int h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, workspace, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_status(e, "qgemm_tc_status");
  if (h != 0) {
    const int z = 0;
    cudaMemcpy(workspace, &z, sizeof(int), cudaMemcpyHostToDevice);
    axb::set_error("qgemm_tc: a bounded tensor-core wait ran out");
    return AXB_ETIMEOUT;
  }
  return AXB_OK;
}

}  // extern "C"
