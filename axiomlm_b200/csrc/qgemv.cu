// Quantized weight formats and the W4A16 GEMV / small-M GEMM for sm_100a.
//
// Replaces qmv_q4_marlin / qmm_q4_marlin (axiomlm/kernels/quant.py:637-684)
// and the Metal kernels qmv_q4_marlin_apple_kernel / qmm_q4_marlin_*
// (metal_kernels.metal:2135, :2268, :2404).  The reference dequantizes into
// fp16 and runs F.linear; here the 4-bit codes stream from HBM straight into
// mma.sync A-fragments (q4t layout, one 128-bit load per lane per 16x64 block)
// and the activations are the B operand, so M <= 64 tokens share one weight
// pass.  Work is split "stream-K" at group granularity over every warp of a
// persistent grid; tiles split between warps are reduced deterministically by
// the last warp to arrive (fixed summation order, per-tile arrival counter).
#include <algorithm>

#include "q4t.cuh"

namespace axb {

// ------------------------------------------------------------------ layout
// q4t: tile t (16 rows) x k-block b (64 columns) = 512 B at ((t*KB)+b)*512.
// Lane l = 4*g + t4 owns, in word j, rows {g, g+8} x columns
// 64*b + 16*t4 + 4*j + {0..3}; nibble i = low half of fragment register a_i,
// nibble i+4 = its high half (registers: a0 (g, +0/+1), a1 (g+8, +0/+1),
// a2 (g, +2/+3), a3 (g+8, +2/+3)).
// Scales per (tile, group): SYM 8 x half2 (s[g], s[g+8]); AFFINE 8 x
// (s[g], b[g], s[g+8], b[g+8]).

__device__ __forceinline__ void q4t_word_coords(int lane, int j, int nib, int& row, int& kk) {
  int g = lane >> 2, t4 = lane & 3;
  int reg = nib & 3, hi = nib >> 2;
  row = g + ((reg & 1) ? 8 : 0);
  kk = 16 * t4 + 4 * j + ((reg & 2) ? 2 : 0) + hi;
}

// ---- packing from fp32 weights (RTN) ---------------------------------------
__global__ void q4t_pack_kernel(const float* __restrict__ w, int N, int K, int G, int sym, int gu,
                                uint32_t* __restrict__ words, __half* __restrict__ scales) {
  const int KB = K / 64, tile = blockIdx.y, kb = blockIdx.x;
  const int grp = (kb * 64) / G;
  __shared__ float s_sc[16], s_bi[16];
  // stats: 16 rows x 16 threads each
  {
    int r = threadIdx.x >> 4, part = threadIdx.x & 15;
    int src = gu_src_row(tile * 16 + r, N, gu);
    float mn = INFINITY, mx = -INFINITY, am = 0.f;
    if (src < N) {
      const float* row = w + (size_t)src * K + (size_t)grp * G;
      for (int e = part; e < G; e += 16) {
        float v = row[e];
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
        am = fmaxf(am, fabsf(v));
      }
    } else {
      mn = mx = am = 0.f;
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    }
    if (part == 0) {
      if (sym) {
        __half s = __float2half_rn(__fdiv_rn(fmaxf(am, 1e-8f), 7.0f));
        s_sc[r] = __half2float(s);
        s_bi[r] = 0.f;
      } else {
        // quant.py:475-486
        float denom = fmaxf(__fsub_rn(mx, mn), 1e-8f);
        s_sc[r] = __half2float(__float2half_rn(__fdiv_rn(denom, 15.0f)));
        s_bi[r] = __half2float(__float2half_rn(mn));
      }
    }
  }
  __syncthreads();
  if (kb * 64 % G == 0 && threadIdx.x < 8) {
    int g = threadIdx.x;
    size_t base = ((size_t)tile * (K / G) + grp) * 8 + g;
    if (sym) {
      scales[base * 2 + 0] = __float2half_rn(s_sc[g]);
      scales[base * 2 + 1] = __float2half_rn(s_sc[g + 8]);
    } else {
      scales[base * 4 + 0] = __float2half_rn(s_sc[g]);
      scales[base * 4 + 1] = __float2half_rn(s_bi[g]);
      scales[base * 4 + 2] = __float2half_rn(s_sc[g + 8]);
      scales[base * 4 + 3] = __float2half_rn(s_bi[g + 8]);
    }
  }
  if (threadIdx.x < 128) {
    int lane = threadIdx.x >> 2, j = threadIdx.x & 3;
    uint32_t word = 0;
#pragma unroll
    for (int nib = 0; nib < 8; ++nib) {
      int row, kk;
      q4t_word_coords(lane, j, nib, row, kk);
      int src = gu_src_row(tile * 16 + row, N, gu);
      int q;
      float sc = s_sc[row];
      if (src >= N) {
        q = sym ? 8 : 0;
      } else {
        float v = w[(size_t)src * K + kb * 64 + kk];
        if (sym) {
          if (sc == 0.f) {
            q = 8;
          } else {
            float r = rintf(__fdiv_rn(v, sc));
            q = (int)fminf(fmaxf(r, -8.f), 7.f) + 8;
          }
        } else {
          float r = rintf(__fdiv_rn(__fsub_rn(v, s_bi[row]), fmaxf(sc, 1e-8f)));
          q = (int)fminf(fmaxf(r, 0.f), 15.f);
        }
      }
      word |= (uint32_t)(q & 0xF) << (4 * nib);
    }
    words[((size_t)tile * KB + kb) * 128 + lane * 4 + j] = word;
  }
}

// ---- relayout of the reference MARLIN-ladder format -----------------------
__device__ __forceinline__ int ladder_code(const uint32_t* wm, int KG, int row, int k) {
  int t8 = row >> 3, c = row & 7, kb = k >> 6, kk = k & 63;
  int wsel = kk >> 5, s = (kk >> 3) & 3, r = kk & 7;
  int c0 = c & 6;
  int lane = (((r >> 2) & 1) << 4) | (((c0 >> 2) & 1) << 3) | (((r >> 1) & 1) << 2) | ((r & 1) << 1) |
             ((c0 >> 1) & 1);
  uint32_t word = wm[(((size_t)t8 * KG + kb) * 32 + lane) * 2 + wsel];
  int shift = ((c & 1) ? 16 : 0) + 4 * s;
  return (word >> shift) & 0xF;
}

__global__ void q4t_from_marlin_kernel(const uint32_t* __restrict__ wm, const __half* __restrict__ sb, int n_rows8,
                                       int K, int n_out, int gu, uint32_t* __restrict__ words,
                                       __half* __restrict__ scales) {
  const int KB = K / 64, tile = blockIdx.y, kb = blockIdx.x;
  int t = threadIdx.x;
  if (t < 128) {
    int lane = t >> 2, j = t & 3;
    uint32_t word = 0;
#pragma unroll
    for (int nib = 0; nib < 8; ++nib) {
      int row, kk;
      q4t_word_coords(lane, j, nib, row, kk);
      int src = gu_src_row(tile * 16 + row, n_out, gu);
      int q = 0;
      if (src < n_out && src < n_rows8) q = ladder_code(wm, KB, src, kb * 64 + kk);
      word |= (uint32_t)q << (4 * nib);
    }
    words[((size_t)tile * KB + kb) * 128 + lane * 4 + j] = word;
  } else if (t < 136) {
    int g = t - 128;
    size_t base = ((size_t)tile * KB + kb) * 8 + g;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int src = gu_src_row(tile * 16 + g + 8 * h, n_out, gu);
      __half s = __float2half_rn(0.f), b = __float2half_rn(0.f);
      if (src < n_out && src < n_rows8) {
        int t8 = src >> 3, c = src & 7;
        const __half* p = sb + (((size_t)t8 * KB + kb) * 8 + c) * 2;
        s = p[0];
        b = p[1];
      }
      scales[base * 4 + 2 * h + 0] = s;
      scales[base * 4 + 2 * h + 1] = b;
    }
  }
}

// ---- relayout of the reference's legacy Q4_G64 format --------------------
// pack_linear_q4_g64 (quant.py:17-69): code k of row n in bits 4 (k % 8) of
// word n * K/8 + k / 8; scale and bias per (row, 64-wide group).  The same
// affine values as q4t AFFINE G64, in a different order.
__global__ void q4t_from_q4g64_kernel(const uint32_t* __restrict__ wl, const __half* __restrict__ sb, int N, int K,
                                      int gu, uint32_t* __restrict__ words, __half* __restrict__ scales) {
  const int KB = K / 64, tile = blockIdx.y, kb = blockIdx.x;
  const int t = threadIdx.x;
  if (t < 128) {
    const int lane = t >> 2, j = t & 3;
    uint32_t word = 0;
#pragma unroll
    for (int nib = 0; nib < 8; ++nib) {
      int row, kk;
      q4t_word_coords(lane, j, nib, row, kk);
      const int src = gu_src_row(tile * 16 + row, N, gu);
      uint32_t q = 0;
      if (src < N) {
        const int k = kb * 64 + kk;
        q = (wl[(size_t)src * (K / 8) + (k >> 3)] >> (4 * (k & 7))) & 0xFu;
      }
      word |= q << (4 * nib);
    }
    words[((size_t)tile * KB + kb) * 128 + lane * 4 + j] = word;
  } else if (t < 136) {
    const int g = t - 128;
    const size_t base = ((size_t)tile * KB + kb) * 8 + g;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int src = gu_src_row(tile * 16 + g + 8 * h, N, gu);
      __half sc = __float2half_rn(0.f), bi = __float2half_rn(0.f);
      if (src < N) {
        const __half* p = sb + ((size_t)src * KB + kb) * 2;
        sc = p[0];
        bi = p[1];
      }
      scales[base * 4 + 2 * h + 0] = sc;
      scales[base * 4 + 2 * h + 1] = bi;
    }
  }
}

// ---- dequant (bit-exact statements of the reference formulas) --------------
__global__ void q4t_dequant_kernel(const uint32_t* __restrict__ words, const __half* __restrict__ scales, int N,
                                   int K, int G, int sym, int gu, __half* __restrict__ out) {
  const int KB = K / 64, tile = blockIdx.y, kb = blockIdx.x;
  int t = threadIdx.x;  // 128 threads: one word each
  int lane = t >> 2, j = t & 3;
  uint32_t word = words[((size_t)tile * KB + kb) * 128 + lane * 4 + j];
  int grp = kb * 64 / G;
#pragma unroll
  for (int nib = 0; nib < 8; ++nib) {
    int row, kk;
    q4t_word_coords(lane, j, nib, row, kk);
    int p = tile * 16 + row;
    int dst = gu_src_row(p, N, gu);
    if (dst >= N) continue;
    int q = (word >> (4 * nib)) & 0xF;
    int g = row & 7, h = row >> 3;
    size_t base = ((size_t)tile * (K / G) + grp) * 8 + g;
    float v;
    if (sym) {
      float s = __half2float(scales[base * 2 + h]);
      v = __fmul_rn((float)(q - 8), s);
    } else {
      float s = __half2float(scales[base * 4 + 2 * h]);
      float b = __half2float(scales[base * 4 + 2 * h + 1]);
      v = __fadd_rn(__fmul_rn((float)q, s), b);  // quant.py:627-631: two fp32 ops
    }
    out[(size_t)dst * K + kb * 64 + kk] = __float2half_rn(v);
  }
}

__global__ void marlin_dequant_kernel(const uint32_t* __restrict__ wm, const __half* __restrict__ sb, int K,
                                      int n_out, __half* __restrict__ out) {
  int row = blockIdx.y, KG = K / 64;
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < K; k += gridDim.x * blockDim.x) {
    int q = ladder_code(wm, KG, row, k);
    int t8 = row >> 3, c = row & 7, kb = k >> 6;
    const __half* p = sb + (((size_t)t8 * KG + kb) * 8 + c) * 2;
    float v = __fadd_rn(__fmul_rn((float)q, __half2float(p[0])), __half2float(p[1]));
    out[(size_t)row * K + k] = __float2half_rn(v);
  }
}

// quant.py:72-129: Q8_G64 RTN pack (one warp per (row, group))
__global__ void q8_pack_kernel(const float* __restrict__ w, int N, int K, uint32_t* __restrict__ out,
                               __half* __restrict__ sb) {
  const int lane = threadIdx.x & 31;
  const long long item = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int G = K / 64;
  if (item >= (long long)N * G) return;
  const int row = (int)(item / G), grp = (int)(item % G);
  const float* src = w + (size_t)row * K + grp * 64;
  float v0 = src[2 * lane], v1 = src[2 * lane + 1];
  float mn = fminf(v0, v1), mx = fmaxf(v0, v1);
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const float denom = fmaxf(__fsub_rn(mx, mn), 1e-8f);
  const __half sc = __float2half_rn(__fdiv_rn(denom, 255.0f));
  const __half bi = __float2half_rn(mn);
  const float scf = fmaxf(__half2float(sc), 1e-8f), bif = __half2float(bi);
  int q0 = (int)fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(v0, bif), scf)), 0.f), 255.f);
  int q1 = (int)fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(v1, bif), scf)), 0.f), 255.f);
  // two bytes per lane: lanes 2i, 2i+1 form word i
  uint32_t part = (uint32_t)q0 | ((uint32_t)q1 << 8);
  uint32_t other = __shfl_xor_sync(0xffffffffu, part, 1);
  if ((lane & 1) == 0) out[(size_t)row * (K / 4) + grp * 16 + lane / 2] = part | (other << 16);
  if (lane == 0) {
    sb[((size_t)row * G + grp) * 2] = sc;
    sb[((size_t)row * G + grp) * 2 + 1] = bi;
  }
}

__global__ void q8_rows_kernel(const uint32_t* __restrict__ w, const __half* __restrict__ sb,
                               const int32_t* __restrict__ idx, int K, __half* __restrict__ out) {
  int i = blockIdx.x;
  int r = idx[i];
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    uint32_t word = w[(size_t)r * (K / 4) + k / 4];
    int q = (word >> (8 * (k & 3))) & 0xFF;
    const __half* p = sb + ((size_t)r * (K / 64) + k / 64) * 2;
    float v = __fadd_rn(__fmul_rn((float)q, __half2float(p[0])), __half2float(p[1]));
    out[(size_t)i * K + k] = __float2half_rn(v);
  }
}

__global__ void ternary_dequant_kernel(const uint8_t* __restrict__ w, const __half* __restrict__ s, int K,
                                       int per_tensor, __half* __restrict__ out) {
  int row = blockIdx.y;
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < K; k += gridDim.x * blockDim.x) {
    int b = w[(size_t)row * (K / 4) + k / 4] >> (2 * (k & 3));
    int q = (b & 1) - ((b >> 1) & 1);
    float sc = __half2float(per_tensor ? s[0] : s[(size_t)row * (K / 64) + k / 64]);
    out[(size_t)row * K + k] = __float2half_rn(__fmul_rn((float)q, sc));
  }
}

__global__ void q2_dequant_kernel(const uint8_t* __restrict__ w, const __half* __restrict__ sb, int K,
                                  __half* __restrict__ out) {
  int row = blockIdx.y;
  for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < K; k += gridDim.x * blockDim.x) {
    int q = (w[(size_t)row * (K / 4) + k / 4] >> (2 * (k & 3))) & 3;
    const __half* p = sb + ((size_t)row * (K / 64) + k / 64) * 2;
    // quant.py:399-401: q*scale and +bias are separate fp16 tensor ops
    __half t = __float2half_rn(__fmul_rn((float)q, __half2float(p[0])));
    out[(size_t)row * K + k] = __float2half_rn(__fadd_rn(__half2float(t), __half2float(p[1])));
  }
}

// ------------------------------------------------------------------ GEMV
// Work split: "stream-K" over quantization groups ("units") at CTA level.
// CTA c owns units [c*U/C, (c+1)*U/C) of the tile-major unit sequence; inside
// the CTA the 4 warps split every tile segment's K range into 4 contiguous
// chunks, stream them through per-warp bulk-copy rings, and reduce the 4
// partial fragments in shared memory in warp order.  A tile whose units span
// several CTAs is finished by the last CTA to arrive (per-tile counter), which
// sums the CTA partials in CTA order: the result is deterministic.
struct GemmArgs {
  const uint4* W;
  const char* S;
  int N, K, M, KB, GB, upt;
  long long U;
  long long C;  // CTAs
  const __half* x;
  int ldx;
  const float* norm_w;
  float eps;
  void* y;
  int ldy;
  const __half* bias;
  int epi, gu;
  float* partials;
  int* counters;
  int* err;
  int xs_stride;  // smem row stride (halves); 0 = read x from global
  int xs_bytes;   // bytes of the staged-x region at the start of shared memory
  int early_trigger;  // release the dependent launch right after staging x
};

#ifndef AXB_GEMV_WARPS
#define AXB_GEMV_WARPS 4
#endif
#ifndef AXB_GEMV_CTAS_PER_SM
#define AXB_GEMV_CTAS_PER_SM 4
#endif
#ifndef AXB_GEMV_CH
#define AXB_GEMV_CH 4
#endif
#ifndef AXB_GEMV_STAGES
#define AXB_GEMV_STAGES 3
#endif
constexpr int kWarps = AXB_GEMV_WARPS;            // warps per CTA (K-split of each tile)
constexpr int kCtasPerSm = AXB_GEMV_CTAS_PER_SM;  // resident CTAs per SM the grid is sized for
constexpr int kCH = AXB_GEMV_CH;                  // k-blocks (512 B each) per pipeline stage
constexpr int kStages = AXB_GEMV_STAGES;          // stages per warp
constexpr int kStageW = kCH * 512;  // weight bytes per stage
constexpr int kStageS = kCH * 64;   // scale bytes per stage (max: affine, one group per k-block)
// per-warp ring: stages of weights, stages of scales, mbarriers; the stride is
// rounded to 128 B so every warp's bulk-copy destinations stay 16-B aligned
constexpr int kWarpRing = (kStages * (kStageW + kStageS) + kStages * 8 + 127) / 128 * 128;
static_assert(kStageW % 16 == 0 && kStageS % 16 == 0 && kWarpRing % 128 == 0, "bulk-copy alignment");
static_assert((kStages * (kStageW + kStageS)) % 8 == 0, "mbarrier alignment");
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ __forceinline__ int cta_start(long long c, long long U, long long C) { return (int)(c * U / C); }
__device__ __forceinline__ int cta_of_unit(long long u, long long U, long long C) {
  return (int)(((u + 1) * C - 1) / U);
}

template <int NT>
__device__ __forceinline__ void epilogue(const GemmArgs& a, int tile, const float (&acc)[NT][4], int lane) {
  const int g = lane >> 2, t4 = lane & 3;
  const int r0 = tile * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int n = nt * 8 + 2 * t4 + e;
      if (n >= a.M) continue;
      const float v0 = acc[nt][e], v1 = acc[nt][2 + e];
      if (a.epi == AXB_EPI_SWIGLU) {
        const int j = tile * 8 + g;
        if (j < (a.N >> 1)) {
          // gate and up are fp16-rounded GEMV outputs
          const float gg = __half2float(__float2half_rn(v0));
          const float uu = __half2float(__float2half_rn(v1));
          reinterpret_cast<__half*>(a.y)[(size_t)n * a.ldy + j] = swiglu_h(gg, uu);
        }
        continue;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int p = h ? r1 : r0;
        const int col = gu_src_row(p, a.N, a.gu);
        if (col >= a.N) continue;
        float v = h ? v1 : v0;
        if (a.bias) v = __fadd_rn(v, __half2float(a.bias[col]));
        __half vh = __float2half_rn(v);
        if (a.epi == AXB_EPI_RESIDUAL) {
          __half* yp = reinterpret_cast<__half*>(a.y) + (size_t)n * a.ldy + col;
          *yp = __float2half_rn(__fadd_rn(__half2float(*yp), __half2float(vh)));
        } else if (a.epi == AXB_EPI_F32) {
          reinterpret_cast<float*>(a.y)[(size_t)n * a.ldy + col] = __half2float(vh);
        } else if (a.epi == AXB_EPI_F32_ACC) {
          reinterpret_cast<float*>(a.y)[(size_t)n * a.ldy + col] = v;
        } else {
          reinterpret_cast<__half*>(a.y)[(size_t)n * a.ldy + col] = vh;
        }
      }
    }
  }
}

// Stage x (optionally RMS-normalized: modules.py:41-43 with an fp32 weight,
// rms = 1/sqrt(mean(x^2) + eps), h = fp16((x * rms) * w)) into shared memory.
// All threads of the CTA share each row so the row's loads are all in flight.
__device__ void stage_x(const GemmArgs& a, __half* xs, float* red) {
  const int tid = threadIdx.x, nth = blockDim.x;
  const int lane = tid & 31, wid = tid >> 5, nw = nth >> 5;
  const int K8 = a.K >> 3;  // uint4 chunks per row
  for (int m = 0; m < a.M; ++m) {
    const uint4* xr = reinterpret_cast<const uint4*>(a.x + (size_t)m * a.ldx);
    uint4* sr = reinterpret_cast<uint4*>(xs + (size_t)m * a.xs_stride);
    if (!a.norm_w) {
      for (int c = tid; c < K8; c += nth) sr[c] = xr[c];
      continue;
    }
    float ss = 0.f;
    for (int c0 = tid; c0 < K8; c0 += nth * 4) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + u * nth < K8) v[u] = xr[c0 + u * nth];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (c0 + u * nth >= K8) continue;
        const __half2* h = reinterpret_cast<const __half2*>(&v[u]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float2 f = __half22float2(h[q]);
          ss = __fmaf_rn(f.x, f.x, ss);
          ss = __fmaf_rn(f.y, f.y, ss);
        }
        sr[c0 + u * nth] = v[u];  // raw x, scaled below
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) red[wid] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < nw; ++w) tot += red[w];
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)a.K), a.eps)));
    for (int c = tid; c < K8; c += nth) {
      uint4 v = sr[c];
      const __half2* h = reinterpret_cast<const __half2*>(&v);
      uint4 o;
      __half2* oh = reinterpret_cast<__half2*>(&o);
      const float4 w0 = reinterpret_cast<const float4*>(a.norm_w)[2 * c];
      const float4 w1 = reinterpret_cast<const float4*>(a.norm_w)[2 * c + 1];
      const float ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 f = __half22float2(h[q]);
        oh[q] = __floats2half2_rn(__fmul_rn(__fmul_rn(f.x, rms), ws[2 * q]),
                                  __fmul_rn(__fmul_rn(f.y, rms), ws[2 * q + 1]));
      }
      sr[c] = o;
    }
    __syncthreads();  // red[] reuse
  }
}

// chunk of tile t handled by warp w: global k-block range [lo, hi)
__device__ __forceinline__ void warp_chunk(int upt, int GB, int U0, int U1, int t, int w, int& lo, int& hi) {
  const int s0 = max(U0, t * upt), s1 = min(U1, (t + 1) * upt);
  const int ns = s1 - s0;
  lo = (s0 + ns * w / kWarps) * GB;
  hi = (s0 + ns * (w + 1) / kWarps) * GB;
}

template <int NT, bool SYM, int GB, bool XS>
__global__ void __launch_bounds__(kWarps * 32, (NT == 1 ? 28 : (NT == 2 ? 20 : 12)) / kWarps) qgemm_kernel(const GemmArgs a) {
  extern __shared__ __align__(128) char smem[];
  __half* xs = reinterpret_cast<__half*>(smem);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int c = blockIdx.x;
  const int U0 = cta_start(c, a.U, a.C), U1 = cta_start(c + 1, a.U, a.C);
  const int t_first = U0 / a.upt, t_last = (U1 - 1) / a.upt;
  constexpr int UB = SYM ? 32 : 64;  // scale bytes per group

  char* ring = smem + a.xs_bytes + (size_t)wid * kWarpRing;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + kStages * (kStageW + kStageS));
  float* red = reinterpret_cast<float*>(smem + a.xs_bytes + kWarps * kWarpRing);  // [kWarps][32][4*NT]
  float* nred = red + kWarps * 32 * 4 * NT;                                       // [kWarps] norm partials
  if (lane == 0) {
    for (int st = 0; st < kStages; ++st) mbar_init(bars + st, 1);
    fence_mbar_init();
  }
  __syncwarp();

  // producer state (lane 0): next stage to issue
  int p_t = t_first, p_kb = 0, p_end = 0, p_i = 0;
  if (lane == 0) warp_chunk(a.upt, GB, U0, U1, p_t, wid, p_kb, p_end);
  auto issue = [&]() {
    if (lane != 0) return;
    while (p_kb >= p_end && p_t < t_last) {
      ++p_t;
      warp_chunk(a.upt, GB, U0, U1, p_t, wid, p_kb, p_end);
    }
    if (p_kb >= p_end) return;
    const int st = p_i % kStages;
    const int n = min(kCH, p_end - p_kb);
    const uint32_t bw = n * 512, bs = (n / GB) * UB;
    fence_proxy_async();
    mbar_expect_tx(bars + st, bw + bs);
    bulk_g2s(ring + st * kStageW, a.W + (size_t)p_kb * 32, bw, bars + st);
    bulk_g2s(ring + kStages * kStageW + st * kStageS, a.S + (size_t)(p_kb / GB) * UB, bs, bars + st);
    p_kb += n;
    ++p_i;
  };
  // weights do not depend on the producer kernel: start streaming now
  for (int i = 0; i < kStages; ++i) issue();

  pdl_wait();
  if (XS) {
    stage_x(a, xs, nred);
    __syncthreads();
  }
  if (a.early_trigger) pdl_trigger();

  int ci = 0;  // stages consumed by this warp
  bool failed = false;
  // B-fragment rows: token nt*8 + g, clamped to a valid row (columns >= M are
  // computed but never stored, so no per-lane branch is needed)
  const uint4* xrow[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int nn = min(nt * 8 + g, a.M - 1);
    xrow[nt] = reinterpret_cast<const uint4*>((XS ? xs + (size_t)nn * a.xs_stride : a.x + (size_t)nn * a.ldx) +
                                              16 * t4);
  }
  // independent accumulation chains per group (the mma results of one
  // k-block's 4 words go to different registers, so consecutive HMMAs do not
  // wait on each other); summed when the group's scale is applied
  constexpr int CH = NT == 1 ? 2 : 1;
  for (int t = t_first; t <= t_last; ++t) {
    int kb_lo, kb_hi;
    warp_chunk(a.upt, GB, U0, U1, t, wid, kb_lo, kb_hi);
    float acc[NT][4];
    float tmp[CH][NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[nt][q] = 0.f;
#pragma unroll
        for (int c2 = 0; c2 < CH; ++c2) tmp[c2][nt][q] = 0.f;
      }
    // activation fragments of the next k-block, loaded one k-block ahead
    uint4 xn[NT][2];
    if (!XS && kb_lo < kb_hi) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        xn[nt][0] = xrow[nt][(kb_lo - t * a.KB) * 8];
        xn[nt][1] = xrow[nt][(kb_lo - t * a.KB) * 8 + 1];
      }
    }
    for (int kb0 = kb_lo; kb0 < kb_hi && !failed;) {
      const int st = ci % kStages;
      if (!mbar_wait(bars + st, (uint32_t)((ci / kStages) & 1), kWaitLimit)) {
        // record the failure; copies still in flight get a bounded wait
        if (lane == 0) atomicExch(a.err, AXB_ETIMEOUT);
        for (int k2 = 1; k2 < kStages; ++k2)
          mbar_wait(bars + ((ci + k2) % kStages), (uint32_t)(((ci + k2) / kStages) & 1), kWaitLimit);
        failed = true;
        break;
      }
      const int n = min(kCH, kb_hi - kb0);
      const uint4* wst = reinterpret_cast<const uint4*>(ring + st * kStageW) + lane;
      const char* sst = ring + kStages * kStageW + st * kStageS;
      const int kbt = kb0 - t * a.KB;  // k-block of the stage within the tile
      auto kblock = [&](const int j) {
          const uint4 cur = wst[j * 32];
          uint32_t bf[NT][8];
          if (XS) {  // staged activations: shared-memory loads, scheduled freely in the unrolled stage
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint4 v0 = xrow[nt][(kbt + j) * 8], v1 = xrow[nt][(kbt + j) * 8 + 1];
              bf[nt][0] = v0.x; bf[nt][1] = v0.y; bf[nt][2] = v0.z; bf[nt][3] = v0.w;
              bf[nt][4] = v1.x; bf[nt][5] = v1.y; bf[nt][6] = v1.z; bf[nt][7] = v1.w;
            }
          } else {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              bf[nt][0] = xn[nt][0].x; bf[nt][1] = xn[nt][0].y; bf[nt][2] = xn[nt][0].z; bf[nt][3] = xn[nt][0].w;
              bf[nt][4] = xn[nt][1].x; bf[nt][5] = xn[nt][1].y; bf[nt][6] = xn[nt][1].z; bf[nt][7] = xn[nt][1].w;
            }
          }
          if (!XS && kb0 + j + 1 < kb_hi) {  // prefetch the next k-block's fragments
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              xn[nt][0] = xrow[nt][(kbt + j + 1) * 8];
              xn[nt][1] = xrow[nt][(kbt + j + 1) * 8 + 1];
            }
          }
          const uint32_t words[4] = {cur.x, cur.y, cur.z, cur.w};
          if (SYM) {
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              uint32_t af[4];
              unpack_word<8>(words[jj], af);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
                mma_16816(tmp[jj % CH][nt], af, bf[nt][2 * jj], bf[nt][2 * jj + 1], tmp[jj % CH][nt]);
            }
            if (GB == 1 || (j & 1)) {  // group complete (stages start on a group boundary)
              const uint32_t sp = reinterpret_cast<const uint32_t*>(sst)[(j / GB) * 8 + g];
              const float2 sc = __half22float2(u32_as_h2(sp));
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                float s4[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  float v = tmp[0][nt][q];
#pragma unroll
                  for (int c2 = 1; c2 < CH; ++c2) v += tmp[c2][nt][q];
                  s4[q] = v;
#pragma unroll
                  for (int c2 = 0; c2 < CH; ++c2) tmp[c2][nt][q] = 0.f;
                }
                acc[nt][0] = __fmaf_rn(sc.x, s4[0], acc[nt][0]);
                acc[nt][1] = __fmaf_rn(sc.x, s4[1], acc[nt][1]);
                acc[nt][2] = __fmaf_rn(sc.y, s4[2], acc[nt][2]);
                acc[nt][3] = __fmaf_rn(sc.y, s4[3], acc[nt][3]);
              }
            }
          } else {
            const uint2 sb = reinterpret_cast<const uint2*>(sst)[(j / GB) * 8 + g];
            const __half2 s01 = u32_as_h2(sb.x), s23 = u32_as_h2(sb.y);
            const __half2 sg = __half2half2(__low2half(s01)), bg = __half2half2(__high2half(s01));
            const __half2 sg8 = __half2half2(__low2half(s23)), bg8 = __half2half2(__high2half(s23));
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              uint32_t af[4];
              unpack_word<0>(words[jj], af);
              // w = fp16(q * s + b): the reference's dequantized fp16 weight
              af[0] = h2_as_u32(__hfma2(u32_as_h2(af[0]), sg, bg));
              af[1] = h2_as_u32(__hfma2(u32_as_h2(af[1]), sg8, bg8));
              af[2] = h2_as_u32(__hfma2(u32_as_h2(af[2]), sg, bg));
              af[3] = h2_as_u32(__hfma2(u32_as_h2(af[3]), sg8, bg8));
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
                mma_16816(tmp[jj % CH][nt], af, bf[nt][2 * jj], bf[nt][2 * jj + 1], tmp[jj % CH][nt]);
            }
          }
      };
      if (n == kCH) {  // full stage: no guards, the 4 k-blocks interleave freely
#pragma unroll
        for (int j = 0; j < kCH; ++j) kblock(j);
      } else {
#pragma unroll
        for (int j = 0; j < kCH; ++j)
          if (j < n) kblock(j);
      }
      __syncwarp();
      issue();
      ++ci;
      kb0 += n;
    }
    if (!SYM) {  // affine: the chains carry scaled values already
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float v = tmp[0][nt][q];
#pragma unroll
          for (int c2 = 1; c2 < CH; ++c2) v += tmp[c2][nt][q];
          acc[nt][q] = v;
        }
    }
    // CTA reduction of the 4 warps' fragments, in warp order
    float* my = red + ((size_t)wid * 32 + lane) * (4 * NT);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      *reinterpret_cast<float4*>(my + 4 * nt) = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
    __syncthreads();
    if (wid == 0) {
      float sum[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int q = 0; q < 4; ++q) sum[nt][q] = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float* pw = red + ((size_t)w * 32 + lane) * (4 * NT);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float4 v = *reinterpret_cast<const float4*>(pw + 4 * nt);
          sum[nt][0] += v.x;
          sum[nt][1] += v.y;
          sum[nt][2] += v.z;
          sum[nt][3] += v.w;
        }
      }
      const bool complete = t * a.upt >= U0 && (t + 1) * a.upt <= U1;
      if (complete) {
        epilogue<NT>(a, t, sum, lane);
      } else {
        const int slot = (t == t_first) ? 0 : 1;
        float* p = a.partials + ((size_t)(c * 2 + slot) * 32 + lane) * (4 * NT);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          *reinterpret_cast<float4*>(p + 4 * nt) = make_float4(sum[nt][0], sum[nt][1], sum[nt][2], sum[nt][3]);
        __threadfence();
        __syncwarp();
        int old = 0;
        if (lane == 0) old = atomicAdd(a.counters + t, 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        const int cf = cta_of_unit((long long)t * a.upt, a.U, a.C);
        const int cl = cta_of_unit((long long)(t + 1) * a.upt - 1, a.U, a.C);
        if (old == (int)(cl - cf)) {  // last contributor: reduce in CTA order
          __threadfence();
          float tot[NT][4];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int q = 0; q < 4; ++q) tot[nt][q] = 0.f;
          for (int cc0 = cf; cc0 <= cl; cc0 += 4) {
            float4 v[4][NT];
#pragma unroll
            for (int u = 0; u < 4; ++u) {  // independent loads, all in flight
              const int cc = cc0 + u;
              if (cc > cl) continue;
              const int sl = (cta_start(cc, a.U, a.C) / a.upt == t) ? 0 : 1;
              const float* pp = a.partials + ((size_t)(cc * 2 + sl) * 32 + lane) * (4 * NT);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) v[u][nt] = __ldcg(reinterpret_cast<const float4*>(pp + 4 * nt));
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              if (cc0 + u > cl) continue;
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                tot[nt][0] += v[u][nt].x;
                tot[nt][1] += v[u][nt].y;
                tot[nt][2] += v[u][nt].z;
                tot[nt][3] += v[u][nt].w;
              }
            }
          }
          epilogue<NT>(a, t, tot, lane);
          if (lane == 0) a.counters[t] = 0;
        }
      }
    }
    __syncthreads();  // red[] reuse
  }
}

// ------------------------------------------------------------------ host
static size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
static int nt_for(int M) { return M <= 8 ? 1 : M <= 16 ? 2 : M <= 32 ? 4 : 8; }
static long long max_ctas() { return (long long)num_sms() * kCtasPerSm; }
static constexpr size_t kSmemLimit = 227 * 1024;
static constexpr size_t kRingBytes = (size_t)kWarps * kWarpRing;
static size_t red_bytes(int NT) { return (size_t)kWarps * 32 * 4 * NT * 4 + 64; }
// staged x is kept small so that two GEMV grids fit on an SM at once (the
// next kernel prefetches its weights under PDL while this one finishes)
static constexpr size_t kXsLimit = 64 * 1024;

template <int NT, bool SYM, int GB, bool XS>
static cudaError_t launch_one(const GemmArgs& ga, int ctas, int threads, size_t smem, cudaStream_t s, bool pdl) {
  return launch_pdl(qgemm_kernel<NT, SYM, GB, XS>, dim3(ctas), dim3(threads), smem, s, pdl, ga);
}

template <int NT, bool XS>
static cudaError_t dispatch_fmt(const GemmArgs& ga, bool sym, int GB, int ctas, int threads, size_t smem,
                                cudaStream_t s, bool pdl) {
  if (sym)
    return GB == 2 ? launch_one<NT, true, 2, XS>(ga, ctas, threads, smem, s, pdl)
                   : launch_one<NT, true, 1, XS>(ga, ctas, threads, smem, s, pdl);
  return GB == 2 ? launch_one<NT, false, 2, XS>(ga, ctas, threads, smem, s, pdl)
                 : launch_one<NT, false, 1, XS>(ga, ctas, threads, smem, s, pdl);
}

bool qgemm_can_fuse_norm(int M, int K) {
  return nt_for(M) <= 4 && round_up((size_t)M * (K + 8) * sizeof(__half), 128) <= kXsLimit;
}

// Set the shared-memory attribute of every instantiation once per device,
// outside any stream capture.
int qgemm_prepare() {
  int dev = 0;
  cudaGetDevice(&dev);
  static DeviceOnce once;
  if (once.done(dev)) return AXB_OK;
#define AXB_SET(NT, SYM, GB, XS)                                                                             \
  {                                                                                                         \
    cudaError_t e = cudaFuncSetAttribute(qgemm_kernel<NT, SYM, GB, XS>,                                      \
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit);     \
    if (e != cudaSuccess) return cuda_status(e, "qgemm attribute");                                         \
  }
#define AXB_SET4(NT, XS) AXB_SET(NT, true, 1, XS) AXB_SET(NT, true, 2, XS) AXB_SET(NT, false, 1, XS) AXB_SET(NT, false, 2, XS)
  AXB_SET4(1, true) AXB_SET4(1, false) AXB_SET4(2, true) AXB_SET4(2, false) AXB_SET4(4, true) AXB_SET4(4, false)
  AXB_SET4(8, false)
#undef AXB_SET4
#undef AXB_SET
  once.set(dev);
  return AXB_OK;
}

// Workspace: [error word | 256 B][tile counters | kMaxTiles ints][partials].
// Every region sits at a fixed offset, so one zeroed workspace serves calls of
// any N and M: counters are only ever touched by the arrival logic, which
// returns each one to zero.
constexpr size_t kMaxTiles = 1 << 17;
constexpr size_t kCountersOff = 256;
constexpr size_t kPartialsOff = kCountersOff + kMaxTiles * 4;

size_t qgemm_workspace(int N, int M) {
  (void)N;
  return kPartialsOff + (size_t)2 * max_ctas() * 32 * 4 * nt_for(M) * sizeof(float);
}

int qgemm(const axb_qgemm_desc* d, cudaStream_t stream) {
  AXB_CHECK_ARG(d, "null descriptor");
  AXB_CHECK_ARG(d->fmt == AXB_W_Q4T_SYM || d->fmt == AXB_W_Q4T_AFFINE, "qgemm: unsupported fmt %d", d->fmt);
  AXB_CHECK_ARG(d->group == 64 || d->group == 128, "qgemm: group must be 64 or 128");
  AXB_CHECK_ARG(d->N > 0 && d->K > 0 && d->K % d->group == 0, "qgemm: bad N/K (%d, %d)", d->N, d->K);
  AXB_CHECK_ARG(d->M >= 1 && d->M <= 64, "qgemm: M must be in [1, 64], got %d", d->M);
  AXB_CHECK_ARG(d->words && d->scales && d->x && d->y, "qgemm: null pointer");
  AXB_CHECK_ARG((reinterpret_cast<uintptr_t>(d->words) & 15) == 0 && (reinterpret_cast<uintptr_t>(d->scales) & 15) == 0,
                "qgemm: weights and scales must be 16-byte aligned");
  AXB_CHECK_ARG(d->ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(d->x) & 15) == 0,
                "qgemm: x must be 16-byte aligned with ldx %% 8 == 0");
  AXB_CHECK_ARG(!d->norm_w || (reinterpret_cast<uintptr_t>(d->norm_w) & 15) == 0,
                "qgemm: norm weight must be 16-byte aligned");
  AXB_CHECK_ARG(!d->gate_up_interleave || d->N % 16 == 0, "qgemm: gate/up interleave needs N %% 16 == 0");
  AXB_CHECK_ARG(d->epilogue != AXB_EPI_SWIGLU || d->gate_up_interleave, "qgemm: SWIGLU needs interleaved rows");
  AXB_CHECK_ARG(d->workspace && d->workspace_bytes >= qgemm_workspace(d->N, d->M),
                "qgemm: workspace too small (%zu < %zu)", d->workspace_bytes, qgemm_workspace(d->N, d->M));
  if (int rc = qgemm_prepare()) return rc;
  GemmArgs ga = {};
  ga.W = reinterpret_cast<const uint4*>(d->words);
  ga.S = reinterpret_cast<const char*>(d->scales);
  ga.N = d->N;
  ga.K = d->K;
  ga.M = d->M;
  ga.KB = d->K / 64;
  ga.GB = d->group / 64;
  ga.upt = d->K / d->group;
  const int n_tiles = (d->N + 15) / 16;
  AXB_CHECK_ARG((size_t)n_tiles <= kMaxTiles && (long long)n_tiles * (d->K / 64) < (1ll << 30),
                "qgemm: matrix too large (%d x %d)", d->N, d->K);
  ga.U = (long long)n_tiles * ga.upt;
  ga.x = reinterpret_cast<const __half*>(d->x);
  ga.ldx = d->ldx;
  ga.norm_w = d->norm_w;
  ga.eps = d->eps;
  ga.y = d->y;
  ga.ldy = d->ldy;
  ga.bias = reinterpret_cast<const __half*>(d->bias);
  ga.epi = d->epilogue;
  ga.gu = d->gate_up_interleave;
  ga.early_trigger = d->pdl >= 2 ? 0 : 1;  // pdl == 2: dependent launch at exit only
  char* ws = reinterpret_cast<char*>(d->workspace);
  ga.err = reinterpret_cast<int*>(ws);
  ga.counters = reinterpret_cast<int*>(ws + kCountersOff);
  ga.partials = reinterpret_cast<float*>(ws + kPartialsOff);
  const int nt = nt_for(d->M);
  const size_t xsb = round_up((size_t)d->M * (d->K + 8) * sizeof(__half), 128);
  const bool xs = nt <= 4 && (d->norm_w != nullptr || xsb <= 32 * 1024) && xsb <= kXsLimit;
  AXB_CHECK_ARG(xs || !d->norm_w, "qgemm: fused RMSNorm needs M <= 32 and M*K*2 <= %zu bytes", kXsLimit);
  ga.xs_stride = xs ? d->K + 8 : 0;
  ga.xs_bytes = xs ? (int)xsb : 0;
  const size_t smem = (size_t)ga.xs_bytes + kRingBytes + red_bytes(nt);
  // persistent grid: every CTA resident at once (up to kCtasPerSm per SM, fewer
  // when the staged activations make CTAs larger) and owning >= 1 group
  const int fit = (int)std::min<size_t>(kCtasPerSm, (kSmemLimit - 1024) / smem);
  ga.C = std::min<long long>((long long)num_sms() * std::max(1, fit), ga.U);
  const int ctas = (int)ga.C, threads = kWarps * 32;
  const bool sym = d->fmt == AXB_W_Q4T_SYM;
  cudaError_t e;
  switch (nt) {
    case 1:
      e = xs ? dispatch_fmt<1, true>(ga, sym, ga.GB, ctas, threads, smem, stream, d->pdl)
             : dispatch_fmt<1, false>(ga, sym, ga.GB, ctas, threads, smem, stream, d->pdl);
      break;
    case 2:
      e = xs ? dispatch_fmt<2, true>(ga, sym, ga.GB, ctas, threads, smem, stream, d->pdl)
             : dispatch_fmt<2, false>(ga, sym, ga.GB, ctas, threads, smem, stream, d->pdl);
      break;
    case 4:
      e = xs ? dispatch_fmt<4, true>(ga, sym, ga.GB, ctas, threads, smem, stream, d->pdl)
             : dispatch_fmt<4, false>(ga, sym, ga.GB, ctas, threads, smem, stream, d->pdl);
      break;
    default: e = dispatch_fmt<8, false>(ga, sym, ga.GB, ctas, threads, smem, stream, d->pdl); break;
  }
  return cuda_status(e, "qgemm launch");
}

int qgemm_status(void* workspace, cudaStream_t s) {
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e, "qgemm status");
  if (v != 0) {
    set_error("qgemm: a weight-stream wait ran out (status %d)", v);
    int z = 0;
    cudaMemcpyAsync(workspace, &z, sizeof(int), cudaMemcpyHostToDevice, s);
    cudaStreamSynchronize(s);
    return v;
  }
  return AXB_OK;
}

// ---------------------------------------------------------------- no-alloc GEMV
// Scratch of axb_qgemm_noalloc: the same layout axb_qgemm expects in a caller
// workspace (error word, tile counters, CTA partials for M <= 8), held in a
// file-scope device array.  Every GPU that loads this library keeps one copy
// (kNoAllocBytes) until the process exits.
constexpr int kNoAllocMaxM = 8;
constexpr size_t kNoAllocMaxCtas = 1024;
constexpr size_t kNoAllocBytes = kPartialsOff + 2 * kNoAllocMaxCtas * 32 * 4 * sizeof(float);
static __device__ __align__(256) char g_noalloc_scratch[kNoAllocBytes];

// Device address of g_noalloc_scratch, looked up once per device with that
// device current (a host-side symbol is not a device address).  Host threads
// may race on a device's first call: both look the same address up.
static void* noalloc_scratch(int* status) {
  static std::atomic<void*> addr[64];  // null-initialized (static storage)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    *status = e != cudaSuccess ? cuda_status(e, "qgemm_noalloc: cudaGetDevice") : AXB_EINVAL;
    if (*status == AXB_EINVAL) set_error("qgemm_noalloc: device index %d out of range", dev);
    return nullptr;
  }
  void* p = addr[dev].load(std::memory_order_acquire);
  if (!p) {
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      *status = cuda_status(e, "qgemm_noalloc: cudaGetSymbolAddress");
      return nullptr;
    }
    addr[dev].store(p, std::memory_order_release);
  }
  *status = AXB_OK;
  return p;
}

int qgemm_noalloc(const axb_qgemm_desc* d, cudaStream_t stream) {
  AXB_CHECK_ARG(d, "null descriptor");
  AXB_CHECK_ARG(d->M >= 1 && d->M <= kNoAllocMaxM, "qgemm_noalloc: M must be in [1, %d] (got %d); use axb_qgemm",
                kNoAllocMaxM, d->M);
  AXB_CHECK_ARG(max_ctas() <= (long long)kNoAllocMaxCtas, "qgemm_noalloc: device has too many SMs for the scratch");
  AXB_CHECK_ARG(d->N > 0 && (size_t)((d->N + 15) / 16) <= kMaxTiles, "qgemm_noalloc: N out of range (%d)", d->N);
  int rc = AXB_OK;
  char* ws = reinterpret_cast<char*>(noalloc_scratch(&rc));
  if (rc) return rc;
  // the array keeps the previous call's contents: clear the tile counters this
  // call uses (a call that ended early may leave them set).  The error word is
  // left alone: it holds until axb_qgemm_noalloc_status reads and clears it.
  cudaError_t e = cudaMemsetAsync(ws + kCountersOff, 0, (size_t)((d->N + 15) / 16) * 4, stream);
  if (e != cudaSuccess) return cuda_status(e, "qgemm_noalloc: clear scratch");
  axb_qgemm_desc dd = *d;
  dd.workspace = ws;
  dd.workspace_bytes = kNoAllocBytes;
  return qgemm(&dd, stream);
}

// The error word of the library-held scratch: same contract as qgemm_status.
int qgemm_noalloc_status(cudaStream_t stream) {
  int rc = AXB_OK;
  void* ws = noalloc_scratch(&rc);
  if (rc) return rc;
  return qgemm_status(ws, stream);
}

}  // namespace axb

using namespace axb;

extern "C" {

size_t axb_q4t_words_bytes(int N, int K) { return (size_t)((N + 15) / 16) * (K / 64) * 512; }
size_t axb_q4t_scales_bytes(int N, int K, int group, int fmt) {
  return (size_t)((N + 15) / 16) * (K / group) * 16 * (fmt == AXB_W_Q4T_AFFINE ? 2 : 1) * sizeof(uint16_t);
}

int axb_q4t_pack(const float* w, int N, int K, int group, int fmt, int gu, void* words, void* scales, void* stream) {
  AXB_CHECK_ARG(w && words && scales, "q4t_pack: null pointer");
  AXB_CHECK_ARG(K % 64 == 0 && (group == 64 || group == 128) && K % group == 0, "q4t_pack: bad K/group");
  AXB_CHECK_ARG(fmt == AXB_W_Q4T_SYM || fmt == AXB_W_Q4T_AFFINE, "q4t_pack: bad fmt");
  AXB_CHECK_ARG(!gu || N % 16 == 0, "q4t_pack: gate/up interleave needs N %% 16 == 0");
  dim3 grid(K / 64, (N + 15) / 16);
  q4t_pack_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(w, N, K, group, fmt == AXB_W_Q4T_SYM, gu,
                                                          (uint32_t*)words, (__half*)scales);
  return launch_status("q4t_pack");
}

int axb_q4t_from_q4g64(const int32_t* w_packed, const uint16_t* sb, int N, int K, int gu, void* words, void* scales,
                       void* stream) {
  AXB_CHECK_ARG(w_packed && sb && words && scales, "q4t_from_q4g64: null pointer");
  AXB_CHECK_ARG(N > 0 && K > 0 && K % 64 == 0, "q4t_from_q4g64: bad shape (%d, %d)", N, K);
  AXB_CHECK_ARG(!gu || N % 16 == 0, "q4t_from_q4g64: gate/up interleave needs N %% 16 == 0");
  dim3 grid(K / 64, (N + 15) / 16);
  q4t_from_q4g64_kernel<<<grid, 160, 0, (cudaStream_t)stream>>>((const uint32_t*)w_packed, (const __half*)sb, N, K, gu,
                                                                 (uint32_t*)words, (__half*)scales);
  return launch_status("q4t_from_q4g64");
}

int axb_q4t_from_marlin(const int32_t* wm, const uint16_t* sb, int n_tiles8, int K, int n_out, int gu, void* words,
                        void* scales, void* stream) {
  AXB_CHECK_ARG(wm && sb && words && scales, "q4t_from_marlin: null pointer");
  AXB_CHECK_ARG(K % 64 == 0 && n_out > 0 && n_out <= n_tiles8 * 8, "q4t_from_marlin: bad shape");
  AXB_CHECK_ARG(!gu || n_out % 16 == 0, "q4t_from_marlin: gate/up interleave needs N %% 16 == 0");
  dim3 grid(K / 64, (n_out + 15) / 16);
  q4t_from_marlin_kernel<<<grid, 160, 0, (cudaStream_t)stream>>>((const uint32_t*)wm, (const __half*)sb,
                                                                 n_tiles8 * 8, K, n_out, gu, (uint32_t*)words,
                                                                 (__half*)scales);
  return launch_status("q4t_from_marlin");
}

int axb_q4t_dequant(const void* words, const void* scales, int N, int K, int group, int fmt, int gu, uint16_t* out,
                    void* stream) {
  AXB_CHECK_ARG(words && scales && out, "q4t_dequant: null pointer");
  AXB_CHECK_ARG(K % 64 == 0 && (group == 64 || group == 128) && K % group == 0, "q4t_dequant: bad K/group");
  dim3 grid(K / 64, (N + 15) / 16);
  q4t_dequant_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>((const uint32_t*)words, (const __half*)scales, N, K,
                                                             group, fmt == AXB_W_Q4T_SYM, gu, (__half*)out);
  return launch_status("q4t_dequant");
}

int axb_q4_marlin_dequant(const int32_t* wm, const uint16_t* sb, int n_tiles8, int K, int n_out, uint16_t* out,
                          void* stream) {
  AXB_CHECK_ARG(wm && sb && out && K % 64 == 0 && n_out <= n_tiles8 * 8 && n_out > 0, "marlin_dequant: bad args");
  dim3 grid((K + 255) / 256, n_out);
  marlin_dequant_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const uint32_t*)wm, (const __half*)sb, K, n_out,
                                                                (__half*)out);
  return launch_status("marlin_dequant");
}

int axb_q8_pack(const float* w, int N, int K, int32_t* out, uint16_t* sb, void* stream) {
  AXB_CHECK_ARG(w && out && sb && N > 0 && K % 64 == 0, "q8_pack: bad args");
  long long items = (long long)N * (K / 64);
  q8_pack_kernel<<<(unsigned)((items + 7) / 8), 256, 0, (cudaStream_t)stream>>>(w, N, K, (uint32_t*)out, (__half*)sb);
  return launch_status("q8_pack");
}

int axb_q8_rows(const int32_t* w, const uint16_t* sb, const int32_t* idx, int n_idx, int K, uint16_t* out,
                void* stream) {
  AXB_CHECK_ARG(w && sb && idx && out && K % 64 == 0 && n_idx >= 0, "q8_rows: bad args");
  if (n_idx == 0) return AXB_OK;
  q8_rows_kernel<<<n_idx, 256, 0, (cudaStream_t)stream>>>((const uint32_t*)w, (const __half*)sb, idx, K,
                                                          (__half*)out);
  return launch_status("q8_rows");
}

int axb_ternary_dequant(const uint8_t* w, const uint16_t* s, int N, int K, int per_tensor, uint16_t* out,
                        void* stream) {
  AXB_CHECK_ARG(w && s && out && K % 64 == 0 && N > 0, "ternary_dequant: bad args");
  dim3 grid((K + 255) / 256, N);
  ternary_dequant_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(w, (const __half*)s, K, per_tensor, (__half*)out);
  return launch_status("ternary_dequant");
}

int axb_q2_dequant(const uint8_t* w, const uint16_t* sb, int N, int K, uint16_t* out, void* stream) {
  AXB_CHECK_ARG(w && sb && out && K % 64 == 0 && N > 0, "q2_dequant: bad args");
  dim3 grid((K + 255) / 256, N);
  q2_dequant_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(w, (const __half*)sb, K, (__half*)out);
  return launch_status("q2_dequant");
}

size_t axb_qgemm_workspace_bytes(int N, int K, int M, int group) {
  (void)K;
  (void)group;
  return qgemm_workspace(N, M);
}

int axb_qgemm(const axb_qgemm_desc* d, void* stream) { return qgemm(d, (cudaStream_t)stream); }

int axb_qgemm_noalloc(const axb_qgemm_desc* d, void* stream) { return qgemm_noalloc(d, (cudaStream_t)stream); }

size_t axb_qgemm_noalloc_scratch_bytes(void) { return kNoAllocBytes; }

int axb_qgemm_noalloc_status(void* stream) { return qgemm_noalloc_status((cudaStream_t)stream); }

int axb_qgemm_status(void* workspace, void* stream) {
  AXB_CHECK_ARG(workspace, "qgemm_status: null workspace");
  return qgemm_status(workspace, (cudaStream_t)stream);
}

}  // extern "C"
