// 2-bit weight formats on the tensor cores: BitNet b1.58 ternary and 2-bit
// affine ("Q2_K" in the reference), GEMV / small-M GEMM for sm_100a.
//
// Replaces qmv_ternary / qmm_ternary (axiomlm/kernels/quant.py:298-336, Metal
// qmv_ternary_half_kernel :3990 / qmm_ternary_half_kernel :4074) and
// qmv_q2_k / qmm_q2_k (quant.py:406-444, Metal :4167 / :4246), plus the
// benchmark-only layouts (no reference implementation) (per-tensor ternary scale; K-quant-style 256-element
// super-blocks with 4-bit sub-scales and sub-mins).
//
// Layout q2t.  The reference's row-major codes (4 per byte, element i of a
// byte at bits 2i) are relaid out once into 16-row tiles and 128-wide
// k-blocks of 512 bytes.  Lane l = 4g + c of a warp owns 16 bytes of a block:
// word j (0..3) holds the A fragments of two m16n8k16 steps h = 0, 1 for rows
// g and g + 8.  Fragment register rho = 4h + reg (reg 0..3 = a0..a3) holds
// the codes of k = 32j + 8c + 4h + 2(reg >> 1) + {0, 1}: its low element at
// bits [2 rho, 2 rho + 2), its high element at bits [16 + 2 rho, ...).  One
// shift and one lop3 with 0x64006400 give the fp16 pair (1024 + u_lo,
// 1024 + u_hi).  The k order inside a 32-wide span is a permutation shared by
// the A and B fragments, chosen so that lane c reads its 8 activations
// x[32j + 8c .. + 7] as one 128-bit load.
//
// Values.  u is the unsigned code.  Ternary: u = q + 1 (q in {-1, 0, 1}),
// w = q * s.  2-bit affine: w = u * s + b.  K-quant: w = d * sc * u -
// dmin * mn per 16-element sub-block.  The GEMV removes the 1024 offset
// exactly (hsub2), runs the MMA on q (ternary) or u (affine) and folds the
// group's scale (and bias times the group sum of x) into the fp32 accumulator
// once per 64-wide group; K-quant weights are dequantized in registers to
// fp16 first (one hfma2) because their sub-blocks are 16 wide.
#include <algorithm>

#include "axb_common.cuh"

namespace axb {

constexpr int kQ2KB = 128;     // k per q2t block
constexpr int kLbWarps = 8;    // warps per GEMV CTA (they split the k-blocks of one tile)
constexpr int kLbMaxM = 8;     // tokens per GEMV call

__host__ __device__ inline bool lb_fmt_ok(int fmt) {
  return fmt == AXB_W_TERNARY_G64 || fmt == AXB_W_TERNARY_PT || fmt == AXB_W_Q2_G64 || fmt == AXB_W_Q2K_SB256;
}

// ---- reference codes ----------------------------------------------------
// code of (row, k) in the reference's row-major packing (quant.py:264-274 /
// :370-381): byte k / 4 of the row, bits 2 (k % 4).
__device__ __forceinline__ int ref_code(const uint8_t* codes, int K, int row, int k) {
  return (codes[(size_t)row * (K / 4) + (k >> 2)] >> (2 * (k & 3))) & 3;
}
// ternary 2-bit code (0 -> 0, 1 -> +1, 2 -> -1; quant.py:287-291) as u = q + 1
__device__ __forceinline__ int ternary_u(int code) { return (code & 1) - ((code >> 1) & 1) + 1; }

// k of fragment register rho (element e) of word j for lane c
__host__ __device__ __forceinline__ int q2t_k(int j, int c, int rho, int e) {
  return 32 * j + 8 * c + 4 * (rho >> 2) + 2 * ((rho & 3) >> 1) + e;
}

// ---- relayout ------------------------------------------------------------
// One thread per (tile, k-block, lane): builds the lane's 4 words and, for
// c == 0 lanes, the metadata of rows g and g + 8.
__global__ void q2t_relayout_kernel(int fmt, const uint8_t* __restrict__ codes, const __half* __restrict__ s1,
                                    const uint8_t* __restrict__ sub, const __half* __restrict__ dm, int N, int K,
                                    uint32_t* __restrict__ words, uint8_t* __restrict__ meta,
                                    __half2* __restrict__ meta2) {
  const int KB = K / kQ2KB;
  const long long total = (long long)((N + 15) / 16) * KB * 32;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int lane = (int)(i & 31);
    const long long tb = i >> 5;  // tile * KB + kb
    const int kb = (int)(tb % KB), t = (int)(tb / KB);
    const int g = lane >> 2, c = lane & 3;
    uint32_t w4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t w = 0;
#pragma unroll
      for (int rho = 0; rho < 8; ++rho) {
        const int row = t * 16 + g + 8 * (rho & 1);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int k = kb * kQ2KB + q2t_k(j, c, rho, e);
          int u = 0;
          if (row < N) {
            const int code = ref_code(codes, K, row, k);
            u = (fmt == AXB_W_TERNARY_G64 || fmt == AXB_W_TERNARY_PT) ? ternary_u(code) : code;
          }
          w |= (uint32_t)u << (2 * rho + 16 * e);
        }
      }
      w4[j] = w;
    }
    reinterpret_cast<uint4*>(words)[i] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    if (c != 0) continue;
    const int rg = t * 16 + g, rg8 = rg + 8;
    if (fmt == AXB_W_TERNARY_G64) {  // (s[g], s[g+8]) per 64-wide group: [tb][g][grp] half2
      __half2* m = reinterpret_cast<__half2*>(meta) + (tb * 8 + g) * 2;
#pragma unroll
      for (int grp = 0; grp < 2; ++grp) {
        const int G = kb * 2 + grp;
        const __half a = rg < N ? s1[(size_t)rg * (K / 64) + G] : __float2half(0.f);
        const __half b = rg8 < N ? s1[(size_t)rg8 * (K / 64) + G] : __float2half(0.f);
        m[grp] = __halves2half2(a, b);
      }
    } else if (fmt == AXB_W_Q2_G64) {  // (scale, bias) of rows g, g+8 per group: [tb][g][grp][rr] half2
      __half2* m = reinterpret_cast<__half2*>(meta) + (tb * 8 + g) * 4;
#pragma unroll
      for (int grp = 0; grp < 2; ++grp)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int row = rr ? rg8 : rg;
          const int G = kb * 2 + grp;
          m[grp * 2 + rr] = row < N ? reinterpret_cast<const __half2*>(s1)[(size_t)row * (K / 64) + G]
                                    : __float2half2_rn(0.f);
        }
    } else if (fmt == AXB_W_Q2K_SB256) {
      // sub bytes [tb][g][c2][rr][j]: sub-block kb*8 + 2j + c2 of row g + 8 rr
      uint8_t* m = meta + (tb * 8 + g) * 16;
#pragma unroll
      for (int c2 = 0; c2 < 2; ++c2)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int row = rr ? rg8 : rg;
            m[c2 * 8 + rr * 4 + j] = row < N ? sub[(size_t)row * (K / 16) + kb * 8 + 2 * j + c2] : 0;
          }
      if ((kb & 1) == 0) {  // (d, dmin) of rows g, g+8 per super-block: [t][sb][g][rr] half2
        const int sb = kb / 2;
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int row = rr ? rg8 : rg;
          meta2[(((size_t)t * (K / 256) + sb) * 8 + g) * 2 + rr] =
              row < N ? reinterpret_cast<const __half2*>(dm)[(size_t)row * (K / 256) + sb] : __float2half2_rn(0.f);
        }
      }
    }
  }
}

// ---- dequant (the reference's value rule, for checking the relayout) -----
// out (N, K) fp16.  Ternary: fp16(q * s) (quant.py:293-295; exact).  2-bit
// affine: fp16(fp16(u * s) + b) (quant.py:399-401, two fp16 ops).  K-quant:
// fp16(fp32(d) * sc * u - fp32(dmin) * mn).
__global__ void q2t_dequant_kernel(int fmt, const uint32_t* __restrict__ words, const uint8_t* __restrict__ meta,
                                   const __half2* __restrict__ meta2, const __half* __restrict__ pt_scale, int N,
                                   int K, __half* __restrict__ out) {
  const int KB = K / kQ2KB;
  const long long total = (long long)((N + 15) / 16) * KB * 32;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int lane = (int)(i & 31);
    const long long tb = i >> 5;
    const int kb = (int)(tb % KB), t = (int)(tb / KB);
    const int g = lane >> 2, c = lane & 3;
    const uint4 wv = reinterpret_cast<const uint4*>(words)[i];
    const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int rho = 0; rho < 8; ++rho)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int rr = rho & 1, row = t * 16 + g + 8 * rr;
          if (row >= N) continue;
          const int kk = q2t_k(j, c, rho, e), k = kb * kQ2KB + kk;
          const int u = (w4[j] >> (2 * rho + 16 * e)) & 3;
          const int grp = kk >> 6;
          __half v;
          if (fmt == AXB_W_TERNARY_G64 || fmt == AXB_W_TERNARY_PT) {
            __half s;
            if (fmt == AXB_W_TERNARY_PT) {
              s = pt_scale[0];
            } else {
              const __half2 sp = reinterpret_cast<const __half2*>(meta)[(tb * 8 + g) * 2 + grp];
              s = rr ? __high2half(sp) : __low2half(sp);
            }
            v = __float2half_rn((float)(u - 1) * __half2float(s));
          } else if (fmt == AXB_W_Q2_G64) {
            const __half2 sb = reinterpret_cast<const __half2*>(meta)[(tb * 8 + g) * 4 + grp * 2 + rr];
            const __half p = __float2half_rn((float)u * __low2float(sb));
            v = __float2half_rn(__half2float(p) + __high2float(sb));
          } else {
            const int jc = kk >> 4;  // sub-block in the k-block = 2 j + (c >> 1)
            const uint8_t sbyte = meta[(tb * 8 + g) * 16 + (jc & 1) * 8 + rr * 4 + (jc >> 1)];
            const __half2 d2 = meta2[(((size_t)t * (K / 256) + kb / 2) * 8 + g) * 2 + rr];
            const float a = __low2float(d2) * (float)(sbyte & 15), b = __high2float(d2) * (float)(sbyte >> 4);
            v = __float2half_rn((float)u * a - b);
          }
          out[(size_t)row * K + k] = v;
        }
  }
}

// ---- group sums of x (2-bit affine: the bias term) ----------------------
__global__ void lb_xsum_kernel(const __half* __restrict__ x, int ldx, int M, int K, float* __restrict__ xsum) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // group * kLbMaxM + token
  const int grp = i / kLbMaxM, m = i % kLbMaxM;
  if (grp >= K / 64) return;
  float s = 0.f;
  if (m < M)
    for (int k = 0; k < 64; ++k) s += __half2float(x[(size_t)m * ldx + grp * 64 + k]);
  xsum[i] = s;
}

// ---- GEMV ---------------------------------------------------------------
__device__ __forceinline__ uint32_t q2_raw(uint32_t w, int rho) {
  return lop3_and_or(w >> (2 * rho), 0x00030003u, 0x64006400u);  // (1024 + u_lo, 1024 + u_hi)
}
__device__ __forceinline__ void mma_16816_acc(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  mma_16816(d, a, b0, b1, d);
}

// One CTA per 16-row tile; its 8 warps take k-blocks kb = warp, warp + 8, ...
// and meet in shared memory in warp order.
template <int FMT>
__global__ void __launch_bounds__(kLbWarps * 32) lbgemv_kernel(const uint4* __restrict__ words,
                                                               const uint8_t* __restrict__ meta,
                                                               const __half2* __restrict__ meta2,
                                                               const __half* __restrict__ pt_scale,
                                                               const __half* __restrict__ x, int ldx,
                                                               const float* __restrict__ xsum, int N, int K, int M,
                                                               __half* __restrict__ y, int ldy,
                                                               const __half* __restrict__ bias, int nsplit,
                                                               float* __restrict__ part) {
  __shared__ float4 red[kLbWarps][32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int t = blockIdx.x, KB = K / kQ2KB;
  const int sp = blockIdx.y, kb0 = (int)((long long)sp * KB / nsplit), kb1 = (int)((long long)(sp + 1) * KB / nsplit);
  constexpr bool TER = FMT == AXB_W_TERNARY_G64 || FMT == AXB_W_TERNARY_PT;
  const __half2 off = TER ? __float2half2_rn(1025.f) : __float2half2_rn(1024.f);  // exact: raw - off = q or u
  const bool tok = g < M;  // B-fragment token of this lane
  const __half* xr = x + (size_t)(tok ? g : 0) * ldx + 8 * c;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  // the k-blocks of a warp are few (K / 128 / warps): issue the weight and
  // metadata loads of up to kLbAhead of them before any math, so their latencies overlap
  constexpr int kLbAhead = 4;
  auto load_kb = [&](int kb, uint4& wv, uint4& mv, uint2& dmv) {
    const size_t tb = (size_t)t * KB + kb;
    wv = ldg_nc_v4(words + tb * 32 + lane);
    mv = make_uint4(0, 0, 0, 0);
    dmv = make_uint2(0, 0);
    if (FMT == AXB_W_TERNARY_G64) {
      const uint2 m2 = __ldg(reinterpret_cast<const uint2*>(meta) + tb * 8 + g);
      mv.x = m2.x;
      mv.y = m2.y;
    } else if (FMT == AXB_W_Q2_G64) {
      mv = __ldg(reinterpret_cast<const uint4*>(meta) + tb * 8 + g);
    } else if (FMT == AXB_W_Q2K_SB256) {
      const uint2 s8 = __ldg(reinterpret_cast<const uint2*>(meta + (tb * 8 + g) * 16 + (c >> 1) * 8));
      mv.x = s8.x;  // row g: sub-blocks of words 0..3
      mv.y = s8.y;  // row g + 8
      dmv = __ldg(reinterpret_cast<const uint2*>(meta2) + ((size_t)t * (K / 256) + kb / 2) * 8 + g);
    }
  };
  auto compute_kb = [&](int kb, const uint4 wv, const uint4 mv, const uint2 dmv) {
    const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
    float tmp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 xv = tok ? __ldg(reinterpret_cast<const uint4*>(xr + kb * kQ2KB + 32 * j)) : make_uint4(0, 0, 0, 0);
      uint32_t r[8];
#pragma unroll
      for (int rho = 0; rho < 8; ++rho) r[rho] = q2_raw(w4[j], rho);
      if (FMT == AXB_W_Q2K_SB256) {
        // w = fp16(A u + B) per row and sub-block (A = d sc, B = -dmin mn)
        float2 d0 = __half22float2(u32_as_h2(dmv.x)), d1 = __half22float2(u32_as_h2(dmv.y));
        const uint32_t sb0 = (mv.x >> (8 * j)) & 0xFF, sb1 = (mv.y >> (8 * j)) & 0xFF;
        const __half2 A0 = __float2half2_rn(d0.x * (float)(sb0 & 15)), B0 = __float2half2_rn(-d0.y * (float)(sb0 >> 4));
        const __half2 A1 = __float2half2_rn(d1.x * (float)(sb1 & 15)), B1 = __float2half2_rn(-d1.y * (float)(sb1 >> 4));
#pragma unroll
        for (int rho = 0; rho < 8; ++rho) {
          const __half2 u = __hsub2(u32_as_h2(r[rho]), off);
          r[rho] = h2_as_u32(__hfma2(u, (rho & 1) ? A1 : A0, (rho & 1) ? B1 : B0));
        }
      } else {
#pragma unroll
        for (int rho = 0; rho < 8; ++rho) r[rho] = h2_as_u32(__hsub2(u32_as_h2(r[rho]), off));
      }
      const uint32_t a0[4] = {r[0], r[1], r[2], r[3]}, a1[4] = {r[4], r[5], r[6], r[7]};
      float(&dst)[4] = (FMT == AXB_W_Q2K_SB256 || FMT == AXB_W_TERNARY_PT) ? acc : tmp;
      mma_16816_acc(dst, a0, xv.x, xv.y);
      mma_16816_acc(dst, a1, xv.z, xv.w);
      if ((FMT == AXB_W_TERNARY_G64 || FMT == AXB_W_Q2_G64) && (j & 1)) {  // a 64-wide group is complete
        const int grp = j >> 1;
        if (FMT == AXB_W_TERNARY_G64) {
          const float2 s = __half22float2(u32_as_h2(grp ? mv.y : mv.x));  // (row g, row g + 8)
          acc[0] = __fmaf_rn(s.x, tmp[0], acc[0]);
          acc[1] = __fmaf_rn(s.x, tmp[1], acc[1]);
          acc[2] = __fmaf_rn(s.y, tmp[2], acc[2]);
          acc[3] = __fmaf_rn(s.y, tmp[3], acc[3]);
        } else {
          const float2 sb0 = __half22float2(u32_as_h2(grp ? mv.z : mv.x));  // (scale, bias) of row g
          const float2 sb1 = __half22float2(u32_as_h2(grp ? mv.w : mv.y));  // row g + 8
          const float2 X = *reinterpret_cast<const float2*>(xsum + ((size_t)kb * 2 + grp) * kLbMaxM + 2 * c);
          acc[0] = __fmaf_rn(sb0.x, tmp[0], __fmaf_rn(sb0.y, X.x, acc[0]));
          acc[1] = __fmaf_rn(sb0.x, tmp[1], __fmaf_rn(sb0.y, X.y, acc[1]));
          acc[2] = __fmaf_rn(sb1.x, tmp[2], __fmaf_rn(sb1.y, X.x, acc[2]));
          acc[3] = __fmaf_rn(sb1.x, tmp[3], __fmaf_rn(sb1.y, X.y, acc[3]));
        }
        tmp[0] = tmp[1] = tmp[2] = tmp[3] = 0.f;
      }
    }
    };
  for (int kb = kb0 + wid; kb < kb1; kb += kLbAhead * kLbWarps) {
    uint4 wv[kLbAhead], mv[kLbAhead];
    uint2 dmv[kLbAhead];
#pragma unroll
    for (int u = 0; u < kLbAhead; ++u)
      if (kb + u * kLbWarps < kb1) load_kb(kb + u * kLbWarps, wv[u], mv[u], dmv[u]);
#pragma unroll
    for (int u = 0; u < kLbAhead; ++u)
      if (kb + u * kLbWarps < kb1) compute_kb(kb + u * kLbWarps, wv[u], mv[u], dmv[u]);
  }
  red[wid][lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  __syncthreads();
  if (wid != 0) return;
  float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int w = 0; w < kLbWarps; ++w) {
    const float4 p = red[w][lane];
    v[0] += p.x;
    v[1] += p.y;
    v[2] += p.z;
    v[3] += p.w;
  }
  const float pts = FMT == AXB_W_TERNARY_PT ? __half2float(pt_scale[0]) : 1.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int n = 2 * c + (q & 1), row = t * 16 + g + 8 * (q >> 1);
    if (n >= M || row >= N) continue;
    if (nsplit > 1) {  // this split's fp32 partial; lb_reduce_kernel finishes the row
      part[((size_t)sp * M + n) * N + row] = v[q];
      continue;
    }
    float o = FMT == AXB_W_TERNARY_PT ? v[q] * pts : v[q];
    if (bias) o += __half2float(bias[row]);
    y[(size_t)n * ldy + row] = __float2half_rn(o);
  }
}

// split-K: y[n][row] = fp16(sum of the splits in order (x the per-tensor scale) + bias)
__global__ void lb_reduce_kernel(const float* __restrict__ part, int S, int M, int N, const __half* __restrict__ pt,
                                 const __half* __restrict__ bias, __half* __restrict__ y, int ldy) {
  const size_t total = (size_t)M * N;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int n = (int)(i / N), row = (int)(i % N);
    float o = 0.f;
    for (int q = 0; q < S; ++q) o += part[(size_t)q * total + i];
    if (pt) o *= __half2float(pt[0]);
    if (bias) o += __half2float(bias[row]);
    y[(size_t)n * ldy + row] = __float2half_rn(o);
  }
}

// k splits: enough CTAs (8 warps each) to fill the GPU when the tiles alone do not
int lb_splits(int N, int K) {
  const int tiles = (N + 15) / 16, KB = K / kQ2KB;
  int S = (4 * num_sms() + tiles - 1) / tiles;
  return std::max(1, std::min(S, std::max(1, KB / kLbWarps)));
}

}  // namespace axb

using namespace axb;

extern "C" {

size_t axb_q2t_words_bytes(int N, int K) {
  if (N <= 0 || K <= 0 || K % kQ2KB) return 0;
  return (size_t)((N + 15) / 16) * (K / kQ2KB) * 512;
}

size_t axb_q2t_meta_bytes(int fmt, int N, int K) {
  if (N <= 0 || K <= 0 || K % kQ2KB || !lb_fmt_ok(fmt)) return 0;
  const size_t tb = (size_t)((N + 15) / 16) * (K / kQ2KB);
  switch (fmt) {
    case AXB_W_TERNARY_G64: return tb * 8 * 8;
    case AXB_W_Q2_G64: return tb * 8 * 16;
    case AXB_W_Q2K_SB256: return tb * 8 * 16;
    default: return 0;
  }
}

size_t axb_q2t_meta2_bytes(int fmt, int N, int K) {
  if (fmt != AXB_W_Q2K_SB256 || N <= 0 || K <= 0 || K % 256) return 0;
  return (size_t)((N + 15) / 16) * (K / 256) * 8 * 2 * 4;
}

int axb_q2t_from_ref(int fmt, const uint8_t* codes, const void* s1, const void* s2, int N, int K, void* words,
                     void* meta, void* meta2, void* stream) {
  AXB_CHECK_ARG(lb_fmt_ok(fmt), "q2t_from_ref: format %d is not a 2-bit format", fmt);
  AXB_CHECK_ARG(N > 0 && K > 0 && K % kQ2KB == 0, "q2t_from_ref: K=%d must be a positive multiple of 128", K);
  AXB_CHECK_ARG(fmt != AXB_W_Q2K_SB256 || K % 256 == 0, "q2t_from_ref: K-quant needs K %% 256 == 0");
  AXB_CHECK_ARG(codes && words, "q2t_from_ref: null codes / words");
  AXB_CHECK_ARG(fmt == AXB_W_TERNARY_PT || (s1 && meta), "q2t_from_ref: scales and meta are required");
  AXB_CHECK_ARG(fmt != AXB_W_Q2K_SB256 || (s2 && meta2), "q2t_from_ref: K-quant needs (d, dmin) and meta2");
  const long long total = (long long)((N + 15) / 16) * (K / kQ2KB) * 32;
  const int grid = (int)std::min<long long>((total + 255) / 256, 65535);
  q2t_relayout_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      fmt, codes, (const __half*)s1, (const uint8_t*)s1, (const __half*)s2, N, K, (uint32_t*)words, (uint8_t*)meta,
      (__half2*)meta2);
  return launch_status("q2t_from_ref");
}

int axb_q2t_dequant(int fmt, const void* words, const void* meta, const void* meta2, const uint16_t* pt_scale, int N,
                    int K, uint16_t* out, void* stream) {
  AXB_CHECK_ARG(lb_fmt_ok(fmt), "q2t_dequant: format %d is not a 2-bit format", fmt);
  AXB_CHECK_ARG(N > 0 && K > 0 && K % kQ2KB == 0 && words && out, "q2t_dequant: bad args");
  AXB_CHECK_ARG(fmt != AXB_W_TERNARY_PT || pt_scale, "q2t_dequant: per-tensor ternary needs its scale");
  AXB_CHECK_ARG(fmt == AXB_W_TERNARY_PT || meta, "q2t_dequant: meta is required");
  AXB_CHECK_ARG(fmt != AXB_W_Q2K_SB256 || meta2, "q2t_dequant: K-quant needs meta2");
  const long long total = (long long)((N + 15) / 16) * (K / kQ2KB) * 32;
  const int grid = (int)std::min<long long>((total + 255) / 256, 65535);
  q2t_dequant_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(fmt, (const uint32_t*)words, (const uint8_t*)meta,
                                                             (const __half2*)meta2, (const __half*)pt_scale, N, K,
                                                             (__half*)out);
  return launch_status("q2t_dequant");
}

static size_t lb_xsum_bytes(int fmt, int K) {
  return fmt == AXB_W_Q2_G64 ? ((size_t)(K / 64) * kLbMaxM * sizeof(float) + 255) / 256 * 256 : 0;
}

size_t axb_lbgemv_workspace_bytes(int fmt, int N, int K, int M) {
  if (N <= 0 || K <= 0 || K % kQ2KB || M < 1) return 0;
  const int S = lb_splits(N, K);
  return lb_xsum_bytes(fmt, K) + (S > 1 ? (size_t)S * kLbMaxM * N * sizeof(float) : 0);
}

int axb_lbgemv(const axb_lbgemv_desc* d, void* stream) {
  AXB_CHECK_ARG(d, "lbgemv: null descriptor");
  AXB_CHECK_ARG(lb_fmt_ok(d->fmt), "lbgemv: format %d is not a 2-bit format", d->fmt);
  AXB_CHECK_ARG(d->N > 0 && d->K > 0 && d->K % kQ2KB == 0, "lbgemv: N=%d K=%d (K must be a multiple of 128)", d->N,
                d->K);
  AXB_CHECK_ARG(d->M >= 1 && d->M <= kLbMaxM, "lbgemv: M=%d out of [1, %d]", d->M, kLbMaxM);
  AXB_CHECK_ARG(d->words && d->x && d->y && d->ldx >= d->K && d->ldy >= d->N, "lbgemv: bad pointers / strides");
  AXB_CHECK_ARG((reinterpret_cast<uintptr_t>(d->x) & 15) == 0 && d->ldx % 8 == 0,
                "lbgemv: x must be 16-byte aligned with ldx a multiple of 8");
  AXB_CHECK_ARG(d->fmt == AXB_W_TERNARY_PT || d->meta, "lbgemv: meta is required");
  AXB_CHECK_ARG(d->fmt != AXB_W_TERNARY_PT || d->pt_scale, "lbgemv: per-tensor ternary needs its scale");
  AXB_CHECK_ARG(d->fmt != AXB_W_Q2K_SB256 || (d->meta2 && d->K % 256 == 0), "lbgemv: K-quant needs meta2");
  const size_t need = axb_lbgemv_workspace_bytes(d->fmt, d->N, d->K, d->M);
  AXB_CHECK_ARG(need == 0 || (d->workspace && d->workspace_bytes >= need), "lbgemv: workspace %zu < %zu bytes",
                d->workspace_bytes, need);
  cudaStream_t st = (cudaStream_t)stream;
  float* xsum = (float*)d->workspace;
  const int S = lb_splits(d->N, d->K);
  float* part = S > 1 ? (float*)((char*)d->workspace + lb_xsum_bytes(d->fmt, d->K)) : nullptr;
  if (lb_xsum_bytes(d->fmt, d->K)) {
    const int n = d->K / 64 * kLbMaxM;
    lb_xsum_kernel<<<(n + 127) / 128, 128, 0, st>>>((const __half*)d->x, d->ldx, d->M, d->K, xsum);
  }
  const int tiles = (d->N + 15) / 16;
#define AXB_LB(F)                                                                                              \
  case F:                                                                                                      \
    lbgemv_kernel<F><<<dim3(tiles, S), kLbWarps * 32, 0, st>>>(                                               \
        (const uint4*)d->words, (const uint8_t*)d->meta, (const __half2*)d->meta2, (const __half*)d->pt_scale, \
        (const __half*)d->x, d->ldx, xsum, d->N, d->K, d->M, (__half*)d->y, d->ldy, (const __half*)d->bias, S,   \
        part);                                                                                                 \
    break;
  switch (d->fmt) {
    AXB_LB(AXB_W_TERNARY_G64)
    AXB_LB(AXB_W_TERNARY_PT)
    AXB_LB(AXB_W_Q2_G64)
    AXB_LB(AXB_W_Q2K_SB256)
  }
#undef AXB_LB
  if (int rc = launch_status("lbgemv")) return rc;
  if (S > 1) {
    const size_t total = (size_t)d->M * d->N;
    const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)num_sms() * 4);
    lb_reduce_kernel<<<blocks, 256, 0, st>>>(part, S, d->M, d->N,
                                             d->fmt == AXB_W_TERNARY_PT ? (const __half*)d->pt_scale : nullptr,
                                             (const __half*)d->bias, (__half*)d->y, d->ldy);
    return launch_status("lbgemv reduce");
  }
  return AXB_OK;
}

}  // extern "C"
