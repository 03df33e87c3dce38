// q4t weight-format device helpers shared by the GEMV and the step kernel.
#pragma once

#include "axb_common.cuh"

namespace axb {

__host__ __device__ inline int gu_src_row(int p, int N, int gu) {
  // packed row p -> source row; gate/up interleave by 8 for the SwiGLU epilogue
  if (!gu) return p;
  int F = N >> 1;
  int tile = p >> 4, h = (p >> 3) & 1, i = p & 7;
  int j = tile * 8 + i;
  if (j >= F) return N;  // padding
  return h ? F + j : j;
}

// nibble pairs of one word -> four A-fragment registers holding (q - Z)
template <int Z>
__device__ __forceinline__ void unpack_word(uint32_t w, uint32_t (&a)[4]) {
  const uint32_t MAGIC = 0x64006400u;
  uint32_t lo0 = lop3_and_or(w, 0x000F000Fu, MAGIC);
  uint32_t hi0 = lop3_and_or(w, 0x00F000F0u, MAGIC);
  uint32_t w8 = w >> 8;
  uint32_t lo1 = lop3_and_or(w8, 0x000F000Fu, MAGIC);
  uint32_t hi1 = lop3_and_or(w8, 0x00F000F0u, MAGIC);
  // lo: 1024 + q ; hi: 1024 + 16 q  (exact fp16 values)
  const __half2 sub = __halves2half2(__ushort_as_half(0x6400 + Z), __ushort_as_half(0x6400 + Z));  // 1024+Z
  const __half2 mul = __float2half2_rn(1.0f / 16.0f);
  const __half2 add = __float2half2_rn(-(64.0f + (float)Z));
  a[0] = h2_as_u32(__hsub2(u32_as_h2(lo0), sub));
  a[1] = h2_as_u32(__hfma2(u32_as_h2(hi0), mul, add));
  a[2] = h2_as_u32(__hsub2(u32_as_h2(lo1), sub));
  a[3] = h2_as_u32(__hfma2(u32_as_h2(hi1), mul, add));
}

}  // namespace axb
