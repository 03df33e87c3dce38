// KV-cache quantization and row-load helpers shared by the attention kernels
// and the step kernel.
#pragma once

#include "axb_common.cuh"

namespace axb {

// ---------------------------------------------------------------- quantize
// The reference's rule (quant.py:709-719, :788-797) for one group, evaluated
// on fp32 inputs (the model path: K after RoPE and V are fp32 tensors there) or
// on fp16 inputs (the op path).  Returns the fp16 scale and writes the ratio
// x / scale, rounded to fp16 first on the fp16 path.
__device__ __forceinline__ float kv_scale(float amax, float qmax, bool fp32_in) {
  float r = __fdiv_rn(amax, qmax);
  if (fp32_in) r = fmaxf(r, 1e-8f);  // the fp16 clamp at 1e-8 is a no-op
  return __half2float(__float2half_rn(r));
}
__device__ __forceinline__ float kv_ratio(float x, float scale, bool fp32_in) {
  float r = __fdiv_rn(x, scale);
  if (!fp32_in) r = __half2float(__float2half_rn(r));
  return r;
}
__device__ __forceinline__ uint8_t fp8_code(float x, float scale, bool fp32_in) {
  // scale 0 (amax below fp16 range): the reference divides by zero and stores
  // NaN codes; write zero codes instead so the cache stays finite.
  if (scale == 0.f) return 0;
  return float_to_e4m3(kv_ratio(x, scale, fp32_in));
}
__device__ __forceinline__ int int4_code(float x, float scale, bool fp32_in) {
  if (scale == 0.f) return x > 0.f ? 7 : (x < 0.f ? -8 : 0);  // +-inf clamp, NaN -> 0 (as the reference)
  float r = rintf(kv_ratio(x, scale, fp32_in));
  return (int)fminf(fmaxf(r, -8.f), 7.f);
}

// lanes in the same scale group: group of G elements over EPL elements/lane
__device__ __forceinline__ float group_max(float v, int lanes_per_group) {
  for (int o = 1; o < lanes_per_group; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// one warp quantizes one hd-vector held EPL = hd/32 elements per lane
// (not inlined: it runs once per row written, and its FP8 rounding is long).
// Returns this lane's bytes of the row (EPL fp16 values, EPL FP8 codes or
// EPL/2 INT4 bytes, little-endian in .x then .y) and, in *scale_out, the fp16
// scale of its group, so a caller can also place the row elsewhere.
template <int EPL>
__device__ __noinline__ uint2 store_kv_row(const float (&v)[EPL], int lane, int kv_type, int G, bool fp32_in,
                                           uint8_t* row, __half* srow, float* scale_out = nullptr) {
  uint32_t pk[2] = {0u, 0u};
  if (kv_type == AXB_KV_F16) {
    __half* r = reinterpret_cast<__half*>(row);
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const __half h = __float2half_rn(v[e]);
      r[lane * EPL + e] = h;
      pk[e >> 1] |= (uint32_t)__half_as_ushort(h) << (16 * (e & 1));
    }
    if (scale_out) *scale_out = 1.f;
    return make_uint2(pk[0], pk[1]);
  }
  float am = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) am = fmaxf(am, fabsf(v[e]));
  const int lpg = G / EPL;  // lanes per scale group
  am = group_max(am, lpg);
  const float qmax = kv_type == AXB_KV_FP8 ? 448.f : 7.f;
  const float sc = kv_scale(am, qmax, fp32_in);
  if (srow && (lane % lpg) == 0) srow[(lane * EPL) / G] = __float2half_rn(sc);
  if (scale_out) *scale_out = sc;
  if (kv_type == AXB_KV_FP8) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const uint8_t b = fp8_code(v[e], sc, fp32_in);
      row[lane * EPL + e] = b;
      pk[e >> 2] |= (uint32_t)b << (8 * (e & 3));
    }
  } else {
#pragma unroll
    for (int e = 0; e < EPL; e += 2) {
      int lo = int4_code(v[e], sc, fp32_in), hi = int4_code(v[e + 1], sc, fp32_in);
      const uint8_t b = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
      row[(lane * EPL + e) >> 1] = b;
      pk[0] |= (uint32_t)b << (8 * (e >> 1));
    }
  }
  return make_uint2(pk[0], pk[1]);
}

__host__ __device__ __forceinline__ int kv_row_bytes(int kv_type, int hd) {
  return kv_type == AXB_KV_F16 ? hd * 2 : (kv_type == AXB_KV_FP8 ? hd : hd / 2);
}

// ---------------------------------------------------------------- row loads
// K/V row loaders: element e of the row as fp32 *without* the group scale.
__device__ __forceinline__ float kv_elem(const uint8_t* row, int type, int e) {
  if (type == AXB_KV_F16) return __half2float(reinterpret_cast<const __half*>(row)[e]);
  if (type == AXB_KV_FP8) return e4m3x2_to_float2((uint16_t)row[e]).x;
  uint8_t c = row[e >> 1];
  int nib = (e & 1) ? (c >> 4) : (c & 0xF);
  return (float)((nib ^ 8) - 8);
}

// Load 16 consecutive elements [e0, e0+16) of a row as fp32 (16-byte aligned
// chunks: 32 B fp16, 16 B fp8, 8 B int4).
__device__ __forceinline__ void kv_load16(const uint8_t* row, int type, int e0, float (&o)[16]) {
  if (type == AXB_KV_F16) {
    const uint4* p = reinterpret_cast<const uint4*>(row + e0 * 2);
    uint4 a = p[0], b = p[1];
    const __half2* ha = reinterpret_cast<const __half2*>(&a);
    const __half2* hb = reinterpret_cast<const __half2*>(&b);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __half22float2(ha[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
      f = __half22float2(hb[i]);
      o[8 + 2 * i] = f.x;
      o[8 + 2 * i + 1] = f.y;
    }
  } else if (type == AXB_KV_FP8) {
    uint4 a = *reinterpret_cast<const uint4*>(row + e0);
    const uint16_t* u = reinterpret_cast<const uint16_t*>(&a);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float2 f = e4m3x2_to_float2(u[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  } else {
    uint2 a = *reinterpret_cast<const uint2*>(row + e0 / 2);
    const uint8_t* u = reinterpret_cast<const uint8_t*>(&a);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[2 * i] = (float)(((u[i] & 0xF) ^ 8) - 8);
      o[2 * i + 1] = (float)(((u[i] >> 4) ^ 8) - 8);
    }
  }
}

}  // namespace axb
