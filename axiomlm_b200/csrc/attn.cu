// KV-cache write (RoPE + FP8/INT4 quantization) and GQA attention for sm_100a.
//
// Replaces rope_kv_cache_write_quantized (axiomlm/kernels/quant.py:896-1008),
// StaticKVCache.update (engine/paged_cache.py:218-361), gqa_flash_decode_mps
// (kernels/ops.py:552-654), gqa_tree_verify_mps (ops.py:657-797) and
// compact_tree_path (paged_cache.py:376-462); Metal counterparts
// rope_kv_cache_write_{half,fp8,int4}_kernel, gqa_flash_decode_split_kv_*,
// gqa_tree_verify_split_kv_*, compact_tree_kv_* (metal_kernels.metal).
#include <algorithm>

#include "kv.cuh"

namespace axb {

// ---------------------------------------------------------------- rope + write
template <int EPL>
__global__ void rope_kv_write_kernel(const axb_kv_write_desc d) {
  pdl_wait();  // qkv comes from the preceding GEMV
  const int lane = threadIdx.x & 31;
  const int heads = d.n_head + 2 * d.n_kv_head;
  const long long item = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long rows = (long long)d.B * d.T;
  if (item >= rows * heads) return;
  const int row = (int)(item / heads), h = (int)(item % heads);
  const int b = row / d.T, t = row % d.T;
  const int hd = d.head_dim;
  const __half* src = reinterpret_cast<const __half*>(d.qkv) + (size_t)row * heads * hd + (size_t)h * hd;
  float v[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    float x = __half2float(src[lane * EPL + e]);
    if (d.bias) x = __half2float(__float2half_rn(__fadd_rn(x, __half2float(reinterpret_cast<const __half*>(d.bias)[h * hd + lane * EPL + e]))));
    v[e] = x;
  }
  const bool is_v = h >= d.n_head + d.n_kv_head;
  if (!is_v) {
    // RoPE on interleaved pairs: complex multiply as torch does on the CPU,
    // (a + bi)(c + di) = (ac - bd) + (ad + bc)i, every product rounded.
    const int off = d.depths ? d.depths[t] : t;
    const int rp = d.dev_params ? d.dev_params[0] : d.rope_pos;
    const int pos = (int)(((long long)rp + off) % d.rope_len);
    const float* f = d.rope + (size_t)pos * hd;  // (hd/2, 2)
#pragma unroll
    for (int e = 0; e < EPL; e += 2) {
      const int i = (lane * EPL + e) >> 1;
      const float c = f[2 * i], s = f[2 * i + 1];
      const float a = v[e], bb = v[e + 1];
      v[e] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(bb, s));
      v[e + 1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(bb, c));
    }
  }
  if (h < d.n_head) {
    float* q = d.q_out + (size_t)row * d.n_head * hd + (size_t)h * hd;
#pragma unroll
    for (int e = 0; e < EPL; ++e) q[lane * EPL + e] = v[e];
    return;
  }
  const int kvh = is_v ? h - d.n_head - d.n_kv_head : h - d.n_head;
  const int wp = d.dev_params ? d.dev_params[1] : d.write_pos;
  const int slot = (int)(((long long)wp + t) % d.max_seq);
  const size_t ridx = ((size_t)b * d.n_kv_head + kvh) * d.max_seq + slot;
  const int rb = kv_row_bytes(d.kv_type, hd);
  uint8_t* base = reinterpret_cast<uint8_t*>(is_v ? d.v_cache : d.k_cache) + ridx * rb;
  __half* sbase = nullptr;
  if (d.kv_type != AXB_KV_F16)
    sbase = reinterpret_cast<__half*>(is_v ? d.v_scale : d.k_scale) + ridx * (hd / d.kv_group);
  // K/V values are fp32 on the model path; on the fp16 op path round first
  if (!d.k_is_fp32) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) v[e] = __half2float(__float2half_rn(v[e]));
  }
  store_kv_row<EPL>(v, lane, d.kv_type, d.kv_group, d.k_is_fp32 != 0, base, sbase);
}

// standalone quantize of (rows, hd) fp16/fp32 vectors
template <int EPL>
__global__ void kv_quantize_kernel(const void* x, int fp32_in, int rows, int hd, int kv_type, int G, uint8_t* q,
                                   __half* sc) {
  const int lane = threadIdx.x & 31;
  const long long r = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  float v[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    size_t i = (size_t)r * hd + lane * EPL + e;
    v[e] = fp32_in ? reinterpret_cast<const float*>(x)[i] : __half2float(reinterpret_cast<const __half*>(x)[i]);
  }
  store_kv_row<EPL>(v, lane, kv_type, G, fp32_in != 0, q + (size_t)r * kv_row_bytes(kv_type, hd),
                    sc + (size_t)r * (hd / G));
}

// dequant: fp16(decoded fp16 value * fp16 scale) (quant.py:764-767, :846-851)
__global__ void kv_dequantize_kernel(const uint8_t* q, const __half* sc, long long n, int hd, int kv_type, int G,
                                     __half* out) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    long long r = i / hd;
    int e = (int)(i % hd);
    float s = __half2float(sc[r * (hd / G) + e / G]);
    float val;
    if (kv_type == AXB_KV_FP8) {
      uint8_t c = q[r * hd + e];
      val = e4m3x2_to_float2((uint16_t)c).x;
    } else {
      uint8_t c = q[r * (hd / 2) + e / 2];
      int nib = (e & 1) ? (c >> 4) : (c & 0xF);
      val = (float)((nib ^ 8) - 8);
    }
    out[i] = __float2half_rn(__fmul_rn(val, s));
  }
}

// ---------------------------------------------------------------- attention
constexpr int kMaxRep = 8;    // q heads per kv head
constexpr int kDecTile = 64;  // tokens per K/V stage (and online-softmax tile)
constexpr uint32_t kAttnWaitLimit = 1u << 22;

// Optional fusion of RoPE + KV write into decode attention (T = 1): q and the
// new token's K/V come straight from the QKV GEMV output.
struct DecodeFuse {
  const __half* qkv;  // (B, (Hq + 2 Hkv) hd) fp16, or nullptr: q in d.q, cache already written
  const float* rope;  // (rope_len, hd/2, 2)
  int rope_len;
};

// Split-K flash decode, T = 1 per sequence.  grid (max_splits, Hkv, B), 128
// threads.  A CTA owns one (sequence, kv head) and a chunk of <= kMaxChunk
// tokens.  Its K/V rows (contiguous per head) are bulk-copied into shared
// memory in one go -- issued before the PDL wait, since cached rows do not
// depend on the preceding kernel -- and the chunk is processed in a single
// pass (scores, softmax, PV) by all n_rep q heads of the group.  With fusion,
// the CTA whose chunk holds the new slot rotates and quantizes the new K/V
// row, writes it to the cache and patches its staged copy.  Split partials
// (O, m, l) are combined by the last CTA of the (sequence, head) in split
// order, all splits loaded in parallel.
constexpr int kMaxChunk = 256;

__host__ __device__ inline int decode_chunk_cap(int kv_type, int hd) {
  const int rb = kv_type == AXB_KV_F16 ? hd * 2 : (kv_type == AXB_KV_FP8 ? hd : hd / 2);
  const int cap = 32768 / rb;  // K and V stages together <= 64 KB
  return cap < kMaxChunk ? cap : kMaxChunk;
}

__host__ __device__ inline void decode_split(int active, int max_splits, int cap, int& nsplit, int& chunk) {
  int ns = (active + cap - 1) / cap;
  if (ns < max_splits) ns = max_splits;
  chunk = (active + ns - 1) / ns;
  chunk = (chunk + 15) / 16 * 16;
  if (chunk > cap) chunk = cap;
  ns = (active + chunk - 1) / chunk;
  nsplit = ns;
}

constexpr int kMaxSplits = 256;

template <int HD>
__global__ void __launch_bounds__(128) decode_attn_kernel(const axb_attn_desc d, int target_splits, int max_splits,
                                                          float* part_o, float* part_ml, int* counters, int* err,
                                                          const DecodeFuse f) {
  constexpr int DPL = HD / 32;  // dims per lane in PV
  constexpr int EPT = HD / 16;  // threads per token in the score pass (16 elements each)
  extern __shared__ __align__(128) char sm[];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int n_rep = d.n_head / d.n_kv_head;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int active = d.dev_params ? d.dev_params[2] : d.active_len;
  const int wpos = d.dev_params ? d.dev_params[1] : d.write_pos;
  const int cap = decode_chunk_cap(d.kv_type, HD);
  int nsplit, chunk;
  decode_split(active, target_splits, cap, nsplit, chunk);
  if (split >= nsplit) return;
  const int t0 = split * chunk, t1 = min(active, t0 + chunk), nt = t1 - t0;
  const int hq0 = kvh * n_rep;
  const int rb = kv_row_bytes(d.kv_type, HD);
  const int G = d.kv_group, ng = HD / G;
  const bool quant = d.kv_type != AXB_KV_F16;

  // shared memory: K rows, V rows, q, probabilities, scales, softmax stats
  char* kst = sm;                                   // [cap][rb]
  char* vst = kst + (size_t)cap * rb;               // [cap][rb]
  float* q_s = reinterpret_cast<float*>(vst + (size_t)cap * rb);  // [8][HD]
  float* p_s = q_s + kMaxRep * HD;                  // [8][cap]
  float* ks_s = p_s + kMaxRep * cap;                // [cap][ng]
  float* vs_s = ks_s + cap * 4;                     // [cap][ng]
  float* ml_s = vs_s + cap * 4;                     // m[8], l[8], scratch
  float* coef = ml_s + 4 * kMaxRep;                 // [8][kMaxSplits] combine weights
  uint64_t* bar = reinterpret_cast<uint64_t*>(coef + kMaxRep * kMaxSplits);
  float* o_red = reinterpret_cast<float*>(sm);      // [4][8][HD], reuses the K/V rows at the end

  const size_t head_base = ((size_t)b * d.n_kv_head + kvh) * d.max_seq;
  const uint8_t* kc = reinterpret_cast<const uint8_t*>(d.k_cache) + head_base * rb;
  const uint8_t* vc = reinterpret_cast<const uint8_t*>(d.v_cache) + head_base * rb;
  const __half* ksc = quant ? reinterpret_cast<const __half*>(d.k_scale) + head_base * ng : nullptr;
  const __half* vsc = quant ? reinterpret_cast<const __half*>(d.v_scale) + head_base * ng : nullptr;

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    fence_proxy_async();
    mbar_expect_tx(bar, 2u * nt * rb);
    bulk_g2s(kst, kc + (size_t)t0 * rb, nt * rb, bar);
    bulk_g2s(vst, vc + (size_t)t0 * rb, nt * rb, bar);
  }
  // scales of the chunk (plain loads; the new slot's is patched below)
  if (quant)
    for (int j = tid; j < nt * ng; j += 128) {
      ks_s[j] = __half2float(ksc[(size_t)t0 * ng + j]);
      vs_s[j] = __half2float(vsc[(size_t)t0 * ng + j]);
    }

  pdl_wait();  // q / the new K,V row come from the preceding GEMV

  // ---- q (rotated in fp32 when fused) and the new K/V row
  const int qkv_dim = (d.n_head + 2 * d.n_kv_head) * HD;
  float nkv[DPL];
  const bool covers_new = f.qkv != nullptr && wpos >= t0 && wpos < t1;
  if (f.qkv) {
    const __half* row = f.qkv + (size_t)b * qkv_dim;
    const int rp = d.dev_params ? d.dev_params[0] : 0;
    const float* fr = f.rope + (size_t)(rp % f.rope_len) * HD;
    for (int i = tid; i < n_rep * HD / 2; i += 128) {
      const int r = i / (HD / 2), pr = i % (HD / 2);
      const __half2 x2 = reinterpret_cast<const __half2*>(row + (hq0 + r) * HD)[pr];
      const float a0 = __low2float(x2), a1 = __high2float(x2);
      const float c = fr[2 * pr], sn = fr[2 * pr + 1];
      q_s[r * HD + 2 * pr] = __fsub_rn(__fmul_rn(a0, c), __fmul_rn(a1, sn));
      q_s[r * HD + 2 * pr + 1] = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(a1, c));
    }
    if (covers_new && wid < 2) {
      const __half* src = row + (size_t)(d.n_head + (wid == 0 ? 0 : d.n_kv_head) + kvh) * HD;
#pragma unroll
      for (int e = 0; e < DPL; ++e) nkv[e] = __half2float(src[lane * DPL + e]);
      if (wid == 0) {  // RoPE on K (transformer.py:1105-1127 rounding)
#pragma unroll
        for (int e = 0; e < DPL; e += 2) {
          const int pr = (lane * DPL + e) >> 1;
          const float c = fr[2 * pr], sn = fr[2 * pr + 1], a0 = nkv[e], a1 = nkv[e + 1];
          nkv[e] = __fsub_rn(__fmul_rn(a0, c), __fmul_rn(a1, sn));
          nkv[e + 1] = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(a1, c));
        }
      }
      // quantize (fp32 rule) and write the cache row + scale
      uint8_t* crow = const_cast<uint8_t*>((wid == 0 ? kc : vc) + (size_t)wpos * rb);
      __half* srow = quant ? const_cast<__half*>((wid == 0 ? ksc : vsc) + (size_t)wpos * ng) : nullptr;
      store_kv_row<DPL>(nkv, lane, d.kv_type, G, true, crow, srow);
    }
  } else {
    for (int i = tid; i < n_rep * HD; i += 128) {
      const int r = i / HD, e = i % HD;
      const size_t qi = ((size_t)b * d.n_head + hq0 + r) * HD + e;
      q_s[i] = d.q_is_fp32 ? reinterpret_cast<const float*>(d.q)[qi]
                           : __half2float(reinterpret_cast<const __half*>(d.q)[qi]);
    }
  }
  if (!mbar_wait(bar, 0, kAttnWaitLimit)) {
    if (tid == 0) atomicExch(err, AXB_ETIMEOUT);
    return;  // the only copy in flight is the one that timed out
  }
  if (covers_new && wid < 2) {
    // patch the staged copy (the prefetch read the slot before this step wrote it)
    uint8_t* rowp = reinterpret_cast<uint8_t*>(wid == 0 ? kst : vst) + (size_t)(wpos - t0) * rb;
    store_kv_row<DPL>(nkv, lane, d.kv_type, G, true, rowp, nullptr);
  }
  __syncthreads();  // global scale writes of the new slot are visible inside the CTA
  if (covers_new && quant && tid < 2 * ng) {
    const int which = tid / ng, gi = tid % ng;
    (which == 0 ? ks_s : vs_s)[(wpos - t0) * ng + gi] = __half2float((which == 0 ? ksc : vsc)[(size_t)wpos * ng + gi]);
  }
  __syncthreads();

  const float sm_scale = 1.0f / sqrtf((float)HD);
  // ---- scores for the whole chunk: EPT threads per token, 16 elements each
  for (int base = 0; base < nt; base += 128 / EPT) {
    const int tk = base + tid / EPT, ch = tid % EPT;
    float part[kMaxRep];
#pragma unroll
    for (int r = 0; r < kMaxRep; ++r) part[r] = 0.f;
    if (tk < nt) {
      float kv[16];
      kv_load16(reinterpret_cast<const uint8_t*>(kst) + (size_t)tk * rb, d.kv_type, ch * 16, kv);
      const float s = quant ? ks_s[tk * ng + (ch * 16) / G] : 1.f;
#pragma unroll
      for (int r = 0; r < kMaxRep; ++r) {
        if (r < n_rep) {
          float acc = 0.f;
#pragma unroll
          for (int e = 0; e < 16; ++e) acc = __fmaf_rn(q_s[r * HD + ch * 16 + e], kv[e], acc);
          part[r] = acc * s;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kMaxRep; ++r) {
      float v = part[r];
      for (int o = 1; o < EPT; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (ch == 0 && tk < nt && r < n_rep) p_s[r * cap + tk] = v * sm_scale;
    }
  }
  __syncthreads();
  // ---- softmax over the chunk: warp w handles heads w, w+4
  for (int r = wid; r < n_rep; r += 4) {
    float mx = -INFINITY;
    for (int tk = lane; tk < nt; tk += 32) mx = fmaxf(mx, p_s[r * cap + tk]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int tk = lane; tk < nt; tk += 32) {
      const float e = __expf(p_s[r * cap + tk] - mx);
      p_s[r * cap + tk] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    if (lane == 0) {
      ml_s[r] = mx;
      ml_s[kMaxRep + r] = sum;
    }
  }
  __syncthreads();
  // ---- PV: warp w takes tokens w, w+4, ...; lane covers DPL consecutive dims
  float acc[kMaxRep][DPL];
#pragma unroll
  for (int r = 0; r < kMaxRep; ++r)
#pragma unroll
    for (int e = 0; e < DPL; ++e) acc[r][e] = 0.f;
  for (int tk = wid; tk < nt; tk += 4) {
    const uint8_t* vrow = reinterpret_cast<const uint8_t*>(vst) + (size_t)tk * rb;
    float vv[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) vv[e] = kv_elem(vrow, d.kv_type, lane * DPL + e);
    const float s = quant ? vs_s[tk * ng + (lane * DPL) / G] : 1.f;
#pragma unroll
    for (int r = 0; r < kMaxRep; ++r) {
      if (r < n_rep) {
        const float pw = p_s[r * cap + tk] * s;
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[r][e] = __fmaf_rn(pw, vv[e], acc[r][e]);
      }
    }
  }
  __syncthreads();  // K/V rows are dead: o_red may reuse them
#pragma unroll
  for (int r = 0; r < kMaxRep; ++r)
    if (r < n_rep)
#pragma unroll
      for (int e = 0; e < DPL; ++e) o_red[(wid * kMaxRep + r) * HD + lane * DPL + e] = acc[r][e];
  __syncthreads();
  const size_t pidx = ((size_t)b * d.n_head + hq0);
  for (int i = tid; i < n_rep * HD; i += 128) {
    const int r = i / HD, e = i % HD;
    const float o = o_red[(0 * kMaxRep + r) * HD + e] + o_red[(1 * kMaxRep + r) * HD + e] +
                    o_red[(2 * kMaxRep + r) * HD + e] + o_red[(3 * kMaxRep + r) * HD + e];
    if (nsplit == 1)
      reinterpret_cast<__half*>(d.out)[(pidx + r) * HD + e] = __float2half_rn(__fdiv_rn(o, ml_s[kMaxRep + r]));
    else
      part_o[((pidx + r) * max_splits + split) * HD + e] = o;
  }
  if (nsplit == 1) return;
  if (tid < n_rep) {
    part_ml[((pidx + tid) * max_splits + split) * 2 + 0] = ml_s[tid];
    part_ml[((pidx + tid) * max_splits + split) * 2 + 1] = ml_s[kMaxRep + tid];
  }
  __threadfence();
  __syncthreads();
  __shared__ int last;
  if (tid == 0) last = (atomicAdd(counters + b * d.n_kv_head + kvh, 1) == nsplit - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  // ---- combine, split order fixed: per-head weights first (warp per head)
  for (int r = wid; r < n_rep; r += 4) {
    const size_t hb = (pidx + r) * max_splits;
    float M = -INFINITY;
    for (int sp = lane; sp < nsplit; sp += 32) M = fmaxf(M, __ldcg(part_ml + (hb + sp) * 2));
    M = warp_max(M);
    float L = 0.f;
    for (int sp = lane; sp < nsplit; sp += 32) {
      const float m = __ldcg(part_ml + (hb + sp) * 2), l = __ldcg(part_ml + (hb + sp) * 2 + 1);
      const float cwt = (m == -INFINITY) ? 0.f : __expf(m - M);
      coef[r * kMaxSplits + sp] = cwt;
      L += l * cwt;
    }
    L = warp_sum(L);
    if (lane == 0) ml_s[kMaxRep + r] = L;
  }
  __syncthreads();
  for (int i = tid; i < n_rep * HD; i += 128) {
    const int r = i / HD, e = i % HD;
    const size_t hb = (pidx + r) * max_splits;
    float O = 0.f;
    for (int sp0 = 0; sp0 < nsplit; sp0 += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = (sp0 + u < nsplit) ? __ldcg(part_o + (hb + sp0 + u) * HD + e) : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (sp0 + u < nsplit) O += v[u] * coef[r * kMaxSplits + sp0 + u];
    }
    reinterpret_cast<__half*>(d.out)[(pidx + r) * HD + e] = __float2half_rn(__fdiv_rn(O, ml_s[kMaxRep + r]));
  }
  if (tid == 0) counters[b * d.n_kv_head + kvh] = 0;
}

size_t decode_smem(int kv_type, int hd) {
  const int rb = kv_type == AXB_KV_F16 ? hd * 2 : (kv_type == AXB_KV_FP8 ? hd : hd / 2);
  const int cap = decode_chunk_cap(kv_type, hd);
  size_t rows = std::max((size_t)2 * cap * rb, (size_t)4 * kMaxRep * hd * 4);
  size_t rest = (size_t)(kMaxRep * hd + kMaxRep * cap + 8 * cap + 4 * kMaxRep + kMaxRep * kMaxSplits) * 4 + 16;
  return rows + rest;
}

// Tree / chunked-prefill attention on the tensor cores: T query tokens per
// sequence, each sees the prefix [0, prefix_len) and tree slot write_pos + j
// iff bit j of masks[t].  Query rows are (token, head) pairs of one KV head,
// token-major; a CTA of 4 warps takes 64 rows (16 per warp) against 64-key
// tiles, flash-attention style:
//  * K and V tiles are staged as exact fp16 codes (fp16 values, e4m3 codes, or
//    int4 codes (n ^ 8) - 8) with their per-(token, group) scales;
//  * S = q K^T with q as fp16 hi + lo (m16n8k16, fp32 accumulate), each K
//    scale group's partial sum multiplied by the token's scale;
//  * online softmax in registers (the C fragment of S is the A fragment of P);
//  * O += P V with the V scale folded into P (normalized by the tile's largest
//    scale of the group, so P' stays in [0, 1]) and P' as hi + lo.
// Split-K over the keys: with nsplit > 1, CTA (rows, split) covers keys
// [split * chunk, ...) and writes its unnormalized (O, m, l) to po / pml
// (tree_combine_kernel merges the splits in order); with nsplit == 1 it
// writes the output directly.
constexpr int kTreeRows = 64;  // query rows per CTA (4 warps x 16)
constexpr int kTreeKeys = 64;  // keys per tile

template <int HD>
struct TreeSmem {
  static constexpr int LD = HD + 8;  // fp16 row pitch: conflict-free ldmatrix / fragment loads
  static constexpr int kQ = 0;                                  // [hi, lo][64 rows][LD] fp16
  static constexpr int kK = kQ + 2 * kTreeRows * LD * 2;        // [64 keys][LD] fp16 codes
  static constexpr int kV = kK + kTreeKeys * LD * 2;            // [64 keys][LD]
  static constexpr int kKs = kV + kTreeKeys * LD * 2;           // [2 tiles][64 keys][8 groups] fp32 K scales
  static constexpr int kVs = kKs + 2 * kTreeKeys * 8 * 4;       // [2 tiles][64 keys][8 groups] fp32 V scales
  static constexpr int kVmax = kVs + 2 * kTreeKeys * 8 * 4;     // [8 groups] fp32
  static constexpr int kMask = kVmax + 8 * 4;                   // [64 rows] uint64
  static constexpr int kRaw = kMask + kTreeRows * 8;            // [2 tiles][K, V][64 keys][row bytes] cache codes
  // shared memory of a launch: the fixed part and the double-buffered raw codes
  static constexpr int bytes(int row_bytes) { return kRaw + 2 * 2 * kTreeKeys * row_bytes; }
};
// 16-byte asynchronous copy global -> shared; src_bytes 0 writes zeros
__device__ __forceinline__ void tree_cp16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void tree_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void tree_cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// fp32 pair -> fp16 (hi, lo) pairs with hi + lo = the value to about 22 bits
__device__ __forceinline__ void tree_split_h2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const float2 hf = __half22float2(h);
  hi = h2_as_u32(h);
  lo = h2_as_u32(__floats2half2_rn(x0 - hf.x, x1 - hf.y));
}
// 16 exact fp16 codes of a staged row piece: fp16 copy, e4m3 -> fp16, int4 (n ^ 8) - 8
__device__ __forceinline__ void tree_codes16(const uint8_t* src, int type, uint4 (&o)[2]) {
  if (type == AXB_KV_F16) {
    o[0] = reinterpret_cast<const uint4*>(src)[0];
    o[1] = reinterpret_cast<const uint4*>(src)[1];
  } else if (type == AXB_KV_FP8) {
    const uint4 a = *reinterpret_cast<const uint4*>(src);
    const uint16_t* u = reinterpret_cast<const uint16_t*>(&a);
    uint32_t* w = reinterpret_cast<uint32_t*>(o);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(u[i], __NV_E4M3);
      w[i] = (uint32_t)h.x | ((uint32_t)h.y << 16);
    }
  } else {
    const uint2 a = *reinterpret_cast<const uint2*>(src);
    const uint8_t* cb = reinterpret_cast<const uint8_t*>(&a);
    uint32_t* w = reinterpret_cast<uint32_t*>(o);
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // low nibble = element 2i, high = 2i + 1
      const uint32_t c = cb[i];
      const uint32_t t = (((c & 0xFu) | ((c & 0xF0u) << 12)) ^ 0x00080008u) | 0x64006400u;
      w[i] = h2_as_u32(__hsub2(u32_as_h2(t), __float2half2_rn(1032.f)));
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(128) tree_attn_kernel(axb_attn_desc d, int nsplit, int chunk, float* po, float* pml) {
  using SM = TreeSmem<HD>;
  constexpr int LD = SM::LD, KS = HD / 16, NBO = HD / 8;
  extern __shared__ __align__(16) char tsm[];
  __half* q_s = reinterpret_cast<__half*>(tsm + SM::kQ);
  __half* k_s = reinterpret_cast<__half*>(tsm + SM::kK);
  __half* v_s = reinterpret_cast<__half*>(tsm + SM::kV);
  float* ks_s = reinterpret_cast<float*>(tsm + SM::kKs);
  float* vs_s = reinterpret_cast<float*>(tsm + SM::kVs);
  float* vmax_s = reinterpret_cast<float*>(tsm + SM::kVmax);
  unsigned long long* mask_s = reinterpret_cast<unsigned long long*>(tsm + SM::kMask);
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int n_rep = d.n_head / d.n_kv_head;
  const int split = blockIdx.x % nsplit;
  const int r0 = (blockIdx.x / nsplit) * kTreeRows;  // first (token, head) row of the CTA
  const int R = min(kTreeRows, d.T * n_rep - r0);
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, c = lane & 3;
  const bool quant = d.kv_type != AXB_KV_F16;
  const int G = quant ? d.kv_group : HD, ng = HD / G;
  const float sm_scale = 1.0f / sqrtf((float)HD);
  pdl_wait();
  if (d.dev_params) {
    d.write_pos = d.dev_params[1];
    d.prefix_len = d.dev_params[3];
  }
  // ---- q rows as fp16 hi / lo (rows past R zero), masks
  for (int i = tid; i < kTreeRows * (HD / 2); i += 128) {
    const int r = i / (HD / 2), e = 2 * (i % (HD / 2));
    float x0 = 0.f, x1 = 0.f;
    if (r < R) {
      const int u = (r0 + r) / n_rep, hq = kvh * n_rep + (r0 + r) % n_rep;
      const size_t qi = (((size_t)b * d.T + u) * d.n_head + hq) * HD + e;
      if (d.q_is_fp32) {
        const float2 f = *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(d.q) + qi);
        x0 = f.x;
        x1 = f.y;
      } else {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(reinterpret_cast<const __half*>(d.q) + qi));
        x0 = f.x;
        x1 = f.y;
      }
    }
    uint32_t hi, lo;
    tree_split_h2(x0, x1, hi, lo);
    *reinterpret_cast<uint32_t*>(q_s + r * LD + e) = hi;
    *reinterpret_cast<uint32_t*>(q_s + (kTreeRows + r) * LD + e) = lo;
  }
  for (int r = tid; r < kTreeRows; r += 128) mask_s[r] = r < R ? d.masks[(r0 + r) / n_rep] : 0ull;

  const int rb = kv_row_bytes(d.kv_type, HD);
  const size_t head_base = ((size_t)b * d.n_kv_head + kvh) * d.max_seq;
  const uint8_t* kc = reinterpret_cast<const uint8_t*>(d.k_cache) + head_base * rb;
  const uint8_t* vc = reinterpret_cast<const uint8_t*>(d.v_cache) + head_base * rb;
  const __half* ksg = quant ? reinterpret_cast<const __half*>(d.k_scale) + head_base * ng : nullptr;
  const __half* vsg = quant ? reinterpret_cast<const __half*>(d.v_scale) + head_base * ng : nullptr;
  // code bytes of 16 elements, and pieces of 16 elements per row
  constexpr int PPR = HD / 16;
  const int piece_bytes = d.kv_type == AXB_KV_F16 ? 32 : (d.kv_type == AXB_KV_FP8 ? 16 : 8);

  // this thread's rows g and g + 8 of the warp's 16: online-softmax state
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  float oacc[NBO][4];
#pragma unroll
  for (int nb = 0; nb < NBO; ++nb)
#pragma unroll
    for (int q = 0; q < 4; ++q) oacc[nb][q] = 0.f;
  const uint32_t q_base = smem_u32(q_s), k_base = smem_u32(k_s), v_base = smem_u32(v_s);
  const int mrow = lane & 7, msel = lane >> 3;  // ldmatrix: this lane's row within matrix msel

  const int n_keys_all = d.prefix_len + d.T;
  const int k_begin = split * chunk, n_keys = min(n_keys_all, k_begin + chunk);
  // ---- K / V staging, double-buffered: the raw codes of the next tile are
  // copied (cp.async) and its scales loaded into registers while the current
  // tile is in the MMAs
  char* raw = tsm + SM::kRaw;
  const int p16 = rb / 16;  // 16-byte pieces per cached row
  auto slot_of = [&](int key) { return key < d.prefix_len ? key : (d.write_pos + key - d.prefix_len) % d.max_seq; };
  auto issue_tile = [&](int kt_i, int buf) {
    const int nk_i = min(kTreeKeys, n_keys - kt_i);
    char* rawb = raw + (size_t)buf * 2 * kTreeKeys * rb;
    for (int i = tid; i < 2 * kTreeKeys * p16; i += 128) {
      const int isv = i / (kTreeKeys * p16), j = (i / p16) % kTreeKeys, pc = i % p16;
      const uint8_t* src = isv ? vc : kc;
      uint32_t nb = 0;
      if (j < nk_i) {
        src += (size_t)slot_of(kt_i + j) * rb + pc * 16;
        nb = 16;
      }
      tree_cp16(rawb + ((size_t)(isv * kTreeKeys + j) * rb + pc * 16), src, nb);
    }
  };
  float sreg[8];  // this thread's scales of the next tile: element tid + 128 q, q < ng
  auto load_sc = [&](int kt_i) {
    const int nk_i = min(kTreeKeys, n_keys - kt_i);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (q < ng) {
        const int e = tid + 128 * q, isv = e / (kTreeKeys * ng), j = (e / ng) % kTreeKeys, gi = e % ng;
        sreg[q] = j < nk_i ? __half2float((isv ? vsg : ksg)[(size_t)slot_of(kt_i + j) * ng + gi]) : 0.f;
      }
  };
  auto store_sc = [&](int buf) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (q < ng) {
        const int e = tid + 128 * q, isv = e / (kTreeKeys * ng), j = (e / ng) % kTreeKeys, gi = e % ng;
        (isv ? vs_s : ks_s)[buf * kTreeKeys * 8 + j * 8 + gi] = sreg[q];
      }
  };
  if (k_begin < n_keys) {
    issue_tile(k_begin, 0);
    if (quant) {
      load_sc(k_begin);
      store_sc(0);
    }
  }
  tree_cp_commit();
  int it = 0;
  for (int kt = k_begin; kt < n_keys; kt += kTreeKeys, ++it) {
    const int nk = min(kTreeKeys, n_keys - kt), buf = it & 1;
    const bool has_next = kt + kTreeKeys < n_keys;
    __syncthreads();  // the previous tile's K / V, raw codes and scales are no longer read
    if (has_next) issue_tile(kt + kTreeKeys, buf ^ 1);
    tree_cp_commit();
    if (quant && has_next) load_sc(kt + kTreeKeys);
    tree_cp_wait<1>();  // this thread's copies of the current tile have landed
    __syncthreads();
    // ---- codes as fp16 (keys past nk are zeros)
    {
      const char* rawb = raw + (size_t)buf * 2 * kTreeKeys * rb;
      for (int i = tid; i < 2 * kTreeKeys * PPR; i += 128) {
        const int isv = i / (kTreeKeys * PPR), j = (i / PPR) % kTreeKeys, pc = i % PPR;
        uint4 o[2];
        tree_codes16(reinterpret_cast<const uint8_t*>(rawb) + (size_t)(isv * kTreeKeys + j) * rb + pc * piece_bytes,
                     d.kv_type, o);
        __half* dst = (isv ? v_s : k_s) + j * LD + 16 * pc;
        reinterpret_cast<uint4*>(dst)[0] = o[0];
        reinterpret_cast<uint4*>(dst)[1] = o[1];
      }
    }
    const float* ksb = ks_s + buf * kTreeKeys * 8;
    const float* vsb = vs_s + buf * kTreeKeys * 8;
    __syncthreads();
    if (quant && w == 0) {  // the tile's largest V scale per group
      for (int gi = 0; gi < ng; ++gi) {
        float mx = fmaxf(vsb[lane * 8 + gi], vsb[(lane + 32) * 8 + gi]);
        mx = warp_max(mx);
        if (lane == 0) vmax_s[gi] = mx > 0.f ? mx : 1.f;
      }
    }
    // ---- S = q K^T (16 rows x 64 keys per warp)
    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int q = 0; q < 4; ++q) s[nb][q] = 0.f;
    {
      float gacc[8][4];
#pragma unroll
      for (int nb = 0; nb < 8; ++nb)
#pragma unroll
        for (int q = 0; q < 4; ++q) gacc[nb][q] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t ahi[4], alo[4];
        {
          // A: m0 rows 0-7 / k 0-7, m1 rows 8-15 / k 0-7, m2 rows 0-7 / k 8-15, m3 rows 8-15 / k 8-15
          const int row = w * 16 + 8 * (msel & 1) + mrow, col = 16 * ks + 8 * (msel >> 1);
          ldsm_x4(ahi, q_base + (uint32_t)(row * LD + col) * 2);
          ldsm_x4(alo, q_base + (uint32_t)((kTreeRows + row) * LD + col) * 2);
        }
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          // B (K^T): m0 keys 0-7 / k 0-7, m1 keys 0-7 / k 8-15, m2 keys 8-15 / k 0-7, m3 keys 8-15 / k 8-15
          uint32_t kb[4];
          const int key = 16 * np + 8 * (msel >> 1) + mrow, col = 16 * ks + 8 * (msel & 1);
          ldsm_x4(kb, k_base + (uint32_t)(key * LD + col) * 2);
          mma_16816(gacc[2 * np], ahi, kb[0], kb[1], gacc[2 * np]);
          mma_16816(gacc[2 * np], alo, kb[0], kb[1], gacc[2 * np]);
          mma_16816(gacc[2 * np + 1], ahi, kb[2], kb[3], gacc[2 * np + 1]);
          mma_16816(gacc[2 * np + 1], alo, kb[2], kb[3], gacc[2 * np + 1]);
        }
        if ((16 * (ks + 1)) % G == 0) {  // a K scale group is complete: fold it in with each key's scale
          const int gi = (16 * ks) / G;
#pragma unroll
          for (int nb = 0; nb < 8; ++nb) {
            const int j0 = 8 * nb + 2 * c;
            const float s0 = quant ? ksb[j0 * 8 + gi] : 1.f, s1 = quant ? ksb[(j0 + 1) * 8 + gi] : 1.f;
            s[nb][0] = __fmaf_rn(gacc[nb][0], s0, s[nb][0]);
            s[nb][1] = __fmaf_rn(gacc[nb][1], s1, s[nb][1]);
            s[nb][2] = __fmaf_rn(gacc[nb][2], s0, s[nb][2]);
            s[nb][3] = __fmaf_rn(gacc[nb][3], s1, s[nb][3]);
#pragma unroll
            for (int q = 0; q < 4; ++q) gacc[nb][q] = 0.f;
          }
        }
      }
    }
    // ---- visibility, scale, online softmax (rows g: q 0/1, g + 8: q 2/3)
    const unsigned long long mk[2] = {mask_s[w * 16 + g], mask_s[w * 16 + g + 8]};
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = 8 * nb + 2 * c + (q & 1), key = kt + j;
        const int hr = q >> 1;
        const bool vis = j < nk && (key < d.prefix_len || ((mk[hr] >> (key - d.prefix_len)) & 1ull));
        s[nb][q] = vis ? s[nb][q] * sm_scale : -INFINITY;
        mx[hr] = fmaxf(mx[hr], s[nb][q]);
      }
    float alpha[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 1));
      mx[hr] = fmaxf(mx[hr], __shfl_xor_sync(0xffffffffu, mx[hr], 2));
      const float m_new = fmaxf(m_r[hr], mx[hr]);
      alpha[hr] = m_new == -INFINITY ? 1.f : (m_r[hr] == -INFINITY ? 0.f : __expf(m_r[hr] - m_new));
      m_r[hr] = m_new;
    }
    float lsum[2] = {0.f, 0.f};
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int hr = q >> 1;
        const float p = s[nb][q] == -INFINITY ? 0.f : __expf(s[nb][q] - m_r[hr]);
        s[nb][q] = p;
        lsum[hr] += p;
      }
    l_r[0] = l_r[0] * alpha[0] + lsum[0];
    l_r[1] = l_r[1] * alpha[1] + lsum[1];
    if (quant) __syncthreads();  // vmax_s
    // ---- O = alpha O + vmax (P' V), P' = p vscale / vmax, per V scale group
#pragma unroll
    for (int gi = 0; gi < HD / 16; ++gi) {  // at most ng groups; G >= 16
      if (gi >= ng) break;
      const float vm = quant ? vmax_s[gi] : 1.f, inv = 1.f / vm;
      const int nb0 = gi * (G / 8), nb1 = nb0 + G / 8;
      // rescale this group's accumulators into units of vm
#pragma unroll
      for (int nb = 0; nb < NBO; ++nb)
        if (nb >= nb0 && nb < nb1) {
          oacc[nb][0] *= alpha[0] * inv;
          oacc[nb][1] *= alpha[0] * inv;
          oacc[nb][2] *= alpha[1] * inv;
          oacc[nb][3] *= alpha[1] * inv;
        }
#pragma unroll
      for (int kq = 0; kq < 4; ++kq) {  // 16 keys per k-step
        float pv[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int j = 16 * kq + 8 * h + 2 * c + (q & 1);
            pv[h][q] = quant ? s[2 * kq + h][q] * (vsb[j * 8 + gi] * inv) : s[2 * kq + h][q];
          }
        uint32_t phi[4], plo[4];
        tree_split_h2(pv[0][0], pv[0][1], phi[0], plo[0]);  // row g, keys 2c, 2c + 1
        tree_split_h2(pv[0][2], pv[0][3], phi[1], plo[1]);  // row g + 8
        tree_split_h2(pv[1][0], pv[1][1], phi[2], plo[2]);  // row g, keys 8 + 2c
        tree_split_h2(pv[1][2], pv[1][3], phi[3], plo[3]);  // row g + 8, keys 8 + 2c
#pragma unroll
        for (int nb = 0; nb < NBO; nb += 2)
          if (nb >= nb0 && nb < nb1) {
            // V (transposed): m0 keys 0-7 / dims nb, m1 keys 8-15 / dims nb, m2 / m3 the same for dims nb + 1
            uint32_t vb[4];
            const int key = 16 * kq + 8 * (msel & 1) + mrow, col = 8 * (nb + (msel >> 1));
            ldsm_x4_t(vb, v_base + (uint32_t)(key * LD + col) * 2);
            mma_16816(oacc[nb], phi, vb[0], vb[1], oacc[nb]);
            mma_16816(oacc[nb], plo, vb[0], vb[1], oacc[nb]);
            mma_16816(oacc[nb + 1], phi, vb[2], vb[3], oacc[nb + 1]);
            mma_16816(oacc[nb + 1], plo, vb[2], vb[3], oacc[nb + 1]);
          }
      }
#pragma unroll
      for (int nb = 0; nb < NBO; ++nb)
        if (nb >= nb0 && nb < nb1)
#pragma unroll
          for (int q = 0; q < 4; ++q) oacc[nb][q] *= vm;
    }
    if (quant && has_next) store_sc(buf ^ 1);  // the next tile's scales (their loads have landed)
  }
  tree_cp_wait<0>();  // no copy may still be landing when the CTA exits
  // ---- row sums across the quad; outputs
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 1);
    l_r[hr] += __shfl_xor_sync(0xffffffffu, l_r[hr], 2);
  }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int r = w * 16 + g + 8 * hr;
    if (r >= R) continue;
    const int u = (r0 + r) / n_rep, hq = kvh * n_rep + (r0 + r) % n_rep;
    const size_t row = ((size_t)b * d.T + u) * d.n_head + hq;
    if (nsplit == 1) {
      __half* o = reinterpret_cast<__half*>(d.out) + row * HD;
      const float l = l_r[hr];
#pragma unroll
      for (int nb = 0; nb < NBO; ++nb)
        *reinterpret_cast<__half2*>(o + 8 * nb + 2 * c) =
            __floats2half2_rn(__fdiv_rn(oacc[nb][2 * hr], l), __fdiv_rn(oacc[nb][2 * hr + 1], l));
    } else {
      float* o = po + (row * nsplit + split) * HD;
#pragma unroll
      for (int nb = 0; nb < NBO; ++nb)
        *reinterpret_cast<float2*>(o + 8 * nb + 2 * c) = make_float2(oacc[nb][2 * hr], oacc[nb][2 * hr + 1]);
      if (c == 0) {
        pml[(row * nsplit + split) * 2 + 0] = m_r[hr];
        pml[(row * nsplit + split) * 2 + 1] = l_r[hr];
      }
    }
  }
}

// out[row] = sum_s w_s O_s / sum_s w_s l_s, w_s = exp(m_s - max m), in split order
__global__ void tree_combine_kernel(const float* __restrict__ po, const float* __restrict__ pml, int nsplit, int hd,
                                    __half* __restrict__ out) {
  const size_t row = blockIdx.x;
  const int e = threadIdx.x;
  float M = -INFINITY;
  for (int q = 0; q < nsplit; ++q) M = fmaxf(M, pml[(row * nsplit + q) * 2]);
  float L = 0.f, O = 0.f;
  for (int q = 0; q < nsplit; ++q) {
    const float m = pml[(row * nsplit + q) * 2], l = pml[(row * nsplit + q) * 2 + 1];
    const float w = m == -INFINITY ? 0.f : __expf(m - M);
    L += l * w;
    if (e < hd) O += po[(row * nsplit + q) * hd + e] * w;
  }
  if (e < hd) out[row * hd + e] = __float2half_rn(__fdiv_rn(O, L));
}

// ---------------------------------------------------------------- compaction
__global__ void compact_kv_kernel(uint8_t* cache, __half* scales, int max_batch, int n_kv_head, int max_seq,
                                  int row_bytes, int n_groups, int write_pos, const int32_t* acc, int n_acc,
                                  const int32_t* n_dev) {
  // blockIdx.x = ((layer*2 + kv)*max_batch + b)*Hkv + h
  extern __shared__ uint8_t stage[];
  if (n_dev) {  // count from the device-side tree walk; an identity path moves nothing
    n_acc = min(max(n_dev[0], 0), n_acc);
    bool same = true;
    for (int m = 0; m < n_acc; ++m) same &= acc[m] == m;
    if (same) return;
  }
  const size_t head = blockIdx.x;
  uint8_t* rows = cache + head * max_seq * (size_t)row_bytes;
  __half* srow = scales ? scales + head * max_seq * (size_t)n_groups : nullptr;
  __half* sstage = reinterpret_cast<__half*>(stage + (size_t)n_acc * row_bytes);
  for (int i = threadIdx.x; i < n_acc * row_bytes; i += blockDim.x) {
    int m = i / row_bytes, e = i % row_bytes;
    int src = (write_pos + acc[m]) % max_seq;
    stage[i] = rows[(size_t)src * row_bytes + e];
  }
  if (srow)
    for (int i = threadIdx.x; i < n_acc * n_groups; i += blockDim.x) {
      int m = i / n_groups, e = i % n_groups;
      sstage[i] = srow[(size_t)((write_pos + acc[m]) % max_seq) * n_groups + e];
    }
  __syncthreads();
  for (int i = threadIdx.x; i < n_acc * row_bytes; i += blockDim.x) {
    int m = i / row_bytes, e = i % row_bytes;
    rows[(size_t)((write_pos + m) % max_seq) * row_bytes + e] = stage[i];
  }
  if (srow)
    for (int i = threadIdx.x; i < n_acc * n_groups; i += blockDim.x) {
      int m = i / n_groups, e = i % n_groups;
      srow[(size_t)((write_pos + m) % max_seq) * n_groups + e] = sstage[i];
    }
}

// ---------------------------------------------------------------- host
static size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// CTAs of one (sequence, kv head) the split count aims for: ~2 CTAs per SM
int decode_max_splits(int B, int n_kv_head) {
  int ctas = B * n_kv_head;
  int want = (2 * num_sms() + ctas - 1) / ctas;
  return std::max(1, std::min(64, want));
}

// grid width (and partial-buffer stride) covering every active length <= max_seq
int decode_grid_splits(int target, int max_seq, int kv_type, int hd) {
  const int cap = decode_chunk_cap(kv_type, hd);
  return std::max(target, (max_seq + cap - 1) / cap);
}

// Workspace: [combine counters | kAttnCounters ints][m, l partials][O partials].
// The counters sit at a fixed offset for every (B, heads, splits), so one
// zeroed workspace serves any call; the combining CTA returns each to zero.
constexpr size_t kAttnCounters = 1 << 16;
constexpr size_t kAttnHead = 256;  // error word

// tree / chunked-prefill mode: splits of the key range and their partials
int tree_splits(int B, int T, int n_head, int n_kv_head, int n_keys) {
  const int n_rep = n_head / n_kv_head;
  const int base = ((T * n_rep + kTreeRows - 1) / kTreeRows) * n_kv_head * B;
  int S = (2 * num_sms() + base - 1) / base;  // about two CTAs per SM (registers)
  S = std::min(S, std::max(1, n_keys / (2 * kTreeKeys)));
  return std::max(1, std::min(S, 64));
}
// The partials follow the workspace's fixed header (error word and the decode
// path's arrival counters, which must stay zero); they may reuse the decode
// partial regions, which every decode launch rewrites before reading.
size_t tree_partials_offset() { return round_up(kAttnHead + kAttnCounters * 4, 256); }
size_t tree_workspace(int B, int T, int n_head, int head_dim, int nsplit) {
  if (nsplit <= 1) return 0;
  const size_t rows = (size_t)B * T * n_head;
  return tree_partials_offset() + round_up(rows * nsplit * head_dim * 4, 256) + round_up(rows * nsplit * 2 * 4, 256);
}

size_t attn_workspace(int B, int n_head, int head_dim, int max_splits) {
  size_t o = (size_t)B * n_head * max_splits * head_dim * 4;
  size_t ml = (size_t)B * n_head * max_splits * 2 * 4;
  return kAttnHead + kAttnCounters * 4 + round_up(ml, 256) + round_up(o, 256);
}

int rope_kv_write(const axb_kv_write_desc* d, cudaStream_t s, bool pdl) {
  AXB_CHECK_ARG(d && d->qkv && d->rope && d->q_out && d->k_cache && d->v_cache, "rope_kv_write: null pointer");
  AXB_CHECK_ARG(d->head_dim == 64 || d->head_dim == 128, "rope_kv_write: head_dim must be 64 or 128");
  AXB_CHECK_ARG(d->n_kv_head > 0 && d->n_head % d->n_kv_head == 0, "rope_kv_write: bad head counts");
  AXB_CHECK_ARG(d->kv_type == AXB_KV_F16 || (d->k_scale && d->v_scale), "rope_kv_write: quantized cache needs scales");
  AXB_CHECK_ARG(d->kv_type == AXB_KV_F16 || (d->kv_group >= 32 && d->head_dim % d->kv_group == 0 &&
                                              d->kv_group >= d->head_dim / 32),
                "rope_kv_write: kv_group must divide head_dim and be >= 32");
  AXB_CHECK_ARG(d->B >= 1 && d->B <= d->max_batch && d->T >= 1 && d->rope_len > 0, "rope_kv_write: bad B/T");
  long long items = (long long)d->B * d->T * (d->n_head + 2 * d->n_kv_head);
  int blocks = (int)((items + 3) / 4);
  cudaError_t e;
  if (d->head_dim == 128)
    e = launch_pdl(rope_kv_write_kernel<4>, dim3(blocks), dim3(128), 0, s, pdl, *d);
  else
    e = launch_pdl(rope_kv_write_kernel<2>, dim3(blocks), dim3(128), 0, s, pdl, *d);
  return cuda_status(e, "rope_kv_write launch");
}

int attention_fused(const axb_attn_desc* d, const DecodeFuse& f, cudaStream_t s);

// Raise the dynamic shared-memory limit of the decode kernels once per device
// (outside any stream capture).
int attn_prepare() {
  static DeviceOnce once;
  int dev = 0;
  cudaGetDevice(&dev);
  if (once.done(dev)) return AXB_OK;
  cudaError_t e = cudaFuncSetAttribute(decode_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tree_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             TreeSmem<128>::bytes(kv_row_bytes(AXB_KV_F16, 128)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tree_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             TreeSmem<64>::bytes(kv_row_bytes(AXB_KV_F16, 64)));
  if (e != cudaSuccess) return cuda_status(e, "attention attribute");
  once.set(dev);
  return AXB_OK;
}

int attention(const axb_attn_desc* d, cudaStream_t s) {
  DecodeFuse f = {};
  return attention_fused(d, f, s);
}

int attention_fused(const axb_attn_desc* d, const DecodeFuse& f, cudaStream_t s) {
  AXB_CHECK_ARG(d && d->q && d->k_cache && d->v_cache && d->out, "attention: null pointer");
  AXB_CHECK_ARG(d->head_dim == 64 || d->head_dim == 128, "attention: head_dim must be 64 or 128");
  AXB_CHECK_ARG(d->n_kv_head > 0 && d->n_head % d->n_kv_head == 0 && d->n_head / d->n_kv_head <= kMaxRep,
                "attention: n_head / n_kv_head must be an integer <= %d", kMaxRep);
  AXB_CHECK_ARG(d->kv_type == AXB_KV_F16 || (d->k_scale && d->v_scale && d->kv_group >= 32 &&
                                              d->head_dim % d->kv_group == 0),
                "attention: bad quantized-cache scales / group (kv_group must divide head_dim, >= 32)");
  if (d->masks == nullptr) {
    AXB_CHECK_ARG(d->active_len >= 1 && d->active_len <= d->max_seq, "attention: bad active_len %d", d->active_len);
    const int target = d->num_splits > 0 ? std::min(64, d->num_splits) : decode_max_splits(d->B, d->n_kv_head);
    const int ms = decode_grid_splits(target, d->max_seq, d->kv_type, d->head_dim);
    AXB_CHECK_ARG(ms <= kMaxSplits, "attention: max_seq %d needs %d splits (> %d)", d->max_seq, ms, kMaxSplits);
    AXB_CHECK_ARG(d->workspace && d->workspace_bytes >= attn_workspace(d->B, d->n_head, d->head_dim, ms),
                  "attention: workspace too small");
    AXB_CHECK_ARG((size_t)d->B * d->n_kv_head <= kAttnCounters, "attention: too many sequences x heads");
    char* ws = reinterpret_cast<char*>(d->workspace);
    int* err = reinterpret_cast<int*>(ws);
    int* cnt = reinterpret_cast<int*>(ws + kAttnHead);
    float* pml = reinterpret_cast<float*>(ws + kAttnHead + kAttnCounters * 4);
    size_t ml_b = round_up((size_t)d->B * d->n_head * ms * 2 * 4, 256);
    float* po = reinterpret_cast<float*>(ws + kAttnHead + kAttnCounters * 4 + ml_b);
    AXB_CHECK_ARG((reinterpret_cast<uintptr_t>(d->k_cache) & 15) == 0 && (reinterpret_cast<uintptr_t>(d->v_cache) & 15) == 0,
                  "attention: caches must be 16-byte aligned");
    dim3 grid(ms, d->n_kv_head, d->B);
    const size_t smem = decode_smem(d->kv_type, d->head_dim);
    if (int rc = attn_prepare()) return rc;
    cudaError_t e;
    if (d->head_dim == 128)
      e = launch_pdl(decode_attn_kernel<128>, grid, dim3(128), smem, s, d->pdl != 0, *d, target, ms, po, pml, cnt, err,
                     f);
    else
      e = launch_pdl(decode_attn_kernel<64>, grid, dim3(128), smem, s, d->pdl != 0, *d, target, ms, po, pml, cnt, err,
                     f);
    return cuda_status(e, "decode attention launch");
  }
  AXB_CHECK_ARG(d->T >= 1 && d->T <= 64, "attention: tree mode needs 1 <= T <= 64");
  AXB_CHECK_ARG(d->prefix_len >= 0 && d->prefix_len <= d->max_seq, "attention: bad prefix_len");
  AXB_CHECK_ARG(d->kv_type == AXB_KV_F16 || (d->kv_group >= 16 && d->head_dim % d->kv_group == 0),
                "attention: tree mode needs kv_group >= 16 dividing head_dim");
  AXB_CHECK_ARG((reinterpret_cast<uintptr_t>(d->k_cache) & 15) == 0 && (reinterpret_cast<uintptr_t>(d->v_cache) & 15) == 0,
                "attention: caches must be 16-byte aligned");
  if (int rc = attn_prepare()) return rc;
  const int n_rep = d->n_head / d->n_kv_head;
  // split the keys across CTAs when the workspace holds the partials; the
  // prefix length is read on the device, so the split plan uses its maximum
  int S = tree_splits(d->B, d->T, d->n_head, d->n_kv_head, d->max_seq);
  if (!d->workspace || d->workspace_bytes < tree_workspace(d->B, d->T, d->n_head, d->head_dim, S)) S = 1;
  const int chunk = S > 1 ? ((d->max_seq + S - 1) / S + kTreeKeys - 1) / kTreeKeys * kTreeKeys : 1 << 30;
  char* tws = reinterpret_cast<char*>(d->workspace) + tree_partials_offset();
  float* po = S > 1 ? reinterpret_cast<float*>(tws) : nullptr;
  const size_t rows = (size_t)d->B * d->T * d->n_head;
  float* pml = S > 1 ? reinterpret_cast<float*>(tws + round_up(rows * S * d->head_dim * 4, 256)) : nullptr;
  dim3 grid(((d->T * n_rep + kTreeRows - 1) / kTreeRows) * S, d->n_kv_head, d->B);
  cudaError_t e;
  if (d->head_dim == 128)
    e = launch_pdl(tree_attn_kernel<128>, grid, dim3(128),
                   (size_t)TreeSmem<128>::bytes(kv_row_bytes(d->kv_type, 128)), s, d->pdl != 0, *d, S, chunk, po, pml);
  else
    e = launch_pdl(tree_attn_kernel<64>, grid, dim3(128), (size_t)TreeSmem<64>::bytes(kv_row_bytes(d->kv_type, 64)),
                   s, d->pdl != 0, *d, S, chunk, po, pml);
  if (e != cudaSuccess) return cuda_status(e, "tree attention launch");
  if (S > 1) {
    tree_combine_kernel<<<(unsigned)rows, 128, 0, s>>>(po, pml, S, d->head_dim, reinterpret_cast<__half*>(d->out));
    return launch_status("tree combine");
  }
  return AXB_OK;
}

}  // namespace axb

using namespace axb;

extern "C" {

int axb_rope_kv_write(const axb_kv_write_desc* d, void* stream) { return rope_kv_write(d, (cudaStream_t)stream, false); }

int axb_kv_quantize(const void* x, int x_is_fp32, int rows, int hd, int kv_type, int G, void* q, uint16_t* sc,
                    void* stream) {
  AXB_CHECK_ARG(x && q && sc && rows >= 0, "kv_quantize: null pointer");
  AXB_CHECK_ARG(kv_type == AXB_KV_FP8 || kv_type == AXB_KV_INT4, "kv_quantize: kv_type must be FP8 or INT4");
  AXB_CHECK_ARG((hd == 64 || hd == 128) && G >= 32 && hd % G == 0, "kv_quantize: bad head_dim/group");
  if (rows == 0) return AXB_OK;
  int blocks = (rows + 3) / 4;
  if (hd == 128)
    kv_quantize_kernel<4><<<blocks, 128, 0, (cudaStream_t)stream>>>(x, x_is_fp32, rows, hd, kv_type, G, (uint8_t*)q,
                                                                    (__half*)sc);
  else
    kv_quantize_kernel<2><<<blocks, 128, 0, (cudaStream_t)stream>>>(x, x_is_fp32, rows, hd, kv_type, G, (uint8_t*)q,
                                                                    (__half*)sc);
  return launch_status("kv_quantize");
}

int axb_kv_dequantize(const void* q, const uint16_t* sc, int rows, int hd, int kv_type, int G, uint16_t* out,
                      void* stream) {
  AXB_CHECK_ARG(q && sc && out && rows >= 0 && hd > 0 && G > 0 && hd % G == 0, "kv_dequantize: bad args");
  AXB_CHECK_ARG(kv_type == AXB_KV_FP8 || kv_type == AXB_KV_INT4, "kv_dequantize: kv_type must be FP8 or INT4");
  long long n = (long long)rows * hd;
  if (n == 0) return AXB_OK;
  int blocks = (int)std::min<long long>((n + 255) / 256, 4096);
  kv_dequantize_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((const uint8_t*)q, (const __half*)sc, n, hd, kv_type,
                                                                 G, (__half*)out);
  return launch_status("kv_dequantize");
}

size_t axb_attn_workspace_bytes(int B, int n_head, int n_kv_head, int head_dim, int max_seq, int kv_type,
                                int num_splits) {
  const int target = num_splits > 0 ? std::min(64, num_splits) : decode_max_splits(B, n_kv_head);
  return attn_workspace(B, n_head, head_dim, decode_grid_splits(target, max_seq, kv_type, head_dim));
}

int axb_attention(const axb_attn_desc* d, void* stream) { return attention(d, (cudaStream_t)stream); }

int axb_compact_kv(void* cache, uint16_t* scales, int n_layer, int max_batch, int n_kv_head, int max_seq,
                   int row_bytes, int n_groups, int write_pos, const int32_t* accepted, int n_acc, void* stream) {
  AXB_CHECK_ARG(cache && accepted && n_acc >= 0 && n_acc <= 64 && row_bytes > 0, "compact_kv: bad args");
  if (n_acc == 0) return AXB_OK;
  size_t smem = (size_t)n_acc * row_bytes + (size_t)n_acc * n_groups * 2;
  int heads = n_layer * 2 * max_batch * n_kv_head;
  compact_kv_kernel<<<heads, 256, smem, (cudaStream_t)stream>>>((uint8_t*)cache, (__half*)scales, max_batch,
                                                                n_kv_head, max_seq, row_bytes, n_groups, write_pos,
                                                                accepted, n_acc, nullptr);
  return launch_status("compact_kv");
}

int axb_compact_kv_dev(void* cache, uint16_t* scales, int n_layer, int max_batch, int n_kv_head, int max_seq,
                       int row_bytes, int n_groups, int write_pos, const int32_t* accepted, const int32_t* n_acc_dev,
                       int max_acc, void* stream) {
  AXB_CHECK_ARG(cache && accepted && n_acc_dev && row_bytes > 0, "compact_kv_dev: null pointer");
  AXB_CHECK_ARG(max_acc >= 1 && max_acc <= 64 && max_acc <= max_seq, "compact_kv_dev: max_accepted must be 1..64");
  size_t smem = (size_t)max_acc * row_bytes + (size_t)max_acc * n_groups * 2;
  AXB_CHECK_ARG(smem <= 48 * 1024, "compact_kv_dev: %d rows of %d bytes exceed the staging", max_acc, row_bytes);
  int heads = n_layer * 2 * max_batch * n_kv_head;
  compact_kv_kernel<<<heads, 256, smem, (cudaStream_t)stream>>>((uint8_t*)cache, (__half*)scales, max_batch,
                                                                n_kv_head, max_seq, row_bytes, n_groups, write_pos,
                                                                accepted, max_acc, n_acc_dev);
  return launch_status("compact_kv_dev");
}

}  // extern "C"
