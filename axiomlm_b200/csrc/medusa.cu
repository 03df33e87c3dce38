// Medusa speculative decoding on the device: the greedy tree walk, the
// Medusa-head residual step, a per-row top-k and the next draft's token
// gather.  Together with the runner's tree step and the device-counted KV
// compaction these keep a whole speculative step on the GPU; the host reads
// back one small result block per step (how many tokens were accepted and
// which) instead of the full (T, V) logits.
//
// Reference behaviour followed:
//  * greedy walk: engine/medusa.py:312-330 (emit argmax at the current node,
//    descend to the first child, in child order, whose draft token equals it);
//  * Medusa head: models/medusa.py:44-53 and eval_medusa_heads,
//    models/transformer.py:414-445 (h' = x_norm + silu(fp16 W_res x_norm) in
//    fp32, logits = W_head fp16(h'));
//  * draft tokens: engine/medusa.py:231-246 and :290-298 (top-k per head,
//    node u takes rank topk_rank[u] of head head_idx[u]; node 0 is the last
//    emitted token).
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "axb_common.cuh"

namespace axb {

constexpr int kTopkThreads = 1024;
constexpr int kTopkWarps = kTopkThreads / 32;

// ---------------------------------------------------------------- tree walk
// One warp.  Node u (< 64) is held by lane u & 31 in slot u >> 5; children of
// a node are the nodes whose parent it is, in increasing index order (the
// order compile_medusa_tree appends them).  The first matching child is the
// lowest set bit of a ballot.
__global__ void tree_accept_kernel(int T, const int32_t* __restrict__ parent, const int32_t* __restrict__ verif,
                                   const int32_t* __restrict__ preds, int budget, int32_t* __restrict__ result) {
  const int lane = threadIdx.x;
  int par[2], tok[2];
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int u = lane + 32 * s;
    par[s] = u < T ? parent[u] : -2;
    tok[s] = u < T ? verif[u] : 0;
  }
  int32_t* acc = result + AXB_TREE_RESULT_HDR;
  int32_t* emitted = acc + AXB_TREE_MAX_NODES;
  int cur = 0, n = 1, ne = 0, last = 0;
  if (lane == 0) acc[0] = 0;
  // a path visits at most T nodes; the bound also ends the walk on a table
  // that is not a tree
  for (int it = 0; it < T && ne < budget; ++it) {
    const int p = preds[cur];
    if (lane == 0) emitted[ne] = p;
    ++ne;
    last = p;
    const unsigned b0 = __ballot_sync(0xffffffffu, par[0] == cur && tok[0] == p);
    const unsigned b1 = __ballot_sync(0xffffffffu, par[1] == cur && tok[1] == p);
    const int nxt = b0 ? __ffs(b0) - 1 : (b1 ? 31 + __ffs(b1) : -1);
    if (nxt < 0 || ne >= budget) break;
    cur = nxt;
    if (lane == 0) acc[n] = cur;
    ++n;
  }
  if (lane == 0) {
    result[0] = n;
    result[1] = cur;
    result[2] = ne;
    result[3] = last;
  }
}

// ------------------------------------------------------------- head inputs
// x32 = norm[leaf] (fp32), x16 = fp16(x32): the head GEMV input.
__global__ void medusa_leaf_kernel(const float* __restrict__ norm, int d, const int32_t* __restrict__ leaf_dev,
                                   int leaf, float* __restrict__ x32, __half* __restrict__ x16) {
  const int row = leaf_dev ? leaf_dev[0] : leaf;
  const float* src = norm + (size_t)row * d;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d; i += gridDim.x * blockDim.x) {
    const float v = src[i];
    x32[i] = v;
    x16[i] = __float2half_rn(v);
  }
}

// h16[k] = fp16(x32 + silu(r16[k])) for each of the K heads' residual outputs
__global__ void medusa_silu_add_kernel(int K, int d, const float* __restrict__ x32, const __half* __restrict__ r16,
                                       __half* __restrict__ h16) {
  const size_t n = (size_t)K * d;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float r = __half2float(r16[i]);
    h16[i] = __float2half_rn(__fadd_rn(x32[i % d], silu_f(r)));
  }
}

// ------------------------------------------------------------------- top-k
// fp16 bits -> an unsigned key with the same order as the values
__device__ __forceinline__ uint32_t h_key(uint16_t b) { return (b & 0x8000u) ? (0xFFFFu ^ b) : (b | 0x8000u); }

// Block-wide exclusive scan of one count per thread (thread order), with the
// block total.  Uses red[kTopkWarps + 1].
__device__ __forceinline__ int block_excl_scan(int v, int* red, int* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) red[w] = inc;
  __syncthreads();
  if (w == 0) {
    int x = lane < kTopkWarps ? red[lane] : 0, xi = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, xi, o);
      if (lane >= o) xi += t;
    }
    if (lane < kTopkWarps) red[lane] = xi - x;
    if (lane == 31) red[kTopkWarps] = xi;
  }
  __syncthreads();
  const int r = red[w] + inc - v;
  *total = red[kTopkWarps];
  __syncthreads();
  return r;
}

// Each thread owns 8 consecutive elements of each 8*1024-element tile, so
// thread order is index order within a tile.
template <typename F>
__device__ __forceinline__ void for_tile8(const __half* row, int n, int base, bool vec, F&& f) {
  const int i0 = base + 8 * threadIdx.x;
  uint16_t v[8];
  if (vec && i0 + 8 <= n) {
    const uint4 q = *reinterpret_cast<const uint4*>(row + i0);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = (uint16_t)(w[j] & 0xFFFFu);
      v[2 * j + 1] = (uint16_t)(w[j] >> 16);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = i0 + j < n ? __half_as_ushort(row[i0 + j]) : 0;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) f(i0 + j, i0 + j < n, h_key(v[j]));
}

constexpr int kTopkCand = 2048;  // candidate capacity of the fast path

// Top-k (k <= AXB_TOPK_MAX) of each row by value, ties to the lower index.
// One CTA per row.  Fast path: the k-th largest of the threads' own maxima
// bounds the row's k-th largest from below, so one more pass collecting the
// keys at or above it (few, for logits) and a bitonic sort of those give the
// answer.  When more than kTopkCand keys tie at the bound (flat rows), the
// exact path runs instead: the k-th largest key by a two-pass 8-bit radix
// select, then an ordered pass collects the larger keys and the
// lowest-indexed ties, and one warp sorts the k survivors.
__global__ void __launch_bounds__(kTopkThreads) topk_rows_kernel(const __half* __restrict__ x, int n, int ld, int k,
                                                                 int32_t* __restrict__ out_idx) {
  __shared__ unsigned long long cand[kTopkCand];  // (key << 32) | ~index: larger is better
  __shared__ uint32_t tmax_s[kTopkThreads];
  __shared__ int hist[256];
  __shared__ int red[kTopkWarps + 1];
  __shared__ uint32_t s_sel[2];
  __shared__ int s_cnt;
  __shared__ uint32_t c_key[AXB_TOPK_MAX];
  __shared__ int c_idx[AXB_TOPK_MAX];
  const __half* row = x + (size_t)blockIdx.x * ld;
  const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  const int tile = 8 * kTopkThreads;
  const int tid = threadIdx.x;

  // ---- fast path: per-thread maxima, their k-th largest as the bound
  uint32_t tmax = 0;
  for (int base = 0; base < n; base += tile)
    for_tile8(row, n, base, vec, [&](int, bool ok, uint32_t key) {
      if (ok) tmax = max(tmax, key);
    });
  tmax_s[tid] = tmax;
  if (tid == 0) s_cnt = 0;
  __syncthreads();
  // bitonic sort of the maxima, descending: the k-th is the bound (k distinct
  // elements are >= it)
  for (int size = 2; size <= kTopkThreads; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (tid < kTopkThreads / 2) {
        const int lo = 2 * tid - (tid & (stride - 1)), hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint32_t a = tmax_s[lo], b = tmax_s[hi];
        if ((a < b) == desc) {
          tmax_s[lo] = b;
          tmax_s[hi] = a;
        }
      }
      __syncthreads();
    }
  const uint32_t bound = tmax_s[k - 1];
  for (int base = 0; base < n; base += tile)
    for_tile8(row, n, base, vec, [&](int i, bool ok, uint32_t key) {
      if (ok && key >= bound) {
        const int slot = atomicAdd(&s_cnt, 1);
        if (slot < kTopkCand) cand[slot] = ((unsigned long long)key << 32) | (0xFFFFFFFFu - (uint32_t)i);
      }
    });
  __syncthreads();
  const int nc = s_cnt;
  if (nc <= kTopkCand) {
    int P = 64;
    while (P < nc) P <<= 1;
    for (int i = nc + tid; i < P; i += blockDim.x) cand[i] = 0ull;
    __syncthreads();
    // bitonic sort, descending
    for (int size = 2; size <= P; size <<= 1)
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < P / 2; i += blockDim.x) {
          const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
          const bool desc = (lo & size) == 0;
          const unsigned long long a = cand[lo], b = cand[hi];
          if ((a < b) == desc) {
            cand[lo] = b;
            cand[hi] = a;
          }
        }
        __syncthreads();
      }
    for (int j = tid; j < k; j += blockDim.x)
      out_idx[(size_t)blockIdx.x * k + j] = (int32_t)(0xFFFFFFFFu - (uint32_t)(cand[j] & 0xFFFFFFFFull));
    return;
  }

  // ---- exact path for flat rows
  uint32_t prefix = 0;  // selected high byte, then the whole key
  int want = k;         // rank still to find inside the selected bucket
  for (int pass = 0; pass < 2; ++pass) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int base = 0; base < n; base += tile)
      for_tile8(row, n, base, vec, [&](int, bool ok, uint32_t key) {
        // lanes with the same bin add once (logits crowd into few bins)
        const uint32_t bin = !ok ? 0xFFFFu : pass == 0 ? key >> 8 : (key >> 8) == prefix ? (key & 0xFFu) : 0xFFFFu;
        const unsigned m = __match_any_sync(0xffffffffu, bin);
        if (bin != 0xFFFFu && (tid & 31) == __ffs(m) - 1) atomicAdd(&hist[bin], __popc(m));
      });
    __syncthreads();
    if (tid == 0) {
      int above = 0, b = 255;
      for (; b > 0; --b) {
        if (above + hist[b] >= want) break;
        above += hist[b];
      }
      s_sel[0] = (uint32_t)b;
      s_sel[1] = (uint32_t)(want - above);
    }
    __syncthreads();
    prefix = pass == 0 ? s_sel[0] : (prefix << 8) | s_sel[0];
    want = (int)s_sel[1];
    __syncthreads();
  }
  const uint32_t thr = prefix;  // the k-th largest key; `want` ties of it are taken
  if (tid == 0) s_cnt = 0;
  __syncthreads();
  const int n_gt = k - want;
  int ties_before = 0;
  for (int base = 0; base < n; base += tile) {
    int mine = 0;
    for_tile8(row, n, base, vec, [&](int i, bool ok, uint32_t key) {
      if (!ok) return;
      if (key > thr) {
        const int s = atomicAdd(&s_cnt, 1);
        if (s < AXB_TOPK_MAX) {
          c_key[s] = key;
          c_idx[s] = i;
        }
      }
      mine += key == thr;
    });
    int total;
    int r = ties_before + block_excl_scan(mine, red, &total);
    if (mine && r < want)
      for_tile8(row, n, base, vec, [&](int i, bool ok, uint32_t key) {
        if (ok && key == thr && r < want) {
          c_key[n_gt + r] = key;
          c_idx[n_gt + r] = i;
          ++r;
        }
      });
    ties_before += total;
  }
  __syncthreads();
  // rank sort of the k survivors: (key desc, index asc)
  if (tid < 32)
    for (int a = tid; a < k; a += 32) {
      const uint32_t ka = c_key[a];
      const int ia = c_idx[a];
      int pos = 0;
      for (int b = 0; b < k; ++b) {
        const uint32_t kb = c_key[b];
        pos += kb > ka || (kb == ka && c_idx[b] < ia);
      }
      out_idx[(size_t)blockIdx.x * k + pos] = ia;
    }
}

// tokens[0] = root token; tokens[u] = topk[head_idx[u]][rank[u]]
__global__ void draft_tokens_kernel(int T, const int32_t* __restrict__ head_idx, const int32_t* __restrict__ rank,
                                    const int32_t* __restrict__ topk, int kmax, const int32_t* __restrict__ root,
                                    int32_t* __restrict__ tokens) {
  for (int u = threadIdx.x; u < T; u += blockDim.x)
    tokens[u] = u == 0 ? root[0] : topk[(size_t)head_idx[u] * kmax + rank[u]];
}

}  // namespace axb

using namespace axb;

extern "C" {

int axb_tree_accept(int T, const int32_t* parent, const int32_t* verif, const int32_t* preds, int budget,
                    int32_t* result, void* stream) {
  AXB_CHECK_ARG(parent && verif && preds && result, "tree_accept: null pointer");
  AXB_CHECK_ARG(T >= 1 && T <= AXB_TREE_MAX_NODES, "tree_accept: T must be 1..%d", AXB_TREE_MAX_NODES);
  AXB_CHECK_ARG(budget >= 1, "tree_accept: budget must be >= 1");
  tree_accept_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(T, parent, verif, preds, budget, result);
  return launch_status("tree_accept");
}

int axb_medusa_leaf(const float* norm, int d, const int32_t* leaf_dev, int leaf, float* x32, uint16_t* x16,
                    void* stream) {
  AXB_CHECK_ARG(norm && x32 && x16 && d > 0 && (leaf_dev || leaf >= 0), "medusa_leaf: bad args");
  medusa_leaf_kernel<<<(d + 255) / 256, 256, 0, (cudaStream_t)stream>>>(norm, d, leaf_dev, leaf, x32, (__half*)x16);
  return launch_status("medusa_leaf");
}

int axb_medusa_silu_add(int K, int d, const float* x32, const uint16_t* r16, uint16_t* h16, void* stream) {
  AXB_CHECK_ARG(x32 && r16 && h16 && K > 0 && d > 0, "medusa_silu_add: bad args");
  const size_t n = (size_t)K * d;
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 4 * (size_t)num_sms());
  medusa_silu_add_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(K, d, x32, (const __half*)r16, (__half*)h16);
  return launch_status("medusa_silu_add");
}

int axb_topk_rows(const uint16_t* x, int rows, int n, int ld, int k, int32_t* out_idx, void* stream) {
  AXB_CHECK_ARG(x && out_idx && rows >= 0 && n > 0 && ld >= n, "topk_rows: bad args");
  AXB_CHECK_ARG(k >= 1 && k <= AXB_TOPK_MAX && k <= n, "topk_rows: k must be 1..min(n, %d)", AXB_TOPK_MAX);
  if (rows == 0) return AXB_OK;
  topk_rows_kernel<<<rows, kTopkThreads, 0, (cudaStream_t)stream>>>((const __half*)x, n, ld, k, out_idx);
  return launch_status("topk_rows");
}

int axb_draft_tokens(int T, const int32_t* head_idx, const int32_t* rank, const int32_t* topk, int kmax,
                     const int32_t* root, int32_t* tokens, void* stream) {
  AXB_CHECK_ARG(head_idx && rank && topk && root && tokens && kmax >= 1, "draft_tokens: null pointer");
  AXB_CHECK_ARG(T >= 1 && T <= AXB_TREE_MAX_NODES, "draft_tokens: T must be 1..%d", AXB_TREE_MAX_NODES);
  draft_tokens_kernel<<<1, 64, 0, (cudaStream_t)stream>>>(T, head_idx, rank, topk, kmax, root, tokens);
  return launch_status("draft_tokens");
}

}  // extern "C"
