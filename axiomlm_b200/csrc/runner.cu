// Whole-model quantized decode runner: one CUDA graph per (batch, tokens, mode).
//
// Replaces MPSQuantizedDecodeRunner / QuantizedDecodeGraphState
// (axiomlm/kernels/mps_kernels.mm:2982-3737: step 3195, verify_tree_step 3265,
// verify_step 3359, get_last_norm 3732), which encodes every layer into one
// Metal command buffer per step.  Here the per-step kernel sequence
//   embed -> L x [qkv GEMV(+RMSNorm) -> RoPE+KV write -> attention ->
//   o GEMV(+residual) -> gate_up GEMV(+RMSNorm, SwiGLU) -> down GEMV(+residual)]
//   -> lm_head GEMV(+final RMSNorm) -> argmax
// is captured once into a CUDA graph (kernels chained with programmatic
// dependent launch) and replayed; per-step positions live in a device buffer
// written by one tiny kernel before each replay.
#include <cstdlib>
#include <map>
#include <tuple>
#include <vector>

#include "step.cuh"
#include "tp.cuh"

namespace axb {

int qgemm(const axb_qgemm_desc* d, cudaStream_t stream);
int qgemm_prepare();
bool qgemm_can_fuse_norm(int M, int K);
size_t qgemm_workspace(int N, int M);
int rope_kv_write(const axb_kv_write_desc* d, cudaStream_t s, bool pdl);
int attention(const axb_attn_desc* d, cudaStream_t s);
struct DecodeFuse {
  const __half* qkv;
  const float* rope;
  int rope_len;
};
int attention_fused(const axb_attn_desc* d, const DecodeFuse& f, cudaStream_t s);
int attn_prepare();
int q8_gemv(const __half* x, int ldx, int M, int K, const uint32_t* w, const __half2* sb, int N, __half* y, int ldy,
            cudaStream_t st, const __half* bias = nullptr);
size_t attn_workspace(int B, int n_head, int head_dim, int max_splits);
int tree_splits(int B, int T, int n_head, int n_kv_head, int n_keys);
size_t tree_workspace(int B, int T, int n_head, int head_dim, int nsplit);
int decode_max_splits(int B, int n_kv_head);
int decode_grid_splits(int target, int max_seq, int kv_type, int hd);
int rmsnorm(const __half* x, const float* w, int M, int K, float eps, __half* out, cudaStream_t s);

// many-token projections on the tcgen05 tensor cores (qgemm_tc.cu); their
// residual / SwiGLU epilogues, with the GEMV's rounding points
__global__ void residual_add_kernel(__half* __restrict__ x, const __half* __restrict__ y, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    x[i] = __float2half_rn(__fadd_rn(__half2float(x[i]), __half2float(y[i])));
}
// gate / up rows interleaved by 8 (tile = 8 gate + 8 up rows): sw[m][j] = swiglu_h(g, u)
__global__ void swiglu_packed_kernel(const __half* __restrict__ gu, int ld, int F, int rows, __half* __restrict__ sw) {
  const size_t total = (size_t)rows * F;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / F), j = (int)(i % F);
    const int p = (j >> 3) * 16 + (j & 7);
    const float g = __half2float(gu[(size_t)m * ld + p]), u = __half2float(gu[(size_t)m * ld + p + 8]);
    sw[(size_t)m * F + j] = swiglu_h(g, u);
  }
}
// gate rows first, then up rows (the reference's gate_up = cat(w_gate, w_up),
// transformer.py:959-964, as Q8 projections keep it): sw[m][j] = swiglu_h(g, u)
__global__ void swiglu_split_kernel(const __half* __restrict__ gu, int ld, int F, int rows, __half* __restrict__ sw) {
  const size_t total = (size_t)rows * F;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / F), j = (int)(i % F);
    const float g = __half2float(gu[(size_t)m * ld + j]), u = __half2float(gu[(size_t)m * ld + F + j]);
    sw[(size_t)m * F + j] = swiglu_h(g, u);
  }
}
int argmax(const __half* x, int rows, int n, int ld, int32_t* out, cudaStream_t s);

struct StepParams {
  int32_t p[4];  // rope_pos, write_pos, active_len, prefix_len
  int32_t T;
  uint64_t masks[64];
  int32_t depths[64];
};

__global__ void set_params_kernel(StepParams sp, int32_t* params, uint64_t* masks, int32_t* depths) {
  int t = threadIdx.x;
  if (t < 4) params[t] = sp.p[t];
  if (t < sp.T) {
    masks[t] = sp.masks[t];
    depths[t] = sp.depths[t];
  }
}

// dequant_q8_rows (quant.py:132-163) for the step's tokens; grid (rows, K/256):
// each thread produces 4 consecutive dims from one 32-bit word.
__global__ void embed_q8_kernel(const uint32_t* __restrict__ w, const __half* __restrict__ sb,
                                const int32_t* __restrict__ tok, int K, int V, __half* __restrict__ out,
                                int* __restrict__ err) {
  pdl_wait();
  const int i = blockIdx.x;
  const int r = tok[i];
  const int k = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
  if (k >= K) return;
  __half* o = out + (size_t)i * K + k;
  if (r < 0 || r >= V) {  // out-of-vocabulary id: zero row, flag the error
    o[0] = o[1] = o[2] = o[3] = __float2half_rn(0.f);
    if (k == 0) atomicExch(err, AXB_EINVAL);
    return;
  }
  const uint32_t word = w[(size_t)r * (K / 4) + k / 4];
  const __half2 p = reinterpret_cast<const __half2*>(sb)[(size_t)r * (K / 64) + k / 64];
  const float s = __low2float(p), bi = __high2float(p);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    o[j] = __float2half_rn(__fadd_rn(__fmul_rn((float)((word >> (8 * j)) & 0xFF), s), bi));
}

// Greedy argmax over the vocabulary (torch.argmax: first index of the max),
// split over many CTAs; the last CTA of a row combines the partials in order.
__global__ void argmax_part_kernel(const __half* __restrict__ x, int n, int ld, int chunk, float* __restrict__ pv,
                                   int* __restrict__ pi, int* __restrict__ cnt, int32_t* __restrict__ out) {
  pdl_wait();
  const int part = blockIdx.x, row = blockIdx.y, nparts = gridDim.x;
  const __half* xr = x + (size_t)row * ld;
  const int k0 = part * chunk, k1 = min(n, k0 + chunk);
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int k = k0 + threadIdx.x * 8; k < k1; k += blockDim.x * 8) {
    if (k + 8 <= k1 && ((((uintptr_t)(xr + k)) & 15) == 0)) {
      uint4 v = *reinterpret_cast<const uint4*>(xr + k);
      const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float f = __half2float(h[j]);
        if (f > best) {
          best = f;
          bi = k + j;
        }
      }
    } else {
      for (int j = k; j < min(k + 8, k1); ++j) {
        float f = __half2float(xr[j]);
        if (f > best) {
          best = f;
          bi = j;
        }
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ int last;
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
    pv[row * nparts + part] = best;
    pi[row * nparts + part] = bi;
    __threadfence();
    last = atomicAdd(cnt + row, 1) == nparts - 1;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  float b = -INFINITY;
  int id = 0x7fffffff;
  for (int p = 0; p < nparts; ++p) {  // parts in index order: strict > keeps the lowest index
    float v = __ldcg(pv + row * nparts + p);
    int ii = __ldcg(pi + row * nparts + p);
    if (v > b || (v == b && ii < id)) {
      b = v;
      id = ii;
    }
  }
  out[row] = id == 0x7fffffff ? 0 : id;
  cnt[row] = 0;
}

// final-norm hidden state in fp32 (the reference's x_norm / get_last_norm)
template <typename OutT>
__global__ void rmsnorm_kernel(const __half* __restrict__ x, const float* __restrict__ w, int K, float eps,
                               OutT* __restrict__ out) {
  pdl_wait();
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
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = __fmul_rn(__fmul_rn(__half2float(xr[k]), rms), w[k]);
    if constexpr (sizeof(OutT) == 2) out[(size_t)row * K + k] = __float2half_rn(v);
    else out[(size_t)row * K + k] = v;
  }
}

static size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// 2-bit projections (q2t; axb_lbgemv)
static bool is_q2t(int f) {
  return f == AXB_W_TERNARY_G64 || f == AXB_W_TERNARY_PT || f == AXB_W_Q2_G64 || f == AXB_W_Q2K_SB256;
}
// formats served by their own GEMV followed by separate residual-add / SwiGLU
// passes, with gate_up in the reference's row order, cat(w_gate, w_up)
static bool ext_fmt(int f) { return f == AXB_W_Q8_G64 || is_q2t(f); }
constexpr int kLbMaxM = 8;  // rows per axb_lbgemv launch

constexpr int kArgmaxParts = 256;
constexpr int kTcMinRows = 16;  // tree / prefill steps above this many rows use the tcgen05 GEMM

struct Layout {
  size_t tokens, params, masks, depths, x, h, qkv, q, attn, sw, logits, amax, xnorm, gemm_ws, attn_ws, total;
  size_t lb_ws, lb_ws_bytes;  // 2-bit GEMV workspace
  size_t am_v, am_i, am_cnt;
  size_t tp_part, tp_keys;  // tensor parallel: row-parallel partial sums (fp32), argmax keys
  size_t gu_tmp, tc_ws, tc_ws_bytes;  // tensor-core projections for many-token steps
  size_t gemm_ws_bytes, attn_ws_bytes;
  // persistent step kernel (decode, B <= 8)
  size_t st_layers, st_part, st_po, st_pml, st_acnt, st_keys, st_exit, st_trace, st_hdump, st_maps;
  size_t st_h, st_qkv, st_attn, st_sw;  // the step kernel's flagged activations: one 8-byte word per 2 halves
  size_t st_trace_bytes, st_hdump_bytes;
};

static Layout make_layout(const axb_model_cfg& c) {
  Layout L = {};
  const size_t rows = (size_t)c.max_batch * c.max_tokens;
  const size_t qkv_dim = (size_t)(c.n_head + 2 * c.n_kv_head) * c.head_dim;
  const size_t qd = (size_t)c.n_head * c.head_dim;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += align256(bytes);
    return o;
  };
  L.tokens = take(rows * 4);
  L.params = take(32);  // [rope_pos, write_pos, active_len, prefix_len, error]
  L.masks = take(64 * 8);
  L.depths = take(64 * 4);
  L.x = take(rows * c.d_model * 2);
  L.h = take(rows * c.d_model * 2);
  L.qkv = take(rows * qkv_dim * 2);
  L.q = take(rows * qd * 4);
  L.attn = take(rows * qd * 2);
  L.sw = take(rows * (size_t)c.ffn * 2);
  L.logits = take(rows * (size_t)c.vocab * 2);
  L.amax = take(rows * 4);
  L.xnorm = take(rows * (size_t)c.d_model * 4);
  L.am_v = take(rows * kArgmaxParts * 4);
  L.am_i = take(rows * kArgmaxParts * 4);
  L.am_cnt = take(rows * 4);
  L.tp_part = take(c.tp_world > 1 ? rows * c.d_model * 4 : 0);
  // tensor-core path (rows > 16): gate_up output in packed order, tcgen05 workspace
  const bool tc = rows > kTcMinRows && c.tp_world <= 1;
  // (Q8 / 2-bit gate_up projections also leave their product there before the SwiGLU pass)
  L.gu_tmp = take(tc || ext_fmt(c.wfmt) ? rows * 2 * (size_t)c.ffn * 2 : 0);
  {
    const int dn = c.dn_fmt ? c.dn_fmt : c.wfmt;
    const int qd_ = c.n_head * c.head_dim;
    const int FNK[5][3] = {{c.wfmt, (int)qkv_dim, c.d_model}, {c.wfmt, c.d_model, qd_}, {c.wfmt, 2 * c.ffn, c.d_model},
                           {dn, c.d_model, c.ffn}, {c.lm_fmt, c.vocab, c.d_model}};
    size_t lb = 0;
    for (auto& f : FNK)
      if (is_q2t(f[0])) lb = std::max(lb, axb_lbgemv_workspace_bytes(f[0], f[1], f[2], kLbMaxM));
    L.lb_ws_bytes = lb;
    L.lb_ws = take(lb);
  }
  size_t tcw = 0;
  if (tc) {
    const int qd_ = c.n_head * c.head_dim;
    const int NK[5][2] = {{(int)qkv_dim, c.d_model}, {c.d_model, qd_}, {2 * c.ffn, c.d_model}, {c.d_model, c.ffn},
                          {c.vocab, c.d_model}};
    for (auto& nk : NK) tcw = std::max(tcw, axb_qgemm_tc_workspace_bytes(nk[0], nk[1], 64));
  }
  L.tc_ws_bytes = tcw;
  L.tc_ws = take(tcw);
  L.tp_keys = take(c.tp_world > 1 ? rows * 8 : 0);
  int m = (int)std::min<size_t>(rows, 64);
  size_t g = 0;
  for (int n : {(int)qkv_dim, c.d_model, 2 * c.ffn, c.vocab}) g = std::max(g, qgemm_workspace(n, m));
  L.gemm_ws_bytes = g;
  L.gemm_ws = take(g);
  size_t a = 0;
  for (int b = 1; b <= c.max_batch; ++b)
    a = std::max(a, attn_workspace(b, c.n_head, c.head_dim,
                                   decode_grid_splits(decode_max_splits(b, c.n_kv_head), c.max_seq, c.kv_type,
                                                      c.head_dim)));
  // tree / prefill steps split their keys across CTAs: room for the partials
  if (c.max_tokens > 1)
    for (int b = 1; b <= c.max_batch; ++b)
      for (int t = 1; t <= c.max_tokens; ++t)
        a = std::max(a, tree_workspace(b, t, c.n_head, c.head_dim,
                                       tree_splits(b, t, c.n_head, c.n_kv_head, c.max_seq)));
  L.attn_ws_bytes = a;
  L.attn_ws = take(a);
  const int sb = std::min(c.max_batch, kStepMaxM);
  L.st_layers = take((size_t)c.n_layer * sizeof(StepLayer));
  L.st_part = take((size_t)num_sms() * step_num_warps() * 32 * 8 * sizeof(float));  // (value, flag) pairs
  L.st_po = take((size_t)sb * c.n_head * kStepMaxSplits * c.head_dim * sizeof(float));
  L.st_pml = take((size_t)sb * c.n_head * kStepMaxSplits * 2 * sizeof(float));
  L.st_acnt = take((size_t)sb * c.n_kv_head * 4);
  L.st_keys = take((size_t)kStepMaxM * 8);
  L.st_exit = take(16);
  L.st_trace_bytes = (size_t)num_sms() * step_trace_slots(c.n_layer) * 8;
  L.st_trace = take(L.st_trace_bytes);
  L.st_hdump_bytes = (size_t)c.n_layer * sb * c.d_model * 2;
  L.st_hdump = take(L.st_hdump_bytes);
  L.st_maps = take((size_t)c.n_layer * 2 * kStepMapBytes);  // 256-aligned (tensor maps need 64)
  L.st_h = take((size_t)sb * c.d_model * 4);
  L.st_qkv = take((size_t)sb * qkv_dim * 4);
  L.st_attn = take((size_t)sb * c.n_head * c.head_dim * 4);
  L.st_sw = take((size_t)sb * c.ffn * 4);
  L.total = off;
  return L;
}

struct Runner {
  axb_model_cfg c;
  bool pdl = true;  // chain kernels with programmatic dependent launch (env AXB_PDL=0 disables)
  int pdl_mode = 1;  // AXB_PDL=2: programmatic edges, GEMVs release dependents only at exit
  Layout L;
  char* ws;
  const void *emb_w, *emb_s, *lm_w, *lm_s;
  const float *ln_f, *rope;
  std::vector<const void*> qkv_w, qkv_s, qkv_b, o_w, o_s, gu_w, gu_s, dn_w, dn_s;
  std::vector<axb_q2t_meta> q2m;  // copies of the 2-bit projections' metadata (the *_s pointers point here)
  std::vector<const float*> ln1, ln2;
  std::vector<void*> kc, vc, ks, vs;
  void* tp_comm = nullptr;  // tensor parallel communicator (tp_world > 1)
  cudaStream_t cap = nullptr;
  std::map<std::tuple<int, int, int>, cudaGraphExec_t> graphs;
  std::map<std::tuple<int, int, int>, int> graph_kernels;  // kernel nodes per captured step
  // persistent step kernel: decode steps of B <= 8 sequences run as one launch
  bool step_ok = false;
  bool step_graph_ok = true;  // cleared if the cooperative launch cannot be captured
  StepArgs sa = {};

  template <typename T>
  T* buf(size_t off) const {
    return reinterpret_cast<T*>(ws + off);
  }

  int gemv(const void* w, const void* s, int fmt, int group, int N, int K, int M, const __half* x, int ldx,
           void* y, int ldy, const void* bias, const float* norm_w, int epi, int gu, cudaStream_t st) const {
    if (ext_fmt(fmt)) return ext_proj(fmt, w, s, N, K, M, x, ldx, y, ldy, bias, norm_w, epi, st);
    // rows beyond 64 are processed in 64-row chunks (one weight pass each)
    for (int m0 = 0; m0 < M; m0 += 64) {
      axb_qgemm_desc d = {};
      d.fmt = fmt;
      d.group = group;
      d.words = w;
      d.scales = s;
      d.N = N;
      d.K = K;
      d.M = std::min(64, M - m0);
      d.x = x + (size_t)m0 * ldx;
      d.ldx = ldx;
      size_t esz = (epi == AXB_EPI_F32 || epi == AXB_EPI_F32_ACC) ? 4 : 2;
      d.y = reinterpret_cast<char*>(y) + (size_t)m0 * ldy * esz;
      d.ldy = ldy;
      d.bias = bias;
      d.norm_w = norm_w;
      d.eps = c.eps;
      d.epilogue = epi;
      d.gate_up_interleave = gu;
      d.workspace = buf<void>(L.gemm_ws);
      d.workspace_bytes = L.gemm_ws_bytes;
      d.pdl = pdl ? pdl_mode : 0;
      int rc = qgemm(&d, st);
      if (rc) return rc;
    }
    return AXB_OK;
  }

  // y = x W^T (+ bias) for a Q8_G64 or 2-bit projection, fp16 out
  int ext_gemv(int fmt, const void* w, const void* s, int N, int K, int M, const __half* x, int ldx, __half* y,
               int ldy, const __half* b, cudaStream_t st) const {
    if (fmt == AXB_W_Q8_G64)
      return q8_gemv(x, ldx, M, K, static_cast<const uint32_t*>(w), static_cast<const __half2*>(s), N, y, ldy, st, b);
    const axb_q2t_meta* m = static_cast<const axb_q2t_meta*>(s);
    for (int m0 = 0; m0 < M; m0 += kLbMaxM) {
      axb_lbgemv_desc d = {};
      d.fmt = fmt;
      d.words = w;
      d.meta = m->meta;
      d.meta2 = m->meta2;
      d.pt_scale = m->pt_scale;
      d.N = N;
      d.K = K;
      d.M = std::min(kLbMaxM, M - m0);
      d.x = x + (size_t)m0 * ldx;
      d.ldx = ldx;
      d.y = y + (size_t)m0 * ldy;
      d.ldy = ldy;
      d.bias = b;
      d.workspace = buf<void>(L.lb_ws);
      d.workspace_bytes = L.lb_ws_bytes;
      if (int rc = axb_lbgemv(&d, st)) return rc;
    }
    return AXB_OK;
  }

  // Q8_G64 projections (the reference's q8 and q4_k_m modes, transformer.py:847-858)
  // and 2-bit ones: the GEMV rounds its product to fp16 (for Q8, then adds the
  // bias and rounds again, as _qlin does), and the residual add or SwiGLU runs
  // as its own pass with the rounding of the fused Q4 epilogues.  The product
  // lands in h (free during the o / down projections) or gu_tmp (gate_up).
  int ext_proj(int fmt, const void* w, const void* s, int N, int K, int M, const __half* x, int ldx, void* y, int ldy,
               const void* bias, const float* norm_w, int epi, cudaStream_t st) const {
    const __half* b = static_cast<const __half*>(bias);
    AXB_CHECK_ARG(norm_w == nullptr, "runner: Q8 / 2-bit projections take normalized rows");
    if (epi == AXB_EPI_STORE) return ext_gemv(fmt, w, s, N, K, M, x, ldx, static_cast<__half*>(y), ldy, b, st);
    const int grid = std::min((M * N + 255) / 256, 4 * num_sms());
    if (epi == AXB_EPI_RESIDUAL) {
      AXB_CHECK_ARG(ldy == N && N == c.d_model, "runner: residual projection shape");
      if (int rc = ext_gemv(fmt, w, s, N, K, M, x, ldx, buf<__half>(L.h), N, b, st)) return rc;
      residual_add_kernel<<<grid, 256, 0, st>>>(static_cast<__half*>(y), buf<__half>(L.h), M * N);
      return launch_status("residual add");
    }
    if (epi == AXB_EPI_SWIGLU) {
      AXB_CHECK_ARG(N == 2 * c.ffn && ldy == c.ffn && L.gu_tmp, "runner: gate_up projection shape");
      if (int rc = ext_gemv(fmt, w, s, N, K, M, x, ldx, buf<__half>(L.gu_tmp), N, b, st)) return rc;
      swiglu_split_kernel<<<grid, 256, 0, st>>>(buf<__half>(L.gu_tmp), N, c.ffn, M, static_cast<__half*>(y));
      return launch_status("swiglu");
    }
    set_error("runner: epilogue %d is not available for Q8 / 2-bit projections", epi);
    return AXB_EINVAL;
  }

  // norm + GEMV: fused prologue when the normalized rows fit in shared memory
  int norm_gemv(const float* nw, const void* w, const void* s, int N, int K, int M, void* y, int ldy,
                const void* bias, int epi, int gu, int fmt, int group, cudaStream_t st) const {
    const __half* x = buf<__half>(L.x);
    if (!ext_fmt(fmt) && qgemm_can_fuse_norm(M, K))
      return gemv(w, s, fmt, group, N, K, M, x, K, y, ldy, bias, nw, epi, gu, st);
    int rc = rmsnorm(x, nw, M, K, c.eps, buf<__half>(L.h), st);
    if (rc) return rc;
    return gemv(w, s, fmt, group, N, K, M, buf<__half>(L.h), K, y, ldy, bias, nullptr, epi, gu, st);
  }

  // the tcgen05 kernel is built for Q4 symmetric group 128 and affine group 64
  static bool tc_fmt(int fmt, int group) {
    return (fmt == AXB_W_Q4T_SYM && group == 128) || (fmt == AXB_W_Q4T_AFFINE && group == 64);
  }
  bool tc_ok = true;  // env AXB_TC=0 keeps many-token steps on the warp-level GEMV
  bool use_tc(int rows) const {
    return tc_ok && rows > kTcMinRows && c.tp_world <= 1 && L.tc_ws_bytes > 0 && tc_fmt(c.wfmt, c.group) &&
           tc_fmt(c.dn_fmt, c.dn_group) &&
           tc_fmt(c.lm_fmt, c.lm_group);
  }

  // y = x W^T (+ bias) for many rows on the tcgen05 kernel (64 rows per launch)
  int tc_gemm(const void* w, const void* s, int fmt, int group, int N, int K, int M, const __half* x, int ldx,
              __half* y, int ldy, const void* bias, cudaStream_t st) const {
    for (int m0 = 0; m0 < M; m0 += 64) {
      axb_qgemm_desc d = {};
      d.fmt = fmt;
      d.group = group;
      d.words = w;
      d.scales = s;
      d.N = N;
      d.K = K;
      d.M = std::min(64, M - m0);
      d.x = x + (size_t)m0 * ldx;
      d.ldx = ldx;
      d.y = y + (size_t)m0 * ldy;
      d.ldy = ldy;
      d.bias = bias;
      d.epilogue = AXB_EPI_STORE;
      d.workspace = buf<void>(L.tc_ws);
      d.workspace_bytes = L.tc_ws_bytes;
      if (int rc = axb_qgemm_tc(&d, st)) return rc;
    }
    return AXB_OK;
  }

  // RMSNorm (fp16 rows into h) then the tensor-core GEMM
  int norm_tc(const float* nw, const void* w, const void* s, int fmt, int group, int N, int K, int M, __half* y,
              int ldy, const void* bias, cudaStream_t st) const {
    int rc = rmsnorm(buf<__half>(L.x), nw, M, K, c.eps, buf<__half>(L.h), st);
    if (rc) return rc;
    return tc_gemm(w, s, fmt, group, N, K, M, buf<__half>(L.h), K, y, ldy, bias, st);
  }

  // x += W a for the o / down projections.  Tensor parallel: this rank's
  // K-slice gives an fp32 partial, the ranks' partials meet in one allreduce,
  // then the residual add rounds as the single-GPU path does.
  int row_parallel(const void* w, const void* s, int fmt, int group, int K, int rows, const __half* act,
                   cudaStream_t st) const {
    const int d = c.d_model;
    if (use_tc(rows)) {  // h is free here: the product lands there, then the residual add
      int rc = tc_gemm(w, s, fmt, group, d, K, rows, act, K, buf<__half>(L.h), d, nullptr, st);
      if (rc) return rc;
      const int n = rows * d;
      residual_add_kernel<<<std::min((n + 255) / 256, 4 * num_sms()), 256, 0, st>>>(buf<__half>(L.x),
                                                                                   buf<__half>(L.h), n);
      return launch_status("residual add");
    }
    if (c.tp_world <= 1)
      return gemv(w, s, fmt, group, d, K, rows, act, K, buf<void>(L.x), d, nullptr, nullptr, AXB_EPI_RESIDUAL, 0, st);
    int rc = gemv(w, s, fmt, group, d, K, rows, act, K, buf<void>(L.tp_part), d, nullptr, nullptr,
                  AXB_EPI_F32_ACC, 0, st);
    if (rc) return rc;
    rc = tp_allreduce(tp_comm, buf<void>(L.tp_part), (size_t)rows * d, AXB_TP_SUM_F32, st);
    if (rc) return rc;
    return tp_residual(buf<__half>(L.x), buf<float>(L.tp_part), rows * d, st);
  }

  int step_forward(int B, cudaStream_t st) const {
    StepArgs a = sa;
    a.B = B;
    return step_launch(a, st);
  }

  int forward(int B, int T, bool tree, bool want_norm, cudaStream_t st) const {
    const int rows = B * T;
    const int d = c.d_model, hd = c.head_dim, Hq = c.n_head, Hkv = c.n_kv_head;
    const int qkv_dim = (Hq + 2 * Hkv) * hd, qd = Hq * hd;
    cudaError_t e = launch_pdl(embed_q8_kernel, dim3(rows, (d / 4 + 127) / 128), dim3(128), 0, st, pdl,
                               (const uint32_t*)emb_w,
                               (const __half*)emb_s, (const int32_t*)buf<int32_t>(L.tokens), d,
                               c.vocab * c.tp_world,  // the embedding table is whole on every rank
                               buf<__half>(L.x), buf<int>(L.params) + 4);
    if (e != cudaSuccess) return cuda_status(e, "embed launch");
    for (int l = 0; l < c.n_layer; ++l) {
      int rc = use_tc(rows) ? norm_tc(ln1[l], qkv_w[l], qkv_s[l], c.wfmt, c.group, qkv_dim, d, rows,
                                      buf<__half>(L.qkv), qkv_dim, qkv_b[l], st)
                            : norm_gemv(ln1[l], qkv_w[l], qkv_s[l], qkv_dim, d, rows, buf<void>(L.qkv), qkv_dim,
                                        qkv_b[l], AXB_EPI_STORE, 0, c.wfmt, c.group, st);
      if (rc) return rc;
      axb_kv_write_desc kw = {};
      kw.kv_type = c.kv_type;
      kw.kv_group = c.kv_group;
      kw.B = B;
      kw.T = T;
      kw.n_head = Hq;
      kw.n_kv_head = Hkv;
      kw.head_dim = hd;
      kw.max_seq = c.max_seq;
      kw.max_batch = c.max_batch;
      kw.qkv = buf<uint16_t>(L.qkv);
      kw.rope = rope;
      kw.rope_len = c.rope_len;
      kw.depths = tree ? buf<int>(L.depths) : nullptr;
      kw.q_out = buf<float>(L.q);
      kw.dev_params = buf<int32_t>(L.params);
      kw.k_cache = kc[l];
      kw.v_cache = vc[l];
      kw.k_scale = (uint16_t*)ks[l];
      kw.v_scale = (uint16_t*)vs[l];
      kw.k_is_fp32 = 1;
      if (tree) {  // decode (T = 1) fuses RoPE + KV write into the attention kernel
        rc = rope_kv_write(&kw, st, pdl);
        if (rc) return rc;
      }
      axb_attn_desc ad = {};
      ad.kv_type = c.kv_type;
      ad.kv_group = c.kv_group;
      ad.B = B;
      ad.n_head = Hq;
      ad.n_kv_head = Hkv;
      ad.head_dim = hd;
      ad.max_seq = c.max_seq;
      ad.max_batch = c.max_batch;
      ad.q = buf<void>(L.q);
      ad.q_is_fp32 = 1;
      ad.k_cache = kc[l];
      ad.v_cache = vc[l];
      ad.k_scale = (const uint16_t*)ks[l];
      ad.v_scale = (const uint16_t*)vs[l];
      ad.out = buf<void>(L.attn);
      ad.active_len = 1;  // overridden by dev_params
      ad.T = T;
      ad.prefix_len = 0;
      ad.masks = tree ? buf<uint64_t>(L.masks) : nullptr;
      ad.dev_params = buf<int32_t>(L.params);
      ad.workspace = buf<void>(L.attn_ws);
      ad.workspace_bytes = L.attn_ws_bytes;
      ad.pdl = pdl ? 1 : 0;
      if (tree) {
        rc = attention(&ad, st);
      } else {
        DecodeFuse f = {buf<__half>(L.qkv), rope, c.rope_len};
        rc = attention_fused(&ad, f, st);
      }
      if (rc) return rc;
      rc = row_parallel(o_w[l], o_s[l], c.wfmt, c.group, qd, rows, buf<__half>(L.attn), st);
      if (rc) return rc;
      if (use_tc(rows)) {
        rc = norm_tc(ln2[l], gu_w[l], gu_s[l], c.wfmt, c.group, 2 * c.ffn, d, rows, buf<__half>(L.gu_tmp), 2 * c.ffn,
                     nullptr, st);
        if (rc) return rc;
        const size_t n = (size_t)rows * c.ffn;
        swiglu_packed_kernel<<<(int)std::min<size_t>((n + 255) / 256, 4 * num_sms()), 256, 0, st>>>(
            buf<__half>(L.gu_tmp), 2 * c.ffn, c.ffn, rows, buf<__half>(L.sw));
        rc = launch_status("swiglu");
      } else {
        rc = norm_gemv(ln2[l], gu_w[l], gu_s[l], 2 * c.ffn, d, rows, buf<void>(L.sw), c.ffn, nullptr, AXB_EPI_SWIGLU,
                       1, c.wfmt, c.group, st);
      }
      if (rc) return rc;
      rc = row_parallel(dn_w[l], dn_s[l], c.dn_fmt, c.dn_group, c.ffn, rows, buf<__half>(L.sw), st);
      if (rc) return rc;
    }
    int rc;
    if (c.lm_fmt == AXB_W_Q8_G64) {
      // tied lm_head: the Q8_G64 embedding matrix, on the final-norm rows
      // (fp16, the reference's qlin cast) staged in the attention buffer
      e = launch_pdl(rmsnorm_kernel<__half>, dim3(rows), dim3(256), 0, st, pdl, (const __half*)buf<__half>(L.x), ln_f,
                     d, c.eps, buf<__half>(L.attn));
      if (e != cudaSuccess) return cuda_status(e, "lm_head norm launch");
      rc = q8_gemv(buf<__half>(L.attn), d, rows, d, static_cast<const uint32_t*>(lm_w),
                   static_cast<const __half2*>(lm_s), c.vocab, buf<__half>(L.logits), c.vocab, st);
    } else {
      rc = use_tc(rows) ? norm_tc(ln_f, lm_w, lm_s, c.lm_fmt, c.lm_group, c.vocab, d, rows, buf<__half>(L.logits),
                                  c.vocab, nullptr, st)
                        : norm_gemv(ln_f, lm_w, lm_s, c.vocab, d, rows, buf<void>(L.logits), c.vocab, nullptr,
                                    AXB_EPI_STORE, 0, c.lm_fmt, c.lm_group, st);
    }
    if (rc) return rc;
    if (want_norm) {
      e = launch_pdl(rmsnorm_kernel<float>, dim3(rows), dim3(256), 0, st, pdl, (const __half*)buf<__half>(L.x), ln_f,
                     d, c.eps, buf<float>(L.xnorm));
      if (e != cudaSuccess) return cuda_status(e, "final norm launch");
    }
    const int chunk = ((c.vocab + kArgmaxParts - 1) / kArgmaxParts + 7) / 8 * 8;
    const int parts = (c.vocab + chunk - 1) / chunk;
    e = launch_pdl(argmax_part_kernel, dim3(parts, rows), dim3(128), 0, st, pdl, (const __half*)buf<__half>(L.logits),
                   c.vocab, c.vocab, chunk, buf<float>(L.am_v), buf<int>(L.am_i), buf<int>(L.am_cnt),
                   buf<int32_t>(L.amax));
    if (e != cudaSuccess) return cuda_status(e, "argmax launch");
    if (c.tp_world > 1)  // vocab-parallel lm_head: the ranks' winners meet in a max of (value, -index) keys
      return tp_argmax(buf<__half>(L.logits), c.vocab, buf<int32_t>(L.amax), rows, c.tp_rank * c.vocab,
                       buf<unsigned long long>(L.tp_keys), tp_comm, st);
    return AXB_OK;
  }
};

}  // namespace axb

using namespace axb;

extern "C" {

size_t axb_runner_workspace_bytes(const axb_model_cfg* cfg) {
  if (!cfg) return 0;
  return make_layout(*cfg).total;
}

int axb_runner_create(const axb_model_cfg* cfg, const axb_model_ptrs* p, void* ws, size_t ws_bytes, void** out) {
  AXB_CHECK_ARG(cfg && p && ws && out, "runner_create: null argument");
  const axb_model_cfg& c = *cfg;
  AXB_CHECK_ARG(c.n_layer > 0 && c.d_model % 64 == 0 && c.ffn % 64 == 0 && c.vocab > 0, "runner_create: bad dims");
  AXB_CHECK_ARG(c.head_dim == 64 || c.head_dim == 128, "runner_create: head_dim must be 64 or 128");
  const int tpw = c.tp_world > 1 ? c.tp_world : 1;
  AXB_CHECK_ARG(c.tp_world <= 1 || (c.tp_rank >= 0 && c.tp_rank < c.tp_world && p && p->tp_comm),
                "runner_create: tensor parallel needs a rank in [0, tp_world) and a communicator");
  AXB_CHECK_ARG(c.n_head * c.head_dim * tpw == c.d_model,
                "runner_create: n_head * head_dim * tp_world must equal d_model");
  AXB_CHECK_ARG(c.wfmt == AXB_W_Q4T_SYM || c.wfmt == AXB_W_Q4T_AFFINE ||
                    (c.wfmt == AXB_W_Q8_G64 && c.group == 64 && c.tp_world <= 1) ||
                    (is_q2t(c.wfmt) && c.tp_world <= 1),
                "runner_create: unsupported weight format %d", c.wfmt);
  // the down projection: the projections' format, or Q8_G64 (the q4_k_m mode)
  const int dn_fmt = c.dn_fmt ? c.dn_fmt : c.wfmt, dn_group = c.dn_fmt ? c.dn_group : c.group;
  AXB_CHECK_ARG((dn_fmt == c.wfmt && dn_group == c.group) ||
                    (dn_fmt == AXB_W_Q8_G64 && dn_group == 64 && c.tp_world <= 1),
                "runner_create: down projection format %d (group %d) not supported", dn_fmt, dn_group);
  AXB_CHECK_ARG(c.lm_fmt == AXB_W_Q4T_SYM || c.lm_fmt == AXB_W_Q4T_AFFINE ||
                    (c.lm_fmt == AXB_W_Q8_G64 && c.lm_group == 64 && c.tp_world <= 1) ||
                    (is_q2t(c.lm_fmt) && c.tp_world <= 1),
                "runner_create: lm_head format %d not supported by the runner", c.lm_fmt);
  if (is_q2t(c.wfmt) || is_q2t(c.lm_fmt))  // 2-bit k-blocks are 128 wide
    AXB_CHECK_ARG(c.d_model % 128 == 0 && (c.n_head * c.head_dim) % 128 == 0 && c.ffn % 128 == 0,
                  "runner_create: 2-bit projections need d_model, n_head * head_dim and ffn multiples of 128");
  AXB_CHECK_ARG(c.max_tokens >= 1 && c.max_tokens <= 64 && c.max_batch >= 1, "runner_create: bad max_tokens/batch");
  AXB_CHECK_ARG(c.ffn % 8 == 0, "runner_create: ffn must be a multiple of 8");
  Layout L = make_layout(c);
  AXB_CHECK_ARG(ws_bytes >= L.total, "runner_create: workspace %zu < %zu bytes", ws_bytes, L.total);
  AXB_CHECK_ARG(p->emb_w && p->emb_s && p->lm_w && p->lm_s && p->ln_f && p->rope, "runner_create: null model pointer");
  for (int l = 0; l < c.n_layer; ++l) {
    AXB_CHECK_ARG(p->qkv_w[l] && p->qkv_s[l] && p->o_w[l] && p->o_s[l] && p->gu_w[l] && p->gu_s[l] && p->dn_w[l] &&
                      p->dn_s[l] && p->ln1[l] && p->ln2[l] && p->k_cache[l] && p->v_cache[l],
                  "runner_create: null pointer for layer %d", l);
    AXB_CHECK_ARG(c.kv_type == AXB_KV_F16 || (p->k_scale && p->v_scale && p->k_scale[l] && p->v_scale[l]),
                  "runner_create: quantized KV cache needs scales (layer %d)", l);
  }
  if (int rc = qgemm_prepare()) return rc;
  if (int rc = attn_prepare()) return rc;
  Runner* r = new Runner();
  r->c = c;
  r->c.dn_fmt = dn_fmt;
  r->c.dn_group = dn_group;
  if (c.tp_world <= 1) {
    r->c.tp_world = 1;
    r->c.tp_rank = 0;
  }
  r->tp_comm = c.tp_world > 1 ? p->tp_comm : nullptr;
  if (const char* tv = getenv("AXB_TC")) r->tc_ok = atoi(tv) != 0;
  if (const char* ev = getenv("AXB_PDL")) {
    r->pdl = atoi(ev) != 0;
    r->pdl_mode = atoi(ev) == 2 ? 2 : 1;
  }
  r->L = L;
  r->ws = reinterpret_cast<char*>(ws);
  r->emb_w = p->emb_w;
  r->emb_s = p->emb_s;
  r->lm_w = p->lm_w;
  r->lm_s = p->lm_s;
  r->ln_f = p->ln_f;
  r->rope = p->rope;
  for (int l = 0; l < c.n_layer; ++l) {
    r->qkv_w.push_back(p->qkv_w[l]);
    r->qkv_s.push_back(p->qkv_s[l]);
    r->qkv_b.push_back(p->qkv_b ? p->qkv_b[l] : nullptr);
    r->o_w.push_back(p->o_w[l]);
    r->o_s.push_back(p->o_s[l]);
    r->gu_w.push_back(p->gu_w[l]);
    r->gu_s.push_back(p->gu_s[l]);
    r->dn_w.push_back(p->dn_w[l]);
    r->dn_s.push_back(p->dn_s[l]);
    r->ln1.push_back(p->ln1[l]);
    r->ln2.push_back(p->ln2[l]);
    r->kc.push_back(p->k_cache[l]);
    r->vc.push_back(p->v_cache[l]);
    r->ks.push_back(p->k_scale ? p->k_scale[l] : nullptr);
    r->vs.push_back(p->v_scale ? p->v_scale[l] : nullptr);
  }
  // 2-bit projections: the scale pointers address host metadata structs, copied
  // here (reserved up front, so the pointers into q2m stay valid)
  r->q2m.reserve(4 * (size_t)c.n_layer + 1);
  auto own_meta = [&](int fmt, const void*& sp) {
    if (!is_q2t(fmt)) return;
    r->q2m.push_back(*static_cast<const axb_q2t_meta*>(sp));
    sp = &r->q2m.back();
  };
  for (int l = 0; l < c.n_layer; ++l) {
    own_meta(c.wfmt, r->qkv_s[l]);
    own_meta(c.wfmt, r->o_s[l]);
    own_meta(c.wfmt, r->gu_s[l]);
    own_meta(dn_fmt, r->dn_s[l]);
  }
  own_meta(c.lm_fmt, r->lm_s);
  cudaError_t e = cudaStreamCreateWithFlags(&r->cap, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete r;
    return cuda_status(e, "runner stream");
  }
  // persistent step kernel (env AXB_STEP=0 keeps decode on the per-kernel graph)
  const char* sv = getenv("AXB_STEP");
  const StepPlan plan = step_plan(c.max_batch, c.d_model, c.ffn, c.n_head, c.n_kv_head, c.head_dim, c.kv_type,
                                  c.kv_type == AXB_KV_F16 ? c.head_dim : c.kv_group, c.group, c.max_seq);
  // (the step kernel's phase flags allow 127 layers; deeper models take the graph path)
  r->step_ok = !(sv && atoi(sv) == 0) && c.tp_world <= 1 && dn_fmt == c.wfmt && c.n_layer <= 127 &&
               step_supported(c.wfmt, c.group, c.lm_fmt, c.lm_group, c.head_dim, c.n_head, c.n_kv_head, c.d_model,
                              c.kv_type, c.kv_group, c.max_seq) &&
               c.ffn % 64 == 0 && plan.smem > 0;
  if (r->step_ok) {
    if (int rc = step_prepare()) {
      axb_runner_destroy(r);
      return rc;
    }
    std::vector<StepLayer> tab(c.n_layer);
    // TMA tensor maps over every layer's K / V cache, stored in the workspace
    std::vector<char> maps((size_t)c.n_layer * 2 * kStepMapBytes);
    if (int rc = step_kv_maps(maps.data(), c.n_layer, p->k_cache, p->v_cache, c.max_batch * c.n_kv_head * c.max_seq,
                              c.kv_type, c.head_dim)) {
      axb_runner_destroy(r);
      return rc;
    }
    e = cudaMemcpy(r->buf<void>(L.st_maps), maps.data(), maps.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      axb_runner_destroy(r);
      return cuda_status(e, "step tensor maps");
    }
    for (int l = 0; l < c.n_layer; ++l) {
      StepLayer& t = tab[l];
      t.w[0] = (const char*)p->qkv_w[l];
      t.s[0] = (const char*)p->qkv_s[l];
      t.w[1] = (const char*)p->o_w[l];
      t.s[1] = (const char*)p->o_s[l];
      t.w[2] = (const char*)p->gu_w[l];
      t.s[2] = (const char*)p->gu_s[l];
      t.w[3] = (const char*)p->dn_w[l];
      t.s[3] = (const char*)p->dn_s[l];
      t.qkv_b = p->qkv_b ? (const __half*)p->qkv_b[l] : nullptr;
      t.ln1 = p->ln1[l];
      t.ln2 = p->ln2[l];
      t.kc = (uint8_t*)p->k_cache[l];
      t.vc = (uint8_t*)p->v_cache[l];
      t.ks = p->k_scale ? (__half*)p->k_scale[l] : nullptr;
      t.vs = p->v_scale ? (__half*)p->v_scale[l] : nullptr;
      t.kmap = r->buf<char>(L.st_maps) + (size_t)(2 * l) * kStepMapBytes;
      t.vmap = r->buf<char>(L.st_maps) + (size_t)(2 * l + 1) * kStepMapBytes;
    }
    e = cudaMemcpy(r->buf<void>(L.st_layers), tab.data(), tab.size() * sizeof(StepLayer), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      axb_runner_destroy(r);
      return cuda_status(e, "step layer table");
    }
    StepArgs& a = r->sa;
    a.layers = r->buf<StepLayer>(L.st_layers);
    a.L = c.n_layer;
    a.d = c.d_model;
    a.Hq = c.n_head;
    a.Hkv = c.n_kv_head;
    a.hd = c.head_dim;
    a.F = c.ffn;
    a.V = c.vocab;
    a.S = c.max_seq;
    a.kv_type = c.kv_type;
    a.kv_group = c.kv_type == AXB_KV_F16 ? c.head_dim : c.kv_group;
    a.group = c.group;
    a.sym = c.wfmt == AXB_W_Q4T_SYM ? 1 : 0;
    a.eps = c.eps;
    a.emb_w = (const uint32_t*)p->emb_w;
    a.emb_s = (const __half*)p->emb_s;
    a.lm_w = (const char*)p->lm_w;
    a.lm_s = (const char*)p->lm_s;
    a.ln_f = p->ln_f;
    a.rope = p->rope;
    a.rope_len = c.rope_len;
    a.tokens = r->buf<int32_t>(L.tokens);
    a.params = r->buf<int32_t>(L.params);
    a.err = r->buf<int>(L.params) + 4;
    a.h = r->buf<uint2>(L.st_h);
    a.qkv = r->buf<uint2>(L.st_qkv);
    a.attn = r->buf<uint2>(L.st_attn);
    a.sw = r->buf<uint2>(L.st_sw);
    a.logits = r->buf<__half>(L.logits);
    a.amax = r->buf<int32_t>(L.amax);
    a.partials = r->buf<float>(L.st_part);
    a.part_o = r->buf<float>(L.st_po);
    a.part_ml = r->buf<float>(L.st_pml);
    a.attn_cnt = r->buf<int>(L.st_acnt);
    a.keys = r->buf<unsigned long long>(L.st_keys);
    a.exit_cnt = r->buf<int>(L.st_exit);
    a.plan = plan;
    a.pref_kb = 0;  // L2 prefetch past the rings: measured slower (the rings alone saturate HBM)
    if (const char* pv = getenv("AXB_STEP_PREF")) a.pref_kb = atoi(pv);
    a.spin_limit = kStepSpinLimit;
    a.mbar_limit = kStepMbarLimit;
    a.hdump = nullptr;
    const char* tr = getenv("AXB_STEP_TRACE");  // phase timeline into runner buffer 5
    a.trace = (tr && atoi(tr) != 0) ? r->buf<unsigned long long>(L.st_trace) : nullptr;
  }
  *out = r;
  return AXB_OK;
}

int axb_runner_destroy(void* h) {
  Runner* r = reinterpret_cast<Runner*>(h);
  if (!r) return AXB_OK;
  for (auto& kv : r->graphs) cudaGraphExecDestroy(kv.second);
  if (r->cap) cudaStreamDestroy(r->cap);
  delete r;
  return AXB_OK;
}

int axb_runner_buffer(void* h, int which, size_t* off, size_t* bytes) {
  Runner* r = reinterpret_cast<Runner*>(h);
  AXB_CHECK_ARG(r && off && bytes, "runner_buffer: null argument");
  const size_t rows = (size_t)r->c.max_batch * r->c.max_tokens;
  switch (which) {
    case 0: *off = r->L.tokens; *bytes = rows * 4; break;
    case 1: *off = r->L.logits; *bytes = rows * r->c.vocab * 2; break;
    case 2: *off = r->L.amax; *bytes = rows * 4; break;
    case 3: *off = r->L.xnorm; *bytes = rows * r->c.d_model * 4; break;
    case 4: *off = r->L.params + 16; *bytes = 4; break;
    case 5: *off = r->L.st_trace; *bytes = r->L.st_trace_bytes; break;
    case 6: *off = r->L.st_hdump; *bytes = r->L.st_hdump_bytes; break;
    default: axb::set_error("runner_buffer: unknown buffer %d", which); return AXB_EINVAL;
  }
  return AXB_OK;
}

int axb_runner_set_debug(void* h, int flags, uint32_t spin_limit, uint32_t mbar_limit) {
  Runner* r = reinterpret_cast<Runner*>(h);
  AXB_CHECK_ARG(r, "runner_set_debug: null handle");
  AXB_CHECK_ARG((flags & ~3) == 0, "runner_set_debug: unknown flags 0x%x", flags);
  if (!r->step_ok) return AXB_OK;  // the per-kernel graph path has no step-kernel hooks
  StepArgs& a = r->sa;
  a.hdump = (flags & AXB_DEBUG_HDUMP) ? r->buf<__half>(r->L.st_hdump) : nullptr;
  a.trace = (flags & AXB_DEBUG_TRACE) ? r->buf<unsigned long long>(r->L.st_trace) : nullptr;
  a.spin_limit = spin_limit ? spin_limit : kStepSpinLimit;
  a.mbar_limit = mbar_limit ? mbar_limit : kStepMbarLimit;
  // captured step graphs hold the old arguments: drop them
  for (auto it = r->graphs.begin(); it != r->graphs.end();) {
    if (std::get<2>(it->first) == 2) {
      cudaGraphExecDestroy(it->second);
      it = r->graphs.erase(it);
    } else {
      ++it;
    }
  }
  return AXB_OK;
}

int axb_runner_step_launches(void* h, int B, int T, int tree) {
  Runner* r = static_cast<Runner*>(h);
  if (!r) return -1;
  const bool step_mode = !tree && T == 1 && B <= kStepMaxM && r->step_ok;
  auto it = r->graph_kernels.find(std::make_tuple(B, T, step_mode ? 2 : (tree ? 1 : 0)));
  return it == r->graph_kernels.end() ? -1 : it->second + 1;  // + the parameter kernel launched beside the graph
}

int axb_runner_uses_step_kernel(void* h) {
  Runner* r = reinterpret_cast<Runner*>(h);
  return r && r->step_ok ? 1 : 0;
}

int axb_runner_step(void* h, int B, int T, int rope_pos, int write_pos, int active_len, int prefix_len,
                    const uint64_t* masks, const int32_t* depths, int use_graph, void* stream) {
  Runner* r = reinterpret_cast<Runner*>(h);
  AXB_CHECK_ARG(r, "runner_step: null handle");
  const axb_model_cfg& c = r->c;
  AXB_CHECK_ARG(B >= 1 && B <= c.max_batch && T >= 1 && T <= c.max_tokens, "runner_step: bad B/T (%d, %d)", B, T);
  const bool tree = masks != nullptr;
  AXB_CHECK_ARG(tree || T == 1, "runner_step: T > 1 needs masks (tree / chunked-prefill mode)");
  AXB_CHECK_ARG(!tree || (depths != nullptr), "runner_step: tree mode needs depths");
  AXB_CHECK_ARG(tree || (active_len >= 1 && active_len <= c.max_seq), "runner_step: bad active_len %d", active_len);
  AXB_CHECK_ARG(write_pos >= 0 && write_pos < c.max_seq, "runner_step: bad write_pos %d", write_pos);
  AXB_CHECK_ARG(!tree || (prefix_len >= 0 && prefix_len + T <= c.max_seq && write_pos + T <= c.max_seq),
                "runner_step: tree slots must fit in the cache");
  if (tree)
    for (int t = 0; t < T; ++t) {
      AXB_CHECK_ARG((masks[t] >> t) & 1ull, "runner_step: masks[%d] must include the node itself", t);
      AXB_CHECK_ARG(T == 64 || (masks[t] >> T) == 0, "runner_step: masks[%d] has bits beyond T", t);
    }
  cudaStream_t st = (cudaStream_t)stream;
  StepParams sp = {};
  sp.p[0] = rope_pos;
  sp.p[1] = write_pos;
  sp.p[2] = active_len;
  sp.p[3] = prefix_len;
  sp.T = tree ? T : 0;
  if (tree)
    for (int t = 0; t < T; ++t) {
      sp.masks[t] = masks[t];
      sp.depths[t] = depths[t];
    }
  set_params_kernel<<<1, 64, 0, st>>>(sp, r->buf<int32_t>(r->L.params), r->buf<uint64_t>(r->L.masks),
                                      r->buf<int32_t>(r->L.depths));
  int rc = launch_status("set_params");
  if (rc) return rc;
  const bool want_norm = tree;
  const bool step_mode = !tree && T == 1 && B <= kStepMaxM && r->step_ok;
  if (step_mode && (!use_graph || !r->step_graph_ok)) return r->step_forward(B, st);
  if (!use_graph) return r->forward(B, T, tree, want_norm, st);
  auto key = std::make_tuple(B, T, step_mode ? 2 : (tree ? 1 : 0));
  auto it = r->graphs.find(key);
  if (it == r->graphs.end()) {
    cudaError_t e = cudaStreamBeginCapture(r->cap, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return cuda_status(e, "begin capture");
    rc = step_mode ? r->step_forward(B, r->cap) : r->forward(B, T, tree, want_norm, r->cap);
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(r->cap, &g);
    cudaGraphExec_t ex = nullptr;
    if (!rc && e == cudaSuccess) e = cudaGraphInstantiate(&ex, g, 0);
    if (g && ex) {  // count the step's kernel launches
      size_t n = 0;
      if (cudaGraphGetNodes(g, nullptr, &n) == cudaSuccess && n) {
        std::vector<cudaGraphNode_t> nodes(n);
        int k = 0;
        if (cudaGraphGetNodes(g, nodes.data(), &n) == cudaSuccess)
          for (size_t i = 0; i < n; ++i) {
            cudaGraphNodeType t;
            if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++k;
          }
        r->graph_kernels[key] = k;
      }
    }
    if (g) cudaGraphDestroy(g);
    if (step_mode && (rc || e != cudaSuccess)) {
      // the cooperative step launch could not go into a graph: launch it directly from now on
      cudaGetLastError();
      r->step_graph_ok = false;
      return r->step_forward(B, st);
    }
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_status(e, "graph capture");
    it = r->graphs.emplace(key, ex).first;
  }
  return cuda_status(cudaGraphLaunch(it->second, st), "graph launch");
}

}  // extern "C"
