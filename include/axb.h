/*
 * AxiomLM-B200: C ABI of the quantized decode hot path (libaxb.so).
 *
 * Plain pointers and sizes only.  Every pointer argument named *_dev is CUDA
 * device memory on the current device; `stream` is a cudaStream_t passed as
 * void*.  Every entry point returns an int status (AXB_OK == 0, negative on
 * error; axb_last_error() has the message) and never allocates device memory
 * in a steady-state call: scratch space ("workspace") is passed in by the
 * caller, sized by the matching *_workspace_bytes() function and zero-filled
 * once before first use (the kernels leave it zeroed again).
 *
 * Each entry point names the reference interface it replaces (paths inside
 * the AxiomLM project).  Those reference functions are PyTorch/Metal; the host
 * mirror in axiomlm_b200/ops.py keeps their Python names and argument meaning
 * and calls these.
 */
#ifndef AXB_H
#define AXB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status ---------------------------------------------------------------- */
#define AXB_OK 0
#define AXB_EINVAL (-1)       /* bad argument / shape / unsupported combination */
#define AXB_ECUDA (-2)        /* a CUDA runtime call or launch failed */
#define AXB_EUNSUPPORTED (-3) /* device is not sm_100 */
#define AXB_ETIMEOUT (-4)     /* a bounded device-side wait ran out */

/* ---- formats ----------------------------------------------------------------- */
/* Projection weights: q4t = 16-row tiles of mma A-fragments, 64207531 nibble
 * interleave.  A tile (16 rows) stores its K range contiguously as 64-wide
 * k-blocks of 512 B; lane l = 4g + t of a warp owns, in 32-bit word j, rows
 * {g, g + 8} x columns 64b + 16t + 4j + {0..3}.  SYM: w = (q - 8) * s;
 * AFFINE: w = q * s + b. */
#define AXB_W_Q4T_SYM 1
#define AXB_W_Q4T_AFFINE 2
#define AXB_W_Q8_G64 3 /* reference Q8_G64 row-major (quant.py:72) */
/* 2-bit formats (q2t layout on the device, relaid out from these reference packings):
 * TERNARY_G64: pack_linear_ternary (quant.py:236-274): codes (N, K/4) u8 (0 -> 0,
 *   1 -> +1, 2 -> -1), scales (N, K/64) fp16, w = q * s.
 * TERNARY_PT:  same codes, one per-tensor fp16 absmean scale (the format of the GEMV sweep's ternary case).
 * Q2_G64:      pack_linear_q2_k (quant.py:339-381): codes (N, K/4) u8 (u in 0..3),
 *   (scale, bias) (N, K/64, 2) fp16, w = fp16(fp16(u * s) + b).
 * Q2K_SB256:   K-quant-style super-blocks (the long-context low-bit configuration's format): codes (N, K/4) u8,
 *   sub (N, K/16) u8 = sc | mn << 4, (d, dmin) (N, K/256, 2) fp16,
 *   w = d * sc * u - dmin * mn. */
#define AXB_W_TERNARY_G64 4
#define AXB_W_TERNARY_PT 5
#define AXB_W_Q2_G64 6
#define AXB_W_Q2K_SB256 7

/* KV cache element types (StaticKVCache cache_dtype, paged_cache.py:122) */
#define AXB_KV_F16 0
#define AXB_KV_FP8 1  /* e4m3fn + one fp16 scale per kv_group elements */
#define AXB_KV_INT4 2 /* symmetric int4, 2 per byte, low nibble = even element */

/* GEMV epilogues */
#define AXB_EPI_STORE 0    /* y = fp16(acc [+ bias]) */
#define AXB_EPI_RESIDUAL 1 /* y = fp16(y + fp16(acc)) in place (x = x + proj(..)) */
#define AXB_EPI_SWIGLU 2   /* rows interleaved gate/up by 8: y[j] = fp16(silu(g) * u) */
#define AXB_EPI_F32 3      /* y (fp32) = fp16-rounded acc, stored as fp32 */
#define AXB_EPI_F32_ACC 4  /* y (fp32) = acc (+ bias), unrounded: a row-parallel partial sum */

const char* axb_last_error(void);
int axb_version(void);
/* 0 when the current device is sm_100 (B200), AXB_EUNSUPPORTED otherwise */
int axb_check_device(void);

/* ---- weight packing / relayout / dequant -------------------------------- */

/* Bytes of the q4t words / scales arrays for an (N, K) matrix. */
size_t axb_q4t_words_bytes(int N, int K);
size_t axb_q4t_scales_bytes(int N, int K, int group, int fmt);

/* Round-to-nearest pack of fp32 (N, K) row-major weights into q4t.
 * fmt AXB_W_Q4T_AFFINE reproduces pack_linear_q4_marlin(clip_search=False)
 * values (quant.py:475-486) at any group; AXB_W_Q4T_SYM is the
 * benchmark's group-128 symmetric form.  `gate_up_interleave`: rows are [gate(F); up(F)]
 * and are stored interleaved by 8 for the SwiGLU epilogue. */
int axb_q4t_pack(const float* w_dev, int N, int K, int group, int fmt, int gate_up_interleave,
                 void* words_dev, void* scales_dev, void* stream);

/* Relayout reference MARLIN-ladder Q4 (w_marlin int32 (Nt8, K/64, 32, 2),
 * sb_marlin fp16 (Nt8, K/64, 8, 2); quant.py:447-594) into q4t affine G64.
 * Bit-exact on codes, scales and biases. */
int axb_q4t_from_marlin(const int32_t* w_marlin_dev, const uint16_t* sb_marlin_dev, int n_tiles8, int K,
                        int n_out, int gate_up_interleave, void* words_dev, void* scales_dev, void* stream);

/* Relayout the reference's legacy Q4_G64 (w_packed int32 (N, K/8), sb fp16
 * (N, K/64, 2); pack_linear_q4_g64, quant.py:17-69, the "q4_legacy" mode) into
 * q4t affine G64: bit-identical codes, scales and biases. */
int axb_q4t_from_q4g64(const int32_t* w_packed_dev, const uint16_t* sb_dev, int N, int K, int gate_up_interleave,
                       void* words_dev, void* scales_dev, void* stream);

/* fp16 (N, K) dequant of q4t (replaces dequantize_q4_marlin, quant.py:597,
 * on the relaid-out form: identical values). */
int axb_q4t_dequant(const void* words_dev, const void* scales_dev, int N, int K, int group, int fmt,
                    int gate_up_interleave, uint16_t* out_dev, void* stream);

/* Direct dequant of the reference ladder layout (quant.py:597-634). */
int axb_q4_marlin_dequant(const int32_t* w_marlin_dev, const uint16_t* sb_marlin_dev, int n_tiles8, int K,
                          int n_out, uint16_t* out_dev, void* stream);

/* pack_linear_q8_g64 (quant.py:72-129): RTN Q8 G64 of fp32 (N, K) weights into
 * (N, K/4) int32 + (N, K/64, 2) fp16 (scale, bias) */
int axb_q8_pack(const float* w_dev, int N, int K, int32_t* out_dev, uint16_t* sb_dev, void* stream);

/* dequant_q8_rows (quant.py:132-163): out[i] = fp16(q * s + b) of row idx[i] */
int axb_q8_rows(const int32_t* w_dev, const uint16_t* sb_dev, const int32_t* idx_dev, int n_idx, int K,
                uint16_t* out_dev, void* stream);

/* dequantize_ternary (quant.py:277-295) and dequantize_q2_k (quant.py:383-403) */
int axb_ternary_dequant(const uint8_t* w_dev, const uint16_t* s_dev, int N, int K, int per_tensor,
                        uint16_t* out_dev, void* stream);
int axb_q2_dequant(const uint8_t* w_dev, const uint16_t* sb_dev, int N, int K, uint16_t* out_dev, void* stream);

/* ---- 2-bit weights: relayout, dequant, GEMV (qmv_ternary / qmm_ternary,
 *      quant.py:298-336; qmv_q2_k / qmm_q2_k, quant.py:406-444) ----------- */
/* Device bytes of the q2t words / per-group metadata / K-quant super-block
 * metadata for an (N, K) matrix (K a multiple of 128; 256 for Q2K_SB256). */
size_t axb_q2t_words_bytes(int N, int K);
size_t axb_q2t_meta_bytes(int fmt, int N, int K);
size_t axb_q2t_meta2_bytes(int fmt, int N, int K);
/* Relayout a reference packing (see the AXB_W_* 2-bit formats) into q2t.
 * s1: scales (TERNARY_G64), (scale, bias) (Q2_G64), sub bytes (Q2K_SB256),
 * unused for TERNARY_PT; s2: (d, dmin) for Q2K_SB256.  Codes, scales and biases
 * are moved, never recomputed. */
int axb_q2t_from_ref(int fmt, const uint8_t* codes_dev, const void* s1_dev, const void* s2_dev, int N, int K,
                     void* words_dev, void* meta_dev, void* meta2_dev, void* stream);
/* fp16 (N, K) dequant of q2t with the reference's value rule (dequantize_ternary,
 * quant.py:277-295; dequantize_q2_k, quant.py:383-403). */
int axb_q2t_dequant(int fmt, const void* words_dev, const void* meta_dev, const void* meta2_dev,
                    const uint16_t* pt_scale_dev, int N, int K, uint16_t* out_dev, void* stream);
typedef struct {
  int fmt;               /* AXB_W_TERNARY_G64 | TERNARY_PT | Q2_G64 | Q2K_SB256 */
  const void* words;     /* q2t words */
  const void* meta;      /* q2t per-group metadata (NULL for TERNARY_PT) */
  const void* meta2;     /* Q2K_SB256 (d, dmin), else NULL */
  const uint16_t* pt_scale; /* TERNARY_PT fp16 scale, else NULL */
  int N, K, M;           /* y[M, N] = x[M, K] W^T (+ bias); M <= 8 */
  const void* x;         /* fp16 (M, ldx), 16-byte aligned, ldx % 8 == 0 */
  int ldx;
  void* y;               /* fp16 (M, ldy) */
  int ldy;
  const void* bias;      /* fp16 (N) or NULL */
  void* workspace;       /* >= axb_lbgemv_workspace_bytes(fmt, N, K, M): group sums of x, split-K partials */
  size_t workspace_bytes;
} axb_lbgemv_desc;
size_t axb_lbgemv_workspace_bytes(int fmt, int N, int K, int M);
int axb_lbgemv(const axb_lbgemv_desc* d, void* stream);

/* ---- Q8_G64 GEMV / small-M GEMM (qmv_q8_g64 / qmm_q8_g64, quant.py:201-233;
 *      Metal qmv_q8_g64_half_kernel :1941) ------------------------------------
 * y (M, ldy) fp16 = x (M, ldx) fp16 . dequant(W)^T with W in the reference's
 * own Q8_G64 layout: w_packed (N, K/4) int32, scales_biases (N, K/64, 2) fp16,
 * dequantized as dequantize_q8_g64 does (fp16(q * scale + bias) in fp32).
 * K % 64 == 0, ldx % 8 == 0, x and w 16-byte aligned. The tied lm_head (the
 * reference default) runs on it. No workspace. */
int axb_q8g64_gemv(const void* x, int ldx, int M, int K, const int32_t* w_packed, const uint16_t* scales_biases,
                   int N, void* y, int ldy, void* stream);

/* ---- quantized GEMV / small-M GEMM (qmv_q4_marlin / qmm_q4_marlin,
 *      quant.py:637-684; Metal qmv_q4_marlin_apple_kernel) ------------------- */
typedef struct {
  int fmt;            /* AXB_W_Q4T_SYM | AXB_W_Q4T_AFFINE */
  int group;          /* 64 | 128 */
  const void* words;  /* q4t words */
  const void* scales; /* q4t scales */
  int N, K, M;        /* y[M, N] = x[M, K] W^T ; M <= 64 */
  const void* x;      /* fp16 (M, ldx) */
  int ldx;
  void* y; /* fp16 (M, ldy) or fp32 for AXB_EPI_F32 */
  int ldy;
  const void* bias;     /* fp16 (N) or NULL */
  const float* norm_w;  /* if non-NULL: B operand = fp16(rmsnorm(x) * norm_w) (fp32 math) */
  float eps;
  int epilogue;         /* AXB_EPI_* */
  int gate_up_interleave;
  void* workspace; /* >= axb_qgemm_workspace_bytes(...), zeroed once */
  size_t workspace_bytes;
  int pdl; /* 1: programmatic dependent launch, dependents released after the
              x staging; 2: dependents released at exit; 0: plain launch */
} axb_qgemm_desc;

size_t axb_qgemm_workspace_bytes(int N, int K, int M, int group);
int axb_qgemm(const axb_qgemm_desc* d, void* stream);
/* GEMV that allocates nothing, for callers that cannot hand over device
 * memory: hosts that reserve the whole device in their own pool up front,
 * plugin or FFI hosts with no allocator of their own, and latency-critical
 * paths where an allocation's implicit synchronization is not acceptable.
 * Same arguments and results as axb_qgemm, but d->workspace is ignored: the
 * scratch (error word, tile counters, partial sums) is a fixed array of
 * axb_qgemm_noalloc_scratch_bytes() (about 1.5 MiB) inside the library, one
 * per GPU, held until the process exits.  Limits: M <= 8 tokens.  The first
 * call on a device looks the array's device address up (make that call before
 * any stream capture).  All calls share the array: two calls that may run at
 * the same time on the GPU (different streams without ordering) race.  Each
 * call clears the tile counters, which must start at zero; the error word
 * holds until axb_qgemm_noalloc_status reads it.  This entry point has no
 * counterpart in the reference. */
int axb_qgemm_noalloc(const axb_qgemm_desc* d, void* stream);
size_t axb_qgemm_noalloc_scratch_bytes(void);
/* Synchronizes `stream`; returns AXB_ETIMEOUT (and clears the flag) if a
 * bounded weight-stream wait of an earlier axb_qgemm_noalloc on this device
 * ran out, so its y may be incomplete.  No counterpart in the reference. */
int axb_qgemm_noalloc_status(void* stream);
/* Synchronizes `stream`; returns AXB_ETIMEOUT (and clears the flag) if a
 * bounded weight-stream wait in an earlier axb_qgemm on this workspace ran out. */
int axb_qgemm_status(void* workspace, void* stream);

/* The same product on the tcgen05 tensor cores for large M (qmm_q4_marlin,
 * quant.py:664-684, Metal qmm_q4_marlin_apple_kernel :2404): 1 <= M <= 64,
 * fmt SYM group 128 or AFFINE group 64, plain store epilogue (+ bias).  Weights
 * are dequantized to the reference's fp16 values, products accumulate in fp32
 * tensor memory.  The workspace (error word, split-K partials) is
 * zero-filled once; axb_qgemm_tc_status reports a bounded wait that ran out. */
size_t axb_qgemm_tc_workspace_bytes(int N, int K, int M);
int axb_qgemm_tc(const axb_qgemm_desc* d, void* stream);
int axb_qgemm_tc_status(void* workspace, void* stream);

/* ---- RMSNorm (modules.py:30-43) ---------------------------------------- */
/* out fp16 (M, K) = fp16(fp32(x) * rsqrt(mean(x^2) + eps) * w) */
int axb_rmsnorm(const uint16_t* x_dev, const float* w_dev, int M, int K, float eps, uint16_t* out_dev,
                void* stream);

/* ---- KV write with RoPE (rope_kv_cache_write_quantized, quant.py:896-1008;
 *      StaticKVCache.update, paged_cache.py:218-361) --------------------------- */
typedef struct {
  int kv_type;  /* AXB_KV_* */
  int kv_group; /* elements per fp16 scale (64 ref, head_dim, 32) */
  int B, T;     /* sequences, new tokens per sequence */
  int n_head, n_kv_head, head_dim;
  int max_seq;           /* cache S */
  int max_batch;         /* cache batch capacity (stride) */
  const uint16_t* qkv;   /* fp16 (B*T, (Hq + 2*Hkv) * hd) GEMV output */
  const uint16_t* bias;  /* optional fp16 qkv bias or NULL */
  const float* rope;     /* (rope_len, hd/2, 2) fp32 = view_as_real(freqs_cis) */
  int rope_len;
  int rope_pos;          /* position of token 0 */
  const int* depths;     /* optional per-token offsets (tree verify) or NULL: offset = t */
  int write_pos;         /* slot of token 0 (slot t = (write_pos + t) % S) */
  float* q_out;          /* fp32 (B*T, Hq*hd): rotated queries (kept fp32, as the reference) */
  const int32_t* dev_params; /* optional device [rope_pos, write_pos, active_len, prefix_len]
                                overriding the scalar fields (CUDA-graph replay) */
  void* k_cache;         /* (max_batch, Hkv, S, row) */
  void* v_cache;
  uint16_t* k_scale;     /* (max_batch, Hkv, S, hd/kv_group) fp16, or NULL for F16 */
  uint16_t* v_scale;
  int k_is_fp32;         /* quantize K from fp32 (model path) instead of fp16 (op path) */
} axb_kv_write_desc;
int axb_rope_kv_write(const axb_kv_write_desc* d, void* stream);

/* Quantize fp16/fp32 (rows, hd) into the cache formats (quantize_kv_fp8 /
 * quantize_kv_int4, quant.py:692-807). */
int axb_kv_quantize(const void* x_dev, int x_is_fp32, int rows, int head_dim, int kv_type, int kv_group,
                    void* q_dev, uint16_t* scale_dev, void* stream);
/* dequantize_kv_fp8 / dequantize_kv_int4 (quant.py:727-852) */
int axb_kv_dequantize(const void* q_dev, const uint16_t* scale_dev, int rows, int head_dim, int kv_type,
                      int kv_group, uint16_t* out_dev, void* stream);

/* ---- attention (gqa_flash_decode_mps ops.py:552, gqa_tree_verify_mps
 *      ops.py:657; Metal gqa_flash_decode_split_kv_*_kernel) -------------- */
typedef struct {
  int kv_type, kv_group;
  int B, n_head, n_kv_head, head_dim, max_seq, max_batch;
  const void* q; /* fp32 or fp16 (B*T, Hq*hd) */
  int q_is_fp32;
  const void* k_cache;
  const void* v_cache;
  const uint16_t* k_scale;
  const uint16_t* v_scale;
  void* out; /* fp16 (B*T, Hq*hd) */
  /* decode (T == 1): all slots [0, active_len) are visible */
  int active_len;
  int num_splits; /* 0 = auto */
  /* tree (T >= 1): slots [0, prefix_len) plus tree slot write_pos + j when
   * bit j of masks[t] is set */
  int T;
  int prefix_len;
  int write_pos;
  const uint64_t* masks; /* device, T entries; NULL = decode mode */
  const int32_t* dev_params; /* optional device [rope_pos, write_pos, active_len, prefix_len] */
  void* workspace;
  size_t workspace_bytes;
  int pdl;
} axb_attn_desc;
size_t axb_attn_workspace_bytes(int B, int n_head, int n_kv_head, int head_dim, int max_seq, int kv_type,
                                int num_splits);
int axb_attention(const axb_attn_desc* d, void* stream);

/* compact_tree_path (paged_cache.py:376-462): move accepted tree slots
 * (write_pos + acc[m]) % S -> (write_pos + m) % S across all layers. */
int axb_compact_kv(void* cache_dev, uint16_t* scales_dev, int n_layer, int max_batch, int n_kv_head,
                   int max_seq, int row_bytes, int n_groups, int write_pos, const int32_t* accepted_dev,
                   int n_accepted, void* stream);

/* compact_tree_path with the accepted list and its length in device memory
 * (written by axb_tree_accept: accepted = result + AXB_TREE_RESULT_HDR,
 * n_accepted_dev = result), so no host round trip sits between the walk and
 * the compaction.  max_accepted (<= 64) bounds the count and sizes the
 * staging; an identity path (acc[m] == m) moves nothing. */
int axb_compact_kv_dev(void* cache_dev, uint16_t* scales_dev, int n_layer, int max_batch, int n_kv_head,
                       int max_seq, int row_bytes, int n_groups, int write_pos, const int32_t* accepted_dev,
                       const int32_t* n_accepted_dev, int max_accepted, void* stream);

/* Greedy argmax over rows (ties -> lowest index, torch.argmax). */
int axb_argmax(const uint16_t* x_dev, int rows, int n, int ld, int32_t* out_dev, void* stream);

/* ---- whole-model decode runner (replaces MPSQuantizedDecodeRunner,
 *      mps_kernels.mm:2982-3737; Transformer.forward T=1 fast path,
 *      transformer.py:1438-1473, forward_tree_verify transformer.py:581) ---- */
typedef struct {
  int n_layer, d_model, n_head, n_kv_head, head_dim, ffn, vocab;
  float eps;
  int wfmt, group;       /* projection format: AXB_W_Q4T_*, AXB_W_Q8_G64 group 64 (the q8 mode),
                            or a 2-bit AXB_W_TERNARY_* / AXB_W_Q2_* format (group unused) */
  int lm_fmt, lm_group;  /* lm_head: AXB_W_Q4T_* or AXB_W_Q8_G64 (tied, q8, q4_k_m) */
  int kv_type, kv_group; /* cache format */
  int max_batch, max_seq, max_tokens; /* max_tokens = tokens per sequence per step (<= 64) */
  int rope_len;
  int has_qkv_bias;
  /* tensor parallelism (0 or 1: off).  With tp_world > 1, n_head, n_kv_head,
   * ffn and vocab are this rank's shard (heads tp_rank * n_head .., FFN rows
   * tp_rank * ffn .., vocab rows tp_rank * vocab ..); d_model is replicated. */
  int tp_world, tp_rank;
  /* down projection format: 0 = the projections' (wfmt, group), or
   * AXB_W_Q8_G64 group 64 (the q4_k_m mode: Q4 projections, Q8 w_down,
   * transformer.py:847).  Q8 projections keep the reference's own layout,
   * gate_up as cat(w_gate, w_up); they run on the per-kernel graph path. */
  int dn_fmt, dn_group;
} axb_model_cfg;

/* Metadata of a 2-bit projection (q2t, from axb_q2t_from_ref) served by the
 * runner.  For the AXB_W_TERNARY_* / AXB_W_Q2_* formats, a projection's scale
 * pointer (qkv_s[l], o_s[l], gu_s[l], dn_s[l], lm_s) points to one of these
 * in host memory; axb_runner_create copies them.  2-bit gate_up projections
 * keep the reference's row order, cat(w_gate, w_up). */
typedef struct {
  const void* meta;         /* q2t per-group metadata, or NULL (TERNARY_PT) */
  const void* meta2;        /* Q2K_SB256 (d, dmin), else NULL */
  const uint16_t* pt_scale; /* TERNARY_PT fp16 scale (device), else NULL */
} axb_q2t_meta;

typedef struct {
  const void* emb_w;  /* Q8_G64 (V, d/4) int32 */
  const void* emb_s;  /* (V, d/64, 2) fp16 */
  const void* lm_w;
  const void* lm_s;
  const float* ln_f;
  const float* rope; /* (rope_len, hd/2, 2) fp32 */
  const void* const* qkv_w;
  const void* const* qkv_s;
  const void* const* qkv_b; /* may be NULL or entries NULL */
  const void* const* o_w;
  const void* const* o_s;
  const void* const* gu_w; /* gate/up interleaved by 8 */
  const void* const* gu_s;
  const void* const* dn_w;
  const void* const* dn_s;
  const float* const* ln1;
  const float* const* ln2;
  void* const* k_cache; /* per layer (max_batch, Hkv, S, row) */
  void* const* v_cache;
  void* const* k_scale; /* per layer fp16 or NULL */
  void* const* v_scale;
  void* tp_comm; /* from axb_tp_comm_create when tp_world > 1, else NULL */
} axb_model_ptrs;

size_t axb_runner_workspace_bytes(const axb_model_cfg* cfg);
/* workspace: zeroed device memory of the size above, owned by the caller */
int axb_runner_create(const axb_model_cfg* cfg, const axb_model_ptrs* ptrs, void* workspace_dev,
                      size_t workspace_bytes, void** handle_out);
int axb_runner_destroy(void* handle);
/* Offsets (bytes, into the workspace) of the runner's I/O buffers:
 * which = 0 tokens int32 (max_batch*max_tokens), 1 logits fp16 (rows, vocab),
 * 2 argmax int32 (rows), 3 final-norm hidden fp32 (rows, d), 4 error word int32
 * (non-zero after a step that met an out-of-vocabulary token id or a bounded
 * device wait that ran out), 5 step-kernel phase timeline uint64 (SMs,
 * slots per SM) globaltimer stamps, written when AXB_STEP_TRACE=1 was set at
 * creation or AXB_DEBUG_TRACE is on, 6 step-kernel residual stream after each
 * layer fp16 (n_layer, B, d), written when AXB_DEBUG_HDUMP is on */
int axb_runner_buffer(void* handle, int which, size_t* offset_out, size_t* bytes_out);
/* Test and diagnosis hooks of the persistent step kernel (no counterpart in
 * the reference): flags AXB_DEBUG_HDUMP (per-layer hidden states into buffer
 * 6) and AXB_DEBUG_TRACE (phase timeline into buffer 5); spin_limit /
 * mbar_limit: polls of a cross-CTA counter / of a copy's mbarrier before a
 * step gives up with AXB_ETIMEOUT (0 = the defaults, 2^22).  A step that gives
 * up still waits for its own copies in flight and leaves the runner usable.
 * A no-op for runners on the per-kernel graph path. */
#define AXB_DEBUG_HDUMP 1
#define AXB_DEBUG_TRACE 2
int axb_runner_set_debug(void* handle, int flags, uint32_t spin_limit, uint32_t mbar_limit);
/* One forward step over B sequences x T new tokens already placed in the
 * token buffer.  T == 1 and masks == NULL: decode (all active slots visible).
 * Otherwise tree/chunk mode: masks[t] / depths[t] host arrays of length T. */
int axb_runner_step(void* handle, int B, int T, int rope_pos, int write_pos, int active_len, int prefix_len,
                    const uint64_t* masks_host, const int32_t* depths_host, int use_graph, void* stream);
/* 1 when decode steps (T == 1, B <= 8) of this runner run as one persistent
 * kernel launch, 0 when they run as the per-kernel CUDA graph (unsupported
 * format, or AXB_STEP=0 in the environment at creation). */
int axb_runner_uses_step_kernel(void* handle);
/* Kernel launches of one step of shape (B, T, tree) once its CUDA graph has
 * been captured (the graph's kernel nodes + the parameter kernel launched
 * beside it); -1 if no such step has run through a graph yet. */
int axb_runner_step_launches(void* handle, int B, int T, int tree);

/* ---- Medusa speculative decoding on the device (engine/medusa.py:48-116,
 *      :231-330, models/medusa.py:20-54, transformer.py:414-445) ----------- */
#define AXB_TREE_MAX_NODES 64 /* uint64 ancestor masks */
#define AXB_TREE_RESULT_HDR 4
/* result block of axb_tree_accept (int32): [0] accepted node count n (>= 1),
 * [1] last accepted node (the next draft's leaf), [2] emitted token count
 * (== n), [3] last emitted token, then AXB_TREE_MAX_NODES accepted node ids
 * (node 0 first) and AXB_TREE_MAX_NODES emitted tokens. */
#define AXB_TREE_RESULT_WORDS (AXB_TREE_RESULT_HDR + 2 * AXB_TREE_MAX_NODES)
#define AXB_TOPK_MAX 64
/* Greedy walk of engine/medusa.py:312-330 over a tree of T nodes: at node
 * cur emit preds[cur]; descend to the first child c (children = nodes with
 * parent[c] == cur, in increasing index order, as compile_medusa_tree lists
 * them) whose draft token verif[c] equals it; stop when none does or after
 * `budget` (>= 1) emitted tokens.  parent[0] = -1 and parent[u] < u.  All
 * arrays are device int32 (preds: the runner's per-node argmax). */
int axb_tree_accept(int T, const int32_t* parent, const int32_t* verif, const int32_t* preds, int budget,
                    int32_t* result, void* stream);
/* Head input of the next draft: x32 = norm[leaf] (fp32 final-norm rows of
 * width d), x16 = fp16(x32).  leaf_dev (device int32, e.g. result + 1) wins
 * over the host index `leaf` when non-NULL. */
int axb_medusa_leaf(const float* norm, int d, const int32_t* leaf_dev, int leaf, float* x32, uint16_t* x16,
                    void* stream);
/* Residual Medusa heads (MedusaHead.forward with use_residual): for each of
 * the K heads, h16[k] = fp16(x32 + silu(r16[k])) with r16[k] = the fp16
 * output of that head's residual GEMV on x16 (all fp32 math). */
int axb_medusa_silu_add(int K, int d, const float* x32, const uint16_t* r16, uint16_t* h16, void* stream);
/* Top-k indices of each fp16 row (k <= AXB_TOPK_MAX), by value descending,
 * equal values by lower index (torch.topk leaves tie order open): out_idx is
 * (rows, k) int32. */
int axb_topk_rows(const uint16_t* x, int rows, int n, int ld, int k, int32_t* out_idx, void* stream);
/* Next draft (engine/medusa.py:290-298): tokens[0] = *root (the last emitted
 * token), tokens[u] = topk[head_idx[u] * kmax + rank[u]] for u >= 1. */
int axb_draft_tokens(int T, const int32_t* head_idx, const int32_t* rank, const int32_t* topk, int kmax,
                     const int32_t* root, int32_t* tokens, void* stream);

/* ---- tensor parallelism over NVLink (no counterpart in the reference, whose
 *      only collective is a training all_reduce, train.py:296) ------------- */
#define AXB_TP_SUM_F32 0
#define AXB_TP_SUM_F16 1
#define AXB_TP_MAX_U64 2
/* NCCL unique id (128 bytes) made on one rank and shared with the others by
 * the host (torch.distributed, a store, ...). */
int axb_tp_unique_id(void* id_out);
/* Communicator of `world` ranks on the current device; one per rank. */
int axb_tp_comm_create(const void* id, int world, int rank, void** comm_out);
int axb_tp_comm_destroy(void* comm);
/* Abandon a communicator whose peers may be gone (pending collectives end). */
int axb_tp_comm_abort(void* comm);
/* In-place allreduce of `count` elements on `stream` (AXB_TP_*). */
int axb_tp_allreduce(void* comm, void* buf_dev, size_t count, int op, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* AXB_H */
