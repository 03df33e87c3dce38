// Arguments of the persistent decode-step kernel (step.cu), filled by the
// runner (runner.cu).
#pragma once

#include "axb_common.cuh"

namespace axb {

// Per-layer weights and cache, one entry per layer in device memory.
struct StepLayer {
  const char* w[4];  // q4t words: QKV, o, gate_up (interleaved by 8), down
  const char* s[4];  // matching scales
  const __half* qkv_b;
  const float* ln1;
  const float* ln2;
  uint8_t* kc;
  uint8_t* vc;
  __half* ks;
  __half* vs;
  const void* kmap;  // TMA tensor maps (CUtensorMap, device memory) over kc / vc as
  const void* vmap;  // (rows = max_batch * Hkv * S, row bytes) tables
};

// Shared-memory plan of one step-kernel configuration (host-computed once per
// runner): per-warp weight rings of `nslots` slots, a union region that holds
// the staged activations of a GEMV phase or the attention working set, and a
// fixed scratch area.
struct StepPlan {
  int nslots;       // ring slots per warp
  int slot_kb;      // k-blocks (512 B of weights) per slot
  int union_bytes;  // staged activations / attention working set
  int attn_cap;     // cached tokens per attention sub-chunk
  int smem;         // dynamic shared memory of the launch
};

struct StepArgs {
  const StepLayer* layers;
  int L;
  int d, Hq, Hkv, hd, F, V, S, kv_type, kv_group, group;
  int sym;  // 1: AXB_W_Q4T_SYM, 0: AXB_W_Q4T_AFFINE (all projections and the lm_head)
  float eps;
  int B;  // sequences this step (one token each), <= kStepMaxM
  const uint32_t* emb_w;
  const __half* emb_s;
  const char* lm_w;
  const char* lm_s;
  const float* ln_f;
  const float* rope;
  int rope_len;
  const int32_t* tokens;
  const int32_t* params;  // rope_pos, write_pos, active_len, prefix_len
  int* err;
  // activations, as flagged words: word i of a row holds halves 2i, 2i + 1 and
  // the flag of the phase that wrote them (the reader waits for the flag)
  uint2* h;        // (B, d / 2) residual stream
  uint2* qkv;      // (B, (Hq + 2 Hkv) hd / 2)
  uint2* attn;     // (B, Hq hd / 2)
  uint2* sw;       // (B, F / 2)
  __half* logits;  // (B, V)
  int32_t* amax;   // (B,)
  // scratch (zeroed once; every counter returns to zero by the end of a step)
  float* partials;    // split-tile pieces: per CTA two slots (phase parity) of 32 lanes x 4 (value, flag) pairs
  float* part_o;      // attention split partials (B, Hq, kStepMaxSplits, hd)
  float* part_ml;     // (B, Hq, kStepMaxSplits, 2)
  int* attn_cnt;      // (B, Hkv) split arrivals, grow through a step
  unsigned long long* keys;  // per-token argmax keys
  int* exit_cnt;      // [0] CTAs done, [1] abort flag, [2] launch epoch
  StepPlan plan;
  // bounded waits: polls of a flagged word (activations, split-tile pieces)
  // and of a copy's mbarrier
  // before the step gives up with AXB_ETIMEOUT (copies already issued are
  // still waited for, with a fixed limit, before a CTA exits)
  uint32_t spin_limit;
  uint32_t mbar_limit;
  int pref_kb;        // k-blocks ahead of a warp's ring that it also prefetches into L2 (0: off)
  __half* hdump;      // optional (L, B, d): the residual stream after each layer
  unsigned long long* trace;  // optional phase timeline: [CTA][step_trace_slots(L)] globaltimer stamps
};

// Phase timeline slots per CTA: start, 10 per layer, then lm_head wait,
// lm_head done, exit (thread 0); then, per GEMV phase, the time each of the
// CTA's warps finished its share; then, per layer, the time the CTA finished
// its attention items.
constexpr int kStepTraceW = 16;  // warp slots per GEMV phase (the warps per CTA)
__host__ __device__ inline int step_trace_slots(int L) { return 4 + 10 * L + (4 * L + 1) * kStepTraceW + 2 * L; }

constexpr int kStepMaxSplits = 64;
constexpr int kStepMaxM = 8;
constexpr uint32_t kStepSpinLimit = 1u << 22;  // default polls of a flagged word
constexpr uint32_t kStepMbarLimit = 1u << 22;  // default polls of a copy's mbarrier

// host side
int step_prepare();
// Shared-memory plan for a model (batch up to max_batch); plan.smem == 0 when
// the configuration does not fit the kernel.
StepPlan step_plan(int max_batch, int d, int F, int Hq, int Hkv, int hd, int kv_type, int kv_group, int group,
                   int max_seq);
bool step_supported(int wfmt, int group, int lm_fmt, int lm_group, int hd, int n_head, int n_kv_head, int d_model,
                    int kv_type, int kv_group, int max_seq);
int step_num_warps();  // warps per CTA of the step kernel (partials are sized per warp)
int step_launch(const StepArgs& a, cudaStream_t s);
// Encode the tensor maps of every layer's K and V cache into maps_host
// (2 * L CUtensorMap, K then V per layer) for the attention staging.
int step_kv_maps(void* maps_host, int L, void* const* kc, void* const* vc, int rows, int kv_type, int hd);
constexpr int kStepMapBytes = 128;  // sizeof(CUtensorMap)

}  // namespace axb
