// Persistent decode step for sm_100a: one cooperative launch (one CTA per SM)
// runs a whole T = 1 forward pass -- embedding, every layer, lm_head, argmax.
//
// Replaces the decode step of MPSQuantizedDecodeRunner / QuantizedDecodeGraphState
// (axiomlm/kernels/mps_kernels.mm:2982-3737, step at :3195), i.e. the T = 1 path of
// Transformer._forward_quantized_sequence (axiomlm/models/transformer.py:1036-1200)
// with StaticKVCache.update (engine/paged_cache.py:250-361) and
// gqa_flash_decode_mps (kernels/ops.py:552-654) inside it.  Numerics are those of
// the per-kernel runner (runner.cu): fp16 activations, fp32 accumulation, the
// reference's RMSNorm / RoPE / KV-quantization rounding points.
//
// Design.
//  * Every GEMV of the step is split "stream-K" over quantization groups with one
//    rule: warp i of the grid owns units [i*U/W, (i+1)*U/W).  A warp's weight
//    stream for the whole step is therefore known at launch.  Lane 0 streams it
//    through a private ring of bulk copies (TMA, non-tensor form) and runs ahead
//    across phase boundaries -- weights never depend on activations -- with an
//    L2 prefetch further ahead, so HBM keeps streaming while the warp waits for
//    the previous phase's activations.
//  * Phases are ordered by completion counters in global memory (tiles finished,
//    attention heads finished) instead of kernel boundaries.  Every wait is
//    bounded; one that runs out records AXB_ETIMEOUT and the grid winds down.
//  * A tile split between warps is finished by the last warp to arrive, which
//    sums the partials in warp order: results are deterministic.
//  * Attention runs on two groups of four warps per CTA over (sequence, kv head,
//    split) items; the cached rows of an item are bulk-copied before the QKV
//    phase has finished; RoPE and the new K/V row's quantized write are fused.
#include <algorithm>

#include "kv.cuh"
#include "q4t.cuh"
#include "step.cuh"

namespace axb {

#ifndef AXB_STEP_CH
#define AXB_STEP_CH 8
#endif
#ifndef AXB_STEP_WARPS
#define AXB_STEP_WARPS 8
#endif
#ifndef AXB_STEP_STAGES
#define AXB_STEP_STAGES (AXB_STEP_WARPS >= 16 ? 2 : 3)
#endif
#ifndef AXB_STEP_CHAINS
#define AXB_STEP_CHAINS 2
#endif
// 1: the GEMV / attention / norm bodies are separate functions (smaller code, own register budgets)
#ifndef AXB_STEP_OUTLINE
#define AXB_STEP_OUTLINE 0
#endif
// 1: a stage is copied to registers and its ring slot re-armed before the math
#ifndef AXB_STEP_REGSTAGE
#define AXB_STEP_REGSTAGE 1
#endif
#if AXB_STEP_OUTLINE
#define AXB_STEP_FN __noinline__
#else
#define AXB_STEP_FN __forceinline__
#endif
constexpr int kSW = AXB_STEP_WARPS;  // warps per CTA (one CTA per SM)
constexpr int kSThreads = kSW * 32;
constexpr int kSCH = AXB_STEP_CH;          // k-blocks (512 B of weights each) per ring stage
constexpr int kSStages = AXB_STEP_STAGES;  // ring stages per warp
constexpr int kSChains = AXB_STEP_CHAINS;  // independent MMA accumulator chains per warp
constexpr int kSStageW = kSCH * 512;
constexpr int kSStageS = kSCH * 64;  // scale bytes per stage (max: affine, one group per k-block)
constexpr int kSRing = (kSStages * (kSStageW + kSStageS) + kSStages * 8 + 127) / 128 * 128;
// staged activations, or the two attention groups' working sets
constexpr int kSUnion = (kSW >= 16 ? 72 : 96) * 1024;
constexpr int kSMisc = 1024;  // reduction scratch [kSW][kStepMaxM] + attention mbarriers + flags
constexpr size_t kSSmem = (size_t)kSW * kSRing + kSUnion + kSMisc;
constexpr int kSGroups = 2;  // attention groups (4 warps each, warps 0-7) per CTA
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr uint32_t kSMbarLimit = 1u << 22;
constexpr int kMaxRepS = 4;  // q heads per kv head (GQA up to 4:1; larger ratios use the per-kernel runner)
constexpr int kXsumLd = 16;  // tokens per group row of the staged-x sums
// the staged-x sums of a K-wide activation sit at the end of the union, the rows from its start
__host__ __device__ constexpr int xsum_bytes(int K, int G) { return ((K / G) * kXsumLd * 4 + 127) / 128 * 128; }
__host__ __device__ constexpr bool xs_fits(int M, int K, int G) {
  return (long long)M * (K + 8) * 2 <= (long long)(kSUnion - xsum_bytes(K, G));
}
// D = A * B with a zero accumulator (the first MMA of a chain)
__device__ __forceinline__ void mma_16816_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}
static_assert(kSSmem <= 227 * 1024, "step kernel shared memory");
static_assert(kSStageW % 16 == 0 && kSStageS % 16 == 0 && kSRing % 128 == 0, "bulk-copy alignment");
static_assert((kSStages * (kSStageW + kSStageS)) % 8 == 0, "mbarrier alignment");
static_assert(kSW >= 4 * kSGroups, "attention groups are 4 warps");
static_assert(kSW * kStepMaxM * 4 <= 512, "reduction scratch");
static_assert(kSW <= kStepTraceW, "trace slots per phase");

// ------------------------------------------------------------------ helpers
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Hand-offs between CTAs: the writers of a block of results meet at a warp /
// group / CTA barrier, then one thread publishes with a release (or acq_rel)
// atomic; the reader polls with an acquire load and meets its peers at a
// barrier before they read.  No full fences.
__device__ __forceinline__ void red_release_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int atom_acq_rel_add(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void group_bar(int id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }
// barrier of one attention group that also ORs a predicate over its 128 threads
__device__ __forceinline__ bool group_bar_or(int id, bool p) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred q, o;\n setp.ne.u32 q, %1, 0;\n bar.red.or.pred o, %2, 128, q;\n selp.u32 %0, 1, 0, o;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)p), "r"(id)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ int tiles_of(int n) { return (n + 15) >> 4; }

// phase timeline stamp, only when a trace buffer is set: thread 0 of each CTA
// (trace_mark), or the calling thread (trace_at)
__device__ __forceinline__ void trace_at(const StepArgs& a, int slot) {
  if (a.trace == nullptr) return;
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  a.trace[(size_t)blockIdx.x * step_trace_slots(a.L) + slot] = t;
}
__device__ __forceinline__ void trace_mark(const StepArgs& a, int slot) {
  if (threadIdx.x == 0) trace_at(a, slot);
}

// Bounded wait for *ctr >= target.  Gives up early when another CTA has already
// raised the abort flag; on running out it raises the flag and records
// AXB_ETIMEOUT in the error word.
__device__ bool wait_ge(const int* ctr, int target, const StepArgs& a) {
  int* abort_flag = a.exit_cnt + 1;
  for (uint32_t it = 0; it < kSpinLimit; ++it) {
    if (ld_acquire(ctr) >= target) return true;
    if ((it & 15) == 15 && *reinterpret_cast<volatile int*>(abort_flag) != 0) return false;
    __nanosleep(it < 32 ? 20 : 200);
  }
  atomicExch(abort_flag, 1);
  atomicExch(a.err, AXB_ETIMEOUT);
  return false;
}

__device__ void raise_abort(const StepArgs& a) {
  atomicExch(a.exit_cnt + 1, 1);
  atomicExch(a.err, AXB_ETIMEOUT);
}

// CTA-wide wait: thread 0 polls, the barrier publishes the outcome.
__device__ bool cta_wait(const int* ctr, int target, const StepArgs& a, bool ok) {
  int good = 0;
  if (threadIdx.x == 0 && ok) good = wait_ge(ctr, target, a) ? 1 : 0;
  return __syncthreads_or(good) != 0;
}

// ------------------------------------------------------------------ GEMV phases
// phase p: 4*l + {0 QKV, 1 o, 2 gate_up, 3 down}; 4*L = lm_head
struct GPh {
  const char* W;
  const char* S;
  int N, K, upt, kind;
  long long U;
};

// Warps that share a GEMV: min(warps, units), so every participating warp
// owns at least one unit (the arrival count of a split tile relies on it).
// Virtual warp v owns units [v*U/We, (v+1)*U/We); v = wid * C + cta spreads a
// small GEMV over all CTAs.
__device__ __forceinline__ long long eff_warps(long long U, int Wt) { return U < Wt ? U : (long long)Wt; }

__device__ __forceinline__ GPh gph(const StepArgs& a, int ph) {
  GPh g;
  if (ph >= 4 * a.L) {
    g.W = a.lm_w;
    g.S = a.lm_s;
    g.N = a.V;
    g.K = a.d;
    g.kind = 4;
  } else {
    const StepLayer* ly = a.layers + (ph >> 2);
    const int k = ph & 3;
    g.W = ly->w[k];
    g.S = ly->s[k];
    g.kind = k;
    switch (k) {
      case 0: g.N = (a.Hq + 2 * a.Hkv) * a.hd; g.K = a.d; break;
      case 1: g.N = a.d; g.K = a.Hq * a.hd; break;
      case 2: g.N = 2 * a.F; g.K = a.d; break;
      default: g.N = a.d; g.K = a.F; break;
    }
  }
  g.upt = g.K / a.group;
  g.U = (long long)tiles_of(g.N) * g.upt;
  return g;
}

// Producer cursor over a warp's weight stream (lane 0 only).
struct Cur {
  int ph, t, t_last, kb, kb_end, upt;
  long long u0, u1;
  const char* W;
  const char* S;
};

template <int GB>
__device__ __forceinline__ void cur_tile(Cur& c) {
  c.kb = (int)max(c.u0, (long long)c.t * c.upt) * GB;
  c.kb_end = (int)min(c.u1, (long long)(c.t + 1) * c.upt) * GB;
}

template <int GB>
__device__ void cur_load(Cur& c, const StepArgs& a, int gw, int Wt) {
  const GPh g = gph(a, c.ph);
  c.W = g.W;
  c.S = g.S;
  c.upt = g.upt;
  const long long We = eff_warps(g.U, Wt);
  c.u0 = gw < We ? (long long)gw * g.U / We : 0;
  c.u1 = gw < We ? (long long)(gw + 1) * g.U / We : 0;
  if (c.u0 >= c.u1) {
    c.t = 0;
    c.t_last = -1;
    c.kb = c.kb_end = 0;
    return;
  }
  c.t = (int)(c.u0 / c.upt);
  c.t_last = (int)((c.u1 - 1) / c.upt);
  cur_tile<GB>(c);
}

// advance past exhausted tiles / phases; false at the end of the step
template <int GB>
__device__ bool cur_fix(Cur& c, const StepArgs& a, int gw, int Wt) {
  while (c.kb >= c.kb_end) {
    if (c.t < c.t_last) {
      ++c.t;
      cur_tile<GB>(c);
      continue;
    }
    if (c.ph >= 4 * a.L) return false;
    ++c.ph;
    cur_load<GB>(c, a, gw, Wt);
  }
  return true;
}

// Per-warp ring of kSStages slots.  Slot indices and mbarrier parities are
// advanced incrementally (no divisions on the per-stage path).  A slot is
// re-armed by the same warp after its stage has been computed: the generic
// loads of the stage have returned by then, so no proxy fence is needed.
struct Ring {
  char* buf;
  uint64_t* bars;
  int cs, cpar;     // consumer: next slot and the parity its mbarrier completes with
  int ps;           // producer (lane 0): next slot to fill
  int inflight;     // producer (lane 0): stages issued and not yet consumed
};

__device__ __forceinline__ void ring_consumed(Ring& r) {
  if (++r.cs == kSStages) {
    r.cs = 0;
    r.cpar ^= 1;
  }
  --r.inflight;
}

template <bool SYM, int GB>
__device__ __forceinline__ void ring_issue(Ring& r, Cur& pc, const StepArgs& a, int gw, int Wt, int lane) {
  if (lane != 0) return;
  constexpr int UB = SYM ? 32 : 64;  // scale bytes per group
  if (pc.kb >= pc.kb_end && !cur_fix<GB>(pc, a, gw, Wt)) return;
  const int st = r.ps;
  r.ps = st + 1 == kSStages ? 0 : st + 1;
  const int n = min(kSCH, pc.kb_end - pc.kb);
  const uint32_t bw = n * 512, bs = (n / GB) * UB;
  mbar_expect_tx(r.bars + st, bw + bs);
  bulk_g2s(r.buf + st * kSStageW, pc.W + (size_t)pc.kb * 512, bw, r.bars + st);
  bulk_g2s(r.buf + kSStages * kSStageW + st * kSStageS, pc.S + (size_t)(pc.kb / GB) * UB, bs, r.bars + st);
  pc.kb += n;
  ++r.inflight;
}

__device__ __forceinline__ int warp_of_unit(long long u, long long U, long long Wt) {
  return (int)(((u + 1) * Wt - 1) / U);
}

// Tile epilogue: token n = 2*t4 + e, rows tile*16 + g (+8).
__device__ void step_epilogue(const StepArgs& a, const GPh& g, int tile, const float (&acc)[4], int lane) {
  const int gg = lane >> 2, t4 = lane & 3;
  const int r0 = tile * 16 + gg, r1 = r0 + 8;
  const int M = a.B;
  unsigned long long best[2] = {0ull, 0ull};
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int n = 2 * t4 + e;
    if (n >= M) continue;
    const float v0 = acc[e], v1 = acc[2 + e];
    if (g.kind == 2) {  // SwiGLU: rows g (gate) and g + 8 (up) of the interleaved tile
      const int j = tile * 8 + gg;
      if (j < a.F) {
        const float gv = __half2float(__float2half_rn(v0));
        const float uv = __half2float(__float2half_rn(v1));
        a.sw[(size_t)n * a.F + j] = __float2half_rn(__fmul_rn(silu_f(gv), uv));
      }
      continue;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = h ? r1 : r0;
      if (row >= g.N) continue;
      float v = h ? v1 : v0;
      if (g.kind == 0) {
        a.qkv[(size_t)n * g.N + row] = __float2half_rn(v);
      } else if (g.kind == 4) {
        const __half vh = __float2half_rn(v);
        a.logits[(size_t)n * a.V + row] = vh;
        // argmax key: ordered value bits, then the lowest row wins ties
        uint32_t bits = __float_as_uint(__half2float(vh));
        bits = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
        const unsigned long long key = ((unsigned long long)bits << 32) | (0xFFFFFFFFu - (uint32_t)row);
        best[e] = key > best[e] ? key : best[e];
      } else {  // residual add into h (fp16 GEMV output, fp16 sum)
        __half* hp = a.h + (size_t)n * a.d + row;
        const float old = __half2float(__ldcg(hp));
        *hp = __float2half_rn(__fadd_rn(old, __half2float(__float2half_rn(v))));
      }
    }
  }
  if (g.kind == 4) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      unsigned long long k = best[e];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        const unsigned long long ok = __shfl_xor_sync(0xffffffffu, k, o);
        k = ok > k ? ok : k;
      }
      const int n = 2 * t4 + e;
      if (gg == 0 && n < M && k) atomicMax(a.keys + n, k);
    }
  }
}

// QKV bias (c_attn_bs) is folded in by the QKV tile finisher
__device__ __forceinline__ void qkv_bias_fix(const StepArgs& a, const StepLayer* ly, const GPh& g, int tile,
                                             float (&acc)[4], int lane) {
  if (g.kind != 0 || ly == nullptr || ly->qkv_b == nullptr) return;
  const int gg = lane >> 2;
  const int r0 = tile * 16 + gg, r1 = r0 + 8;
  if (r0 < g.N) {
    const float b0 = __half2float(ly->qkv_b[r0]);
    acc[0] = __fadd_rn(acc[0], b0);
    acc[1] = __fadd_rn(acc[1], b0);
  }
  if (r1 < g.N) {
    const float b1 = __half2float(ly->qkv_b[r1]);
    acc[2] = __fadd_rn(acc[2], b1);
    acc[3] = __fadd_rn(acc[3], b1);
  }
}

// One GEMV phase for this warp.  x is staged in shared memory (XS: normalized
// rows + per-group sums) or read from global memory (L2) one k-block ahead.
template <bool SYM, int GB, bool XS>
__device__ AXB_STEP_FN bool gemv_phase(const StepArgs& a, int ph, Ring& r, Cur& pc, const __half* xs, int xs_stride,
                           const float* xsum, const __half* xg, int ldx, int gw, int Wt, int lane,
                           bool ok, int* done_ctr) {
  const GPh g = gph(a, ph);
  const long long We = eff_warps(g.U, Wt);
  if (gw >= We || !ok) return ok;
  const long long u0 = (long long)gw * g.U / We, u1 = (long long)(gw + 1) * g.U / We;
  const StepLayer* ly = ph < 4 * a.L ? a.layers + (ph >> 2) : nullptr;
  const int gq = lane >> 2, t4 = lane & 3;
  const int KB = g.K / 64;
  const int t_first = (int)(u0 / g.upt), t_last = (int)((u1 - 1) / g.upt);
  const int nn = min(gq, a.B - 1);
  const uint4* xrow = reinterpret_cast<const uint4*>((XS ? xs + (size_t)nn * xs_stride : xg + (size_t)nn * ldx) +
                                                     16 * t4);
  int finished = 0;
  constexpr int CH = kSChains;
  for (int t = t_first; t <= t_last && ok; ++t) {
    const int kb_lo = (int)max(u0, (long long)t * g.upt) * GB;
    const int kb_hi = (int)min(u1, (long long)(t + 1) * g.upt) * GB;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    // accumulators per MMA chain, in two sets used by alternate groups: the
    // scale fold of one group overlaps the MMAs of the next
    float tmp2[2][CH][4];
#pragma unroll
    for (int p2 = 0; p2 < 2; ++p2)
#pragma unroll
      for (int c2 = 0; c2 < CH; ++c2)
#pragma unroll
        for (int q = 0; q < 4; ++q) tmp2[p2][c2][q] = 0.f;
    uint4 xn0 = make_uint4(0, 0, 0, 0), xn1 = xn0;
    if (!XS) {
      xn0 = __ldcg(xrow + (kb_lo - t * KB) * 8);
      xn1 = __ldcg(xrow + (kb_lo - t * KB) * 8 + 1);
    }
    for (int kb0 = kb_lo; kb0 < kb_hi;) {
      const int st = r.cs;
      const bool got = mbar_wait(r.bars + st, (uint32_t)r.cpar, kSMbarLimit);
      if (!__all_sync(0xffffffffu, got)) {  // one decision for the whole warp
        if (lane == 0) raise_abort(a);
        ok = false;
        break;
      }
      const int n = min(kSCH, kb_hi - kb0);
      const uint4* wst = reinterpret_cast<const uint4*>(r.buf + st * kSStageW) + lane;
      const char* sst = r.buf + kSStages * kSStageW + st * kSStageS;
      const int kbt = kb0 - t * KB;
      // copy the stage (this lane's words, the scales of its rows) into
      // registers and hand the slot back at once: the next copy is in flight
      // while this stage is computed
      uint4 wreg[AXB_STEP_REGSTAGE ? kSCH : 1];
      uint2 sreg[AXB_STEP_REGSTAGE ? kSCH : 1];  // SYM: .x = (s[g], s[g+8]); AFFINE: (s, b) pairs
      if (AXB_STEP_REGSTAGE) {
#pragma unroll
        for (int j = 0; j < (AXB_STEP_REGSTAGE ? kSCH : 1); ++j) {
          if (j < n) wreg[j] = wst[j * 32];
          if (j < n / GB) {
            if (SYM) sreg[j].x = reinterpret_cast<const uint32_t*>(sst)[j * 8 + gq];
            else sreg[j] = reinterpret_cast<const uint2*>(sst)[j * 8 + gq];
          }
        }
        __syncwarp();
        ring_consumed(r);
        ring_issue<SYM, GB>(r, pc, a, gw, Wt, lane);
      }
      auto wword = [&](const int j) -> uint4 { return AXB_STEP_REGSTAGE ? wreg[AXB_STEP_REGSTAGE ? j : 0] : wst[j * 32]; };
      auto sword = [&](const int gi) -> uint2 {
        if (AXB_STEP_REGSTAGE) return sreg[AXB_STEP_REGSTAGE ? gi : 0];
        return SYM ? make_uint2(reinterpret_cast<const uint32_t*>(sst)[gi * 8 + gq], 0u)
                   : reinterpret_cast<const uint2*>(sst)[gi * 8 + gq];
      };
      auto kblock = [&](const int j) {
        float(&tmp)[CH][4] = tmp2[SYM ? ((j / GB) & 1) : 0];
        const uint4 cur = wword(j);
        uint32_t bf[8];
        if (XS) {
          const uint4 v0 = xrow[(kbt + j) * 8], v1 = xrow[(kbt + j) * 8 + 1];
          bf[0] = v0.x; bf[1] = v0.y; bf[2] = v0.z; bf[3] = v0.w;
          bf[4] = v1.x; bf[5] = v1.y; bf[6] = v1.z; bf[7] = v1.w;
        } else {
          bf[0] = xn0.x; bf[1] = xn0.y; bf[2] = xn0.z; bf[3] = xn0.w;
          bf[4] = xn1.x; bf[5] = xn1.y; bf[6] = xn1.z; bf[7] = xn1.w;
          if (kb0 + j + 1 < kb_hi) {
            xn0 = __ldcg(xrow + (kbt + j + 1) * 8);
            xn1 = __ldcg(xrow + (kbt + j + 1) * 8 + 1);
          }
        }
        const uint32_t words[4] = {cur.x, cur.y, cur.z, cur.w};
        if (SYM && XS) {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            uint32_t af[4];
            unpack_word_raw(words[jj], af);
            // the first MMA of each chain in a group starts from zero
            const bool fresh = (j % GB) == 0 && jj < CH;
            if (fresh)
              mma_16816_z(tmp[jj % CH], af, bf[2 * jj], bf[2 * jj + 1]);
            else
              mma_16816(tmp[jj % CH], af, bf[2 * jj], bf[2 * jj + 1], tmp[jj % CH]);
          }
          if (GB == 1 || (j & 1)) {  // group complete: remove the offsets, apply the scales
            const uint32_t sp = sword(j / GB).x;
            const float2 sc = __half22float2(u32_as_h2(sp));
            const int grp = (kbt + j) / GB;
            const float2 xg2 = *reinterpret_cast<const float2*>(xsum + grp * kXsumLd + 2 * t4);
            float s4[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float v = tmp[0][q];
#pragma unroll
              for (int c2 = 1; c2 < CH; ++c2) v += tmp[c2][q];
              s4[q] = v;
            }
            acc[0] = __fmaf_rn(sc.x, __fmaf_rn(-1032.f, xg2.x, s4[0]), acc[0]);
            acc[1] = __fmaf_rn(sc.x, __fmaf_rn(-1032.f, xg2.y, s4[1]), acc[1]);
            acc[2] = __fmaf_rn(sc.y, __fmaf_rn(0.0625f, s4[2], -72.f * xg2.x), acc[2]);
            acc[3] = __fmaf_rn(sc.y, __fmaf_rn(0.0625f, s4[3], -72.f * xg2.y), acc[3]);
          }
        } else if (SYM) {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            uint32_t af[4];
            unpack_word<8>(words[jj], af);
            const bool fresh = (j % GB) == 0 && jj < CH;
            if (fresh)
              mma_16816_z(tmp[jj % CH], af, bf[2 * jj], bf[2 * jj + 1]);
            else
              mma_16816(tmp[jj % CH], af, bf[2 * jj], bf[2 * jj + 1], tmp[jj % CH]);
          }
          if (GB == 1 || (j & 1)) {
            const uint32_t sp = sword(j / GB).x;
            const float2 sc = __half22float2(u32_as_h2(sp));
            float s4[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float v = tmp[0][q];
#pragma unroll
              for (int c2 = 1; c2 < CH; ++c2) v += tmp[c2][q];
              s4[q] = v;
            }
            acc[0] = __fmaf_rn(sc.x, s4[0], acc[0]);
            acc[1] = __fmaf_rn(sc.x, s4[1], acc[1]);
            acc[2] = __fmaf_rn(sc.y, s4[2], acc[2]);
            acc[3] = __fmaf_rn(sc.y, s4[3], acc[3]);
          }
        } else {
          const uint2 sb = sword(j / GB);
          const __half2 s01 = u32_as_h2(sb.x), s23 = u32_as_h2(sb.y);
          const __half2 sg = __half2half2(__low2half(s01)), bg = __half2half2(__high2half(s01));
          const __half2 sg8 = __half2half2(__low2half(s23)), bg8 = __half2half2(__high2half(s23));
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            uint32_t af[4];
            unpack_word<0>(words[jj], af);
            af[0] = h2_as_u32(__hfma2(u32_as_h2(af[0]), sg, bg));
            af[1] = h2_as_u32(__hfma2(u32_as_h2(af[1]), sg8, bg8));
            af[2] = h2_as_u32(__hfma2(u32_as_h2(af[2]), sg, bg));
            af[3] = h2_as_u32(__hfma2(u32_as_h2(af[3]), sg8, bg8));
            mma_16816(tmp[jj % CH], af, bf[2 * jj], bf[2 * jj + 1], tmp[jj % CH]);
          }
        }
      };
      if (n == kSCH) {
#pragma unroll
        for (int j = 0; j < kSCH; ++j) kblock(j);
      } else {
#pragma unroll
        for (int j = 0; j < kSCH; ++j)
          if (j < n) kblock(j);
      }
      if (!AXB_STEP_REGSTAGE) {
        __syncwarp();
        ring_consumed(r);
        ring_issue<SYM, GB>(r, pc, a, gw, Wt, lane);
      }
      kb0 += n;
    }
    if (!ok) break;
    if (!SYM) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float v = tmp2[0][0][q];
#pragma unroll
        for (int c2 = 1; c2 < CH; ++c2) v += tmp2[0][c2][q];
        acc[q] = v;
      }
    }
    const bool complete = (long long)t * g.upt >= u0 && (long long)(t + 1) * g.upt <= u1;
    if (complete) {
      qkv_bias_fix(a, ly, g, t, acc, lane);
      step_epilogue(a, g, t, acc, lane);
      ++finished;
      continue;
    }
    // A split tile is finished by the warp that owns its first unit: the tile
    // is always that warp's last one (had its range run past the tile, it
    // would own the whole tile).  Every other warp of the tile has it as its
    // first tile: it publishes a partial and moves on without waiting.
    const int wf = warp_of_unit((long long)t * g.upt, g.U, We);
    const int wl = warp_of_unit((long long)(t + 1) * g.upt - 1, g.U, We);
    if (gw != wf) {
      float* p = a.partials + ((size_t)(gw * 2) * 32 + lane) * 4;
      *reinterpret_cast<float4*>(p) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      __syncwarp();
      if (lane == 0) red_release_add(a.tile_cnt + t, 1);
      continue;
    }
    int arrived = 1;
    if (lane == 0) arrived = wait_ge(a.tile_cnt + t, wl - wf, a) ? 1 : 0;
    if (__shfl_sync(0xffffffffu, arrived, 0) == 0) {
      ok = false;
      break;
    }
    // the partials in warp order, this warp's own first
    float tot[4] = {acc[0], acc[1], acc[2], acc[3]};
    for (int w0 = wf + 1; w0 <= wl; w0 += 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)  // independent loads, all in flight
        if (w0 + u <= wl) v[u] = __ldcg(reinterpret_cast<const float4*>(a.partials + ((size_t)((w0 + u) * 2) * 32 + lane) * 4));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (w0 + u > wl) continue;
        tot[0] += v[u].x;
        tot[1] += v[u].y;
        tot[2] += v[u].z;
        tot[3] += v[u].w;
      }
    }
    qkv_bias_fix(a, ly, g, t, tot, lane);
    step_epilogue(a, g, t, tot, lane);
    if (lane == 0) a.tile_cnt[t] = 0;  // published by the done counter's release below
    ++finished;
  }
  if (finished) {
    __syncwarp();
    if (lane == 0) red_release_add(done_ctr, finished);
  }
  return ok;
}

// ------------------------------------------------------------------ staging
// Embedding rows (dequant_q8_rows, quant.py:132-163) into xs; CTA 0 also
// stores them into h (the residual stream).
__device__ void stage_embed(const StepArgs& a, __half* xs, int stride) {
  const int K4 = a.d / 4;
  for (int i = threadIdx.x; i < a.B * K4; i += blockDim.x) {
    const int m = i / K4, k4 = i % K4;
    const int r = a.tokens[m];
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (r >= 0 && r < a.V) {
      const uint32_t word = a.emb_w[(size_t)r * K4 + k4];
      const __half2 p = reinterpret_cast<const __half2*>(a.emb_s)[(size_t)r * (a.d / 64) + k4 / 16];
      const float s = __low2float(p), bi = __high2float(p);
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = __fadd_rn(__fmul_rn((float)((word >> (8 * j)) & 0xFF), s), bi);
    } else if (blockIdx.x == 0 && k4 == 0) {
      atomicExch(a.err, AXB_EINVAL);  // out-of-vocabulary id: zero row
    }
    __half2 h01 = __floats2half2_rn(v[0], v[1]), h23 = __floats2half2_rn(v[2], v[3]);
    uint2 pk = make_uint2(h2_as_u32(h01), h2_as_u32(h23));
    *reinterpret_cast<uint2*>(xs + (size_t)m * stride + 4 * k4) = pk;
    if (blockIdx.x == 0) *reinterpret_cast<uint2*>(a.h + (size_t)m * a.d + 4 * k4) = pk;
  }
}

// Stage M rows of K activations into shared memory (row stride K + 8 halves):
// from global memory (src), or the raw rows already in xs (src null).  With
// an RMSNorm weight w (modules.py:30-43: rms = 1/sqrt(mean(x^2) + eps),
// fp16((x * rms) * w)) the rows are normalized in place.  With sums (SYM
// weights) the fp32 per-group sums of the staged rows follow.
__device__ __noinline__ void stage_x(int B, int G, float eps, const __half* src, int K, const float* w, __half* xs,
                                     int stride, float* xsum, bool sums, float* red) {
  const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, wid = tid >> 5;
  const int K8 = K / 8;
  for (int m = 0; m < B; ++m) {
    float ss = 0.f;
    const uint4* srow = src ? reinterpret_cast<const uint4*>(src + (size_t)m * K) : nullptr;
    uint4* drow = reinterpret_cast<uint4*>(xs + (size_t)m * stride);
    for (int c0 = tid; c0 < K8; c0 += 4 * nth) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)  // all loads of the round in flight together
        if (c0 + u * nth < K8) v[u] = srow ? __ldcg(srow + c0 + u * nth) : drow[c0 + u * nth];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (c0 + u * nth >= K8) continue;
        if (srow) drow[c0 + u * nth] = v[u];
        if (w) {
          const __half2* hh = reinterpret_cast<const __half2*>(&v[u]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = __half22float2(hh[q]);
            ss = __fmaf_rn(f.x, f.x, ss);
            ss = __fmaf_rn(f.y, f.y, ss);
          }
        }
      }
    }
    if (w) {
      ss = warp_sum(ss);
      if (lane == 0) red[wid * kStepMaxM + m] = ss;
    }
  }
  __syncthreads();
  if (w) {
    for (int i = tid; i < B * K8; i += nth) {
      const int m = i / K8, c = i % K8;
      float tot = 0.f;
      for (int ww = 0; ww < (nth >> 5); ++ww) tot += red[ww * kStepMaxM + m];
      const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), eps)));
      uint4* sp = reinterpret_cast<uint4*>(xs + (size_t)m * stride) + c;
      const uint4 v = *sp;
      const __half2* hh = reinterpret_cast<const __half2*>(&v);
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(w) + 2 * c);
      const float4 w1 = __ldg(reinterpret_cast<const float4*>(w) + 2 * c + 1);
      const float ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      uint4 o;
      __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __half22float2(hh[q]);
        oh[q] = __floats2half2_rn(__fmul_rn(__fmul_rn(f.x, rms), ws[2 * q]),
                                  __fmul_rn(__fmul_rn(f.y, rms), ws[2 * q + 1]));
      }
      *sp = o;
    }
    __syncthreads();
  }
  if (sums) {
    const int ngr = K / G, nw = nth >> 5;
    for (int item = wid; item < ngr * B; item += nw) {
      const int grp = item % ngr, m = item / ngr;
      const __half* sx = xs + (size_t)m * stride + grp * G;
      float v = 0.f;
      for (int k = lane * 2; k < G; k += 64) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(sx + k));
        v += f.x + f.y;
      }
      v = warp_sum(v);
      if (lane == 0) xsum[grp * kXsumLd + m] = v;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ attention
struct AttnLayout {
  int rb, ng, kv, ksc, vsc, qh, p, ml, coef, bytes;
};

// Working set of one attention group: staged K and V rows, their fp16 scales
// (bulk-copied with the rows), q as fp16 hi / lo parts (8 rows, the ones past
// n_rep zero), the probabilities, the online-softmax state and the split
// combine weights.
__host__ __device__ inline AttnLayout attn_layout(int kv_type, int hd, int kv_group, int cap) {
  AttnLayout L;
  L.rb = kv_row_bytes(kv_type, hd);
  L.ng = kv_type == AXB_KV_F16 ? 1 : hd / kv_group;
  int off = 0;
  L.kv = off;
  off += 2 * cap * L.rb;
  off = (off + 15) / 16 * 16;
  const int sb = (cap * L.ng * 2 + 15) / 16 * 16;
  L.ksc = off;
  off += sb;
  L.vsc = off;
  off += sb;
  L.qh = off;
  off += 2 * 8 * hd * 2;
  L.p = off;
  off += kMaxRepS * cap * 4;
  L.ml = off;
  off += 32 * 4;  // m[8], l[8], alpha[8], flags
  L.coef = off;
  off += kMaxRepS * kStepMaxSplits * 4;
  L.bytes = (off + 127) / 128 * 128;
  return L;
}

__device__ __forceinline__ void attn_split_plan(int active, int units, int cap, int& nsplit, int& chunk) {
  int target = units;
  if (target > kStepMaxSplits) target = kStepMaxSplits;
  if (target < 1) target = 1;
  chunk = (active + target - 1) / target;
  chunk = (chunk + 15) / 16 * 16;
  if (chunk < 16) chunk = 16;
  nsplit = (active + chunk - 1) / chunk;
  (void)cap;
}

// Issue the bulk copy of cached K/V rows [c0, c0 + nt) of one head and, for
// quantized caches, their scales (rounded up to 8 tokens: 16-byte copies;
// the cache length is a multiple of 8) (group thread 0).
__device__ __forceinline__ void attn_copy(const StepLayer* ly, size_t head_base, int rb, int ng, bool quant, int c0,
                                          int nt, char* gsm, const AttnLayout& Lo, int cap, uint64_t* bar) {
  const int nt8 = (nt + 7) & ~7;
  fence_proxy_async();
  mbar_expect_tx(bar, 2u * nt * rb + (quant ? 2u * nt8 * ng * 2 : 0u));
  bulk_g2s(gsm + Lo.kv, ly->kc + (head_base + c0) * rb, nt * rb, bar);
  bulk_g2s(gsm + Lo.kv + (size_t)cap * rb, ly->vc + (head_base + c0) * rb, nt * rb, bar);
  if (quant) {
    bulk_g2s(gsm + Lo.ksc, ly->ks + (head_base + c0) * ng, nt8 * ng * 2, bar);
    bulk_g2s(gsm + Lo.vsc, ly->vs + (head_base + c0) * ng, nt8 * ng * 2, bar);
  }
}

struct AttnItem {
  int b, kvh, split, t0, t1;
};

__device__ __forceinline__ AttnItem attn_item_of(int item, int nsplit, int chunk, int Hkv, int active) {
  AttnItem it;
  it.split = item % nsplit;
  const int r2 = item / nsplit;
  it.kvh = r2 % Hkv;
  it.b = r2 / Hkv;
  it.t0 = it.split * chunk;
  it.t1 = min(active, it.t0 + chunk);
  return it;
}

// fp16 pair (elements e, e + 1) of a staged K/V row: an MMA fragment register
// holding the cache's exact values (fp16, e4m3 codes, or int4 codes)
__device__ __forceinline__ uint32_t kv_pair_h2(const uint8_t* row, int type, int e) {
  if (type == AXB_KV_F16) return *reinterpret_cast<const uint32_t*>(row + e * 2);
  if (type == AXB_KV_FP8) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(*reinterpret_cast<const uint16_t*>(row + e), __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
  }
  const uint32_t cb = row[e >> 1];  // low nibble = element e, high = e + 1; value (n ^ 8) - 8
  const uint32_t t = (((cb & 0xFu) | ((cb & 0xF0u) << 12)) ^ 0x00080008u) | 0x64006400u;
  return h2_as_u32(__hsub2(u32_as_h2(t), __float2half2_rn(1032.f)));
}
// element e of two staged rows as an fp16 pair (row0, row1); an absent row is 0
__device__ __forceinline__ uint32_t kv_col_pair_h2(const uint8_t* r0, const uint8_t* r1, int type, int e) {
  if (type == AXB_KV_F16) {
    const uint32_t lo = r0 ? reinterpret_cast<const uint16_t*>(r0)[e] : 0u;
    const uint32_t hi = r1 ? reinterpret_cast<const uint16_t*>(r1)[e] : 0u;
    return lo | (hi << 16);
  }
  if (type == AXB_KV_FP8) {
    const uint16_t two = (uint16_t)((r0 ? r0[e] : 0u) | ((r1 ? r1[e] : 0u) << 8));
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(two, __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
  }
  const uint32_t sh = (e & 1) * 4;
  const uint32_t n0 = r0 ? ((r0[e >> 1] >> sh) & 0xFu) ^ 8u : 8u;  // 8 encodes 0 after the offset
  const uint32_t n1 = r1 ? ((r1[e >> 1] >> sh) & 0xFu) ^ 8u : 8u;
  return h2_as_u32(__hsub2(u32_as_h2((n0 | (n1 << 16)) | 0x64006400u), __float2half2_rn(1032.f)));
}
// fp32 pair -> fp16 (hi, lo) pairs with hi + lo = the value to about 22 bits
__device__ __forceinline__ void split_h2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const float2 hf = __half22float2(h);
  hi = h2_as_u32(h);
  lo = h2_as_u32(__floats2half2_rn(x0 - hf.x, x1 - hf.y));
}

// One attention item (sequence b, kv head, split) on a group of 4 warps, on
// the tensor cores: S = q K^T with q as fp16 hi + lo (K codes are exact in
// fp16; the per-token scales apply to the fp32 result), then O += P V with the
// per-token V scale folded into P (normalized by the chunk's largest scale)
// and P as hi + lo.  Warp w owns output dims [w HD / 4, (w + 1) HD / 4).
// gt = thread index in the group, gwarp = warp index in the group.
template <int HD>
__device__ AXB_STEP_FN bool attn_item(const StepArgs& a, const StepLayer* ly, int layer, const AttnItem& it,
                                      int nsplit, bool prefetched, char* gsm, uint64_t* bar, uint32_t& uses, int bar_id,
                                      int gt, int* done_ctr, bool ok) {
  constexpr int DPL = HD / 32, KS = HD / 16, NB = HD / 32;  // NB: n8 output blocks per warp
  const int lane = gt & 31, gwarp = gt >> 5, g = lane >> 2, c = lane & 3;
  const int cap = a.attn_cap;
  const AttnLayout Lo = attn_layout(a.kv_type, HD, a.kv_group, cap);
  const int rb = Lo.rb, ng = Lo.ng, G = a.kv_type == AXB_KV_F16 ? HD : a.kv_group;
  const bool quant = a.kv_type != AXB_KV_F16;
  const int n_rep = a.Hq / a.Hkv, hq0 = it.kvh * n_rep;
  const int rpos = a.params[0], wpos = a.params[1];
  const size_t head_base = ((size_t)it.b * a.Hkv + it.kvh) * a.S;
  char* kst = gsm + Lo.kv;
  char* vst = kst + (size_t)cap * rb;
  __half* ksc_s = reinterpret_cast<__half*>(gsm + Lo.ksc);
  __half* vsc_s = reinterpret_cast<__half*>(gsm + Lo.vsc);
  __half* qh_s = reinterpret_cast<__half*>(gsm + Lo.qh);  // [hi / lo][8 rows][HD]
  float* p_s = reinterpret_cast<float*>(gsm + Lo.p);
  float* ml_s = reinterpret_cast<float*>(gsm + Lo.ml);  // m[8] l[8] alpha[8] flag
  float* coef = reinterpret_cast<float*>(gsm + Lo.coef);

  // ---- q with RoPE (fp32), as fp16 hi / lo rows; the new K/V row rotated, quantized and written
  const int qkv_dim = (a.Hq + 2 * a.Hkv) * HD;
  const __half* row = a.qkv + (size_t)it.b * qkv_dim;
  const float* fr = a.rope + (size_t)(rpos % a.rope_len) * HD;
  for (int i = gt; i < 8 * HD / 2; i += 128) {
    const int rr = i / (HD / 2), pr = i % (HD / 2);
    float q0 = 0.f, q1 = 0.f;
    if (rr < n_rep) {
      const __half2 x2 = __ldcg(reinterpret_cast<const __half2*>(row + (hq0 + rr) * HD) + pr);
      const float a0 = __low2float(x2), a1 = __high2float(x2);
      const float cs = fr[2 * pr], sn = fr[2 * pr + 1];
      q0 = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(a1, sn));
      q1 = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(a1, cs));
    }
    uint32_t hi, lo;
    split_h2(q0, q1, hi, lo);
    reinterpret_cast<uint32_t*>(qh_s)[(rr * HD) / 2 + pr] = hi;
    reinterpret_cast<uint32_t*>(qh_s)[(8 * HD + rr * HD) / 2 + pr] = lo;
  }
  if (gt < 8) {
    ml_s[gt] = -INFINITY;
    ml_s[8 + gt] = 0.f;
  }
  float nkv[DPL];
  const bool covers = wpos >= it.t0 && wpos < it.t1;
  if (covers && gwarp < 2) {
    const __half* src = row + (size_t)(a.Hq + (gwarp == 0 ? 0 : a.Hkv) + it.kvh) * HD;
#pragma unroll
    for (int e = 0; e < DPL; ++e) nkv[e] = __half2float(__ldcg(src + lane * DPL + e));
    if (gwarp == 0) {  // RoPE on K, every product rounded (transformer.py:1105-1127)
#pragma unroll
      for (int e = 0; e < DPL; e += 2) {
        const int pr = (lane * DPL + e) >> 1;
        const float cs = fr[2 * pr], sn = fr[2 * pr + 1], a0 = nkv[e], a1 = nkv[e + 1];
        nkv[e] = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(a1, sn));
        nkv[e + 1] = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(a1, cs));
      }
    }
    uint8_t* crow = (gwarp == 0 ? ly->kc : ly->vc) + (head_base + wpos) * rb;
    __half* srow = quant ? (gwarp == 0 ? ly->ks : ly->vs) + (head_base + wpos) * ng : nullptr;
    store_kv_row<DPL>(nkv, lane, a.kv_type, G, true, crow, srow);
  }
  group_bar(bar_id);

  const float sm_scale = 1.0f / sqrtf((float)HD);
  const int d0 = gwarp * (HD / 4);  // this warp's output dims (one V scale group: kv_group >= HD / 4)
  const int vgrp = quant ? d0 / G : 0;
  float oacc[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int q = 0; q < 4; ++q) oacc[nb][q] = 0.f;
  bool first = true;
  for (int c0 = it.t0; c0 < it.t1 && ok; c0 += cap) {
    const int nt = min(cap, it.t1 - c0);
    if (!(first && prefetched) && gt == 0) attn_copy(ly, head_base, rb, ng, quant, c0, nt, gsm, Lo, cap, bar);
    first = false;
    const bool got = mbar_wait(bar, uses & 1, kSMbarLimit);
    ++uses;
    if (group_bar_or(bar_id, !got)) {  // one decision for the whole group
      if (gt == 0) raise_abort(a);
      ok = false;
      break;
    }
    if (covers && gwarp < 2 && wpos >= c0 && wpos < c0 + nt) {
      // the copy may have read the slot (codes and scale) before this step wrote it
      uint8_t* rowp = reinterpret_cast<uint8_t*>(gwarp == 0 ? kst : vst) + (size_t)(wpos - c0) * rb;
      __half* sp = quant ? (gwarp == 0 ? ksc_s : vsc_s) + (size_t)(wpos - c0) * ng : nullptr;
      store_kv_row<DPL>(nkv, lane, a.kv_type, G, true, rowp, sp);
    }
    group_bar(bar_id);
    // ---- scores: warp w takes 8-token blocks w, w + 4, ...; the fp32 result
    // of each scale group is scaled by the token's K scale when the group ends
    const uint32_t* qh32 = reinterpret_cast<const uint32_t*>(qh_s);
    for (int blk = gwarp; blk * 8 < nt; blk += 4) {
      const int tok = min(blk * 8 + g, nt - 1);  // B-fragment column; columns past nt are discarded
      const uint8_t* krow = reinterpret_cast<const uint8_t*>(kst) + (size_t)tok * rb;
      const int t_a = blk * 8 + 2 * c, t_b = t_a + 1;  // this thread's C-fragment columns
      float sc0 = 0.f, sc1 = 0.f, gacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const uint32_t b0 = kv_pair_h2(krow, a.kv_type, 16 * s + 2 * c);
        const uint32_t b1 = kv_pair_h2(krow, a.kv_type, 16 * s + 2 * c + 8);
        const uint32_t ahi[4] = {qh32[(g * HD + 16 * s + 2 * c) / 2], 0u, qh32[(g * HD + 16 * s + 2 * c + 8) / 2], 0u};
        const uint32_t alo[4] = {qh32[(8 * HD + g * HD + 16 * s + 2 * c) / 2], 0u,
                                 qh32[(8 * HD + g * HD + 16 * s + 2 * c + 8) / 2], 0u};
        mma_16816(gacc, ahi, b0, b1, gacc);
        mma_16816(gacc, alo, b0, b1, gacc);
        if ((16 * (s + 1)) % G == 0) {  // a K scale group is complete
          const int grp = (16 * s) / G;
          const float s0 = quant && t_a < nt ? __half2float(ksc_s[t_a * ng + grp]) : 1.f;
          const float s1 = quant && t_b < nt ? __half2float(ksc_s[t_b * ng + grp]) : 1.f;
          sc0 = __fmaf_rn(gacc[0], s0, sc0);
          sc1 = __fmaf_rn(gacc[1], s1, sc1);
          gacc[0] = gacc[1] = gacc[2] = gacc[3] = 0.f;
        }
      }
      if (g < n_rep) {
        if (t_a < nt) p_s[g * cap + t_a] = sc0 * sm_scale;
        if (t_b < nt) p_s[g * cap + t_b] = sc1 * sm_scale;
      }
    }
    group_bar(bar_id);
    // ---- online softmax over the chunk: warp w handles heads w, w + 4
    for (int r = gwarp; r < n_rep; r += 4) {
      float mx = -INFINITY;
      for (int tk = lane; tk < nt; tk += 32) mx = fmaxf(mx, p_s[r * cap + tk]);
      mx = warp_max(mx);
      const float m_old = ml_s[r];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.f;
      for (int tk = lane; tk < nt; tk += 32) {
        const float e = __expf(p_s[r * cap + tk] - m_new);
        p_s[r * cap + tk] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      __syncwarp();
      if (lane == 0) {
        const float alpha = m_old == -INFINITY ? 0.f : __expf(m_old - m_new);
        ml_s[r] = m_new;
        ml_s[8 + r] = ml_s[8 + r] * alpha + sum;
        ml_s[16 + r] = alpha;
      }
    }
    group_bar(bar_id);
    // ---- O = alpha O + vmax * (P' V), P' = p * vscale / vmax (vmax: the
    // chunk's largest V scale of this warp's group, keeps P' in fp16 range)
    float vmax = 1.f;
    if (quant) {
      float m = 0.f;
      for (int tk = lane; tk < nt; tk += 32) m = fmaxf(m, __half2float(vsc_s[tk * ng + vgrp]));
      m = warp_max(m);
      vmax = m > 0.f ? m : 1.f;
    }
    const float inv_vmax = 1.f / vmax;
    const float alpha = g < n_rep ? ml_s[16 + g] : 0.f;
    float tacc[NB][4];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int q = 0; q < 4; ++q) tacc[nb][q] = 0.f;
    for (int t0 = 0; t0 < nt; t0 += 16) {
      float pv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int t = t0 + 2 * c + (q & 1) + 8 * (q >> 1);
        float v = 0.f;
        if (g < n_rep && t < nt) {
          v = p_s[g * cap + t];
          if (quant) v *= __half2float(vsc_s[t * ng + vgrp]) * inv_vmax;
        }
        pv[q] = v;
      }
      uint32_t h01, l01, h23, l23;
      split_h2(pv[0], pv[1], h01, l01);
      split_h2(pv[2], pv[3], h23, l23);
      const uint32_t ahi[4] = {h01, 0u, h23, 0u}, alo[4] = {l01, 0u, l23, 0u};
      const int ta = t0 + 2 * c, tb = ta + 8;
      const uint8_t* r0 = ta < nt ? reinterpret_cast<const uint8_t*>(vst) + (size_t)ta * rb : nullptr;
      const uint8_t* r1 = ta + 1 < nt ? reinterpret_cast<const uint8_t*>(vst) + (size_t)(ta + 1) * rb : nullptr;
      const uint8_t* r2 = tb < nt ? reinterpret_cast<const uint8_t*>(vst) + (size_t)tb * rb : nullptr;
      const uint8_t* r3 = tb + 1 < nt ? reinterpret_cast<const uint8_t*>(vst) + (size_t)(tb + 1) * rb : nullptr;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        const int d = d0 + nb * 8 + g;  // B-fragment column
        const uint32_t b0 = kv_col_pair_h2(r0, r1, a.kv_type, d);
        const uint32_t b1 = kv_col_pair_h2(r2, r3, a.kv_type, d);
        mma_16816(tacc[nb], ahi, b0, b1, tacc[nb]);
        mma_16816(tacc[nb], alo, b0, b1, tacc[nb]);
      }
    }
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      oacc[nb][0] = __fmaf_rn(vmax, tacc[nb][0], oacc[nb][0] * alpha);
      oacc[nb][1] = __fmaf_rn(vmax, tacc[nb][1], oacc[nb][1] * alpha);
    }
    group_bar(bar_id);  // staged rows and p_s are free for the next chunk
  }
  if (!ok) return false;
  // ---- this thread's outputs: head g, dims d0 + 8 nb + 2c + {0, 1}
  const size_t pidx = (size_t)it.b * a.Hq + hq0;
  if (g < n_rep) {
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      const int d = d0 + nb * 8 + 2 * c;
      if (nsplit == 1) {
        a.attn[(pidx + g) * HD + d] = __float2half_rn(__fdiv_rn(oacc[nb][0], ml_s[8 + g]));
        a.attn[(pidx + g) * HD + d + 1] = __float2half_rn(__fdiv_rn(oacc[nb][1], ml_s[8 + g]));
      } else {
        *reinterpret_cast<float2*>(a.part_o + ((pidx + g) * kStepMaxSplits + it.split) * HD + d) =
            make_float2(oacc[nb][0], oacc[nb][1]);
      }
    }
  }
  if (nsplit == 1) {
    group_bar(bar_id);
    if (gt == 0) red_release_add(done_ctr, 1);
    return true;
  }
  if (gt < n_rep) {
    a.part_ml[((pidx + gt) * kStepMaxSplits + it.split) * 2 + 0] = ml_s[gt];
    a.part_ml[((pidx + gt) * kStepMaxSplits + it.split) * 2 + 1] = ml_s[8 + gt];
  }
  group_bar(bar_id);
  // ---- combine, shared by all the head's split groups.  Every split of the
  // head runs at once (n_items <= attention groups in the grid), so each group
  // waits for all of them and then combines its own slice of the head's
  // n_rep * HD outputs.  The per-head counter only grows during a step (layer l
  // completes at (l + 1) * nsplit arrivals); the step's last CTA clears it.
  int* cnt = a.attn_cnt + it.b * a.Hkv + it.kvh;
  int* flag = reinterpret_cast<int*>(ml_s + 24);
  if (gt == 0) {
    red_release_add(cnt, 1);
    *flag = wait_ge(cnt, (layer + 1) * nsplit, a) ? 1 : 0;
  }
  group_bar(bar_id);
  if (!*flag) return false;
  const int nout = n_rep * HD;
  const int i0 = it.split * nout / nsplit, i1 = (it.split + 1) * nout / nsplit;
  const int r_lo = i0 / HD, r_hi = (i1 - 1) / HD;  // heads touched by the slice
  // per-head split weights: each lane loads the (m, l) of splits lane and lane + 32
  static_assert(kStepMaxSplits <= 64, "two splits per lane");
  for (int r = r_lo + gwarp; r <= r_hi; r += 4) {
    const size_t hb = (pidx + r) * kStepMaxSplits;
    float2 ml[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int sp = lane + 32 * q;
      ml[q] = sp < nsplit ? __ldcg(reinterpret_cast<const float2*>(a.part_ml) + hb + sp) : make_float2(-INFINITY, 0.f);
    }
    const float Mx = warp_max(fmaxf(ml[0].x, ml[1].x));
    float Ls = 0.f;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int sp = lane + 32 * q;
      if (sp < nsplit) {
        const float cw = (ml[q].x == -INFINITY) ? 0.f : __expf(ml[q].x - Mx);
        coef[(r - r_lo) * kStepMaxSplits + sp] = cw;
        Ls += ml[q].y * cw;
      }
    }
    Ls = warp_sum(Ls);
    if (lane == 0) ml_s[8 + (r - r_lo)] = Ls;
  }
  group_bar(bar_id);
  // 8 lanes per output (splits j, j + 8, ...), 16 outputs per pass; the
  // lanes' partial sums meet in a fixed shuffle order
  const int j8 = gt & 7, npass = (i1 - i0 + 15) / 16;  // the same trip count in every lane
  for (int pass = 0; pass < npass; ++pass) {
    const int i = i0 + 16 * pass + (gt >> 3);
    const bool act = i < i1;
    const int ii = act ? i : i0;
    const int r = ii / HD, e = ii % HD;
    const size_t hb = (pidx + r) * kStepMaxSplits;
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int sp = j8 + 8 * u;
      v[u] = (act && sp < nsplit) ? __ldcg(a.part_o + (hb + sp) * HD + e) : 0.f;
    }
    float O = 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int sp = j8 + 8 * u;
      if (act && sp < nsplit) O = __fmaf_rn(v[u], coef[(r - r_lo) * kStepMaxSplits + sp], O);
    }
    O += __shfl_xor_sync(0xffffffffu, O, 1);
    O += __shfl_xor_sync(0xffffffffu, O, 2);
    O += __shfl_xor_sync(0xffffffffu, O, 4);
    if (act && j8 == 0) a.attn[(pidx + r) * HD + e] = __float2half_rn(__fdiv_rn(O, ml_s[8 + (r - r_lo)]));
  }
  group_bar(bar_id);
  if (gt == 0) red_release_add(done_ctr, 1);
  return true;
}

// ------------------------------------------------------------------ kernel
template <bool SYM, int GB, int HD>
__global__ void __launch_bounds__(kSThreads, 1) step_kernel(const StepArgs a) {
  extern __shared__ __align__(128) char smem[];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int C = gridDim.x, Wt = C * kSW, gw = wid * C + blockIdx.x;  // virtual warp id
  char* uni = smem + kSW * kSRing;
  float* red = reinterpret_cast<float*>(uni + kSUnion);  // [kSW][kStepMaxM]
  uint64_t* abar = reinterpret_cast<uint64_t*>(uni + kSUnion + 512);  // one per attention group
  int* s_last = reinterpret_cast<int*>(uni + kSUnion + 512 + 64);

  // staged activations: M rows of K + 8 halves from the union's start, their
  // per-(group, token) sums at its end
  __half* xs = reinterpret_cast<__half*>(uni);
  auto xsum_of = [&](int K) { return reinterpret_cast<float*>(uni + kSUnion - xsum_bytes(K, a.group)); };
  const int xs_stride = a.d + 8;

  Ring ring;
  ring.buf = smem + wid * kSRing;
  ring.bars = reinterpret_cast<uint64_t*>(ring.buf + kSStages * (kSStageW + kSStageS));
  ring.cs = 0;
  ring.cpar = 0;
  ring.ps = 0;
  ring.inflight = 0;
  Cur pc;
  if (lane == 0) {
    for (int s = 0; s < kSStages; ++s) mbar_init(ring.bars + s, 1);
    if (wid < kSGroups) mbar_init(abar + wid, 1);
    fence_mbar_init();
    pc.ph = 0;
    cur_load<GB>(pc, a, gw, Wt);
    for (int s = 0; s < kSStages; ++s) ring_issue<SYM, GB>(ring, pc, a, gw, Wt, lane);
  }
  __syncthreads();

  bool ok = true;
  const int qkv_dim = (a.Hq + 2 * a.Hkv) * a.hd;
  const int t_d = tiles_of(a.d);
  const int grp = wid >> 2, gt = tid & 127;
  uint32_t abar_uses = 0;

  trace_mark(a, 0);
  // embedding rows for the first layer's QKV (every CTA stages its own copy)
  stage_embed(a, xs, xs_stride);
  __syncthreads();
  if (blockIdx.x == 0 && tid == 0) red_release_add(a.done, 1);

  // GEMV phases in order: p = 4 l + {0 QKV, 1 o, 2 gate_up, 3 down}, 4 L = lm_head;
  // attention runs between a layer's QKV and o phases.  One loop, so every
  // GEMV variant is emitted once.
  for (int ph = 0; ph <= 4 * a.L; ++ph) {
    const int l = ph >> 2, kind = ph < 4 * a.L ? (ph & 3) : 4;
    const StepLayer* ly = a.layers + (kind == 4 ? 0 : l);
    int* dn = a.done + 1 + 5 * l;  // QKV, attention, o, gate_up, down counters of layer l
    const int ts = 1 + 10 * l;
    // ---- wait for the phase's input; its source, width and RMSNorm weight
    const __half* src;
    const float* nw = nullptr;
    int K, *done_ctr;
    if (kind == 0) {  // QKV: RMSNorm(h) (the embedding rows already in xs for layer 0)
      if (l > 0) ok = cta_wait(dn - 1, t_d, a, ok);
      trace_mark(a, ts + 0);
      src = l > 0 ? a.h : nullptr;
      K = a.d;
      nw = ly->ln1;
      done_ctr = dn;
    } else if (kind == 1) {  // o: attention output (+ residual)
      {
        int nsplit, chunk;
        attn_split_plan(a.params[2], (kSGroups * C) / (a.B * a.Hkv), a.attn_cap, nsplit, chunk);
        ok = cta_wait(dn + 1, a.B * a.Hkv * nsplit, a, ok);  // every attention item (and its combine slice)
      }
      if (l == 0) ok = cta_wait(a.done, 1, a, ok);  // h holds the embedding rows
      trace_mark(a, ts + 4);
      src = a.attn;
      K = a.Hq * a.hd;
      done_ctr = dn + 2;
    } else if (kind == 2) {  // gate_up: RMSNorm(h), SwiGLU epilogue
      ok = cta_wait(dn + 2, t_d, a, ok);
      trace_mark(a, ts + 6);
      src = a.h;
      K = a.d;
      nw = ly->ln2;
      done_ctr = dn + 3;
    } else if (kind == 3) {  // down: SwiGLU output (+ residual)
      ok = cta_wait(dn + 3, tiles_of(2 * a.F), a, ok);
      trace_mark(a, ts + 8);
      src = a.sw;
      K = a.F;
      done_ctr = dn + 4;
    } else {  // lm_head: final RMSNorm(h); with no layers h holds CTA 0's embedding rows
      ok = a.L > 0 ? cta_wait(a.done + 5 * a.L, t_d, a, ok) : cta_wait(a.done, 1, a, ok);
      trace_mark(a, 1 + 10 * a.L);
      src = a.h;
      K = a.d;
      nw = a.ln_f;
      done_ctr = a.done + 1 + 5 * a.L;
    }
    // ---- the GEMV: activations staged in shared memory when they fit (always
    // for the normalized inputs), else read from L2 one k-block ahead
    const bool staged = xs_fits(a.B, K, a.group);
    if (!staged && (nw != nullptr || src == nullptr)) {
      // normalized inputs (and layer 0's embedding rows) exist only as staged
      // rows; the host guarantees they fit (xs_fits for d_model), so this is a
      // contract violation: report it rather than read an absent source
      if (tid == 0) atomicExch(a.err, AXB_EINVAL);
      ok = false;
    }
    if (staged) {
      if (ok) stage_x(a.B, a.group, a.eps, src, K, nw, xs, K + 8, xsum_of(K), SYM, red);
      ok = gemv_phase<SYM, GB, true>(a, ph, ring, pc, xs, K + 8, xsum_of(K), nullptr, 0, gw, Wt, lane, ok,
                                     done_ctr);
    } else {
      ok = gemv_phase<SYM, GB, false>(a, ph, ring, pc, nullptr, 0, nullptr, src, K, gw, Wt, lane, ok, done_ctr);
    }
    if (lane == 0) trace_at(a, 4 + 10 * a.L + ph * kStepTraceW + wid);  // this warp's share done
    trace_mark(a, kind == 4 ? 2 + 10 * a.L : ts + (kind == 0 ? 1 : 2 * kind + 3));  // QKV, o, gate_up, down done
    if (kind != 0) continue;
    // ---- attention of layer l (RoPE + KV write fused)
    ok = __syncthreads_and(ok) != 0;  // the staged rows are dead: the union holds attention next
    {
      const int active = a.params[2];
      int nsplit, chunk;
      attn_split_plan(active, (kSGroups * C) / (a.B * a.Hkv), a.attn_cap, nsplit, chunk);
      const int n_items = a.B * a.Hkv * nsplit;
      char* gsm = uni + (grp < kSGroups ? grp : 0) * (kSUnion / kSGroups);
      const AttnLayout Lo = attn_layout(a.kv_type, HD, a.kv_group, a.attn_cap);
      // warps beyond the attention groups take no items
      int item = grp < kSGroups ? blockIdx.x * kSGroups + grp : n_items;
      if (ok && item < n_items && gt == 0) {  // cached rows do not depend on this step's QKV
        const AttnItem it = attn_item_of(item, nsplit, chunk, a.Hkv, active);
        const size_t hb = ((size_t)it.b * a.Hkv + it.kvh) * a.S;
        attn_copy(ly, hb, Lo.rb, Lo.ng, a.kv_type != AXB_KV_F16, it.t0, min(a.attn_cap, it.t1 - it.t0), gsm, Lo,
                  a.attn_cap, abar + grp);
      }
      const bool pre_ok = ok;
      ok = cta_wait(dn + 0, tiles_of(qkv_dim), a, ok);
      trace_mark(a, ts + 2);
      bool first = true;
      for (; item < n_items; item += kSGroups * C) {
        if (!ok) {
          // a copy issued above is still owed to this group's mbarrier
          if (first && pre_ok) mbar_wait(abar + grp, abar_uses & 1, kSMbarLimit);
          break;
        }
        const AttnItem it = attn_item_of(item, nsplit, chunk, a.Hkv, active);
        ok = attn_item<HD>(a, ly, l, it, nsplit, first, gsm, abar + grp, abar_uses, 1 + grp, gt, dn + 1, ok);
        first = false;
      }
      if (gt == 0 && grp < kSGroups) trace_at(a, 4 + 10 * a.L + (4 * a.L + 1) * kStepTraceW + 2 * l + grp);
    }
    trace_mark(a, ts + 3);
  }

  // ---- wind down: copies still in flight (only after an abort) get a bounded wait
  if (lane == 0)
    for (int i = 0; i < ring.inflight; ++i) {
      mbar_wait(ring.bars + ring.cs, (uint32_t)ring.cpar, kSMbarLimit);
      if (++ring.cs == kSStages) {
        ring.cs = 0;
        ring.cpar ^= 1;
      }
    }
  __syncthreads();
  trace_mark(a, 3 + 10 * a.L);
  if (tid == 0) *s_last = (atom_acq_rel_add(a.exit_cnt, 1) == C - 1) ? 1 : 0;
  __syncthreads();
  if (!*s_last) return;
  // last CTA: publish the argmax, return every counter to zero
  if (tid < a.B) {
    const unsigned long long k = __ldcg(a.keys + tid);
    a.amax[tid] = k ? (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)) : 0;
    a.keys[tid] = 0ull;
  }
  for (int i = tid; i < 2 + 5 * a.L; i += blockDim.x) a.done[i] = 0;
  for (int i = tid; i < a.B * a.Hkv; i += blockDim.x) a.attn_cnt[i] = 0;  // grow through the step
  if (*reinterpret_cast<volatile int*>(a.exit_cnt + 1) != 0) {  // an aborted step may leave arrivals behind
    for (int i = tid; i < a.max_tiles; i += blockDim.x) a.tile_cnt[i] = 0;
  }
  __syncthreads();
  if (tid == 0) {
    a.exit_cnt[1] = 0;
    a.exit_cnt[0] = 0;
  }
}

// ------------------------------------------------------------------ host
int step_num_warps() { return kSW; }

int step_attn_cap(int kv_type, int hd, int kv_group) {
  for (int cap = 256; cap >= 16; cap -= 16) {
    const AttnLayout L = attn_layout(kv_type, hd, kv_group, cap);
    if (L.bytes <= kSUnion / kSGroups) return cap;
  }
  return 0;
}

bool step_supported(int wfmt, int group, int lm_fmt, int lm_group, int hd, int n_head, int n_kv_head, int d_model,
                    int kv_type, int kv_group, int max_seq) {
  if (wfmt != lm_fmt || group != lm_group) return false;
  if (wfmt != AXB_W_Q4T_SYM && wfmt != AXB_W_Q4T_AFFINE) return false;
  if (group != 64 && group != 128) return false;
  if (hd != 64 && hd != 128) return false;
  if (n_kv_head <= 0 || n_head % n_kv_head != 0 || n_head / n_kv_head > kMaxRepS) return false;
  if (d_model % 128 != 0) return false;
  if (!xs_fits(kStepMaxM, d_model, group)) return false;
  // a K scale group spans whole 16-wide MMA steps, a V scale group a warp's output dims
  if (kv_type != AXB_KV_F16 && (kv_group < 16 || kv_group < hd / 4 || hd % kv_group != 0)) return false;
  if (max_seq % 8) return false;  // scales are bulk-copied in 8-token (16-byte) runs
  return step_attn_cap(kv_type, hd, kv_group) > 0;
}

#define AXB_STEP_KERNELS(X) \
  X(true, 2, 128) X(true, 1, 128) X(false, 2, 128) X(false, 1, 128) X(true, 2, 64) X(true, 1, 64) X(false, 2, 64) X(false, 1, 64)

int step_prepare() {
  int dev = 0;
  cudaGetDevice(&dev);
  static int done_dev = -1;
  if (done_dev == dev) return AXB_OK;
#define AXB_SET(SYM, GB, HD)                                                                                 \
  {                                                                                                         \
    cudaError_t e = cudaFuncSetAttribute(step_kernel<SYM, GB, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                         (int)kSSmem);                                                      \
    if (e != cudaSuccess) return cuda_status(e, "step kernel attribute");                                   \
  }
  AXB_STEP_KERNELS(AXB_SET)
#undef AXB_SET
  done_dev = dev;
  return AXB_OK;
}

int step_launch(const StepArgs& a, cudaStream_t s) {
  AXB_CHECK_ARG(a.B >= 1 && a.B <= kStepMaxM, "step: batch %d out of range", a.B);
  // the shapes the kernel's fixed shared-memory layout is sized for
  AXB_CHECK_ARG(a.group == 64 || a.group == 128, "step: group %d", a.group);
  AXB_CHECK_ARG(a.d > 0 && a.d % 128 == 0 && a.F % 64 == 0 && a.V > 0, "step: bad dims (%d, %d, %d)", a.d, a.F, a.V);
  AXB_CHECK_ARG((a.hd == 64 || a.hd == 128) && a.Hkv > 0 && a.Hq % a.Hkv == 0 && a.Hq / a.Hkv <= kMaxRepS,
                "step: bad heads (%d, %d, %d)", a.Hq, a.Hkv, a.hd);
  AXB_CHECK_ARG(xs_fits(kStepMaxM, a.d, a.group), "step: d_model %d too large for the staged activations", a.d);
  AXB_CHECK_ARG(a.attn_cap >= 16 && attn_layout(a.kv_type, a.hd, a.kv_group, a.attn_cap).bytes <= kSUnion / kSGroups,
                "step: attention chunk %d does not fit", a.attn_cap);
  AXB_CHECK_ARG(a.lm_w && a.lm_s && a.ln_f && a.emb_w && a.emb_s && a.rope && a.tokens && a.params && a.err && a.h &&
                    a.logits && a.amax && a.done && a.tile_cnt && a.partials && a.keys && a.exit_cnt &&
                    (a.L == 0 || (a.layers && a.qkv && a.attn && a.sw && a.part_o && a.part_ml && a.attn_cnt)),
                "step: null pointer in the step arguments");
  AXB_CHECK_ARG((reinterpret_cast<uintptr_t>(a.lm_w) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.lm_s) & 15) == 0,
                "step: lm_head words and scales must be 16-byte aligned");
  if (int rc = step_prepare()) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms());
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = kSSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the phases wait on one another
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaErrorInvalidValue;
  const int GB = a.group / 64;
#define AXB_LAUNCH(SYM, GBv, HD) \
  if (a.sym == (SYM ? 1 : 0) && GB == GBv && a.hd == HD) e = cudaLaunchKernelEx(&cfg, step_kernel<SYM, GBv, HD>, a); else
  AXB_STEP_KERNELS(AXB_LAUNCH) { set_error("step: unsupported format"); return AXB_EINVAL; }
#undef AXB_LAUNCH
  return cuda_status(e, "step kernel launch");
}

}  // namespace axb
