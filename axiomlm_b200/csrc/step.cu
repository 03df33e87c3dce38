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
//    rule: virtual warp i of the grid owns units [i*U/W, (i+1)*U/W).  A warp's
//    weight stream for the whole step is therefore known at launch.  Lane 0
//    streams it through a private ring of bulk copies (TMA, non-tensor form)
//    that runs ahead across phase boundaries -- weights never depend on
//    activations -- so HBM keeps streaming while the warp waits for the
//    previous phase's activations.
//  * 16 warps per SM, each under 128 registers.  The code of every phase is
//    kept small (a one-group-per-iteration k loop read straight from the ring,
//    no unrolled stage copies): the whole step's hot code has to stay in the
//    SM's instruction cache, because each phase runs once per layer and a cold
//    fetch of straight-line code costs microseconds.
//  * Phases hand off through flagged activation words instead of kernel
//    boundaries or counters: each 8-byte word holds two fp16 values and the
//    flag of the phase that wrote it (one vector store), and a reader reloads
//    the words it needs until they carry that flag.  Every wait is bounded
//    (limits in StepArgs); one that runs out records AXB_ETIMEOUT and the grid
//    winds down, waiting for its own copies first.
//  * A tile split between the warps of a CTA is summed in shared memory, in
//    warp order, after one CTA barrier; a tile that continues into later CTAs
//    is finished by the CTA that owns its first unit, which adds their pieces
//    in CTA order (deterministic results).  Those pieces carry their own flags
//    (value, flag pairs), so no fence or counter sits between a piece and its
//    reader.
//  * Attention: one (sequence, kv head, split) item per CTA, on all 16 warps.
//    The item's cached rows are bulk-copied before the QKV phase has finished;
//    RoPE and the new K/V row's quantized write are fused.  The last split of a
//    head to finish combines the head (no CTA waits for another's split).
#include <algorithm>

#include "kv.cuh"
#include "q4t.cuh"
#include "step.cuh"

namespace axb {

constexpr int kSW = 16;  // warps per CTA (one CTA per SM)
constexpr int kSThreads = kSW * 32;
// A ring slot holds plan.slot_kb k-blocks (512 B of weights each) and their
// scales (at most 64 B per k-block: affine, one group per k-block).
constexpr int kSlotPerKb = 512 + 64;
constexpr int kMaxSlots = 8;                  // ring slots per warp (upper bound; the plan picks 2-3)
constexpr int kSBars = kSW * kMaxSlots * 8;   // ring mbarriers
constexpr int kSMisc = 4096;                  // reduction scratch, attention mbarrier, flags, producer cursors
constexpr int kSmemMax = 227 * 1024;
constexpr int kMaxRepS = 8;                   // q heads per kv head (the 8 rows of the score MMA)
constexpr uint32_t kDrainLimit = 1u << 22;    // polls for copies already in flight (not a runtime limit)
constexpr int kSPartBytes = kSW * 2 * 32 * 16;  // split-tile pieces: two per warp, 32 lanes x 4 floats
// misc-region offsets
constexpr int kMiscRed = 0;      // float [kSW][kStepMaxM]
constexpr int kMiscBar = 512;    // uint64 attention mbarrier
constexpr int kMiscFlag = 576;   // int flags
constexpr int kMiscCur = 3072;   // per-warp producer cursors (lane 0), kept out of registers
static_assert(kSW * kStepMaxM * 4 <= kMiscBar, "reduction scratch");
static_assert((4 * kSlotPerKb) % 128 == 0, "bulk-copy alignment of every slot size (a multiple of 4 k-blocks)");
static_assert(kSW <= kStepTraceW, "trace slots per phase");

__host__ __device__ constexpr int round_up_i(int v, int m) { return (v + m - 1) / m * m; }
// staged activations: M rows of K + 8 halves from the union's start
__host__ __device__ constexpr int stage_bytes(int M, int K) { return round_up_i(M * (K + 8) * 2, 128); }

// D = A * B with a zero accumulator (the first MMA of a chain)
__device__ __forceinline__ void mma_16816_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// ------------------------------------------------------------------ helpers
// The attention split count and the CTA exit count: one thread's acq_rel
// atomic after its CTA's barrier (the CTA's writes before it are released).
__device__ __forceinline__ int atom_acq_rel_add(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ int tiles_of(int n) { return (n + 15) >> 4; }

// Split-tile partials travel with their flag: each 16-byte word holds two
// (value, flag) pairs, written by one vector store and read by one vector
// load, and a reader takes a word once both flags carry the current phase's
// value (a per-launch epoch and the phase).  The data is its own signal: no
// fence, counter or atomic on the way.
__device__ __forceinline__ void st_ll(uint4* p, float v0, float v1, uint32_t fl) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(__float_as_uint(v0)), "r"(fl),
               "r"(__float_as_uint(v1)), "r"(fl)
               : "memory");
}
__device__ __forceinline__ uint4 ld_ll(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Activations move the same way: word i of a row holds halves 2i, 2i + 1
// and the flag of the phase that wrote them, in one 8-byte store, so a phase
// starts when the words it reads carry the flag it expects; no counter,
// release or acquire sits between a producer's store and its reader.  The
// flag of phase p (-1: the embedding rows) of launch e is e * 512 + p + 2,
// never 0, the value of a word nobody wrote.
__device__ __forceinline__ uint32_t act_flag(uint32_t epoch, int p) { return epoch * 512u + (uint32_t)(p + 2); }
__device__ __forceinline__ void st_act(uint2* p, uint32_t h2, uint32_t fl) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(h2), "r"(fl) : "memory");
}
__device__ __forceinline__ uint2 ld_act(const uint2* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

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

__device__ __forceinline__ void raise_abort(const StepArgs& a) {
  atomicExch(a.exit_cnt + 1, 1);
  atomicExch(a.err, AXB_ETIMEOUT);
}

// The halves of a flagged activation word once it carries flag fl.  The wait
// is bounded: it gives up after a.spin_limit polls (raising the abort) or as
// soon as another CTA has raised it; the step's outputs are then not valid.
__device__ __forceinline__ bool act_giveup(uint32_t it, const StepArgs& a) {
  if (it >= a.spin_limit) {
    raise_abort(a);
    return true;
  }
  return (it & 15) == 0 && *reinterpret_cast<const volatile int*>(a.exit_cnt + 1) != 0;
}
__device__ __forceinline__ uint32_t act_get(const uint2* p, uint32_t fl, const StepArgs& a) {
  uint2 v = ld_act(p);
  for (uint32_t it = 1; v.y != fl && !act_giveup(it, a); ++it) {
    __nanosleep(32);
    v = ld_act(p);
  }
  return v.x;
}
// Loads are issued first (all in flight) and only then waited on: v holds
// what the first load saw; these reload until the flag(s) match.
__device__ __forceinline__ void act_wait1(const uint2* p, uint2& v, uint32_t fl, const StepArgs& a) {
  for (uint32_t it = 1; v.y != fl && !act_giveup(it, a); ++it) {
    __nanosleep(32);
    v = ld_act(p);
  }
}
// two consecutive flagged words in one 16-byte load: halves 4i .. 4i + 3
__device__ __forceinline__ void act_wait2(const uint2* p, uint4& v, uint32_t fl, const StepArgs& a) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
  for (uint32_t it = 1; (v.y != fl || v.w != fl) && !act_giveup(it, a); ++it) {
    __nanosleep(32);
    v = ld_ll(q);
  }
}

// ------------------------------------------------------------------ GEMV phases
// phase p: 4*l + {0 QKV, 1 o, 2 gate_up, 3 down}; 4*L = lm_head
struct GPh {
  const char* W;
  const char* S;
  int N, K, upt, kind, layer;
  uint32_t U;  // units (tile, group); U * warps < 2^32 for every supported shape (host-checked)
};

// Units of a GEMV phase: CTA c owns the contiguous run [c U / C, (c + 1) U / C),
// and inside it warp w of its min(16, units) participating warps an equal
// contiguous share.  A tile is therefore split between warps of one CTA
// (reduced through shared memory) and between at most a few CTAs (one
// partial per CTA through global memory).  The producer cursor uses the same
// ranges.
struct URange {
  uint32_t u0, u1;
};
__device__ __forceinline__ uint32_t cta_u0(uint32_t U, int c, int C) {
  return (uint32_t)(((unsigned long long)U * (unsigned)c) / (unsigned)C);
}
__device__ __forceinline__ uint32_t cta_warps(uint32_t n) { return n < (uint32_t)kSW ? n : (uint32_t)kSW; }
__device__ __forceinline__ URange warp_range(uint32_t U, int c, int C, int w) {
  const uint32_t c0 = cta_u0(U, c, C), n = cta_u0(U, c + 1, C) - c0, we = cta_warps(n);
  if ((uint32_t)w >= we) return {0u, 0u};
  return {c0 + (uint32_t)(((unsigned long long)n * (unsigned)w) / we),
          c0 + (uint32_t)(((unsigned long long)n * (unsigned)(w + 1)) / we)};
}
// the owner of unit u among n units split as above (warps of a CTA from c0, or CTAs from 0)
__device__ __forceinline__ int owner_of(uint32_t u, uint32_t c0, uint32_t n, uint32_t parts) {
  return (int)(((unsigned long long)(u - c0 + 1) * parts - 1) / n);
}

__device__ __forceinline__ GPh gph(const StepArgs& a, int ph) {
  GPh g;
  if (ph >= 4 * a.L) {
    g.W = a.lm_w;
    g.S = a.lm_s;
    g.N = a.V;
    g.K = a.d;
    g.kind = 4;
    g.layer = a.L;
  } else {
    const StepLayer* ly = a.layers + (ph >> 2);
    const int k = ph & 3;
    g.W = ly->w[k];
    g.S = ly->s[k];
    g.kind = k;
    g.layer = ph >> 2;
    switch (k) {
      case 0: g.N = (a.Hq + 2 * a.Hkv) * a.hd; g.K = a.d; break;
      case 1: g.N = a.d; g.K = a.Hq * a.hd; break;
      case 2: g.N = 2 * a.F; g.K = a.d; break;
      default: g.N = a.d; g.K = a.F; break;
    }
  }
  g.upt = g.K / a.group;
  g.U = (uint32_t)tiles_of(g.N) * (uint32_t)g.upt;
  return g;
}

// Producer cursor over a warp's weight stream (lane 0 only).
struct Cur {
  int ph, t, t_last, kb, kb_end, upt;
  uint32_t u0, u1;
  const char* W;
  const char* S;
};

static_assert(kMiscCur + kSW * sizeof(Cur) <= kSMisc, "producer cursors");

template <int GB>
__device__ __forceinline__ void cur_tile(Cur& c) {
  c.kb = (int)max(c.u0, (uint32_t)(c.t * c.upt)) * GB;
  c.kb_end = (int)min(c.u1, (uint32_t)((c.t + 1) * c.upt)) * GB;
}

template <int GB>
__device__ __forceinline__ void cur_load(Cur& c, const StepArgs& a, int wid) {
  const GPh g = gph(a, c.ph);
  c.W = g.W;
  c.S = g.S;
  c.upt = g.upt;
  const URange r = warp_range(g.U, blockIdx.x, gridDim.x, wid);
  c.u0 = r.u0;
  c.u1 = r.u1;
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
__device__ __forceinline__ bool cur_fix(Cur& c, const StepArgs& a, int wid) {
  while (c.kb >= c.kb_end) {
    if (c.t < c.t_last) {
      ++c.t;
      cur_tile<GB>(c);
      continue;
    }
    if (c.ph >= 4 * a.L) return false;
    ++c.ph;
    cur_load<GB>(c, a, wid);
  }
  return true;
}

// Per-warp ring of n slots.  Slot indices and mbarrier parities are advanced
// incrementally.  A slot is re-armed by the same warp after its last read
// (the warp's generic loads of the slot have returned by then), so no proxy
// fence is needed.  A slot never spans two tiles: the consumer derives each
// slot's k-block count from its own loop, in the producer's order.
struct Ring {
  char* buf;
  uint64_t* bars;
  int n;            // slots
  int cs, cpar;     // consumer: next slot and the parity its mbarrier completes with
  int ps;           // producer (lane 0): next slot to fill
  int inflight;     // producer (lane 0): slots issued and not yet consumed
};

__device__ __forceinline__ void ring_consumed(Ring& r) {
  if (++r.cs == r.n) {
    r.cs = 0;
    r.cpar ^= 1;
  }
  --r.inflight;
}

template <bool SYM, int GB>
__device__ __forceinline__ void ring_issue(Ring& r, Cur& pc, const StepArgs& a, int wid, int lane) {
  if (lane != 0) return;
  constexpr int UB = SYM ? 32 : 64;  // scale bytes per group
  if (pc.kb >= pc.kb_end && !cur_fix<GB>(pc, a, wid)) return;
  const int st = r.ps;
  r.ps = st + 1 == r.n ? 0 : st + 1;
  const int sl = a.plan.slot_kb;
  const int nk = min(sl, pc.kb_end - pc.kb);
  const uint32_t bw = nk * 512, bs = (nk / GB) * UB;
  char* slot = r.buf + (size_t)st * sl * kSlotPerKb;
  const uint64_t pol = l2_evict_first_policy();
  mbar_expect_tx(r.bars + st, bw + bs);
  bulk_g2s_hint(slot, pc.W + (size_t)pc.kb * 512, bw, r.bars + st, pol);
  bulk_g2s_hint(slot + sl * 512, pc.S + (size_t)(pc.kb / GB) * UB, bs, r.bars + st, pol);
  // keep the stream further ahead in flight through L2: the k-blocks a.pref_kb
  // past this slot, while they stay in this warp's range of the phase (the
  // range is one contiguous run of tiles)
  if (a.pref_kb > 0) {
    const int kp = pc.kb + a.pref_kb, kend = (int)pc.u1 * GB;
    if (kp < kend) {
      const int np = min(sl, kend - kp);
      bulk_prefetch_l2(pc.W + (size_t)kp * 512, np * 512);
      if (np >= GB) bulk_prefetch_l2(pc.S + (size_t)(kp / GB) * UB, (np / GB) * UB);
    }
  }
  pc.kb += nk;
  ++r.inflight;
}

// Tile epilogue: token n = 2*t4 + e, rows tile*16 + g (+8).  The kind is
// dispatched once, and the small loops stay rolled (the epilogue runs once
// per tile; its code has to stay small, not fast).
__device__ __forceinline__ void step_epilogue(const StepArgs& a, const GPh& g, int tile, float v00, float v01,
                                           float v10, float v11, const uint2& hres, int lane, uint32_t efl) {
  const int gg = lane >> 2, t4 = lane & 3;
  const int r0 = tile * 16 + gg;
  const int M = a.B;
  const float acc[4] = {v00, v01, v10, v11};
  // outputs go out as flagged words of two halves: rows r and r + 1 live in
  // lanes g and g + 1 (four lanes apart), so the even row's lane takes its
  // neighbour's half and stores the pair
  if (g.kind == 2) {  // SwiGLU: rows g (gate) and g + 8 (up) of the interleaved tile
    const int j = tile * 8 + gg;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int n = 2 * t4 + e;
      const float gv = __half2float(__float2half_rn(acc[e]));
      const float uv = __half2float(__float2half_rn(acc[2 + e]));
      const uint32_t sv = __half_as_ushort(swiglu_h(gv, uv));
      const uint32_t nb = __shfl_down_sync(0xffffffffu, sv, 4);
      if ((gg & 1) == 0 && n < M && j < a.F) st_act(a.sw + ((size_t)n * a.F + j) / 2, sv | (nb << 16), efl);
    }
    return;
  }
  if (g.kind == 4) {  // lm_head: logits + per-token argmax key
#pragma unroll 1
    for (int e = 0; e < 2; ++e) {
      const int n = 2 * t4 + e;
      unsigned long long best = 0ull;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        const int row = r0 + 8 * hh;
        if (n >= M || row >= g.N) continue;
        const __half vh = __float2half_rn(acc[2 * hh + e]);
        a.logits[(size_t)n * a.V + row] = vh;
        // argmax key: ordered value bits, then the lowest row wins ties
        uint32_t bits = __float_as_uint(__half2float(vh));
        if (bits == 0x80000000u) bits = 0u;  // -0 == +0: a tie, which the lower row wins
        bits = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
        const unsigned long long key = ((unsigned long long)bits << 32) | (0xFFFFFFFFu - (uint32_t)row);
        best = key > best ? key : best;
      }
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        const unsigned long long ok = __shfl_xor_sync(0xffffffffu, best, o);
        best = ok > best ? ok : best;
      }
      if (gg == 0 && n < M && best) atomicMax(a.keys + n, best);
    }
    return;
  }
  const __half2 hr01 = u32_as_h2(hres.x), hr23 = u32_as_h2(hres.y);
  const float hrv[4] = {__low2float(hr01), __high2float(hr01), __low2float(hr23), __high2float(hr23)};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int n = 2 * t4 + (q & 1), row = r0 + 8 * (q >> 1);
    __half nv;
    if (g.kind == 0) {
      nv = __float2half_rn(acc[q]);
    } else {  // residual add into h (fp16 GEMV output, fp16 sum); h was read at the tile's start
      nv = __float2half_rn(__fadd_rn(hrv[q], __half2float(__float2half_rn(acc[q]))));
      if (g.kind == 3 && a.hdump && n < M && row < g.N) a.hdump[((size_t)g.layer * M + n) * a.d + row] = nv;
    }
    const uint32_t sv = __half_as_ushort(nv);
    const uint32_t nb = __shfl_down_sync(0xffffffffu, sv, 4);
    if ((gg & 1) == 0 && n < M && row < g.N) {
      uint2* dst = g.kind == 0 ? a.qkv + ((size_t)n * g.N + row) / 2 : a.h + ((size_t)n * a.d + row) / 2;
      st_act(dst, sv | (nb << 16), efl);
    }
  }
}

// The residual values a tile's epilogue adds to (o and down phases): read at
// the tile's start so the load's latency hides under the tile's k loop.
__device__ __forceinline__ uint2 residual_of(const StepArgs& a, const GPh& g, int tile, int lane, uint32_t rfl) {
  if (g.kind != 1 && g.kind != 3) return make_uint2(0u, 0u);
  const int gg = lane >> 2, t4 = lane & 3, r0 = tile * 16 + gg;
  uint2 w[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {  // all four loads in flight, then the flag checks
    const int n = 2 * t4 + (q & 1), row = r0 + 8 * (q >> 1);
    w[q] = (n < a.B && row < g.N) ? ld_act(a.h + ((size_t)n * a.d + row) / 2) : make_uint2(0u, rfl);
  }
  uint32_t h[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int n = 2 * t4 + (q & 1), row = r0 + 8 * (q >> 1);
    if (n < a.B && row < g.N) act_wait1(a.h + ((size_t)n * a.d + row) / 2, w[q], rfl, a);
    h[q] = (w[q].x >> (16 * (row & 1))) & 0xFFFFu;
  }
  return make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
}

// QKV bias (c_attn_bs) is folded in by the QKV tile finisher
__device__ __forceinline__ void qkv_bias_fix(const StepArgs& a, const GPh& g, int tile, float (&acc)[4], int lane) {
  if (g.kind != 0) return;
  const __half* qb = a.layers[g.layer].qkv_b;
  if (qb == nullptr) return;
  const int gg = lane >> 2;
  const int r0 = tile * 16 + gg, r1 = r0 + 8;
  if (r0 < g.N) {
    const float b0 = __half2float(qb[r0]);
    acc[0] = __fadd_rn(acc[0], b0);
    acc[1] = __fadd_rn(acc[1], b0);
  }
  if (r1 < g.N) {
    const float b1 = __half2float(qb[r1]);
    acc[2] = __fadd_rn(acc[2], b1);
    acc[3] = __fadd_rn(acc[3], b1);
  }
}

// One GEMV phase for this warp.  x is staged in shared memory (XS: the rows,
// normalized where the phase has an RMSNorm) or read from global memory (L2)
// one k-block ahead.  The nibbles enter the MMA as exact fp16 (q - 8).
// The k loop handles one quantization group (GB k-blocks) per iteration,
// reading the weights straight from the ring slot.  A tile that lies whole in
// the warp's range is finished at once; a piece of a split tile goes to the
// warp's shared-memory slot (0: its first tile, 1: its last), and after a CTA
// barrier the CTA sums each split tile's pieces in warp order.  A tile that
// began in an earlier CTA is published as this CTA's partial; the CTA that
// owns a tile's first unit adds the later CTAs' partials in CTA order and
// finishes it (deterministic sums).
template <bool SYM, int GB, bool XS>
__device__ __forceinline__ bool gemv_phase(const StepArgs& a, int ph, Ring& r, Cur& pc, const __half* xs,
                                           int xs_stride, const uint2* xg, int ldx, float* spart, int wid,
                                           int lane, bool ok, uint32_t epoch) {
  const GPh g = gph(a, ph);
  const uint32_t fl = epoch * 512u + (uint32_t)ph + 1u;  // split-tile partials (never 0)
  const uint32_t efl = act_flag(epoch, ph);              // this phase's outputs
  const uint32_t rfl = act_flag(epoch, ph - 2);          // the residual: h as the phase two back wrote it
  const uint32_t sfl = act_flag(epoch, ph - 1);          // x read from global memory: the previous phase's output
  const URange wr = warp_range(g.U, blockIdx.x, gridDim.x, wid);
  const uint32_t u0 = wr.u0, u1 = wr.u1;
  const int gq = lane >> 2, t4 = lane & 3;
  const int KB = g.K / 64;
  const int t_first = (int)(u0 / g.upt), t_last = u1 > u0 ? (int)((u1 - 1) / g.upt) : t_first - 1;
  const int nn = min(gq, a.B - 1);
  // staged x: this lane's 16 halves of a k-block as two 16-byte loads; x in
  // global memory: the same halves as 8 flagged words (four 16-byte loads,
  // issued one k-block ahead and checked when used)
  const uint4* xrow = XS ? reinterpret_cast<const uint4*>(xs + (size_t)nn * xs_stride + 16 * t4) : nullptr;
  const uint2* xw = XS ? nullptr : xg + (size_t)nn * (ldx / 2) + 8 * t4;
  for (int t = t_first; t <= t_last && ok; ++t) {
    const int kb_lo = (int)max(u0, (uint32_t)(t * g.upt)) * GB;
    const int kb_hi = (int)min(u1, (uint32_t)((t + 1) * g.upt)) * GB;
    const bool complete = (uint32_t)(t * g.upt) >= u0 && (uint32_t)((t + 1) * g.upt) <= u1;
    const uint2 hres = complete ? residual_of(a, g, t, lane, rfl) : make_uint2(0u, 0u);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    // two accumulator chains (alternate fragment words) so consecutive MMAs
    // do not wait on each other; SYM restarts them per group, AFFINE (weights
    // dequantized before the MMA) runs them over the tile
    float c[2][4];
#pragma unroll
    for (int q = 0; q < 2; ++q)
#pragma unroll
      for (int e = 0; e < 4; ++e) c[q][e] = 0.f;
    uint4 xn[4];
    if (!XS) {
#pragma unroll
      for (int i = 0; i < 4; ++i) xn[i] = ld_ll(reinterpret_cast<const uint4*>(xw + 32 * (kb_lo - t * KB)) + i);
    }
    for (int kb = kb_lo; kb < kb_hi;) {
      const int st = r.cs;
      if (!__all_sync(0xffffffffu, mbar_wait(r.bars + st, (uint32_t)r.cpar, a.mbar_limit))) {
        if (lane == 0) raise_abort(a);
        ok = false;
        break;
      }
      const int sl = a.plan.slot_kb;
      const int nk = min(sl, kb_hi - kb);
      const uint4* wsl = reinterpret_cast<const uint4*>(r.buf + (size_t)st * sl * kSlotPerKb) + lane;
      const char* ssl = r.buf + (size_t)st * sl * kSlotPerKb + sl * 512;
      const int kbt = kb - t * KB;
      // one k-block of the slot; a group's scales are applied after its last k-block
      auto kblock = [&](const int j) {
        const uint4 wv = wsl[j * 32];
        uint32_t bf[8];
        if (XS) {
          const uint4 v0 = xrow[(kbt + j) * 8], v1 = xrow[(kbt + j) * 8 + 1];
          bf[0] = v0.x; bf[1] = v0.y; bf[2] = v0.z; bf[3] = v0.w;
          bf[4] = v1.x; bf[5] = v1.y; bf[6] = v1.z; bf[7] = v1.w;
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            act_wait2(xw + 32 * (kbt + j) + 2 * i, xn[i], sfl, a);
            bf[2 * i] = xn[i].x;
            bf[2 * i + 1] = xn[i].z;
          }
          if (kb + j + 1 < kb_hi) {
#pragma unroll
            for (int i = 0; i < 4; ++i) xn[i] = ld_ll(reinterpret_cast<const uint4*>(xw + 32 * (kbt + j + 1)) + i);
          }
        }
        const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
        if (SYM) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t af[4];
            unpack_word<8>(words[q], af);
            if ((j % GB) == 0 && q < 2) mma_16816_z(c[q & 1], af, bf[2 * q], bf[2 * q + 1]);
            else mma_16816(c[q & 1], af, bf[2 * q], bf[2 * q + 1], c[q & 1]);
          }
          if ((j % GB) == GB - 1) {  // group complete: apply the scales
            const uint32_t sp = reinterpret_cast<const uint32_t*>(ssl)[(j / GB) * 8 + gq];
            const float2 sc = __half22float2(u32_as_h2(sp));
            acc[0] = __fmaf_rn(sc.x, c[0][0] + c[1][0], acc[0]);
            acc[1] = __fmaf_rn(sc.x, c[0][1] + c[1][1], acc[1]);
            acc[2] = __fmaf_rn(sc.y, c[0][2] + c[1][2], acc[2]);
            acc[3] = __fmaf_rn(sc.y, c[0][3] + c[1][3], acc[3]);
          }
        } else {
          const uint2 sb = reinterpret_cast<const uint2*>(ssl)[j * 8 + gq];
          const __half2 s01 = u32_as_h2(sb.x), s23 = u32_as_h2(sb.y);
          const __half2 sg = __half2half2(__low2half(s01)), bg = __half2half2(__high2half(s01));
          const __half2 sg8 = __half2half2(__low2half(s23)), bg8 = __half2half2(__high2half(s23));
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t af[4];
            unpack_word<0>(words[q], af);
            af[0] = h2_as_u32(__hfma2(u32_as_h2(af[0]), sg, bg));
            af[1] = h2_as_u32(__hfma2(u32_as_h2(af[1]), sg8, bg8));
            af[2] = h2_as_u32(__hfma2(u32_as_h2(af[2]), sg, bg));
            af[3] = h2_as_u32(__hfma2(u32_as_h2(af[3]), sg8, bg8));
            mma_16816(c[q & 1], af, bf[2 * q], bf[2 * q + 1], c[q & 1]);
          }
        }
      };
      // one quantization group (GB k-blocks) per iteration: the loop body is
      // the only copy of the GEMV math in the kernel (the step's code has to
      // stay in the instruction cache)
#pragma unroll 1
      for (int j = 0; j < nk; j += GB) {
#pragma unroll
        for (int jj = 0; jj < GB; ++jj) kblock(j + jj);
      }
      __syncwarp();
      ring_consumed(r);
      ring_issue<SYM, GB>(r, pc, a, wid, lane);
      kb += nk;
    }
    if (!ok) break;
    if (!SYM) {
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] = c[0][e] + c[1][e];
    }
    if (complete) {
      qkv_bias_fix(a, g, t, acc, lane);
      step_epilogue(a, g, t, acc[0], acc[1], acc[2], acc[3], hres, lane, efl);
      continue;
    }
    *reinterpret_cast<float4*>(spart + ((wid * 2 + (t == t_first ? 0 : 1)) * 32 + lane) * 4) =
        make_float4(acc[0], acc[1], acc[2], acc[3]);
  }
  // ---- the CTA's split tiles (tile ct0 + i is taken by warp i % 16)
  ok = __syncthreads_and(ok) != 0;
  const int C = gridDim.x, cta = blockIdx.x;
  const uint32_t c0 = cta_u0(g.U, cta, C), n = cta_u0(g.U, cta + 1, C) - c0, we = cta_warps(n);
  const uint32_t upt = (uint32_t)g.upt;
  if (ok && n > 0) {
    const int ct0 = (int)(c0 / upt), ct1 = (int)((c0 + n - 1) / upt);
    for (int t = ct0 + wid; t <= ct1 && ok; t += kSW) {
      const uint32_t ts = (uint32_t)t * upt, te = ts + upt;
      const uint32_t p0 = max(c0, ts), p1 = min(c0 + n, te);
      const int wa = owner_of(p0, c0, n, we), wb = owner_of(p1 - 1, c0, n, we);
      const uint32_t ra0 = c0 + (uint32_t)(((unsigned long long)n * (unsigned)wa) / we);
      const uint32_t ra1 = c0 + (uint32_t)(((unsigned long long)n * (unsigned)(wa + 1)) / we);
      if (wa == wb && ra0 <= ts && ra1 >= te) continue;  // whole in one warp: already finished
      const bool first_cta = p0 == ts;
      const uint2 hres = first_cta ? residual_of(a, g, t, lane, rfl) : make_uint2(0u, 0u);
      float tot[4] = {0.f, 0.f, 0.f, 0.f};
      for (int w0 = wa; w0 <= wb; ++w0) {
        const uint32_t r0 = c0 + (uint32_t)(((unsigned long long)n * (unsigned)w0) / we);
        const float4 v =
            *reinterpret_cast<const float4*>(spart + ((w0 * 2 + ((uint32_t)t == r0 / upt ? 0 : 1)) * 32 + lane) * 4);
        tot[0] += v.x;
        tot[1] += v.y;
        tot[2] += v.z;
        tot[3] += v.w;
      }
      // A CTA's pieces alternate between two slots by phase parity: its next
      // phase's piece never lands on one a slower CTA has yet to read (writing
      // the piece of phase ph + 2 needs phase ph + 1 outputs, hence every
      // phase-ph tile, this one included, finished).
      if (!first_cta) {  // the tile began in an earlier CTA: publish this CTA's piece (one per CTA)
        uint4* p = reinterpret_cast<uint4*>(a.partials) + (((size_t)cta * 2 + (ph & 1)) * 32 + lane) * 2;
        st_ll(p, tot[0], tot[1], fl);
        st_ll(p + 1, tot[2], tot[3], fl);
        continue;
      }
      if (p1 != te) {  // the tile runs on into later CTAs: their pieces, in CTA order
        const int cb = owner_of(te - 1, 0u, g.U, (uint32_t)C);
        for (int cc = cta + 1; cc <= cb; ++cc) {
          if (cta_u0(g.U, cc + 1, C) == cta_u0(g.U, cc, C)) continue;  // a CTA with no units (U < C)
          const uint4* p = reinterpret_cast<const uint4*>(a.partials) + (((size_t)cc * 2 + (ph & 1)) * 32 + lane) * 2;
          uint4 v0 = ld_ll(p), v1 = ld_ll(p + 1);
          uint32_t it = 0;
          while (v0.y != fl || v0.w != fl || v1.y != fl || v1.w != fl) {
            if (++it >= a.spin_limit) break;
            __nanosleep(32);
            v0 = ld_ll(p);
            v1 = ld_ll(p + 1);
          }
          if (__any_sync(0xffffffffu, it >= a.spin_limit)) {
            if (lane == 0) raise_abort(a);
            ok = false;
            break;
          }
          tot[0] += __uint_as_float(v0.x);
          tot[1] += __uint_as_float(v0.z);
          tot[2] += __uint_as_float(v1.x);
          tot[3] += __uint_as_float(v1.z);
        }
        if (!ok) break;
      }
      qkv_bias_fix(a, g, t, tot, lane);
      step_epilogue(a, g, t, tot[0], tot[1], tot[2], tot[3], hres, lane, efl);
    }
  }
  return ok;
}

// ------------------------------------------------------------------ staging
// Embedding rows (dequant_q8_rows, quant.py:132-163) into xs; CTA 0 also
// stores them into h (the residual stream).
__device__ __forceinline__ void stage_embed(const StepArgs& a, __half* xs, int stride, uint32_t efl) {
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
    if (blockIdx.x == 0) {
      uint2* hp = a.h + ((size_t)m * a.d + 4 * k4) / 2;
      st_act(hp, pk.x, efl);
      st_act(hp + 1, pk.y, efl);
    }
  }
}

// Stage M rows of K activations into shared memory (row stride K + 8 halves):
// from global memory (src), or the raw rows already in xs (src null).  With
// an RMSNorm weight w (modules.py:30-43: rms = 1/sqrt(mean(x^2) + eps),
// fp16((x * rms) * w)) the rows are normalized in place.
//
// Every warp of the CTA calls it, whatever its own ok (an abort can leave ok
// different in different warps): the barriers are the same for all, the
// first one makes ok the CTA's, and the copy is skipped where ok is false.
__device__ __forceinline__ bool stage_x(const StepArgs& a, int B, float eps, const uint2* src, uint32_t sfl, int K,
                                        const float* w, __half* xs, int stride, float* red, bool ok) {
  const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, wid = tid >> 5;
  const int K8 = ok ? K / 8 : 0;
  // pass 1: copy (two 8-half chunks in flight per thread, each two 16-byte
  // flagged loads, waited for until they carry the producer's flag) + sums
  // of squares
  for (int m = 0; m < B; ++m) {
    const uint2* srow = src ? src + (size_t)m * (K / 2) : nullptr;
    uint4* drow = reinterpret_cast<uint4*>(xs + (size_t)m * stride);
    float ss = 0.f;
    for (int c0 = tid; c0 < K8; c0 += 2 * nth) {
      uint4 v[2];
      if (srow) {
        uint4 raw[2][2];
#pragma unroll
        for (int u = 0; u < 2; ++u)  // all four loads in flight, then the flag checks
          if (c0 + u * nth < K8) {
            const uint4* q = reinterpret_cast<const uint4*>(srow + 4 * (c0 + u * nth));
            raw[u][0] = ld_ll(q);
            raw[u][1] = ld_ll(q + 1);
          }
#pragma unroll
        for (int u = 0; u < 2; ++u)
          if (c0 + u * nth < K8) {
            act_wait2(srow + 4 * (c0 + u * nth), raw[u][0], sfl, a);
            act_wait2(srow + 4 * (c0 + u * nth) + 2, raw[u][1], sfl, a);
            v[u] = make_uint4(raw[u][0].x, raw[u][0].z, raw[u][1].x, raw[u][1].z);
          }
      } else {
#pragma unroll
        for (int u = 0; u < 2; ++u)
          if (c0 + u * nth < K8) v[u] = drow[c0 + u * nth];
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (c0 + u * nth >= K8) continue;
        if (srow) drow[c0 + u * nth] = v[u];
        const __half2* hh = reinterpret_cast<const __half2*>(&v[u]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __half22float2(hh[q]);
          ss = __fmaf_rn(f.x, f.x, ss);
          ss = __fmaf_rn(f.y, f.y, ss);
        }
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) red[wid * kStepMaxM + m] = ss;
  }
  ok = __syncthreads_and(ok) != 0;
  if (!w || !ok) return ok;
  // pass 2: normalize in place
  for (int m = 0; m < B; ++m) {
    float tot = 0.f;
    for (int ww = 0; ww < (nth >> 5); ++ww) tot += red[ww * kStepMaxM + m];
    const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), eps)));
    uint4* drow = reinterpret_cast<uint4*>(xs + (size_t)m * stride);
    for (int cc = tid; cc < K8; cc += nth) {
      const uint4 v = drow[cc];
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(w) + 2 * cc);
      const float4 w1 = __ldg(reinterpret_cast<const float4*>(w) + 2 * cc + 1);
      const float ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      const __half2* hh = reinterpret_cast<const __half2*>(&v);
      uint4 o;
      __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __half22float2(hh[q]);
        oh[q] = __floats2half2_rn(__fmul_rn(__fmul_rn(f.x, rms), ws[2 * q]),
                                  __fmul_rn(__fmul_rn(f.y, rms), ws[2 * q + 1]));
      }
      drow[cc] = o;
    }
  }
  __syncthreads();
  return ok;
}

// ------------------------------------------------------------------ attention
// K/V rows are staged by TMA tensor copies in boxes of kBoxRows rows and at
// most 128 bytes of a row (a "plane"; fp16 rows of 256 B take two planes),
// with the copy engine's 16-byte-chunk swizzle (the XOR of the chunk index
// with the row's position in the 1 KB swizzle atom): the eight rows one MMA
// fragment reads then fall in different shared-memory banks.
constexpr int kBoxRows = 32;

__host__ __device__ constexpr int kv_box_bytes(int rb) { return rb < 128 ? rb : 128; }

// byte b (< BX) of staged row r of one plane, swizzled as the copy engine
// writes it (the plane starts on a 1 KB boundary)
template <int BX>
__device__ __forceinline__ int swz(int r, int b) {
  return r * BX + ((((b >> 4) ^ ((r * BX >> 7) & (BX / 16 - 1)))) << 4) + (b & 15);
}

struct AttnLayout {
  int rb, bx, np, ng, kv, ksc, vsc, qh, qs, bytes;
};

// Working set of one attention item: the staged K and V planes (1 KB
// aligned; the union start is aligned up at run time, hence the slack), which
// after the last chunk hold the warps' partial results (per warp: m[8], l[8],
// O[n_rep][hd + 4] in fp32), their rows' fp16 scales, and q as fp16 hi / lo parts
// (8 rows, the ones past n_rep zero; rows hd/2 + 4 words apart).  cap is a
// multiple of kBoxRows.
__host__ __device__ inline AttnLayout attn_layout(int kv_type, int hd, int kv_group, int cap, int n_rep) {
  AttnLayout L;
  L.rb = kv_row_bytes(kv_type, hd);
  L.bx = kv_box_bytes(L.rb);
  L.np = L.rb / L.bx;
  L.ng = kv_type == AXB_KV_F16 ? 1 : hd / kv_group;
  L.kv = 0;
  const int stage = 2 * cap * L.rb;
  const int merge = kSW * 16 * 4 + kSW * n_rep * (hd + 4) * 4;
  int off = round_up_i(stage > merge ? stage : merge, 128);
  const int sb = round_up_i(cap * L.ng * 2, 16);
  L.ksc = off;
  off += sb;
  L.vsc = off;
  off += sb;
  L.qs = hd / 2 + 4;
  L.qh = off;
  off += 2 * 8 * L.qs * 4;
  L.bytes = round_up_i(off, 128) + 1024;  // + alignment slack
  return L;
}

// the 1 KB-aligned start of the attention working set inside the union
__device__ __forceinline__ char* attn_base(char* uni) {
  return uni + ((1024u - (smem_u32(uni) & 1023u)) & 1023u);
}

// Splits per (sequence, kv head): one item per CTA when the heads fit, and
// chunks in kBoxRows multiples.
__device__ __forceinline__ void attn_split_plan(int active, int units, int& nsplit, int& chunk) {
  int target = units;
  if (target > kStepMaxSplits) target = kStepMaxSplits;
  if (target < 1) target = 1;
  chunk = (active + target - 1) / target;
  chunk = (chunk + kBoxRows - 1) / kBoxRows * kBoxRows;
  if (chunk < kBoxRows) chunk = kBoxRows;
  nsplit = (active + chunk - 1) / chunk;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const void* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Copy cached K/V rows [c0, c0 + nt) of one head (thread 0): whole boxes of
// kBoxRows rows per plane through the layer's tensor maps (rows past the item
// are staged but never read; rows past the cache are filled with zeros), and
// for quantized caches the rows' scales (rounded up to 8 tokens: 16-byte
// copies; the cache length is a multiple of 8) as plain bulk copies.
__device__ __noinline__ void attn_copy(const StepLayer* ly, size_t head_base, int np, int bx, int ng, int rb,
                                       bool quant, int c0, int nt, int cap, char* kpl, char* ksc, char* vsc,
                                       uint64_t* bar) {
  const int nbox = (nt + kBoxRows - 1) / kBoxRows;
  const int nt8 = (nt + 7) & ~7;
  fence_proxy_async();
  mbar_expect_tx(bar, 2u * np * nbox * kBoxRows * bx + (quant ? 2u * nt8 * ng * 2 : 0u));
  char* vpl = kpl + (size_t)cap * rb;
  const int y0 = (int)(head_base + c0);
  const uint64_t pol = l2_evict_first_policy();  // cached rows are read once per step
  for (int pl = 0; pl < np; ++pl)
    for (int i = 0; i < nbox; ++i) {
      const size_t off = (size_t)pl * cap * bx + (size_t)i * kBoxRows * bx;
      tma_load_2d(kpl + off, ly->kmap, pl * bx, y0 + i * kBoxRows, bar, pol);
      tma_load_2d(vpl + off, ly->vmap, pl * bx, y0 + i * kBoxRows, bar, pol);
    }
  if (quant) {
    bulk_g2s(ksc, ly->ks + (head_base + c0) * ng, nt8 * ng * 2, bar);
    bulk_g2s(vsc, ly->vs + (head_base + c0) * ng, nt8 * ng * 2, bar);
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

// Address of byte `byte` of staged row r (planes of BX bytes, cap rows each).
template <int BX>
__device__ __forceinline__ const uint8_t* kv_at(const char* planes, int cap, int r, int byte) {
  const int pl = byte / BX;
  return reinterpret_cast<const uint8_t*>(planes) + (size_t)pl * cap * BX + swz<BX>(r, byte - pl * BX);
}

// fp16 pair (elements e, e + 1; e even) of staged row r: an MMA fragment
// register holding the cache's exact values (fp16, e4m3 codes, or int4 codes)
template <int type, int BX>
__device__ __forceinline__ uint32_t kv_pair_h2(const char* planes, int cap, int r, int e) {
  if (type == AXB_KV_F16) return *reinterpret_cast<const uint32_t*>(kv_at<BX>(planes, cap, r, 2 * e));
  if (type == AXB_KV_FP8) {
    const __half2_raw h =
        __nv_cvt_fp8x2_to_halfraw2(*reinterpret_cast<const uint16_t*>(kv_at<BX>(planes, cap, r, e)), __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
  }
  const uint32_t cb = *kv_at<BX>(planes, cap, r, e >> 1);  // low nibble = element e, high = e + 1; value (n ^ 8) - 8
  const uint32_t t = (((cb & 0xFu) | ((cb & 0xF0u) << 12)) ^ 0x00080008u) | 0x64006400u;
  return h2_as_u32(__hsub2(u32_as_h2(t), __float2half2_rn(1032.f)));
}
// element e of staged rows r0, r1 as an fp16 pair (row0, row1); a row < 0 is 0
template <int type, int BX>
__device__ __forceinline__ uint32_t kv_col_pair_h2(const char* planes, int cap, int r0, int r1, int e) {
  if (type == AXB_KV_F16) {
    const uint32_t lo = r0 >= 0 ? *reinterpret_cast<const uint16_t*>(kv_at<BX>(planes, cap, r0, 2 * e)) : 0u;
    const uint32_t hi = r1 >= 0 ? *reinterpret_cast<const uint16_t*>(kv_at<BX>(planes, cap, r1, 2 * e)) : 0u;
    return lo | (hi << 16);
  }
  if (type == AXB_KV_FP8) {
    const uint32_t b0 = r0 >= 0 ? *kv_at<BX>(planes, cap, r0, e) : 0u;
    const uint32_t b1 = r1 >= 0 ? *kv_at<BX>(planes, cap, r1, e) : 0u;
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((uint16_t)(b0 | (b1 << 8)), __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
  }
  const uint32_t sh = (e & 1) * 4;
  const uint32_t n0 = r0 >= 0 ? ((*kv_at<BX>(planes, cap, r0, e >> 1) >> sh) & 0xFu) ^ 8u : 8u;  // 8 encodes 0
  const uint32_t n1 = r1 >= 0 ? ((*kv_at<BX>(planes, cap, r1, e >> 1) >> sh) & 0xFu) ^ 8u : 8u;
  return h2_as_u32(__hsub2(u32_as_h2((n0 | (n1 << 16)) | 0x64006400u), __float2half2_rn(1032.f)));
}
// fp16 pair (row A, row B) of element 16 MS + 8 H + g of two staged rows,
// given the rows' byte offsets in a plane (rb = r * BX) and swizzle keys
// (key = (rb >> 7) & (BX / 16 - 1)): the element's 16-byte chunk is a
// compile-time constant, so an access is one XOR, one add and the load.
template <int KVT, int BX>
__device__ __forceinline__ int kv_key(int rb) {
  return (rb >> 7) & (BX / 16 - 1);
}
template <int KVT, int BX, int MS, int H>
__device__ __forceinline__ uint32_t kv_rows_pair(const char* planes, int capBX, int rbA, int keyA, int rbB, int keyB,
                                                 int g) {
  if constexpr (KVT == AXB_KV_FP8) {  // byte 16 MS + 8 H + g
    constexpr int byte0 = 16 * MS, pl = byte0 / BX, ch = (byte0 % BX) >> 4;
    const uint8_t* p = reinterpret_cast<const uint8_t*>(planes) + pl * capBX + 8 * H + g;
    const uint32_t b0 = p[rbA + ((ch ^ keyA) << 4)], b1 = p[rbB + ((ch ^ keyB) << 4)];
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((uint16_t)(b0 | (b1 << 8)), __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
  } else if constexpr (KVT == AXB_KV_F16) {  // bytes 32 MS + 16 H + 2 g, + 1
    constexpr int byte0 = 32 * MS + 16 * H, pl = byte0 / BX, ch = (byte0 % BX) >> 4;
    const char* p = planes + pl * capBX + 2 * g;
    const uint32_t lo = *reinterpret_cast<const uint16_t*>(p + rbA + ((ch ^ keyA) << 4));
    const uint32_t hi = *reinterpret_cast<const uint16_t*>(p + rbB + ((ch ^ keyB) << 4));
    return lo | (hi << 16);
  } else {  // INT4: byte 8 MS + 4 H + g / 2, nibble g & 1 (value (n ^ 8) - 8)
    constexpr int byte0 = 8 * MS + 4 * H, pl = byte0 / BX, ch = (byte0 % BX) >> 4;
    const uint8_t* p = reinterpret_cast<const uint8_t*>(planes) + pl * capBX + (byte0 & 15) + (g >> 1);
    const int sh = (g & 1) * 4;
    const uint32_t n0 = ((p[rbA + ((ch ^ keyA) << 4)] >> sh) & 0xFu) ^ 8u;
    const uint32_t n1 = ((p[rbB + ((ch ^ keyB) << 4)] >> sh) & 0xFu) ^ 8u;
    return h2_as_u32(__hsub2(u32_as_h2((n0 | (n1 << 16)) | 0x64006400u), __float2half2_rn(1032.f)));
  }
}
template <int KVT, int BX, int MS>
__device__ __forceinline__ void kv_v_frag(const char* planes, int capBX, const int (&rb)[4], const int (&key)[4], int g,
                                          uint32_t (&va)[4]) {
  va[0] = kv_rows_pair<KVT, BX, MS, 0>(planes, capBX, rb[0], key[0], rb[1], key[1], g);
  va[1] = kv_rows_pair<KVT, BX, MS, 1>(planes, capBX, rb[0], key[0], rb[1], key[1], g);
  va[2] = kv_rows_pair<KVT, BX, MS, 0>(planes, capBX, rb[2], key[2], rb[3], key[3], g);
  va[3] = kv_rows_pair<KVT, BX, MS, 1>(planes, capBX, rb[2], key[2], rb[3], key[3], g);
}
template <int KVT, int BX, int MS, int NMS>
__device__ __forceinline__ void pv_steps(const char* vst, int capBX, const int (&rb)[4], const int (&key)[4],
                                         const int (&rr)[4], const __half* vsc_s, int ng, int G, int lgG, int g,
                                         uint32_t h01, uint32_t h23, uint32_t l01, uint32_t l23, float al0, float al1,
                                         __half2& s01, __half2& s23, float (&o)[NMS][4]) {
  if constexpr (MS < NMS) {
    constexpr bool quant = KVT != AXB_KV_F16;
    if (quant && (MS == 0 || ((16 * MS) & (G - 1)) == 0)) {  // a new V scale group (groups span 16 dims or more)
      const int gi = (16 * MS) >> lgG;
      s01 = __halves2half2(vsc_s[rr[0] * ng + gi], vsc_s[rr[1] * ng + gi]);
      s23 = __halves2half2(vsc_s[rr[2] * ng + gi], vsc_s[rr[3] * ng + gi]);
    }
    uint32_t va[4];
    kv_v_frag<KVT, BX, MS>(vst, capBX, rb, key, g, va);
    if (quant) {
      va[0] = h2_as_u32(__hmul2(u32_as_h2(va[0]), s01));
      va[1] = h2_as_u32(__hmul2(u32_as_h2(va[1]), s01));
      va[2] = h2_as_u32(__hmul2(u32_as_h2(va[2]), s23));
      va[3] = h2_as_u32(__hmul2(u32_as_h2(va[3]), s23));
    }
    float t[4] = {0.f, 0.f, 0.f, 0.f};
    mma_16816(t, va, h01, h23, t);
    mma_16816(t, va, l01, l23, t);
    o[MS][0] = __fmaf_rn(o[MS][0], al0, t[0]);
    o[MS][1] = __fmaf_rn(o[MS][1], al1, t[1]);
    o[MS][2] = __fmaf_rn(o[MS][2], al0, t[2]);
    o[MS][3] = __fmaf_rn(o[MS][3], al1, t[3]);
    pv_steps<KVT, BX, MS + 1, NMS>(vst, capBX, rb, key, rr, vsc_s, ng, G, lgG, g, h01, h23, l01, l23, al0, al1, s01,
                                   s23, o);
  }
}

// fp32 pair -> fp16 (hi, lo) pairs with hi + lo = the value to about 22 bits
__device__ __forceinline__ void split_h2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const float2 hf = __half22float2(h);
  hi = h2_as_u32(h);
  lo = h2_as_u32(__floats2half2_rn(x0 - hf.x, x1 - hf.y));
}

// One attention item (sequence b, kv head, split) on the whole CTA, on the
// tensor cores.  Warp w takes the 16-token blocks w, w + 16, ... of each
// staged chunk and keeps its own online-softmax state for the (up to 8) q
// heads of the kv head: S = q K^T for the block with q as fp16 hi + lo (a
// quantized K row enters as the reference's dequantized fp16 values,
// fp16(code * scale): one HMUL2 per pair, the product of two fp16 values
// rounded once, so q . k sees the same K as the reference's SDPA); the block's
// probabilities stay in registers (the score MMA's output fragment is the PV
// MMA's input fragment); O += P V with P as hi + lo and V again as its
// dequantized fp16 values.  After the last chunk the warps' states are merged
// in warp order.  A split writes its (O, m, l) partial; the head's last split
// to finish combines all of them in split order and publishes the head.
// Every loop here runs once per block or per output: the code is kept small
// (one copy of the chunk loop, a rolled score loop).
template <int HD, int KVT>
__device__ __forceinline__ bool attn_item(const StepArgs& a, const StepLayer* ly, int layer, const AttnItem& it,
                                       int nsplit, bool prefetched, char* gsm, char* misc, uint32_t& uses,
                                       uint32_t afl, bool ok) {
  constexpr int BX = kv_box_bytes(KVT == AXB_KV_F16 ? HD * 2 : (KVT == AXB_KV_FP8 ? HD : HD / 2));
  constexpr int DPL = HD / 32, KS = HD / 16, OS = HD + 4;  // OS: row stride of the merged O
  constexpr bool quant = KVT != AXB_KV_F16;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, c = lane & 3;
  const int cap = a.plan.attn_cap;
  const int n_rep = a.Hq / a.Hkv, hq0 = it.kvh * n_rep;
  const AttnLayout Lo = attn_layout(KVT, HD, a.kv_group, cap, n_rep);
  const int ng = Lo.ng, G = KVT == AXB_KV_F16 ? HD : a.kv_group;
  const int lgG = __ffs(G) - 1;  // scale groups are powers of two
  const int qs = Lo.qs;
  const int rpos = a.params[0], wpos = a.params[1];
  const size_t head_base = ((size_t)it.b * a.Hkv + it.kvh) * a.S;
  int* flag = reinterpret_cast<int*>(misc + kMiscFlag) + 1;
  uint64_t* bar = reinterpret_cast<uint64_t*>(misc + kMiscBar);
  char* kst = gsm + Lo.kv;  // K planes, then V planes
  char* vst = kst + (size_t)cap * Lo.rb;
  const __half* ksc_s = reinterpret_cast<const __half*>(gsm + Lo.ksc);
  const __half* vsc_s = reinterpret_cast<const __half*>(gsm + Lo.vsc);
  uint32_t* qh32 = reinterpret_cast<uint32_t*>(gsm + Lo.qh);  // [hi / lo][8 rows][qs]

  // ---- q with RoPE (fp32), as fp16 hi / lo rows; the new K/V row rotated, quantized and written
  const int qkv_dim = (a.Hq + 2 * a.Hkv) * HD;
  const uint2* row = a.qkv + (size_t)it.b * qkv_dim / 2;  // flagged words of this token's q, k, v
  const float* fr = a.rope + (size_t)(rpos % a.rope_len) * HD;
  for (int i = tid; i < 8 * HD / 2; i += kSThreads) {
    const int rr = i / (HD / 2), pr = i % (HD / 2);
    float q0 = 0.f, q1 = 0.f;
    if (rr < n_rep) {
      const __half2 x2 = u32_as_h2(act_get(row + (hq0 + rr) * HD / 2 + pr, afl, a));
      const float a0 = __low2float(x2), a1 = __high2float(x2);
      const float cs = fr[2 * pr], sn = fr[2 * pr + 1];
      q0 = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(a1, sn));
      q1 = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(a1, cs));
    }
    uint32_t hi, lo;
    split_h2(q0, q1, hi, lo);
    qh32[rr * qs + pr] = hi;
    qh32[(8 + rr) * qs + pr] = lo;
  }
  uint2 ncode = make_uint2(0u, 0u);
  float nscale = 0.f;
  const bool covers = wpos >= it.t0 && wpos < it.t1;
  if (covers && w < 2) {
    float nkv[DPL];
    const uint2* src = row + (size_t)(a.Hq + (w == 0 ? 0 : a.Hkv) + it.kvh) * HD / 2;
#pragma unroll
    for (int e = 0; e < DPL; e += 2) {
      const __half2 v2 = u32_as_h2(act_get(src + (lane * DPL + e) / 2, afl, a));
      nkv[e] = __low2float(v2);
      nkv[e + 1] = __high2float(v2);
    }
    if (w == 0) {  // RoPE on K, every product rounded (transformer.py:1105-1127)
#pragma unroll
      for (int e = 0; e < DPL; e += 2) {
        const int pr = (lane * DPL + e) >> 1;
        const float cs = fr[2 * pr], sn = fr[2 * pr + 1], a0 = nkv[e], a1 = nkv[e + 1];
        nkv[e] = __fsub_rn(__fmul_rn(a0, cs), __fmul_rn(a1, sn));
        nkv[e + 1] = __fadd_rn(__fmul_rn(a0, sn), __fmul_rn(a1, cs));
      }
    }
    uint8_t* crow = (w == 0 ? ly->kc : ly->vc) + (head_base + wpos) * Lo.rb;
    __half* srow = quant ? (w == 0 ? ly->ks : ly->vs) + (head_base + wpos) * ng : nullptr;
    ncode = store_kv_row<DPL>(nkv, lane, KVT, G, true, crow, srow, &nscale);
  }
  __syncthreads();

  const float sm_scale = 1.0f / sqrtf((float)HD);
  float m_run = -INFINITY, l_run = 0.f;  // head g (the same in the four lanes of a row)
  float o[HD / 16][4];  // dims 16 ms + g (+ 8) x heads 2c, 2c + 1
#pragma unroll
  for (int ms = 0; ms < HD / 16; ++ms) o[ms][0] = o[ms][1] = o[ms][2] = o[ms][3] = 0.f;
  for (int c0 = it.t0; c0 < it.t1; c0 += cap) {
    const int nt = min(cap, it.t1 - c0);
    if (!(c0 == it.t0 && prefetched) && tid == 0) attn_copy(ly, head_base, Lo.np, Lo.bx, Lo.ng, Lo.rb, quant, c0, nt, cap, gsm + Lo.kv, gsm + Lo.ksc, gsm + Lo.vsc, bar);
    const bool got = mbar_wait(bar, uses & 1, a.mbar_limit);
    ++uses;
    if (__syncthreads_or(!got)) {  // one decision for the whole CTA
      if (tid == 0) {
        raise_abort(a);
        mbar_wait(bar, (uses - 1) & 1, kDrainLimit);  // the copies in flight land before the CTA moves on
      }
      ok = false;
      break;
    }
    if (covers && w < 2 && wpos >= c0 && wpos < c0 + nt) {
      // the copy may have read the slot (codes and scale) before this step
      // wrote it: place this step's row (this lane's bytes) and scale
      constexpr int LB = KVT == AXB_KV_F16 ? 2 * DPL : (KVT == AXB_KV_FP8 ? DPL : DPL / 2);  // bytes per lane
      uint8_t* dst = const_cast<uint8_t*>(kv_at<BX>(w == 0 ? kst : vst, cap, wpos - c0, lane * LB));
      if (LB == 8) *reinterpret_cast<uint2*>(dst) = ncode;
      else if (LB == 4) *reinterpret_cast<uint32_t*>(dst) = ncode.x;
      else if (LB == 2) *reinterpret_cast<uint16_t*>(dst) = (uint16_t)ncode.x;
      else *dst = (uint8_t)ncode.x;
      const int lpg = G / DPL;
      if (quant && (lane % lpg) == 0)
        const_cast<__half*>(w == 0 ? ksc_s : vsc_s)[(size_t)(wpos - c0) * ng + (lane * DPL) / G] =
            __float2half_rn(nscale);
    }
    __syncthreads();
    for (int tb = 16 * w; tb < nt; tb += 16 * kSW) {
      // ---- scores of the block's two 8-token halves (B-fragment columns tb + g, tb + 8 + g;
      // columns past the chunk read its last row and are masked below)
      const int k0 = min(tb + g, nt - 1), k1 = min(tb + 8 + g, nt - 1);
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
      for (int s = 0; s < KS; ++s) {
        const uint32_t* qp = qh32 + g * qs + 8 * s + c;
        const uint32_t ahi[4] = {qp[0], 0u, qp[4], 0u};
        const uint32_t alo[4] = {qp[8 * qs], 0u, qp[8 * qs + 4], 0u};
        const int e0 = 16 * s + 2 * c;
        uint32_t b00 = kv_pair_h2<KVT, BX>(kst, cap, k0, e0), b01 = kv_pair_h2<KVT, BX>(kst, cap, k0, e0 + 8);
        uint32_t b10 = kv_pair_h2<KVT, BX>(kst, cap, k1, e0), b11 = kv_pair_h2<KVT, BX>(kst, cap, k1, e0 + 8);
        if (quant) {
          const int gi = (16 * s) >> lgG;
          const __half2 sc0 = __half2half2(ksc_s[k0 * ng + gi]), sc1 = __half2half2(ksc_s[k1 * ng + gi]);
          b00 = h2_as_u32(__hmul2(u32_as_h2(b00), sc0));
          b01 = h2_as_u32(__hmul2(u32_as_h2(b01), sc0));
          b10 = h2_as_u32(__hmul2(u32_as_h2(b10), sc1));
          b11 = h2_as_u32(__hmul2(u32_as_h2(b11), sc1));
        }
        mma_16816(s0, ahi, b00, b01, s0);
        mma_16816(s0, alo, b00, b01, s0);
        mma_16816(s1, ahi, b10, b11, s1);
        mma_16816(s1, alo, b10, b11, s1);
      }
      // ---- online softmax: this thread holds head g at tokens ta, ta + 1, tc, tc + 1
      const int ta = tb + 2 * c, tc = ta + 8;
      const float sv[4] = {ta < nt ? s0[0] * sm_scale : -INFINITY, ta + 1 < nt ? s0[1] * sm_scale : -INFINITY,
                           tc < nt ? s1[0] * sm_scale : -INFINITY, tc + 1 < nt ? s1[1] * sm_scale : -INFINITY};
      float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);  // finite: token tb is in the chunk
      const float alpha = m_run == -INFINITY ? 0.f : __expf(m_run - m_new);
      float p[4], ps = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        p[q] = sv[q] == -INFINITY ? 0.f : __expf(sv[q] - m_new);
        ps += p[q];
      }
      ps += __shfl_xor_sync(0xffffffffu, ps, 1);
      ps += __shfl_xor_sync(0xffffffffu, ps, 2);
      l_run = __fmaf_rn(l_run, alpha, ps);
      m_run = m_new;
      // ---- O^T = alpha O^T + V^T P^T (dims x heads): the A operand is V^T
      // (16 dims x the block's 16 tokens), the B operand this thread's
      // probabilities as the score MMA left them (head g at tokens ta, ta + 1
      // and tc, tc + 1), as fp16 hi + lo
      uint32_t h01, l01, h23, l23;
      split_h2(p[0], p[1], h01, l01);
      split_h2(p[2], p[3], h23, l23);
      // the rescale of this thread's output heads 2c, 2c + 1 (rows 2c, 2c + 1 of the score layout)
      const float al0 = __shfl_sync(0xffffffffu, alpha, 8 * c), al1 = __shfl_sync(0xffffffffu, alpha, 8 * c + 4);
      // this thread's four tokens' rows, clamped into the chunk: an absent
      // token has p = 0 and reads a finite cached row, so it adds exactly 0
      const int rr[4] = {min(ta, nt - 1), min(ta + 1, nt - 1), min(tc, nt - 1), min(tc + 1, nt - 1)};
      int rb[4], key[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        rb[q] = rr[q] * BX;
        key[q] = kv_key<KVT, BX>(rb[q]);
      }
      __half2 s01, s23;
      pv_steps<KVT, BX, 0, HD / 16>(vst, cap * BX, rb, key, rr, vsc_s, ng, G, lgG, g, h01, h23, l01, l23, al0, al1, s01,
                                    s23, o);
    }
    __syncthreads();  // the staged rows are free for the next chunk
  }
  if (!ok) return false;

  // ---- merge the warps' states in warp order (the staged rows are dead)
  float* wm = reinterpret_cast<float*>(gsm + Lo.kv);  // [kSW][8] m, then [kSW][8] l
  float* wo = wm + 2 * kSW * 8;                        // [kSW][n_rep][OS]
  if (c == 0) {
    wm[w * 8 + g] = m_run;
    wm[kSW * 8 + w * 8 + g] = l_run;
  }
#pragma unroll
  for (int ms = 0; ms < HD / 16; ++ms)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int h = 2 * c + (q & 1), dd = 16 * ms + g + 8 * (q >> 1);
      if (h < n_rep) wo[((size_t)w * n_rep + h) * OS + dd] = o[ms][q];
    }
  __syncthreads();
  const size_t pidx = (size_t)it.b * a.Hq + hq0;
  for (int i = tid; i < n_rep * HD; i += kSThreads) {
    const int r = i / HD, e = i % HD;
    float M = -INFINITY;
#pragma unroll 4
    for (int v = 0; v < kSW; ++v) M = fmaxf(M, wm[v * 8 + r]);
    float Ls = 0.f, O = 0.f;
#pragma unroll 4
    for (int v = 0; v < kSW; ++v) {
      const float mv = wm[v * 8 + r];
      const float cw = mv == -INFINITY ? 0.f : __expf(mv - M);
      Ls = __fmaf_rn(wm[kSW * 8 + v * 8 + r], cw, Ls);
      O = __fmaf_rn(wo[((size_t)v * n_rep + r) * OS + e], cw, O);
    }
    if (nsplit == 1) {  // adjacent outputs e, e + 1 sit in adjacent lanes: one flagged word
      const uint32_t hv = __half_as_ushort(__float2half_rn(__fdiv_rn(O, Ls)));
      const uint32_t nb = __shfl_down_sync(0xffffffffu, hv, 1);
      if ((e & 1) == 0) st_act(a.attn + ((pidx + r) * HD + e) / 2, hv | (nb << 16), afl);
    } else {
      a.part_o[((pidx + r) * kStepMaxSplits + it.split) * HD + e] = O;
      if (e == 0)
        *reinterpret_cast<float2*>(a.part_ml + ((pidx + r) * kStepMaxSplits + it.split) * 2) = make_float2(M, Ls);
    }
  }
  __syncthreads();
  if (nsplit == 1) return true;
  // ---- the head's last split to arrive combines it.  The per-head counter
  // only grows during a step (layer l completes at (l + 1) * nsplit arrivals);
  // the step's last CTA clears it.
  if (tid == 0) {
    const int old = atom_acq_rel_add(a.attn_cnt + it.b * a.Hkv + it.kvh, 1);
    *flag = old == (layer + 1) * nsplit - 1 ? 1 : 0;
  }
  __syncthreads();
  if (!*flag) return true;
  // The splits' partials are staged in shared memory first, all loads of a
  // batch in flight at once: every (m, l), then the head group's O rows in
  // groups of gs splits (all of them when they fit, the usual case).  The
  // sums are the same as reading the partials one by one: M over all splits,
  // then l and O accumulated in split order.  One output per thread
  // (n_rep <= 4, HD <= 128).
  static_assert(4 * HD <= kSThreads, "one combined output per thread");
  const int mlb = round_up_i(n_rep * nsplit * 8, 16);
  float2* sml = reinterpret_cast<float2*>(gsm + Lo.kv);  // [n_rep][nsplit]
  float4* so4 = reinterpret_cast<float4*>(gsm + Lo.kv + mlb);  // [n_rep][gs][HD / 4]
  const int gs = min(nsplit, (Lo.ksc - Lo.kv - mlb) / (n_rep * HD * 4));
  for (int i = tid; i < n_rep * nsplit; i += kSThreads) {
    const int hr = i / nsplit, sp = i - hr * nsplit;
    sml[i] = __ldcg(reinterpret_cast<const float2*>(a.part_ml) + (pidx + hr) * kStepMaxSplits + sp);
  }
  const bool mine = tid < n_rep * HD;
  const int r = tid / HD, e = tid % HD;
  float M = -INFINITY, Ls = 0.f, O = 0.f;
  for (int s0 = 0; s0 < nsplit; s0 += gs) {
    const int ns = min(gs, nsplit - s0), per = ns * (HD / 4), n4 = n_rep * per;
    for (int i = tid; i < n4; i += kSThreads) {  // 16-byte async copies through L2: no registers held
      const int hr = i / per;
      cp_async16(so4 + hr * gs * (HD / 4) + (i - hr * per),
                 reinterpret_cast<const float4*>(a.part_o + ((pidx + hr) * kStepMaxSplits + s0) * HD) + (i - hr * per));
    }
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    if (mine) {
      if (s0 == 0) {
#pragma unroll 4
        for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, sml[r * nsplit + sp].x);
      }
      const float* so = reinterpret_cast<const float*>(so4) + (size_t)r * gs * HD + e;
#pragma unroll 4
      for (int sp = 0; sp < ns; ++sp) {
        const float2 v = sml[r * nsplit + s0 + sp];
        const float cw = v.x == -INFINITY ? 0.f : __expf(v.x - M);
        Ls = __fmaf_rn(v.y, cw, Ls);
        O = __fmaf_rn(so[sp * HD], cw, O);
      }
    }
    __syncthreads();
  }
  if (mine) {  // n_rep * HD is a multiple of 32: whole warps
    const uint32_t hv = __half_as_ushort(__float2half_rn(__fdiv_rn(O, Ls)));
    const uint32_t nb = __shfl_down_sync(0xffffffffu, hv, 1);
    if ((e & 1) == 0) st_act(a.attn + ((pidx + r) * HD + e) / 2, hv | (nb << 16), afl);
  }
  return true;
}

// The attention phase of layer l on this CTA: its first item's cached rows
// are copied before the layer's QKV phase has finished (they do not depend on
// it), then the CTA takes items blockIdx.x, + gridDim.x, ...
template <int HD>
__device__ __forceinline__ bool attn_phase(const StepArgs& a, int l, char* uni, char* misc, uint32_t& uses, bool ok,
                                           uint32_t epoch) {
  const int tid = threadIdx.x, C = gridDim.x;
  const StepLayer* ly = a.layers + l;
  uint64_t* bar = reinterpret_cast<uint64_t*>(misc + kMiscBar);
  const uint32_t afl = act_flag(epoch, 4 * l);  // the layer's QKV outputs, and this phase's outputs
  const int active = a.params[2];
  int nsplit, chunk;
  attn_split_plan(active, C / (a.B * a.Hkv), nsplit, chunk);
  const int n_items = a.B * a.Hkv * nsplit;
  const AttnLayout Lo = attn_layout(a.kv_type, HD, a.kv_group, a.plan.attn_cap, a.Hq / a.Hkv);
  char* gsm = attn_base(uni);
  int item = blockIdx.x;
  const bool pre = ok && item < n_items;
  if (pre && tid == 0) {  // cached rows do not depend on this step's QKV
    const AttnItem it = attn_item_of(item, nsplit, chunk, a.Hkv, active);
    const size_t hb = ((size_t)it.b * a.Hkv + it.kvh) * a.S;
    attn_copy(ly, hb, Lo.np, Lo.bx, Lo.ng, Lo.rb, a.kv_type != AXB_KV_F16, it.t0, min(a.plan.attn_cap, it.t1 - it.t0),
              a.plan.attn_cap, gsm + Lo.kv, gsm + Lo.ksc, gsm + Lo.vsc, bar);
  }
  trace_mark(a, 1 + 10 * l + 2);  // an item waits for its own head's q, k, v words
  bool first = true;
  for (; item < n_items; item += C) {
    if (!ok) {
      // the copies issued above land before the union is reused
      if (first && pre && tid == 0) mbar_wait(bar, uses & 1, kDrainLimit);
      if (first && pre) ++uses;
      break;
    }
    const AttnItem it = attn_item_of(item, nsplit, chunk, a.Hkv, active);
    if (a.kv_type == AXB_KV_FP8)
      ok = attn_item<HD, AXB_KV_FP8>(a, ly, l, it, nsplit, first, gsm, misc, uses, afl, ok);
    else if (a.kv_type == AXB_KV_INT4)
      ok = attn_item<HD, AXB_KV_INT4>(a, ly, l, it, nsplit, first, gsm, misc, uses, afl, ok);
    else
      ok = attn_item<HD, AXB_KV_F16>(a, ly, l, it, nsplit, first, gsm, misc, uses, afl, ok);
    first = false;
  }
  if (tid == 0) trace_at(a, 4 + 10 * a.L + (4 * a.L + 1) * kStepTraceW + 2 * l);
  return ok;
}

// ------------------------------------------------------------------ kernel
template <bool SYM, int GB, int HD>
__global__ void __launch_bounds__(kSThreads, 1) step_kernel(const StepArgs a) {
  extern __shared__ __align__(128) char smem[];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int C = gridDim.x;
  const int nsl = a.plan.nslots, slot_b = a.plan.slot_kb * kSlotPerKb;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)kSW * nsl * slot_b);
  char* uni = smem + (size_t)kSW * nsl * slot_b + kSBars;
  char* misc = uni + a.plan.union_bytes;
  float* red = reinterpret_cast<float*>(misc + kMiscRed);
  int* s_last = reinterpret_cast<int*>(misc + kMiscFlag);

  // staged activations: M rows of K + 8 halves from the union's start
  __half* xs = reinterpret_cast<__half*>(uni);
  const int ub = a.plan.union_bytes;
  const int xs_stride = a.d + 8;
  float* spart = reinterpret_cast<float*>(uni + ub - kSPartBytes);  // split-tile pieces, at the union's end

  Ring ring;
  ring.buf = smem + (size_t)wid * nsl * slot_b;
  ring.bars = bars + wid * kMaxSlots;
  ring.n = nsl;
  ring.cs = 0;
  ring.cpar = 0;
  ring.ps = 0;
  ring.inflight = 0;
  Cur& pc = reinterpret_cast<Cur*>(misc + kMiscCur)[wid];
  if (lane == 0) {
    for (int s = 0; s < nsl; ++s) mbar_init(ring.bars + s, 1);
    if (wid == 0) mbar_init(reinterpret_cast<uint64_t*>(misc + kMiscBar), 1);
    fence_mbar_init();
    pc.ph = 0;
    cur_load<GB>(pc, a, wid);
    for (int s = 0; s < nsl; ++s) ring_issue<SYM, GB>(ring, pc, a, wid, lane);
  }
  __syncthreads();

  bool ok = true;
  // launch epoch (advanced by the step's last CTA): split-tile partials of
  // GEMV phase ph carry the flag epoch * 512 + ph + 1 (never 0, the value of
  // an unwritten slot)
  const uint32_t epoch = *reinterpret_cast<volatile const uint32_t*>(a.exit_cnt + 2);
  uint32_t abar_uses = 0;  // completed phases of the attention mbarrier

  trace_mark(a, 0);
  // embedding rows for the first layer's QKV (every CTA stages its own copy)
  stage_embed(a, xs, xs_stride, act_flag(epoch, -1));
  __syncthreads();

  // GEMV phases in order: p = 4 l + {0 QKV, 1 o, 2 gate_up, 3 down}, 4 L = lm_head;
  // attention runs between a layer's QKV and o phases.  One loop, so every
  // GEMV variant is emitted once.
  for (int ph = 0; ph <= 4 * a.L; ++ph) {
    const int l = ph >> 2, kind = ph < 4 * a.L ? (ph & 3) : 4;
    const StepLayer* ly = a.layers + (kind == 4 ? 0 : l);
    const int ts = 1 + 10 * l;
    // ---- the phase's input: its source, width and RMSNorm weight.  There is
    // no wait here: the staging (or the GEMV's own x loads) waits for the
    // words of the previous phase's output to carry that phase's flag.
    const uint2* src;
    const float* nw = nullptr;
    int K;
    if (kind == 0) {  // QKV: RMSNorm(h) (the embedding rows already in xs for layer 0)
      trace_mark(a, ts + 0);
      src = l > 0 ? a.h : nullptr;
      K = a.d;
      nw = ly->ln1;
    } else if (kind == 1) {  // o: attention output (+ residual)
      trace_mark(a, ts + 4);
      src = a.attn;
      K = a.Hq * a.hd;
    } else if (kind == 2) {  // gate_up: RMSNorm(h), SwiGLU epilogue
      trace_mark(a, ts + 6);
      src = a.h;
      K = a.d;
      nw = ly->ln2;
    } else if (kind == 3) {  // down: SwiGLU output (+ residual)
      trace_mark(a, ts + 8);
      src = a.sw;
      K = a.F;
    } else {  // lm_head: final RMSNorm(h); with no layers h holds CTA 0's embedding rows
      trace_mark(a, 1 + 10 * a.L);
      src = a.h;
      K = a.d;
      nw = a.ln_f;
    }
    // ---- the GEMV: activations staged in shared memory when they fit (always
    // for the normalized inputs), else read from L2 one k-block ahead
    const bool staged = stage_bytes(a.B, K) + kSPartBytes <= ub;
    if (!staged && (nw != nullptr || src == nullptr)) {
      // normalized inputs (and layer 0's embedding rows) exist only as staged
      // rows; the host guarantees they fit, so this is a contract violation:
      // report it rather than read an absent source
      if (tid == 0) atomicExch(a.err, AXB_EINVAL);
      ok = false;
    }
    if (staged) {
      ok = stage_x(a, a.B, a.eps, src, act_flag(epoch, ph - 1), K, nw, xs, K + 8, red, ok);
      ok = gemv_phase<SYM, GB, true>(a, ph, ring, pc, xs, K + 8, nullptr, 0, spart, wid, lane, ok, epoch);
    } else {
      ok = gemv_phase<SYM, GB, false>(a, ph, ring, pc, nullptr, 0, src, K, spart, wid, lane, ok, epoch);
    }
    if (lane == 0) trace_at(a, 4 + 10 * a.L + ph * kStepTraceW + wid);  // this warp's share done
    trace_mark(a, kind == 4 ? 2 + 10 * a.L : ts + (kind == 0 ? 1 : 2 * kind + 3));  // QKV, o, gate_up, down done
    if (kind != 0) continue;
    // ---- attention of layer l (RoPE + KV write fused)
    ok = __syncthreads_and(ok) != 0;  // the staged rows are dead: the union holds attention next
    ok = attn_phase<HD>(a, l, uni, misc, abar_uses, ok, epoch);
    trace_mark(a, ts + 3);
  }

  // ---- wind down: copies still in flight (only after an abort) are waited for
  if (lane == 0)
    for (int i = 0; i < ring.inflight; ++i) {
      mbar_wait(ring.bars + ring.cs, (uint32_t)ring.cpar, kDrainLimit);
      if (++ring.cs == ring.n) {
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
  for (int i = tid; i < a.B * a.Hkv; i += blockDim.x) a.attn_cnt[i] = 0;  // grow through the step
  __syncthreads();
  if (tid == 0) {
    a.exit_cnt[2] += 1;  // the next launch's epoch (every CTA read this one at its start)
    a.exit_cnt[1] = 0;
    a.exit_cnt[0] = 0;
  }
}

// ------------------------------------------------------------------ host
int step_num_warps() { return kSW; }

int step_kv_maps(void* maps_host, int L, void* const* kc, void* const* vc, int rows, int kv_type, int hd) {
  static_assert(sizeof(CUtensorMap) == kStepMapBytes, "tensor map size");
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
      set_error("step: cuTensorMapEncodeTiled is not available from the driver");
      return AXB_ECUDA;
    }
    encode = reinterpret_cast<EncodeFn>(fn);
  }
  const int rb = kv_row_bytes(kv_type, hd), bx = kv_box_bytes(rb);
  const CUtensorMapSwizzle sw = bx == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                          : (bx == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  CUtensorMap* maps = reinterpret_cast<CUtensorMap*>(maps_host);
  const cuuint64_t dims[2] = {(cuuint64_t)rb, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)rb};
  const cuuint32_t box[2] = {(cuuint32_t)bx, (cuuint32_t)kBoxRows};
  const cuuint32_t estr[2] = {1, 1};
  for (int l = 0; l < L; ++l)
    for (int kv = 0; kv < 2; ++kv) {
      CUresult r = encode(maps + 2 * l + kv, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, kv ? vc[l] : kc[l], dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) {
        set_error("step: tensor map of layer %d (%s) failed (%d)", l, kv ? "V" : "K", (int)r);
        return AXB_ECUDA;
      }
    }
  return AXB_OK;
}

StepPlan step_plan(int max_batch, int d, int F, int Hq, int Hkv, int hd, int kv_type, int kv_group, int group,
                   int max_seq) {
  (void)F;
  (void)max_seq;
  StepPlan p = {0, 0, 0, 0, 0};
  const int B = std::min(max_batch, kStepMaxM);
  const int need = stage_bytes(B, d) + kSPartBytes;  // normalized inputs are always staged
  // ring shapes, best first: 2 slots of 8 k-blocks, then 3 or 2 slots of 4
  // (the same bytes in flight in fewer, larger copies, as long as the union fits)
  const int shapes[3][2] = {{8, 2}, {4, 3}, {4, 2}};
  for (const auto& sh : shapes) {
    const int sl = sh[0], ns = sh[1];
    const int fixed = kSW * ns * sl * kSlotPerKb + kSBars + kSMisc;
    const int avail = (kSmemMax - fixed) / 128 * 128;
    if (avail < need) continue;
    int cap = 0;
    for (int c = 256; c >= kBoxRows; c -= kBoxRows)
      if (attn_layout(kv_type, hd, kv_group, c, Hq / Hkv).bytes <= avail) {
        cap = c;
        break;
      }
    if (cap == 0) continue;
    p.nslots = ns;
    p.slot_kb = sl;
    p.union_bytes = avail;
    p.attn_cap = cap;
    p.smem = fixed + avail;
    return p;
  }
  return p;
}

bool step_supported(int wfmt, int group, int lm_fmt, int lm_group, int hd, int n_head, int n_kv_head, int d_model,
                    int kv_type, int kv_group, int max_seq) {
  if (wfmt != lm_fmt || group != lm_group) return false;
  if (wfmt != AXB_W_Q4T_SYM && wfmt != AXB_W_Q4T_AFFINE) return false;
  if (group != 64 && group != 128) return false;
  if (hd != 64 && hd != 128) return false;
  if (n_kv_head <= 0 || n_head % n_kv_head != 0 || n_head / n_kv_head > kMaxRepS) return false;
  if (d_model % 128 != 0) return false;
  // a K scale group spans whole 16-wide MMA steps, a V scale group a warp's 8 output dims
  if (kv_type != AXB_KV_F16 && (kv_group < 16 || hd % kv_group != 0)) return false;
  if (max_seq % 8) return false;  // scales are bulk-copied in 8-token (16-byte) runs
  return true;
}

#define AXB_STEP_KERNELS(X) \
  X(true, 2, 128) X(true, 1, 128) X(false, 2, 128) X(false, 1, 128) X(true, 2, 64) X(true, 1, 64) X(false, 2, 64) X(false, 1, 64)

int step_prepare() {
  int dev = 0;
  cudaGetDevice(&dev);
  static DeviceOnce once;
  if (once.done(dev)) return AXB_OK;
#define AXB_SET(SYM, GB, HD)                                                                                 \
  {                                                                                                         \
    cudaError_t e = cudaFuncSetAttribute(step_kernel<SYM, GB, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                         kSmemMax);                                                         \
    if (e != cudaSuccess) return cuda_status(e, "step kernel attribute");                                   \
  }
  AXB_STEP_KERNELS(AXB_SET)
#undef AXB_SET
  once.set(dev);
  return AXB_OK;
}

int step_launch(const StepArgs& a, cudaStream_t s) {
  AXB_CHECK_ARG(a.B >= 1 && a.B <= kStepMaxM, "step: batch %d out of range", a.B);
  // the shapes the kernel's fixed shared-memory layout is sized for
  AXB_CHECK_ARG(a.group == 64 || a.group == 128, "step: group %d", a.group);
  AXB_CHECK_ARG(a.d > 0 && a.d % 128 == 0 && a.F % 64 == 0 && a.V > 0, "step: bad dims (%d, %d, %d)", a.d, a.F, a.V);
  AXB_CHECK_ARG((a.hd == 64 || a.hd == 128) && a.Hkv > 0 && a.Hq % a.Hkv == 0 && a.Hq / a.Hkv <= kMaxRepS,
                "step: bad heads (%d, %d, %d)", a.Hq, a.Hkv, a.hd);
  AXB_CHECK_ARG(a.plan.smem > 0 && a.plan.smem <= kSmemMax && a.plan.nslots >= 2 && a.plan.nslots <= kMaxSlots &&
                    a.plan.slot_kb >= 4 && a.plan.slot_kb % 4 == 0 &&
                    a.plan.union_bytes % 128 == 0,
                "step: no shared-memory plan for this model");
  AXB_CHECK_ARG(stage_bytes(a.B, a.d) + kSPartBytes <= a.plan.union_bytes,
                "step: d_model %d too large for the staged activations at batch %d", a.d, a.B);
  AXB_CHECK_ARG(a.plan.attn_cap >= kBoxRows && a.plan.attn_cap % kBoxRows == 0 &&
                    attn_layout(a.kv_type, a.hd, a.kv_group, a.plan.attn_cap, a.Hq / a.Hkv).bytes <= a.plan.union_bytes,
                "step: attention chunk %d does not fit", a.plan.attn_cap);
  AXB_CHECK_ARG(a.spin_limit > 0 && a.mbar_limit > 0, "step: wait limits must be positive");
  AXB_CHECK_ARG(a.L >= 0 && 4 * a.L + 1 < 511, "step: %d layers (the phase flags allow 127)", a.L);
  AXB_CHECK_ARG(a.lm_w && a.lm_s && a.ln_f && a.emb_w && a.emb_s && a.rope && a.tokens && a.params && a.err && a.h &&
                    a.logits && a.amax && a.partials && a.keys && a.exit_cnt &&
                    (a.L == 0 || (a.layers && a.qkv && a.attn && a.sw && a.part_o && a.part_ml && a.attn_cnt)),
                "step: null pointer in the step arguments");
  AXB_CHECK_ARG((reinterpret_cast<uintptr_t>(a.lm_w) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.lm_s) & 15) == 0,
                "step: lm_head words and scales must be 16-byte aligned");
  if (int rc = step_prepare()) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms());
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = a.plan.smem;
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
