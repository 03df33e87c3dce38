// W4A16 GEMM on the 5th-generation tensor cores (tcgen05) for the token
// counts where the projection becomes a dense contraction: tree verification
// with many candidates, chunked prefill, decode batches of 16-64.
//
// Replaces qmm_q4_marlin (axiomlm/kernels/quant.py:664-684; Metal
// qmm_q4_marlin_apple_kernel :2404, BM=32 x BN=16 simdgroup tiles) for
// M > 16.  At 64 tokens a Q4 weight byte feeds 256 flops, the B200's ridge:
// the legacy warp-level mma path cannot keep up with HBM there.
//
// One CTA computes a 128-row x NT-token tile of y (NT = 32 or 64: the token
// count rounded up) over a K range (split-K across CTAs when the rows alone
// do not fill the GPU), with its warps specialized and linked by mbarriers --
// no CTA-wide barrier in the k loop:
//  * warp 8 streams the weights, two 64-wide k-blocks per slot, into a
//    4-slot ring with one bulk copy per row tile (a q4t tile's k range is
//    contiguous); a slot is released as soon as the dequantizing warps have
//    read it;
//  * warp 10 streams the NT-token activation blocks into a 3-slot ring (one
//    copy per k-block), which a small pre-pass (tc_xlayout_kernel) has laid
//    out in the tensor core's canonical K-major order, zero rows past M (a
//    32-token width for M <= 32 halves this L2 traffic);
//  * warps 0-7 (one row tile each; scales read from global memory a chunk
//    ahead) dequantize the slot's weights to fp16 (the reference's values:
//    fp16((q - 8) s) symmetric, fp16(q s + b) affine) into one of two operand
//    stages, in the canonical no-swizzle layout with a 144-byte core-matrix
//    pitch along K (16-byte rows of 8 lanes land in distinct banks), then
//    signal the stage full;
//  * warp 9 owns the tensor memory; its lane 0 issues tcgen05.mma (M = 128,
//    N = NT, K = 16, fp32 accumulate) per stage and commits the stage's
//    completion to the operand stage and the activation slot;
//  * warps 0-7 finally read the accumulator with tcgen05.ld (warp w: lanes
//    32 (w % 4).., tokens (NT / 2) (w / 4)..) and store fp16 (+ bias), or
//    fp32 partials that tc_reduce_kernel sums in split order.
// Measured limits (B200): with the dequantization and the MMAs both removed,
// this copy-and-barrier skeleton alone streams about 2.4 TB/s; more
// dequantizing warps, deeper rings, larger copies, three operand stages and
// 256-row CTAs (halving the activation traffic) each left the time within a
// few percent, so the ceiling is the per-SM handling of the bulk copies and
// barrier hand-offs, not HBM.
// Every mbarrier wait is bounded; a wait that runs out records AXB_ETIMEOUT,
// raises the CTA's abort flag (the other roles stop at their next stage),
// waits (bounded) for the tensor core and the copies in flight, frees the
// tensor memory and returns.
#include <algorithm>

#include "axb_common.cuh"
#include "q4t.cuh"

namespace axb {

constexpr int kTcHalf = 128;              // MMA M: rows per accumulator
constexpr int kTcHalves = 1;              // 128-row accumulators per CTA
constexpr int kTcRows = kTcHalves * kTcHalf;  // weight rows per CTA
constexpr int kTcTiles = kTcRows / 16;    // q4t row tiles per CTA
constexpr int kTcTok = 64;                // largest MMA N (tokens per CTA)
constexpr int kTcKC = 64;                 // k per chunk (one q4t k-block; one operand stage)
constexpr int kTcSlotK = 2;               // k-blocks per weight slot
constexpr int kTcWSlots = 4;              // weight ring slots (released once dequantized)
constexpr int kTcXSlots = 3;              // activation ring slots, one k-block each (released when its MMAs are done)
constexpr int kTcStages = 2;              // dequantized operand stages
constexpr int kTcDqWarps = kTcTiles;      // dequantize / epilogue warps
constexpr int kTcWarpW = kTcDqWarps, kTcWarpMma = kTcDqWarps + 1, kTcWarpX = kTcDqWarps + 2;
constexpr int kTcThreads = 32 * (kTcDqWarps + 3);
constexpr int kTcX = kTcTok * kTcKC * 2;          // 8 KB activation block per k-block (64 token rows)
constexpr int kTcWSlot = kTcTiles * kTcSlotK * 512;  // q4t words of the CTA's tiles per slot
constexpr int kTcXSlot = kTcX;
constexpr int kTcAK = 144;                // operand stage: core-matrix pitch along K (bytes)
constexpr int kTcAM = 8 * kTcAK;          // ... and along M (8-row groups)
constexpr int kTcAHalf = (kTcHalf / 8) * kTcAM;   // 18 KB per 128-row half
constexpr int kTcA = kTcHalves * kTcAHalf;
constexpr int kTcSmem = kTcWSlots * kTcWSlot + kTcXSlots * kTcXSlot + kTcStages * kTcA + 256;
constexpr uint32_t kTcWaitLimit = 1u << 24;
// instruction descriptor (kind::f16): D fp32, A and B fp16, both K-major,
// N (bits 17-22: N / 8), M = 128 (bits 24-28: M / 16)
__host__ __device__ constexpr uint32_t tc_idesc(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcHalf >> 4) << 24);
}

struct TcArgs {
  const uint32_t* words;
  const __half* scales;
  const __half* xl;  // activations in the canonical layout: [K / 64][8 KB]
  const __half* bias;
  __half* y;
  float* part;  // split-K partials [S][M][N] (summed by tc_reduce_kernel), or null
  int* err;
  int N, K, M, ldy, G;
};

// byte offset of element (n, k) of an activation block: core matrices of 8
// rows x 16 bytes, 128 B apart along K (leading byte offset), 1024 B apart
// along N (stride byte offset); the first NT rows are the first NT * 128 bytes
__device__ __forceinline__ uint32_t tc_off(int r, int k) {
  return (uint32_t)((r >> 3) * 1024 + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}
// byte offset of 16-byte row piece (r, k .. k + 7) of a 128-row operand half
__device__ __forceinline__ uint32_t tc_aoff(int r, int k) {
  return (uint32_t)((r >> 3) * kTcAM + (k >> 3) * kTcAK + (r & 7) * 16);
}

// shared-memory matrix descriptor: start >> 4, leading (K) and stride (M/N)
// byte offsets >> 4, descriptor version 1 (bits 46-47), no swizzle
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
         ((uint64_t)1 << 46);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 16 consecutive fp32 accumulator columns of this warp's 32 lanes
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// activations x (M x K, row pitch ldx) -> [K / 64] blocks of 64 tokens x 64 k
// in the canonical K-major layout, zero rows past M
__global__ void tc_xlayout_kernel(const __half* __restrict__ x, int M, int K, int ldx, __half* __restrict__ xl) {
  const int KB = K / kTcKC;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < KB * kTcTok * 8; i += gridDim.x * blockDim.x) {
    const int kb = i / (kTcTok * 8), n = (i / 8) % kTcTok, kc = i % 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (n < M) v = *reinterpret_cast<const uint4*>(x + (size_t)n * ldx + kb * kTcKC + kc * 8);
    *reinterpret_cast<uint4*>(reinterpret_cast<char*>(xl) + (size_t)kb * kTcX + tc_off(n, kc * 8)) = v;
  }
}

template <bool SYM, int GB, int NT>
__global__ void __launch_bounds__(kTcThreads) qgemm_tc_kernel(const TcArgs a) {
  constexpr int kCols = kTcHalves * NT < 32 ? 32 : kTcHalves * NT;  // tensor-memory columns: each half's NT fp32 tokens
  constexpr uint32_t kIdesc = tc_idesc(NT);
  extern __shared__ __align__(1024) char smem[];
  char* wring = smem;                                  // [slot][16 tiles][kTcSlotK k-blocks] q4t words
  char* xring = wring + kTcWSlots * kTcWSlot;          // [slot][NT rows of an 8 KB block] activations
  char* stA = xring + kTcXSlots * kTcXSlot;            // [stage][2 halves][kTcAHalf] dequantized weights
  uint64_t* wfull = reinterpret_cast<uint64_t*>(stA + kTcStages * kTcA);  // [slot] copies landed
  uint64_t* wempty = wfull + kTcWSlots;                // [slot] dequantized by every warp
  uint64_t* xfull = wempty + kTcWSlots;                // [slot] copies landed
  uint64_t* xempty = xfull + kTcXSlots;                // [slot] its MMAs are done
  uint64_t* afull = xempty + kTcXSlots;                // [stage] dequantized
  uint64_t* aempty = afull + kTcStages;                // [stage] its MMAs are done
  uint64_t* done = aempty + kTcStages;                 // every MMA is done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int tid = threadIdx.x, wid = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int KB = a.K / kTcKC, Nt = (a.N + 15) / 16;
  const int rb = blockIdx.x, S = gridDim.y, sp = blockIdx.y;
  const int kb0 = (int)((long long)sp * KB / S), kb1 = (int)((long long)(sp + 1) * KB / S);
  const int nch = kb1 - kb0;
  const int ntiles = min(kTcTiles, Nt - rb * kTcTiles);

  if (wid == kTcWarpMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < kTcWSlots; ++s) {
      mbar_init(wfull + s, 1);
      mbar_init(wempty + s, kTcDqWarps);
    }
    for (int s = 0; s < kTcXSlots; ++s) {
      mbar_init(xfull + s, 1);
      mbar_init(xempty + s, 1);
    }
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(afull + s, kTcDqWarps);
      mbar_init(aempty + s, 1);
    }
    mbar_init(done, 1);
    *abort_s = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int nfill = (nch + kTcSlotK - 1) / kTcSlotK;
  if (wid == kTcWarpW || wid == kTcWarpX) {
    // ---- producers: the weight warp streams the row tiles' words (a copy per
    // tile and slot), the activation warp the NT-row activation blocks
    const bool isw = wid == kTcWarpW;
    const int nsl = isw ? kTcWSlots : kTcXSlots, nf = isw ? nfill : nch;
    uint64_t* fullb = isw ? wfull : xfull;
    uint64_t* emptyb = isw ? wempty : xempty;
    int f = 0;
    for (; f < nf; ++f) {
      const int sl = f % nsl;
      if (f >= nsl) {
        // every lane that issues a copy into the slot observes its release
        const bool got = __all_sync(0xffffffffu, mbar_wait(emptyb + sl, (uint32_t)((f / nsl - 1) & 1),
                                                           kTcWaitLimit));
        if (!got || *abort_s) {
          if (lane == 0 && !got) {
            *abort_s = 1;
            atomicExch(a.err, AXB_ETIMEOUT);
          }
          break;
        }
      }
      const int kb = kb0 + (isw ? f * kTcSlotK : f), nk = isw ? min(kTcSlotK, kb1 - kb) : 1;
      if (lane == 0) {
        fence_proxy_async();
        mbar_expect_tx(fullb + sl, (uint32_t)(isw ? nk * ntiles * 512 : NT * 128));
      }
      __syncwarp();
      if (isw && lane < ntiles) {
        const int tile = rb * kTcTiles + lane;
        bulk_g2s(wring + sl * kTcWSlot + lane * (kTcSlotK * 512),
                 reinterpret_cast<const char*>(a.words) + ((size_t)tile * KB + kb) * 512, nk * 512, fullb + sl);
      } else if (!isw && lane == 0) {
        bulk_g2s(xring + sl * kTcXSlot, reinterpret_cast<const char*>(a.xl) + (size_t)kb * kTcX, NT * 128,
                 fullb + sl);
      }
    }
    // no copy may still be landing when the CTA exits: wait for the last fill of every slot
    if (lane == 0)
      for (int q = max(0, f - nsl); q < f; ++q)
        if (!mbar_wait(fullb + q % nsl, (uint32_t)((q / nsl) & 1), kTcWaitLimit)) {
          *abort_s = 1;
          atomicExch(a.err, AXB_ETIMEOUT);
        }
  } else if (wid == kTcWarpMma) {
    // ---- MMA issue (lane 0): both 128-row halves of one operand stage per k-block
    if (lane == 0) {
      for (int c = 0; c < nch; ++c) {
        const int sl = c % kTcXSlots, st = c % kTcStages;
        const bool got = mbar_wait(afull + st, (uint32_t)((c / kTcStages) & 1), kTcWaitLimit) &&
                         mbar_wait(xfull + sl, (uint32_t)((c / kTcXSlots) & 1), kTcWaitLimit);
        if (!got || *abort_s) {
          if (!got) {
            *abort_s = 1;
            atomicExch(a.err, AXB_ETIMEOUT);
          }
          break;
        }
        tc_fence_after();
        const uint32_t sb = smem_u32(xring + sl * kTcXSlot);
#pragma unroll
        for (int h = 0; h < kTcHalves; ++h) {
          const uint32_t sa = smem_u32(stA + st * kTcA + h * kTcAHalf);
#pragma unroll
          for (int ks = 0; ks < kTcKC / 16; ++ks)
            tc_mma(tmem + (uint32_t)(h * NT), tc_desc(sa + 2 * kTcAK * ks, kTcAK, kTcAM),
                   tc_desc(sb + 256 * ks, 128, 1024), kIdesc, (c > 0 || ks > 0) ? 1u : 0u);
        }
        tc_commit(aempty + st);
        tc_commit(xempty + sl);
      }
      tc_commit(done);  // covers every MMA issued above
    }
    __syncwarp();
  } else {
    // ---- dequantize: warp w takes row tile w; scales come straight from
    // global memory, loaded one chunk ahead
    const int ng = a.K / a.G;
    const int tile = min(rb * kTcTiles + wid, Nt - 1);  // rows past N: any valid tile
    auto load_sc = [&](int c) {
      const int grp = ((kb0 + c) * kTcKC) / a.G;
      uint2 sc;
      if (SYM) {
        sc.x = __ldg(reinterpret_cast<const uint32_t*>(a.scales) + ((size_t)tile * ng + grp) * 8 + g);
        sc.y = 0;
      } else {
        sc = __ldg(reinterpret_cast<const uint2*>(a.scales) + ((size_t)tile * ng + grp) * 8 + g);
      }
      return sc;
    };
    uint2 sc_cur = nch > 0 ? load_sc(0) : make_uint2(0, 0);
    for (int c = 0; c < nch; ++c) {
      const int fl = c / kTcSlotK, sl = fl % kTcWSlots, st = c % kTcStages, hk = c % kTcSlotK;
      const uint2 sc_nxt = c + 1 < nch ? load_sc(c + 1) : sc_cur;
      // every lane reads the slot and writes the stage: each observes both barriers
      bool mine = mbar_wait(wfull + sl, (uint32_t)((fl / kTcWSlots) & 1), kTcWaitLimit);
      if (mine && c >= kTcStages) mine = mbar_wait(aempty + st, (uint32_t)((c / kTcStages - 1) & 1), kTcWaitLimit);
      const bool got = __all_sync(0xffffffffu, mine);
      if (!got || *abort_s) {
        if (lane == 0 && !got) {
          *abort_s = 1;
          atomicExch(a.err, AXB_ETIMEOUT);
        }
        break;
      }
      const char* slot = wring + sl * kTcWSlot;
      char* A = stA + st * kTcA + (wid >> 3) * kTcAHalf;
      {
        const uint4 wv = *reinterpret_cast<const uint4*>(slot + wid * (kTcSlotK * 512) + hk * 512 + lane * 16);
        const uint2 sc = sc_cur;
        const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t rg[4][2], rg8[4][2];  // [word j][f0 / f2] rows g and g + 8
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t fr[4];
          if (SYM) {
            unpack_word<8>(w4[j], fr);  // exact (q - 8) as fp16
            const __half2 s01 = u32_as_h2(sc.x);
            const __half2 sg = __half2half2(__low2half(s01)), sg8 = __half2half2(__high2half(s01));
            fr[0] = h2_as_u32(__hmul2(u32_as_h2(fr[0]), sg));
            fr[1] = h2_as_u32(__hmul2(u32_as_h2(fr[1]), sg8));
            fr[2] = h2_as_u32(__hmul2(u32_as_h2(fr[2]), sg));
            fr[3] = h2_as_u32(__hmul2(u32_as_h2(fr[3]), sg8));
          } else {
            unpack_word<0>(w4[j], fr);  // q as fp16
            const __half2 p0 = u32_as_h2(sc.x), p1 = u32_as_h2(sc.y);  // (s[g], b[g]), (s[g+8], b[g+8])
            const __half2 sg = __half2half2(__low2half(p0)), bg = __half2half2(__high2half(p0));
            const __half2 sg8 = __half2half2(__low2half(p1)), bg8 = __half2half2(__high2half(p1));
            fr[0] = h2_as_u32(__hfma2(u32_as_h2(fr[0]), sg, bg));
            fr[1] = h2_as_u32(__hfma2(u32_as_h2(fr[1]), sg8, bg8));
            fr[2] = h2_as_u32(__hfma2(u32_as_h2(fr[2]), sg, bg));
            fr[3] = h2_as_u32(__hfma2(u32_as_h2(fr[3]), sg8, bg8));
          }
          // f0 / f2: row g, k = 16 t4 + 4 j + {0, 1} / {2, 3}; f1 / f3: row g + 8
          rg[j][0] = fr[0];
          rg[j][1] = fr[2];
          rg8[j][0] = fr[1];
          rg8[j][1] = fr[3];
        }
        const int r = (wid & 7) * 16 + g, k = 16 * t4;
        *reinterpret_cast<uint4*>(A + tc_aoff(r, k)) = make_uint4(rg[0][0], rg[0][1], rg[1][0], rg[1][1]);
        *reinterpret_cast<uint4*>(A + tc_aoff(r + 8, k)) = make_uint4(rg8[0][0], rg8[0][1], rg8[1][0], rg8[1][1]);
        *reinterpret_cast<uint4*>(A + tc_aoff(r, k + 8)) = make_uint4(rg[2][0], rg[2][1], rg[3][0], rg[3][1]);
        *reinterpret_cast<uint4*>(A + tc_aoff(r + 8, k + 8)) = make_uint4(rg8[2][0], rg8[2][1], rg8[3][0], rg8[3][1]);
      }
      fence_proxy_async();  // the tensor core reads the stage through the async proxy
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(afull + st);
        if (hk == kTcSlotK - 1 || c == nch - 1) mbar_arrive(wempty + sl);  // the slot's words are consumed
      }
      sc_cur = sc_nxt;
    }
  }

  // ---- every MMA of the CTA is done (or the CTA gave up): read the accumulators
  if (wid < kTcDqWarps) {
    const bool got = __all_sync(0xffffffffu, mbar_wait(done, 0u, kTcWaitLimit));
    if (!got && lane == 0) {
      *abort_s = 1;
      atomicExch(a.err, AXB_ETIMEOUT);
    }
  }
  __syncthreads();
  const bool ok = *abort_s == 0 && nch > 0;
  tc_fence_after();
  // ---- epilogue (warps 0-15): warp w reads half w / 8, accumulator lanes 32 (w % 4) .. (its
  // rows) and tokens (NT / 2) ((w / 4) % 2) ..; fp16 (+ bias), or the split's fp32 partial
  if (wid < kTcDqWarps && ok) {
    const int quarter = wid & 3, cpart = (wid >> 2) & 1, h = wid >> 3;
    const int row = rb * kTcRows + h * kTcHalf + 32 * quarter + lane;
    const bool live = row < a.N;
    const float bsum = (S == 1 && a.bias && live) ? __half2float(a.bias[row]) : 0.f;
#pragma unroll
    for (int j = 0; j < NT / 32; ++j) {
      const int n0 = cpart * (NT / 2) + 16 * j;
      uint32_t r[16];
      tc_ld16(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(h * NT + n0), r);
      if (live) {
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int n = n0 + q;
          if (n < a.M) {
            if (S == 1)
              a.y[(size_t)n * a.ldy + row] = __float2half_rn(__uint_as_float(r[q]) + bsum);
            else
              a.part[((size_t)sp * a.M + n) * a.N + row] = __uint_as_float(r[q]);
          }
        }
      }
    }
  }
  // ---- tensor memory is no longer needed
  tc_fence_before();
  __syncthreads();
  if (wid == kTcWarpMma)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

// split-K: y[m][n] = fp16(sum over splits in order + bias)
__global__ void tc_reduce_kernel(const float* __restrict__ part, int S, int M, int N, const __half* __restrict__ bias,
                                 __half* __restrict__ y, int ldy) {
  const size_t total = (size_t)M * N;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(i / N), n = (int)(i % N);
    float o = 0.f;
    for (int q = 0; q < S; ++q) o += __ldcg(part + (size_t)q * total + i);
    if (bias) o += __half2float(bias[n]);
    y[(size_t)m * ldy + n] = __float2half_rn(o);
  }
}

// splits of K so that the CTAs (two per SM) fill the GPU in about one wave
int tc_splits(int N, int K) {
  const int rbs = (N + kTcRows - 1) / kTcRows, KB = K / kTcKC;
  int S = (2 * num_sms() + rbs - 1) / rbs;
  S = std::max(1, std::min(S, std::min(16, KB / 2)));
  return S;
}

}  // namespace axb

using namespace axb;

extern "C" {

// workspace: error word | activations in the canonical layout | split-K partials
static size_t tc_xl_bytes(int K) { return (size_t)(K / kTcKC) * kTcX; }

size_t axb_qgemm_tc_workspace_bytes(int N, int K, int M) {
  (void)M;
  if (N <= 0 || K <= 0 || K % kTcKC) return 0;
  const int S = tc_splits(N, K);
  const size_t part = S > 1 ? (size_t)S * kTcTok * N * sizeof(float) : 0;
  return 256 + tc_xl_bytes(K) + part;
}

int axb_qgemm_tc(const axb_qgemm_desc* d, void* stream) {
  AXB_CHECK_ARG(d, "qgemm_tc: null descriptor");
  AXB_CHECK_ARG(d->fmt == AXB_W_Q4T_SYM || d->fmt == AXB_W_Q4T_AFFINE, "qgemm_tc: unsupported fmt %d", d->fmt);
  AXB_CHECK_ARG((d->fmt == AXB_W_Q4T_SYM && d->group == 128) || (d->fmt == AXB_W_Q4T_AFFINE && d->group == 64),
                "qgemm_tc: (fmt %d, group %d) not built", d->fmt, d->group);
  AXB_CHECK_ARG(d->N > 0 && d->K > 0 && d->K % d->group == 0 && d->K % kTcKC == 0, "qgemm_tc: bad N/K (%d, %d)",
                d->N, d->K);
  AXB_CHECK_ARG(d->M >= 1 && d->M <= kTcTok, "qgemm_tc: M=%d out of [1, %d]", d->M, kTcTok);
  AXB_CHECK_ARG(d->epilogue == AXB_EPI_STORE && d->norm_w == nullptr && !d->gate_up_interleave,
                "qgemm_tc: only the plain store epilogue (+bias) is built");
  AXB_CHECK_ARG(d->words && d->scales && d->x && d->y && d->ldx >= d->K && d->ldy >= d->N,
                "qgemm_tc: bad pointers / strides");
  AXB_CHECK_ARG((reinterpret_cast<uintptr_t>(d->x) & 15) == 0 && d->ldx % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(d->words) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(d->scales) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(d->workspace) & 255) == 0,
                "qgemm_tc: x, words and scales must be 16-byte aligned (workspace 256), ldx a multiple of 8");
  const size_t need = axb_qgemm_tc_workspace_bytes(d->N, d->K, d->M);
  AXB_CHECK_ARG(d->workspace && d->workspace_bytes >= need, "qgemm_tc: workspace %zu < %zu bytes",
                d->workspace_bytes, need);
  static DeviceOnce attr_once;  // per device: alternating between GPUs does not repeat the set-up
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_once.done(dev)) {
    cudaError_t e = cudaSuccess;
    const void* ks[4] = {(const void*)qgemm_tc_kernel<true, 2, 32>, (const void*)qgemm_tc_kernel<true, 2, 64>,
                         (const void*)qgemm_tc_kernel<false, 1, 32>, (const void*)qgemm_tc_kernel<false, 1, 64>};
    for (int i = 0; i < 4 && e == cudaSuccess; ++i)
      e = cudaFuncSetAttribute(ks[i], cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    if (e != cudaSuccess) return cuda_status(e, "qgemm_tc attribute");
    attr_once.set(dev);
  }
  const int S = tc_splits(d->N, d->K);
  const int rbs = (d->N + kTcRows - 1) / kTcRows;
  char* ws = (char*)d->workspace;
  TcArgs a;
  a.words = (const uint32_t*)d->words;
  a.scales = (const __half*)d->scales;
  a.xl = (const __half*)(ws + 256);
  a.bias = (const __half*)d->bias;
  a.y = (__half*)d->y;
  a.err = (int*)ws;
  a.part = S > 1 ? (float*)(ws + 256 + tc_xl_bytes(d->K)) : nullptr;
  a.N = d->N;
  a.K = d->K;
  a.M = d->M;
  a.ldy = d->ldy;
  a.G = d->group;
  {
    const int pieces = (d->K / kTcKC) * kTcTok * 8;
    tc_xlayout_kernel<<<std::min((pieces + 255) / 256, 8 * num_sms()), 256, 0, (cudaStream_t)stream>>>(
        (const __half*)d->x, d->M, d->K, d->ldx, (__half*)(ws + 256));
    if (int rc = launch_status("qgemm_tc layout")) return rc;
  }
  dim3 grid(rbs, S);
  const bool narrow = d->M <= 32;  // one 32-token MMA width: half the activation traffic
  if (d->fmt == AXB_W_Q4T_SYM) {
    if (narrow)
      qgemm_tc_kernel<true, 2, 32><<<grid, kTcThreads, kTcSmem, (cudaStream_t)stream>>>(a);
    else
      qgemm_tc_kernel<true, 2, 64><<<grid, kTcThreads, kTcSmem, (cudaStream_t)stream>>>(a);
  } else {
    if (narrow)
      qgemm_tc_kernel<false, 1, 32><<<grid, kTcThreads, kTcSmem, (cudaStream_t)stream>>>(a);
    else
      qgemm_tc_kernel<false, 1, 64><<<grid, kTcThreads, kTcSmem, (cudaStream_t)stream>>>(a);
  }
  if (int rc = launch_status("qgemm_tc")) return rc;
  if (S > 1) {
    const size_t total = (size_t)d->M * d->N;
    const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)num_sms() * 8);
    tc_reduce_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(a.part, S, d->M, d->N, a.bias, a.y, d->ldy);
    return launch_status("qgemm_tc reduce");
  }
  return AXB_OK;
}

/* Synchronizes `stream`; AXB_ETIMEOUT (and clears it) when a bounded wait of
 * an earlier axb_qgemm_tc on this workspace ran out. */
int axb_qgemm_tc_status(void* workspace, void* stream) {
  AXB_CHECK_ARG(workspace, "qgemm_tc_status: null workspace");
  int h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, workspace, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_status(e, "qgemm_tc_status");
  if (h != 0) {
    const int z = 0;
    cudaMemcpy(workspace, &z, sizeof(int), cudaMemcpyHostToDevice);
    axb::set_error("qgemm_tc: a bounded tensor-core wait ran out");
    return AXB_ETIMEOUT;
  }
  return AXB_OK;
}

}  // extern "C"
