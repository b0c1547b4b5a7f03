// wr_fused.cu — the fused decode-time MoE layer for 1..4 tokens, streamed
// through shared memory with bulk (TMA) copies at HBM bandwidth.
//
// Replaces warp-route's k_fused_moe / k_fused_moe_batched
// (src/fused_moe.cu:76-227, src/fused_moe_batched.cu:66-180): the same
// router -> top-K -> SwiGLU over the selected experts -> weighted combine,
// spread over every SM instead of one warp.
//
// One kernel per layer, k_fused_stream: one persistent CTA per SM (227 KB
// shared memory), launched cooperatively with programmatic dependent launch:
// it waits (griddepcontrol.wait) for the previous kernel on the stream, then
// lets the next one start launching, so back-to-back layers do not pay a
// full launch gap.
//   router   every warp of the grid takes (token, 8-row batch, segment)
//            items of the router sums; one grid-wide counter, then each CTA
//            adds the 8 segment sums of every logit in order and selects;
//   warps 0-7  consumers: dot products out of shared memory;
//   warp 8     producer: lane 0 issues cp.async.bulk copies into a ring of
//              5-12 stages of up to 32 KB (mbarrier full/empty pairs, L2
//              evict-first) and never waits on the math;
//   warp 9     publisher: signals grid-wide when this CTA's activations of a
//              slot are complete (below).
// Every copy is a contiguous run of weight rows (up to 32 KB): B200's TMA
// streams at HBM bandwidth only with large contiguous copies.
//
// The selected experts become "slots"; the layer is then two matvecs:
//   phase A  rows p = slot*I + i of [Wg; Wu] . x -> act[p] =
//            w_slot * silu(g) * u (fp32 workspace, one value per token).
//            A stage holds GA gate rows and the same GA up rows (two copies).
//            Groups of GA row pairs are dealt to the CTAs round robin, slot
//            after slot, so slot 0's activations are complete about halfway.
//   phase B  out[h] = sum over slots of Wd_slot[h, :] . act[slot, :].  The
//            slot's activations sit in shared memory in windows of at most
//            16384 columns; a stage is GB rows of one window.  Output rows
//            are split evenly over the CTAs.
// Phase A rows are owned by one warp each (the CTA's k-th row pair by warp
// k % 8), which computes the whole dot product.  Phase B rows are read by
// PB warps (1 or 2), each taking a column slice; every warp adds into its
// own row accumulators, summed in warp order at the end.  Only the warps
// that read a stage wait for it and release it (the producer pre-arrives
// for the others), so the warps work on different stages at once.  Because
// a warp skips the stages it does not read, a parity wait alone could
// mistake a later use of the ring slot for the one it wants; the producer
// therefore tags each slot with the number of the stage it holds, and a
// reader waits for its tag before its parity wait (the tag is written only
// after the slot's previous use was released, so the parity is then
// unambiguous).  No partial sum crosses a warp except in the fixed final
// sum, so results are deterministic (fixed lane order and trees, fixed
// slot/window order, no floating-point atomics).
// Completion of slot s: each consumer warp arrives on a per-slot mbarrier
// once its share of slot s is written; the publisher warp waits on it and
// adds the CTA to the grid-wide counter of slot s with one GPU-scope
// release.  Phase B of slot s starts once that counter holds every CTA
// (bounded spin); the producer keeps prefetching phase-B weights meanwhile.
#include <cuda_runtime.h>

#include <mutex>
#include <type_traits>

#include "wr_common.cuh"
#include "wr_internal.h"
#include "wr_router.cuh"

namespace wr {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 64;  // + producer warp + publisher warp
constexpr int kTargetStage = 32 * 1024;          // stage size aimed for
constexpr int kMaxStageBytes = 32 * 1024;
constexpr int kMaxStages = 12;
constexpr int kWideStageBytes = 48 * 1024;   // two-row-pair / phase-B stages (make_plan_v)
constexpr int kPairStageBytes = 52 * 1024;   // ... when that makes a window two phase-B stages
constexpr int kWideWindowBytes = 24 * 1024;  // their activation windows, at most
constexpr int kSmemBytes = 232448;  // 227 KB: the sm_100 per-CTA opt-in maximum
constexpr int kMiscBytes = 8192;
constexpr int kMiscOff = kSmemBytes - kMiscBytes;
constexpr int kMaxNT = 4;
constexpr int kMaxRowsPerStage = 32;
constexpr int kRowsPerWarp = kMaxRowsPerStage / kConsumerWarps;  // owned rows per warp per stage
// Room for at least 4 of the largest stages.
constexpr int kVecMaxBytes = kMiscOff - 4 * kMaxStageBytes;  // x / activation window
static_assert(kVecMaxBytes % 64 == 0, "vector region must keep 64-byte alignment");

// Offsets inside the misc region (at the end of shared memory).
constexpr int kOffBars = 0;        // full[12], empty[12]
constexpr int kOffAbort = 256;     // int
constexpr int kOffNSlots = 260;    // int
constexpr int kOffSlotTag = 264;   // int [12]: stage number each ring slot currently holds
constexpr int kOffEpoch = 320;     // uint32: this launch's all-reduce epoch
constexpr int kOffSlotE = 512;     // int [64]: local expert of each slot
constexpr int kOffSlotW = 768;     // float [64 * NT]: routing weight (0: not routed)
constexpr int kOffTokIds = 1792;   // int [NT * 64]
constexpr int kOffTokW = 2816;     // float [NT * 64]
constexpr int kOffSlotBar = 3840;  // mbarrier [64]: the W consumer warps are done with slot s
constexpr int kOffLogits = 4352;   // float [NT * 64]: router logits
constexpr int kMaxActBufs = 16;    // phase B: activation window buffers, at most
constexpr int kOffActBars = 5376;  // mbarrier act_full[16], act_empty[16]
static_assert(kOffBars + 8 * (2 * kMaxStages) <= kOffAbort, "misc");
static_assert(kOffLogits + 4 * kMaxNT * kMaxExperts <= kOffActBars, "misc");
constexpr int kOffLParts = 5632;   // float [T][segment][E]: a small router's partial sums
constexpr int kLPartsBytes = 512;  // (<= 2 items per consumer warp: T * E <= 16)
static_assert(kOffActBars + 16 * kMaxActBufs <= kOffLParts, "misc");
static_assert(kOffLParts + kLPartsBytes <= kMiscBytes, "misc");
static_assert(kOffTokW + 4 * kMaxNT * kMaxExperts <= kOffSlotBar, "misc");
static_assert(kOffSlotBar + 8 * kMaxExperts <= kOffLogits, "misc");
static_assert(kOffLogits + 4 * kMaxNT * kMaxExperts <= kMiscBytes, "misc");

// Workspace: control words, router partial sums, activations.
constexpr int kSyncExit = 1;      // CTAs that have finished (self-reset)
constexpr int kSyncStatus = 2;    // DEV_TIMEOUT_* bits
constexpr int kSyncRouter = 3;    // CTAs whose router partial sums are written
constexpr int kSyncSlot0 = 64;    // [64 + s]: CTAs whose slot-s activations are all written
constexpr size_t kSyncBytes = kWsControlBytes;
static_assert((kSyncSlot0 + kMaxExperts) * 4 <= (int)kSyncBytes, "control words");
// router partial sums [T][segment][E] fp32
constexpr size_t kRouterBytes = (size_t)kMaxNT * kRouterSegments * kMaxExperts * 4;  // 8 KB
constexpr size_t kActOffset = kSyncBytes + kRouterBytes;

// Named barrier 1: the eight consumer warps.
constexpr int kBarConsumers = 1;

// Stage geometry, computed once on the host.
struct Plan {
  int GA;    // phase A: row pairs per stage
  int CWA;   // phase A: columns per stage (H when whole rows fit)
  int WB;    // phase B: activation window width (columns of one slot)
  int nwin;  // phase B: windows per slot
  int GB;    // phase B: rows per stage
  int SB;    // stage bytes
  int nst;   // ring stages
  int PB;      // phase B: warps per row, each taking a column slice (1, 2, 4 or 8)
  int orderA;  // phase A group order (kOrderRoundRobin / kOrderRanges)
  int localR;  // router: every CTA computes all partial sums itself (small routers)
  int NBM;     // phase B: most output rows one CTA holds
  int RA;      // float offset of the per-warp row accumulators [W][NBM][NT] in the vector region
  int AOFF;    // float offset of the activation window buffers in the vector region (0: they
               // overlap x, so the first window may only land once phase A is over)
  int CB;      // activation window buffers (1 .. kMaxActBufs)
  int WBF;     // floats per activation window buffer (WB * NT, 64-byte multiple)
};

struct FusedArgs {
  const void* x;
  const uint8_t* wbuf;
  float* out;
  int32_t* ids_out;
  float* w_out;
  const void* gate_w;   // [E][H]
  const float* bias;    // [E] or null
  float* rparts;        // [T][kRouterSegments][E] router partial sums (workspace)
  float* act;
  uint32_t* sync;
  int E, H, I, K, T;
  int ep_first, ep_num;
  Layout lay;
  Plan pl;
  CommView comm;  // comm.world == 0: no all-reduce (a one-rank communicator still runs it)
  Residual res;   // res.x == null: out = layer(x); else out = x + layer(x) (+ next_x)
};

WR_DEVINL int64_t split_lo(int64_t n, int i, int parts) { return (n * i) / parts; }

// Phase A dot products of one gate row and one up row over chunks [j0, j1)
// (16-byte chunks of VEC elements starting at column c0) against x.
template <typename Tw, int NT>
WR_DEVINL void dot_pair(const uint4* __restrict__ gp, const uint4* __restrict__ up,
                        const float* __restrict__ xs, int H, int c0, int j0, int j1, int lane,
                        float (&g)[NT], float (&u)[NT]) {
  constexpr int VEC = Chunk<Tw>::kVec;
  float g1[NT], u1[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) g1[t] = u1[t] = 0.0f;
#pragma unroll 4
  for (int j = j0 + lane; j < j1; j += 32) {
    float gf[VEC], uf[VEC];
    Chunk<Tw>::widen(gp[j], gf);
    Chunk<Tw>::widen(up[j], uf);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float4* xv = reinterpret_cast<const float4*>(xs + t * H + c0 + j * VEC);
#pragma unroll
      for (int q4 = 0; q4 < VEC / 4; ++q4) {
        const float4 x4 = xv[q4];
        float& ga = (q4 & 1) ? g1[t] : g[t];
        float& ua = (q4 & 1) ? u1[t] : u[t];
        ga = fmaf(gf[4 * q4 + 0], x4.x, ga);
        ga = fmaf(gf[4 * q4 + 1], x4.y, ga);
        ga = fmaf(gf[4 * q4 + 2], x4.z, ga);
        ga = fmaf(gf[4 * q4 + 3], x4.w, ga);
        ua = fmaf(uf[4 * q4 + 0], x4.x, ua);
        ua = fmaf(uf[4 * q4 + 1], x4.y, ua);
        ua = fmaf(uf[4 * q4 + 2], x4.z, ua);
        ua = fmaf(uf[4 * q4 + 3], x4.w, ua);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    g[t] += g1[t];
    u[t] += u1[t];
  }
}

// Two fp32 multiply-adds with bf16 inputs: acc += lo(w) * lo(x), then
// acc += hi(w) * hi(x).  A bf16 product is exact in fp32 and each add rounds
// once, so this equals fmaf on the widened values; the mixed-precision FMA
// just needs no separate widening instruction.
WR_DEVINL float fma2_bf16(uint32_t w, uint32_t x, float acc) {
  asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\t"
      "mov.b32 {wl, wh}, %1;\n\t"
      "mov.b32 {xl, xh}, %2;\n\t"
      "fma.rn.f32.bf16 %0, wl, xl, %0;\n\t"
      "fma.rn.f32.bf16 %0, wh, xh, %0;\n\t}"
      : "+f"(acc)
      : "r"(w), "r"(x));
  return acc;
}

// dot_pair for bf16 weights with x kept as bf16 chunks in shared memory
// ([NT][H]); same elements, order and accumulators as dot_pair, so the same
// fp32 results.
template <int NT>
WR_DEVINL void dot_pair_bf16(const uint4* __restrict__ gp, const uint4* __restrict__ up,
                             const uint4* __restrict__ xs, int H, int c0, int j0, int j1,
                             int lane, float (&g)[NT], float (&u)[NT]) {
  float g1[NT], u1[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) g1[t] = u1[t] = 0.0f;
#pragma unroll 4
  for (int j = j0 + lane; j < j1; j += 32) {
    const uint4 gw = gp[j], uw = up[j];
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const uint4 xv = xs[(t * H + c0) / 8 + j];
      g[t] = fma2_bf16(gw.y, xv.y, fma2_bf16(gw.x, xv.x, g[t]));
      u[t] = fma2_bf16(uw.y, xv.y, fma2_bf16(uw.x, xv.x, u[t]));
      g1[t] = fma2_bf16(gw.w, xv.w, fma2_bf16(gw.z, xv.z, g1[t]));
      u1[t] = fma2_bf16(uw.w, xv.w, fma2_bf16(uw.z, xv.z, u1[t]));
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    g[t] += g1[t];
    u[t] += u1[t];
  }
}

// Phase B dot products of nr <= R rows of one stage (row r's chunks start at
// wp + r * rs) over chunks j0, j0 + js, ... < nch against the activation
// window (layout [column][NT]): acc[r][t] += row r . act[:, t].  Each
// activation chunk is loaded from shared memory once for all the rows (one
// row at a time would read the fp32 window once per row: twice the bytes of
// the bf16 weights).  Per row, products alternate between two accumulators
// by chunk half (acc: even 4-element groups, acc1: odd), added at the end.
template <typename Tw, int NT, int R>
WR_DEVINL void dot_down_rows(const uint4* __restrict__ wp, int rs, const float* __restrict__ av,
                             int nch, int j0, int js, int nr, float (&acc)[R][NT]) {
  constexpr int VEC = Chunk<Tw>::kVec;
  constexpr int UF = R == 1 ? 4 : 2;  // loop unroll: loads of UF chunks in flight
  float acc1[R][NT];
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int t = 0; t < NT; ++t) acc1[r][t] = 0.0f;
  }
  if constexpr (VEC == 8 && NT == 1) {
    // bf16, one token: a lane's 8 activations are 32 bytes, so lanes 4 apart
    // would hit the same shared-memory banks.  Lanes with bit 2 set read the
    // upper 16 bytes first (and take the weight halves in the same swapped
    // order): each group of 8 lanes then covers 8 distinct bank slots.  Those
    // lanes fill acc and acc1 in swapped roles, and acc + acc1 is the same.
    const int hs = (j0 & 4) ? 4 : 0;
#pragma unroll UF
    for (int j = j0; j < nch; j += js) {
      const float4 aA = *reinterpret_cast<const float4*>(av + j * 8 + hs);
      const float4 aB = *reinterpret_cast<const float4*>(av + j * 8 + (4 - hs));
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (r < nr) {
          const uint4 w = wp[r * rs + j];
          const uint32_t wA0 = hs ? w.z : w.x, wA1 = hs ? w.w : w.y;
          const uint32_t wB0 = hs ? w.x : w.z, wB1 = hs ? w.y : w.w;
          acc[r][0] = fmaf(bf16lo(wA0), aA.x, acc[r][0]);
          acc[r][0] = fmaf(bf16hi(wA0), aA.y, acc[r][0]);
          acc[r][0] = fmaf(bf16lo(wA1), aA.z, acc[r][0]);
          acc[r][0] = fmaf(bf16hi(wA1), aA.w, acc[r][0]);
          acc1[r][0] = fmaf(bf16lo(wB0), aB.x, acc1[r][0]);
          acc1[r][0] = fmaf(bf16hi(wB0), aB.y, acc1[r][0]);
          acc1[r][0] = fmaf(bf16lo(wB1), aB.z, acc1[r][0]);
          acc1[r][0] = fmaf(bf16hi(wB1), aB.w, acc1[r][0]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r][0] += acc1[r][0];
  } else {
#pragma unroll UF
    for (int j = j0; j < nch; j += js) {
      float af[VEC * NT];
      const float4* a4p = reinterpret_cast<const float4*>(av + j * VEC * NT);
#pragma unroll
      for (int q4 = 0; q4 < VEC * NT / 4; ++q4) {
        const float4 a4 = a4p[q4];
        af[4 * q4 + 0] = a4.x;
        af[4 * q4 + 1] = a4.y;
        af[4 * q4 + 2] = a4.z;
        af[4 * q4 + 3] = a4.w;
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (r < nr) {
          float wf[VEC];
          Chunk<Tw>::widen(wp[r * rs + j], wf);
#pragma unroll
          for (int flat = 0; flat < VEC * NT; ++flat) {  // flat = q * NT + t
            float& ac = ((flat / NT) & 1) ? acc1[r][flat % NT] : acc[r][flat % NT];
            ac = fmaf(wf[flat / NT], af[flat], ac);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[r][t] += acc1[r][t];
    }
  }
}

template <int NT>
WR_DEVINL void warp_sum(float (&v)[NT]) {
#pragma unroll
  for (int t = 0; t < NT; ++t) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v[t] += __shfl_xor_sync(0xffffffffu, v[t], off);
  }
}

// Position in the ring: stage slot and the parity of its current use,
// advanced one stage at a time without divisions.
struct Cursor {
  int si;
  uint32_t ph;
  WR_DEVINL void next(int nst) {
    if (++si == nst) {
      si = 0;
      ph ^= 1u;
    }
  }
};

// Phase A work of one CTA.  Each slot's I row pairs form ng groups of GA
// consecutive row pairs.  Every CTA finishes its share of slot s before it
// starts slot s + 1, so slot s's activations are complete early.  Two orders:
//   kOrderRoundRobin  the S * ng groups, slot after slot, dealt round robin
//                     (group q to CTA q mod G): the grid sweeps one
//                     contiguous window of the weights;
//   kOrderRanges      in slot s the CTA takes range number (b + 53 s) mod G of
//                     G near-equal contiguous ranges, from a rotated start;
//   kOrderGlobal      one contiguous range of the slot-major list, from a
//                     rotated start (slots are then published only at the end).
enum { kOrderRoundRobin = 0, kOrderRanges = 1, kOrderGlobal = 2 };
// Advanced one group at a time without divisions (except once per slot
// range or wrap), since every consumer warp and the producer step it for
// every stage.
struct GroupsA {
  int mode, b, G, S, ng, GA, I;
  int k, n, lo, rot;  // position k of n in the current range starting at group lo
  int s, j;           // current group: number j of slot s
  int r, g;           // its row pairs [r, r + g)
  WR_DEVINL void set() {
    r = j * GA;
    g = min(GA, I - r);
  }
  // kOrderRanges: the first slot >= `slot` in which this CTA has groups.
  WR_DEVINL void range(int slot) {
    for (s = slot; s < S; ++s) {
      const int c = (int)((b + 53LL * s) % G);
      lo = (int)((int64_t)ng * c / G);
      n = (int)((int64_t)ng * (c + 1) / G) - lo;
      if (n > 0) break;
    }
    k = 0;
    rot = n > 0 ? (int)(((int64_t)b * 37) % n) : 0;
    j = lo + rot;
    if (s < S) set();
  }
  // kOrderGlobal: position on global group number q.
  WR_DEVINL void at(int q) {
    s = q / ng;
    j = q - s * ng;
    set();
  }
  WR_DEVINL void init(int mode_, int b_, int G_, int S_, int ng_, int GA_, int I_) {
    mode = mode_; b = b_; G = G_; S = S_; ng = ng_; GA = GA_; I = I_;
    if (mode == kOrderRanges) {
      range(0);
    } else if (mode == kOrderGlobal) {
      const int64_t Q = (int64_t)S * ng;
      lo = (int)(Q * b / G);
      n = (int)(Q * (b + 1) / G) - lo;
      rot = n > 0 ? (int)(((int64_t)b * 37) % n) : 0;
      k = 0;
      if (n > 0) at(lo + rot); else s = S;
    } else {
      if ((int64_t)b < (int64_t)S * ng) at(b); else s = S;
    }
  }
  WR_DEVINL bool valid() const { return s < S; }
  WR_DEVINL void next() {
    if (mode == kOrderRanges) {
      if (++k == n) {
        range(s + 1);
      } else {
        if (++j == lo + n) j = lo;
        set();
      }
    } else if (mode == kOrderGlobal) {
      if (++k == n) {
        s = S;
      } else if (k == n - rot) {
        at(lo);  // wrap to the start of the range
      } else {
        if (++j == ng) { j = 0; ++s; }
        set();
      }
    } else {
      j += G;
      while (j >= ng && s < S) { j -= ng; ++s; }
      if (s < S) set();
    }
  }
};

template <typename Tw, int NT>
__global__ void __launch_bounds__(kThreads, 1) k_fused_stream(const FusedArgs a) {
  constexpr int VEC = Chunk<Tw>::kVec;
  constexpr int ELT = (int)sizeof(Tw);
  constexpr int W = kConsumerWarps;
  // bf16: x stays bf16 in shared memory and phase A uses mixed-precision FMAs
  constexpr bool kBf16 = std::is_same<Tw, uint16_t>::value;

  extern __shared__ __align__(1024) uint8_t smem[];
  const Plan pl = a.pl;
  const int nst = pl.nst;
  uint8_t* ring = smem;
  float* vreg = reinterpret_cast<float*>(smem + nst * pl.SB);
  uint8_t* misc = smem + kMiscOff;
  uint64_t* full = reinterpret_cast<uint64_t*>(misc + kOffBars);
  uint64_t* empty = full + kMaxStages;
  uint64_t* act_full = reinterpret_cast<uint64_t*>(misc + kOffActBars);
  uint64_t* act_empty = act_full + kMaxActBufs;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + kOffAbort);
  int* s_nslots = reinterpret_cast<int*>(misc + kOffNSlots);
  volatile int* slot_tag = reinterpret_cast<volatile int*>(misc + kOffSlotTag);
  int* slot_e = reinterpret_cast<int*>(misc + kOffSlotE);
  float* slot_w = reinterpret_cast<float*>(misc + kOffSlotW);
  int* tok_ids = reinterpret_cast<int*>(misc + kOffTokIds);
  float* tok_w = reinterpret_cast<float*>(misc + kOffTokW);
  float* s_logits = reinterpret_cast<float*>(misc + kOffLogits);
  float* rowacc = vreg + pl.RA;  // [W][NBM][NT] phase-B partial sums, one set per warp
  uint64_t* slot_bar = reinterpret_cast<uint64_t*>(misc + kOffSlotBar);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int H = a.H, I = a.I, E = a.E, K = a.K, T = a.T;
  const int G = gridDim.x, b = blockIdx.x;

  if (tid == 0) {
    for (int s = 0; s < kMaxExperts; ++s) mbar_init(&slot_bar[s], W);
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
      slot_tag[s] = -1;
    }
    for (int q = 0; q < pl.CB; ++q) {
      mbar_init(&act_full[q], 1);
      mbar_init(&act_empty[q], W);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }

  // The router's inputs into L2 while the previous kernel finishes (each CTA
  // a share): gate_w does not depend on it, and x may, but a prefetch into
  // L2 (the point of coherence) cannot return stale data later.
  if (tid == 32 * W) {
    prefetch_share_l2(a.gate_w, (int64_t)E * H * (kBf16 ? 2 : 4), b, G);
    prefetch_share_l2(a.x, (int64_t)T * H * (kBf16 ? 2 : 4), b, G);
  }
  // The previous kernel on the stream (which may have produced x, or be the
  // previous call on this workspace) is complete from here on.  The next
  // kernel may begin its launch now: its CTAs take over SMs as ours exit.
  griddep_wait();
  griddep_launch_dependents();
  uint32_t* s_epoch = reinterpret_cast<uint32_t*>(misc + kOffEpoch);
  if (tid == 0 && a.comm.world > 0) *s_epoch = *a.comm.epoch + 1;  // read after the previous launch
  // Output value v of token t, row h: into `out`, or with an all-reduce as
  // the word (v | epoch << 32) into this rank's slot of every rank's
  // mailbox (*s_epoch is read after the __syncthreads below, before use).
  auto emit = [&](int t, int h, float v) {
    if (a.comm.world > 0) {
      const uint32_t e = *s_epoch;
      const uint64_t word = ((uint64_t)e << 32) | __float_as_uint(v);
      const size_t off =
          (((size_t)a.comm.rank * 2 + (e & 1u)) * kCommMaxTokens + t) * (size_t)H + h;
      for (int q = 0; q < a.comm.world; ++q) st_relaxed_sys_u64(a.comm.box[q] + off, word);
    } else {
      const int64_t i = (int64_t)t * H + h;
      a.out[i] = residual_out(a.res, i, v);
    }
  };

  // ---- x -> shared memory as fp32 [NT][H] (tokens >= T are zero), by the
  // producer and publisher warps, while the consumer warps compute the router
  // partial sums: item (token t, row batch eb, segment seg) is segment seg of
  // router rows [8 eb, 8 eb + 8) against x_t (the fixed order of
  // wr_router.cuh).  Small routers (pl.localR) are computed whole by every
  // CTA into a small shared-memory area; larger ones are spread over every
  // consumer warp of the grid and meet in the workspace behind one grid-wide
  // counter.
  const int nbat = (E + kRouterRowBatch - 1) / kRouterRowBatch;
  float* lparts = reinterpret_cast<float*>(misc + kOffLParts);  // [T][segment][E] when pl.localR
  if (warp >= W && kBf16) {
    // bf16 x kept as is: [NT][H] chunks (tokens >= T are zero)
    const uint4* xg = static_cast<const uint4*>(a.x);
    uint4* dst = reinterpret_cast<uint4*>(vreg);
    const int nvec = H / VEC;
#pragma unroll 8
    for (int idx = tid - W * 32; idx < NT * nvec; idx += kThreads - W * 32)
      dst[idx] = idx < T * nvec ? ldg_nc_v4(xg + idx) : make_uint4(0u, 0u, 0u, 0u);
  } else if (warp >= W) {
    const Tw* xg = static_cast<const Tw*>(a.x);
    const int nvec = H / VEC;  // the host guarantees H % VEC == 0 on this path
#pragma unroll 8
    for (int idx = tid - W * 32; idx < NT * nvec; idx += kThreads - W * 32) {
      const int t = idx / nvec;
      const int v = idx - t * nvec;
      float f[VEC];
      if (t < T) {
        Chunk<Tw>::widen(ldg_nc_v4(xg + (int64_t)t * H + (int64_t)v * VEC), f);
      } else {
#pragma unroll
        for (int q = 0; q < VEC; ++q) f[q] = 0.0f;
      }
      float4* dst = reinterpret_cast<float4*>(vreg + t * H + v * VEC);
#pragma unroll
      for (int q = 0; q < VEC / 4; ++q)
        dst[q] = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
    }
  } else {
    const Tw* gw = static_cast<const Tw*>(a.gate_w);
    const Tw* xg = static_cast<const Tw*>(a.x);
    const int items = T * nbat * kRouterSegments;
    const int first = pl.localR ? warp : b + G * warp;
    const int step = pl.localR ? W : G * W;
    float* pbase = pl.localR ? lparts : a.rparts;
    for (int it = first; it < items; it += step) {
      const int seg = it % kRouterSegments;
      const int rest = it / kRouterSegments;
      const int eb = rest % nbat, t = rest / nbat;
      const int e0 = eb * kRouterRowBatch;
      router_segment_warp<Tw, XGlobal<Tw>>(
          gw + (int64_t)e0 * H, XGlobal<Tw>{xg + (int64_t)t * H}, min(kRouterRowBatch, E - e0), H,
          seg, lane, true, pbase + ((int64_t)t * kRouterSegments + seg) * E + e0);
    }
  }
  __syncthreads();
  if (!pl.localR) {
    if (tid == 0) {
      // grid-wide: every CTA's partial sums are written
      __threadfence();
      red_release_gpu_add(&a.sync[kSyncRouter], 1u);
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_gpu(&a.sync[kSyncRouter]) < (uint32_t)G) {
        if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(&a.sync[kSyncStatus], DEV_TIMEOUT_GRID);
          *abort_flag = 1;
          break;
        }
      }
    }
    __syncthreads();
  }
  // ---- logits (segment sums added in order, + bias) and top-K per token ----
  for (int i = tid; i < T * E; i += kThreads) {
    const int t = i / E, e = i - t * E;
    float part[kRouterSegments];
    const int64_t pt = (int64_t)t * kRouterSegments * E + e;
#pragma unroll
    for (int j = 0; j < kRouterSegments; ++j)  // workspace sums: read from L2 (other CTAs wrote them)
      part[j] = pl.localR ? lparts[pt + j * E] : __ldcg(a.rparts + pt + j * E);
    float l = part[0];
#pragma unroll
    for (int j = 1; j < kRouterSegments; ++j) l = __fadd_rn(l, part[j]);
    if (a.bias) l = __fadd_rn(l, a.bias[e]);
    s_logits[t * kMaxExperts + e] = l;
  }
  __syncthreads();
  if (warp < T)
    select_topk_warp(s_logits + warp * kMaxExperts, E, K, lane, tok_ids + warp * kMaxExperts,
                     tok_w + warp * kMaxExperts);
  __syncthreads();
  if (tid == 0) {
    int ns = 0;
    for (int t = 0; t < T; ++t) {
      for (int k = 0; k < K; ++k) {
        const int e = tok_ids[t * kMaxExperts + k];
        if (e < a.ep_first || e >= a.ep_first + a.ep_num) continue;
        const int le = e - a.ep_first;
        int s = 0;
        while (s < ns && slot_e[s] != le) ++s;
        if (s == ns) {
          slot_e[ns] = le;
          for (int tt = 0; tt < NT; ++tt) slot_w[ns * NT + tt] = 0.0f;
          ++ns;
        }
        slot_w[s * NT + t] = tok_w[t * kMaxExperts + k];
      }
    }
    *s_nslots = ns;
  }
  if (b == 0) {
    for (int i = tid; i < T * K; i += kThreads) {
      const int t = i / K, k = i - t * K;
      if (a.ids_out) a.ids_out[i] = tok_ids[t * kMaxExperts + k];
      if (a.w_out) a.w_out[i] = tok_w[t * kMaxExperts + k];
    }
  }
  __syncthreads();

  const int S = *s_nslots;
  const int ng = (I + pl.GA - 1) / pl.GA;  // phase A groups per slot (S * I < 2^30)
  const int hb0 = (int)split_lo(H, b, G), hb1 = (int)split_lo(H, b + 1, G);
  const int nb = hb1 - hb0;
  const int nb_u = (nb + pl.GB - 1) / pl.GB;
  const int hb_start = hb0 + (nb_u ? (int)(((int64_t)b * 11) % nb_u) : 0) * pl.GB;
  const int wc_last = I - (pl.nwin - 1) * pl.WB;  // width of a slot's last window

  if (S == 0) {
    // No local expert selected (expert-parallel rank): this rank adds zero.
    for (int idx = tid; idx < T * nb; idx += kThreads) {
      const int t = idx / nb;
      emit(t, hb0 + (idx - t * nb), 0.0f);
    }
  } else if (warp == W) {
    // =========================== producer ===================================
    if (lane == 0) {
      // (nothing but the bulk copies writes the ring, so no proxy fence is
      // needed before the first one)
      const uint64_t pol = l2_policy_evict_first();
      bool ok = true;
      int issued = 0;
      Cursor c{0, 0u};
      // Reserves the next stage: waits for the stage it replaces to be
      // released, then tags the slot with the new stage number.  Returns
      // false on a timeout.
      auto reserve = [&]() -> bool {
        if (issued >= nst && !mbar_wait(&empty[c.si], c.ph ^ 1u, abort_flag)) return false;
        slot_tag[c.si] = issued;
        return true;
      };
      // `owners` warps will release the stage; arrive for the others now.
      auto commit = [&](int owners) {
        if (owners < W) mbar_arrive_cnt(&empty[c.si], (uint32_t)(W - owners));
        c.next(nst);
        ++issued;
      };
      // phase A
      GroupsA ga;
      ga.init(pl.orderA, b, G, S, ng, pl.GA, I);
      for (; ga.valid() && ok; ga.next()) {
        const int g = ga.g;
        const uint8_t* eb =
            a.wbuf + (int64_t)slot_e[ga.s] * a.lay.stride + (int64_t)ga.r * H * ELT;
        for (int c0 = 0; c0 < H; c0 += pl.CWA) {
          if (!(ok = reserve())) break;
          const int cw = min(pl.CWA, H - c0);
          uint8_t* st = ring + c.si * pl.SB;
          const uint32_t piece = (uint32_t)g * cw * ELT;  // g == 1 when cw < H
          mbar_arrive_expect_tx(&full[c.si], 2 * piece);
          const uint8_t* src = eb + (int64_t)c0 * ELT;
          bulk_g2s(st, src + a.lay.off_gate, piece, &full[c.si], pol);
          bulk_g2s(st + pl.GA * pl.CWA * ELT, src + a.lay.off_up, piece, &full[c.si], pol);
          commit(g < W ? g : W);
        }
      }
      // phase B
      for (int s = 0; s < S && ok; ++s) {
        const uint8_t* eb = a.wbuf + (int64_t)slot_e[s] * a.lay.stride + a.lay.off_down;
        for (int win = 0, c0 = 0; win < pl.nwin && ok; ++win, c0 += pl.WB) {
          const int wc = win + 1 < pl.nwin ? pl.WB : wc_last;
          int hb = hb_start;
          for (int uu = 0; uu < nb_u; ++uu) {
            if (!(ok = reserve())) break;
            const int g = min(pl.GB, hb1 - hb);
            uint8_t* st = ring + c.si * pl.SB;
            const uint8_t* src = eb + ((int64_t)hb * I + c0) * ELT;
            mbar_arrive_expect_tx(&full[c.si], (uint32_t)g * wc * ELT);
            if (wc == I) {
              bulk_g2s(st, src, (uint32_t)g * I * ELT, &full[c.si], pol);
            } else {
              for (int r = 0; r < g; ++r)
                bulk_g2s(st + r * pl.WB * ELT, src + (int64_t)r * I * ELT, wc * ELT, &full[c.si],
                         pol);
            }
            commit(min(g, W / pl.PB) * pl.PB);
            hb += pl.GB;
            if (hb >= hb1) hb = hb0;
          }
        }
      }
      if (!ok) {
        // Let every copy already issued land before the CTA can exit.
        *abort_flag = 1;
        const int first = issued > nst ? issued - nst : 0;
        for (int j = first; j < issued; ++j)
          if (!mbar_wait(&full[j % nst], (uint32_t)(j / nst) & 1u, nullptr))
            atomicOr(&a.sync[kSyncStatus], DEV_TIMEOUT_DRAIN);
        atomicOr(&a.sync[kSyncStatus], DEV_TIMEOUT_EMPTY);
      }
    }
  } else if (warp == W + 1) {
    // =========================== publisher ==================================
    // (1) Once all W consumer warps of this CTA have written their slot-s
    // activations (each arrives on slot_bar[s], used once per launch), counts
    // the CTA in on the grid-wide counter of slot s with one GPU-scope
    // release, so the consumers never stall on a GPU-scope release.
    // (2) Phase B's activation windows (slot s, window win; j = s * nwin +
    // win) go into pl.CB buffers round robin: window j is copied into buffer
    // j % CB as soon as slot s is complete grid-wide and the consumers have
    // released the buffer's previous window (act_empty), so a slot's
    // activations are in shared memory before its rows come up instead of
    // each slot costing a grid-wide wait plus a copy in the consumers' path.
    // With AOFF == 0 the buffers overlap x, and the first window waits for
    // the end of phase A in this CTA (every consumer warp has arrived on
    // every slot's barrier; a warp arrives on the slots in order).
    // Both jobs are polled in one loop, so neither waits behind the other;
    // a window that can go is issued before a pending release, which may
    // hold this thread while the SM's bulk copies drain.
    if (lane == 0) {
      const int NW = S * pl.nwin;
      const uint64_t pol = l2_policy_evict_last();
      int pub = 0, done = 0, win_j = 0;  // slots released / seen complete here
      uint64_t t_prog = globaltimer_ns();
      uint32_t spins = 0;
      bool ok = true;
      while (ok && (pub < S || win_j < NW)) {
        bool prog = false;
        while (done < S && mbar_test_wait(&slot_bar[done], 0u)) ++done;
        if (win_j < NW) {
          const int s = win_j / pl.nwin, win = win_j - s * pl.nwin;
          const int ab = win_j % pl.CB;
          const int use = win_j / pl.CB;
          bool ready = use > 0 ? mbar_test_wait(&act_empty[ab], (uint32_t)(use - 1) & 1u)
                               : (pl.AOFF > 0 || done == S);
          if (ready && win == 0) ready = ld_acquire_gpu(&a.sync[kSyncSlot0 + s]) >= (uint32_t)G;
          if (ready) {
            fence_proxy_async_global();  // the peers' activations, then async-proxy reads
            if (use == 0) fence_proxy_async_smem();  // x or nothing was here (generic writes)
            const int c0 = win * pl.WB;
            const int wc = win + 1 < pl.nwin ? pl.WB : I - (pl.nwin - 1) * pl.WB;
            const uint32_t bytes = (uint32_t)wc * NT * 4;
            uint8_t* dst = reinterpret_cast<uint8_t*>(vreg + pl.AOFF + ab * pl.WBF);
            const uint8_t* src =
                reinterpret_cast<const uint8_t*>(a.act + ((int64_t)s * I + c0) * NT);
            mbar_arrive_expect_tx(&act_full[ab], bytes);
            for (uint32_t off = 0; off < bytes; off += 32768u)
              bulk_g2s(dst + off, src + off, min(32768u, bytes - off), &act_full[ab], pol);
            ++win_j;
            prog = true;
          }
        }
        if (pub < done) {
          fence_proxy_async_global();
          red_release_gpu_add(&a.sync[kSyncSlot0 + pub], 1u);
          ++pub;
          prog = true;
        }
        if (prog) {
          t_prog = globaltimer_ns();
        } else if ((++spins & 63u) == 0) {
          if (*abort_flag) {
            ok = false;
          } else if (globaltimer_ns() - t_prog > kWaitLimitNs) {
            atomicOr(&a.sync[kSyncStatus], DEV_TIMEOUT_GRID);
            *abort_flag = 1;
            ok = false;
          }
        }
      }
      // Every window copy issued lands before the CTA can exit (the
      // consumers have waited for all of them unless the launch aborted).
      for (int j = win_j > pl.CB ? win_j - pl.CB : 0; j < win_j; ++j)
        if (!mbar_wait(&act_full[j % pl.CB], (uint32_t)(j / pl.CB) & 1u, nullptr))
          atomicOr(&a.sync[kSyncStatus], DEV_TIMEOUT_DRAIN);
    }
  } else {
    // =========================== consumer warps =============================
    // Only the owners of a stage's rows wait for it, read it and release it.
    // Loop trip counts depend only on the problem, so all warps pass every
    // named barrier exactly once even after a failed wait; `ok` is kept
    // warp-uniform with __all_sync.
    Cursor c{0, 0u};
    int stage = 0;  // number of the stage under the cursor
    bool ok = true;
    // Owner's wait for stage `stage` in slot c.si: its tag, then its data.
    auto wait_owned = [&]() -> bool {
      bool got = true;
      if (slot_tag[c.si] != stage) {
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t spin = 1; slot_tag[c.si] != stage; ++spin) {
          if ((spin & 63u) == 0 && (*abort_flag || globaltimer_ns() - t0 > kWaitLimitNs)) {
            got = false;
            break;
          }
        }
      }
      if (got) got = mbar_wait(&full[c.si], c.ph, abort_flag);
      return __all_sync(0xffffffffu, got);
    };

    // This warp's activations of slot s are written: tell the publisher.
    auto publish = [&](int s) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&slot_bar[s]);
    };

    // ---- phase A: gate/up rows -> activations; the CTA's k-th row pair is
    // owned by warp k % 8 ----
    {
      const int nch_full = pl.CWA / VEC;
      float ga[NT], ua[NT];  // running sums of a row pair split over stages
#pragma unroll
      for (int t = 0; t < NT; ++t) ga[t] = ua[t] = 0.0f;
      GroupsA gr;
      gr.init(pl.orderA, b, G, S, ng, pl.GA, I);
      int lrow = 0;      // row pairs of this CTA before the current group
      int published = 0; // slots [0, published) are published by this warp
      for (; gr.valid(); gr.next()) {
        if (pl.orderA != kOrderGlobal)
          for (; published < gr.s; ++published) publish(published);
        const int g = gr.g;
        const int first = (warp - (lrow & (W - 1)) + W) & (W - 1);  // my first row of the group
        const bool mine = first < g;
        lrow += g;
        for (int c0 = 0; c0 < H; c0 += pl.CWA) {
          const int cw = min(pl.CWA, H - c0);
          if (ok && mine) ok = wait_owned();
          if (ok && mine) {
            const uint8_t* st = ring + c.si * pl.SB;
            if (cw == H) {
              // whole row pairs: rows first, first+8, ... of this stage
              float gg[kRowsPerWarp][NT], uv[kRowsPerWarp][NT];
#pragma unroll
              for (int k = 0; k < kRowsPerWarp; ++k) {
#pragma unroll
                for (int t = 0; t < NT; ++t) gg[k][t] = uv[k][t] = 0.0f;
                const int rr = first + k * W;
                if (rr < g) {
                  const uint4* gp = reinterpret_cast<const uint4*>(st + rr * pl.CWA * ELT);
                  const uint4* up = reinterpret_cast<const uint4*>(st + (pl.GA + rr) * pl.CWA * ELT);
                  if constexpr (kBf16)
                    dot_pair_bf16<NT>(gp, up, reinterpret_cast<const uint4*>(vreg), H, 0, 0,
                                      nch_full, lane, gg[k], uv[k]);
                  else
                    dot_pair<Tw, NT>(gp, up, vreg, H, 0, 0, nch_full, lane, gg[k], uv[k]);
                }
              }
              __syncwarp();
              if (lane == 0) mbar_arrive(&empty[c.si]);
#pragma unroll
              for (int k = 0; k < kRowsPerWarp; ++k) {
                const int rr = first + k * W;
                if (rr < g) {
                  warp_sum<NT>(gg[k]);
                  warp_sum<NT>(uv[k]);
#pragma unroll
                  for (int t = 0; t < NT; ++t) {
                    if (lane == t) {
                      const float wt = slot_w[gr.s * NT + t];
                      a.act[((int64_t)gr.s * I + gr.r + rr) * NT + t] =
                          (wt != 0.0f) ? wt * (silu(gg[k][t]) * uv[k][t]) : 0.0f;
                    }
                  }
                }
              }
            } else {
              // one row pair split over several stages (g == 1, first == 0)
              if constexpr (kBf16)
                dot_pair_bf16<NT>(reinterpret_cast<const uint4*>(st),
                                  reinterpret_cast<const uint4*>(st + pl.GA * pl.CWA * ELT),
                                  reinterpret_cast<const uint4*>(vreg), H, c0, 0, cw / VEC, lane,
                                  ga, ua);
              else
                dot_pair<Tw, NT>(reinterpret_cast<const uint4*>(st),
                                 reinterpret_cast<const uint4*>(st + pl.GA * pl.CWA * ELT), vreg, H,
                                 c0, 0, cw / VEC, lane, ga, ua);
              __syncwarp();
              if (lane == 0) mbar_arrive(&empty[c.si]);
              if (c0 + cw >= H) {
                warp_sum<NT>(ga);
                warp_sum<NT>(ua);
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                  if (lane == t) {
                    const float wt = slot_w[gr.s * NT + t];
                    a.act[((int64_t)gr.s * I + gr.r) * NT + t] =
                        (wt != 0.0f) ? wt * (silu(ga[t]) * ua[t]) : 0.0f;
                  }
                }
#pragma unroll
                for (int t = 0; t < NT; ++t) ga[t] = ua[t] = 0.0f;
              }
            }
          }
          c.next(nst);
          ++stage;
        }
      }
      for (; published < S; ++published) publish(published);
    }
    if (!ok && lane == 0) *abort_flag = 1;
    for (int i = tid; i < W * pl.NBM * NT; i += kConsumerThreads) rowacc[i] = 0.0f;

    // ---- phase B: down rows, slot by slot.  Local row lr of a stage is read
    // by the PB warps of row group lr % GW, each taking a column slice; a
    // warp computes its (up to kRowsPerWarp) rows of the stage together, so
    // they share every activation load.  Warp w adds into its own
    // accumulators rowacc[w][h][t], summed in warp order at the end.  The
    // activation window of (slot s, window win) is the j-th, in buffer j % CB;
    // the publisher warp fills it, and each warp releases it after its rows
    // of the window. ----
    {
      const int GW = W / pl.PB;         // row groups of PB warps
      const int partB = warp % pl.PB;   // my column slice
      const int grpB = warp / pl.PB;    // my row group
      named_bar_sync(kBarConsumers, kConsumerThreads);  // row accumulators zeroed
      const int rs = pl.WB / VEC;  // 16-byte chunks from one stage row to the next
      int j = 0;
      for (int s = 0; s < S; ++s) {
        for (int win = 0; win < pl.nwin; ++win, ++j) {
          const int wc = win + 1 < pl.nwin ? pl.WB : wc_last;
          const int nch = wc / VEC;
          const int ab = j % pl.CB;
          const uint32_t use = (uint32_t)(j / pl.CB);
          if (*abort_flag) ok = false;
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&act_full[ab], use & 1u, abort_flag));
          const float* av = vreg + pl.AOFF + ab * pl.WBF;
          int hb = hb_start;
          for (int uu = 0; uu < nb_u; ++uu) {
            const int g = min(pl.GB, hb1 - hb);
            // local row lr is read by the PB warps of row group lr % GW, warp
            // `part` of them taking chunks part*32 + lane + PB*32*k
            const int lr0 = hb - hb0;  // local row of the stage's first row
            const int first = (grpB - (lr0 & (GW - 1)) + GW) & (GW - 1);  // my first row of it
            const int nr = first < g ? (g - first + GW - 1) / GW : 0;    // my rows: first + k GW
            float* racc = rowacc + ((int64_t)warp * pl.NBM + lr0 + first) * NT;
            if (ok && nr > 0) ok = wait_owned();
            if (ok && nr > 0) {
              const uint4* wp = reinterpret_cast<const uint4*>(ring + c.si * pl.SB) + first * rs;
              const int j0 = partB * 32 + lane, js = pl.PB * 32;
              float v[kRowsPerWarp][NT];
#pragma unroll
              for (int r = 0; r < kRowsPerWarp; ++r) {
#pragma unroll
                for (int t = 0; t < NT; ++t) v[r][t] = 0.0f;
              }
              if (nr == 1) {  // one row: the deeper-unrolled loop
                float v1[1][NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) v1[0][t] = 0.0f;
                dot_down_rows<Tw, NT, 1>(wp, GW * rs, av, nch, j0, js, 1, v1);
#pragma unroll
                for (int t = 0; t < NT; ++t) v[0][t] = v1[0][t];
              } else if (nr == 2) {
                float v2[2][NT];
#pragma unroll
                for (int r = 0; r < 2; ++r) {
#pragma unroll
                  for (int t = 0; t < NT; ++t) v2[r][t] = 0.0f;
                }
                dot_down_rows<Tw, NT, 2>(wp, GW * rs, av, nch, j0, js, 2, v2);
#pragma unroll
                for (int r = 0; r < 2; ++r) {
#pragma unroll
                  for (int t = 0; t < NT; ++t) v[r][t] = v2[r][t];
                }
              } else {
                dot_down_rows<Tw, NT, kRowsPerWarp>(wp, GW * rs, av, nch, j0, js, nr, v);
              }
              __syncwarp();
              if (lane == 0) mbar_arrive(&empty[c.si]);
#pragma unroll
              for (int r = 0; r < kRowsPerWarp; ++r) {
                if (r < nr) {
                  warp_sum<NT>(v[r]);
                  if (lane == 0) {
#pragma unroll
                    for (int t = 0; t < NT; ++t) racc[r * GW * NT + t] += v[r][t];
                  }
                }
              }
            }
            c.next(nst);
            ++stage;
            hb += pl.GB;
            if (hb >= hb1) hb = hb0;
          }
          // this warp is done with the window's buffer
          __syncwarp();
          if (lane == 0) mbar_arrive(&act_empty[ab]);
          if (!ok && lane == 0) *abort_flag = 1;
        }
      }
      named_bar_sync(kBarConsumers, kConsumerThreads);  // all row accumulators final
      // (with an all-reduce the rows are written even after a failed wait,
      // so the peers' waits end; the status word reports the failure)
      if ((ok && !*abort_flag) || a.comm.world > 0) {
        for (int idx = tid; idx < T * nb; idx += kConsumerThreads) {
          const int t = idx / nb;
          const int h = idx - t * nb;
          float o = rowacc[h * NT + t];
#pragma unroll
          for (int w = 1; w < W; ++w) o += rowacc[((int64_t)w * pl.NBM + h) * NT + t];
          emit(t, hb0 + h, o);
        }
      }
      if (lane == 0 && !ok) atomicOr(&a.sync[kSyncStatus], DEV_TIMEOUT_FULL);
    }
  }

  __syncthreads();
  if (a.comm.world > 0) {
    // ---- one-shot all-reduce: this CTA's rows of every rank ----
    // Each word of this rank's mailbox is polled until it carries this
    // launch's epoch; the values are summed in source-rank order.  Every
    // source's word is loaded at once first (one memory latency instead of
    // one per source), then any that is not there yet is polled alone.
    const uint32_t e = *s_epoch;
    const uint64_t t0 = globaltimer_ns();
    bool late = false;
    for (int idx = tid; idx < T * nb; idx += kThreads) {
      const int t = idx / nb;
      const int h = hb0 + (idx - t * nb);
      const uint64_t* pb = a.comm.box[a.comm.rank] + ((size_t)(e & 1u) * kCommMaxTokens + t) * H + h;
      const size_t qs = (size_t)2 * kCommMaxTokens * H;  // words between sources
      uint64_t w[kMaxRanks];
#pragma unroll
      for (int q = 0; q < kMaxRanks; ++q)
        if (q < a.comm.world) w[q] = ld_relaxed_sys_u64(pb + q * qs);
      float o = 0.0f;
#pragma unroll
      for (int q = 0; q < kMaxRanks; ++q) {
        if (q < a.comm.world) {
          for (uint32_t spin = 1; (uint32_t)(w[q] >> 32) != e && !late; ++spin) {
            if ((spin & 63u) == 0 && globaltimer_ns() - t0 > a.comm.peer_wait_ns) {
              atomicOr(&a.sync[kSyncStatus], DEV_TIMEOUT_PEER);
              late = true;
            }
            w[q] = ld_relaxed_sys_u64(pb + q * qs);
          }
          o += __uint_as_float((uint32_t)w[q]);
        }
      }
      const int64_t i = (int64_t)t * H + h;
      a.out[i] = residual_out(a.res, i, o);
    }
  }
  if (tid == 0) {
    // Self-reset of the slot counters: every CTA has left its waits once it
    // counts itself out, so the last one can clear them all.  The fence makes
    // this CTA's counter increments (made by other warps, ordered before by
    // the barrier) visible before its exit count; the clears are plain
    // stores, visible to the next launch once this one has completed.
    __threadfence();
    const uint32_t prev = atomicAdd(&a.sync[kSyncExit], 1u);
    if (prev == (uint32_t)G - 1) {
      for (int s = 0; s < S; ++s) a.sync[kSyncSlot0 + s] = 0u;
      a.sync[kSyncRouter] = 0u;
      if (a.comm.world > 0) *a.comm.epoch = *s_epoch;  // the next launch uses epoch + 1
      a.sync[kSyncExit] = 0u;
    }
  }
}

// Launch mode of the fused kernel, probed once per device: programmatic
// dependent launch together with the cooperative attribute when the driver
// takes both, else each alone.
enum LaunchMode { kModeUnknown = 0, kModeCoopPdl, kModePdl, kModeCoop };

template <typename Tw, int NT>
wr_status_t launch_stream(const FusedArgs& args, int grid, cudaStream_t stream) {
  auto kern = k_fused_stream<Tw, NT>;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  static int mode[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  });
  if (attr_err[dev & 63] != cudaSuccess)
    return cuda_fail(attr_err[dev & 63], "cudaFuncSetAttribute(fused)");

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  int& m = mode[dev & 63];
  const int tries[3] = {kModeCoopPdl, kModePdl, kModeCoop};
  cudaError_t e = cudaSuccess;
  for (int i = 0; i < 3; ++i) {
    const int mm = m != kModeUnknown ? m : tries[i];
    if (mm == kModeCoopPdl) { cfg.attrs = attr; cfg.numAttrs = 2; }
    if (mm == kModePdl) { cfg.attrs = attr + 1; cfg.numAttrs = 1; }
    if (mm == kModeCoop) { cfg.attrs = attr; cfg.numAttrs = 1; }
    e = cudaLaunchKernelEx(&cfg, kern, args);
    if (e == cudaSuccess) {
      m = mm;
      return WR_OK;
    }
    if (m != kModeUnknown) break;
    cudaGetLastError();  // clear, try the next mode
  }
  return cuda_fail(e, "cudaLaunchKernelEx(fused)");
}

int nt_bucket(int T) { return T <= 1 ? 1 : (T <= 2 ? 2 : 4); }

int clamp_rows(int64_t g) {
  if (g < 1) g = 1;
  return (int)(g > kMaxRowsPerStage ? kMaxRowsPerStage : g);
}

// wide: stages of two whole row pairs of more than 16 KB (copies of 2 rows,
// 32-48 KB stages: a one-row-pair stage would issue copies of one row of
// 8-16 KB, which stream from HBM more slowly), with activation windows of at
// most 24 KB so that the ring still holds 4 stages.
Plan make_plan_v(const Problem& p, int nt, int grid, bool wide) {
  const int elt = p.elt, vec = 16 / elt;
  Plan pl;
  // phase A: whole row pairs when one fits in a stage, else pieces of
  // kTargetStage / 2 bytes of one gate row and one up row
  const int64_t pair = 2LL * p.H * elt;
  int stage_a;
  if (wide) {
    pl.GA = 2;
    pl.CWA = p.H;
    stage_a = (int)(2 * pair);
  } else if (pair <= kMaxStageBytes) {
    pl.GA = clamp_rows(kTargetStage / pair);
    pl.CWA = p.H;
    stage_a = (int)(pl.GA * pair);
  } else {
    pl.GA = 1;
    pl.CWA = (kTargetStage / 2 / elt) / vec * vec;
    stage_a = 2 * pl.CWA * elt;
  }
  // phase B: windows of at most kTargetStage bytes of weight columns
  int64_t wmax = (int64_t)kVecMaxBytes / (nt * 4);
  if (wmax > kTargetStage / elt) wmax = kTargetStage / elt;
  if (wide && wmax > kWideWindowBytes / (nt * 4)) wmax = kWideWindowBytes / (nt * 4);
  wmax = wmax / vec * vec;
  if (p.I <= wmax) {
    pl.nwin = 1;
    pl.WB = p.I;
  } else {
    pl.nwin = (int)((p.I + wmax - 1) / wmax);
    int64_t w = (p.I + pl.nwin - 1) / pl.nwin;
    pl.WB = (int)((w + vec - 1) / vec * vec);
  }
  // phase B: the CTA's rows of a window in as few stages of at most
  // kWideStageBytes as they fit, split evenly (the consumers pay a fixed cost
  // per stage, and a short last stage costs as much as a full one)
  const int64_t row_b = (int64_t)pl.WB * elt;
  const int64_t nbm = (p.H + grid - 1) / grid;
  auto rows_within = [&](int64_t cap) {
    int64_t g = cap / row_b;
    if (g > kMaxRowsPerStage) g = kMaxRowsPerStage;
    return g < 1 ? (int64_t)1 : g;
  };
  int64_t gb_max = rows_within(kWideStageBytes);
  // a slightly larger stage when it halves a window's stages to two (the
  // 8-way tensor-parallel Mixtral shard: 28 rows as 14 + 14, not 10 + 9 + 9;
  // measured 27.8 -> 26.6 us, while the same cap cost 4-row-pair stages 3 us)
  if ((nbm + gb_max - 1) / gb_max > 2 &&
      (nbm + rows_within(kPairStageBytes) - 1) / rows_within(kPairStageBytes) <= 2)
    gb_max = rows_within(kPairStageBytes);
  const int64_t nstg = (nbm + gb_max - 1) / gb_max;
  pl.GB = clamp_rows((nbm + nstg - 1) / nstg);
  int sb = stage_a > (int)(pl.GB * row_b) ? stage_a : (int)(pl.GB * row_b);
  sb = (sb + 127) / 128 * 128;
  pl.SB = sb;
  // phase A fills the slots phase B needs (whole row pairs only)
  if (pl.CWA == p.H && (int64_t)pl.GA * pair < sb && sb / pair > pl.GA) pl.GA = clamp_rows(sb / pair);
  // Long rows are split by columns over PB warps (shorter holds of each
  // stage); a warp then reads at most kRowsPerWarp rows of a stage.
  const int nchB = pl.WB / vec;
  pl.PB = nchB >= 1536 ? 2 : 1;
  while (pl.PB > 1 && pl.GB > kRowsPerWarp * (kConsumerWarps / pl.PB)) pl.PB /= 2;
  pl.orderA = kOrderRoundRobin;
  pl.NBM = (p.H + grid - 1) / grid;
  // The vector region holds x (bf16 as is, fp32 widened), the activation
  // window buffers and the per-warp row accumulators; the ring gets the rest.
  // Separate window buffers (after x) let the first windows land during
  // phase A and later ones while earlier windows are read, but not at the
  // cost of the weight stream: the ring keeps the stages the overlapped
  // layout would have, up to 6 (6 x 32 KB in flight per SM covers HBM's
  // latency).  Otherwise one window buffer shares x's space.
  auto r64 = [](int64_t v) { return (v + 63) / 64 * 64; };
  auto stages = [&](int64_t used) -> int64_t {
    const int64_t n = used < kMiscOff ? (kMiscOff - used) / sb : 0;
    return n > kMaxStages ? kMaxStages : n;
  };
  const int64_t xb = r64((int64_t)nt * p.H * (elt == 2 ? 2 : 4));
  const int64_t winb = r64((int64_t)pl.WB * nt * 4);
  const int64_t accb = r64((int64_t)kConsumerWarps * pl.NBM * nt * 4);
  const int64_t ov = xb > winb ? xb : winb;
  const int64_t nst_ov = stages(ov + accb);
  const int64_t slots_max = p.ep_num < (int64_t)p.K * nt ? p.ep_num : (int64_t)p.K * nt;
  int64_t nw_max = slots_max * pl.nwin;
  if (nw_max > kMaxActBufs) nw_max = kMaxActBufs;
  const int64_t keep = nst_ov < 6 ? nst_ov : 6;
  int cb = 0;
  for (int64_t q = nw_max; q >= 1 && cb == 0; --q)
    if (stages(xb + q * winb + accb) >= (keep > 2 ? keep : 2)) cb = (int)q;
  pl.WBF = (int)(winb / 4);
  if (cb > 0) {
    pl.AOFF = (int)(xb / 4);
    pl.CB = cb;
    pl.RA = (int)((xb + cb * winb) / 4);
    pl.nst = (int)stages(xb + cb * winb + accb);
  } else {
    pl.AOFF = 0;
    pl.CB = 1;
    pl.RA = (int)(ov / 4);
    pl.nst = (int)nst_ov;
  }
  // Every CTA computes the whole router when it is small (<= 2 items per
  // consumer warp, <= 64 KB of router weights read from L2 by each CTA; the
  // partial sums then fit in kLPartsBytes of shared memory); otherwise the
  // items are spread over the grid.
  const int64_t items =
      (int64_t)nt * ((p.E + kRouterRowBatch - 1) / kRouterRowBatch) * kRouterSegments;
  pl.localR = (items <= 2 * kConsumerWarps && (int64_t)p.E * p.H * elt <= 64 * 1024 &&
               (int64_t)nt * kRouterSegments * p.E * 4 <= kLPartsBytes)
                  ? 1
                  : 0;
  return pl;
}

Plan make_plan(const Problem& p, int nt, int grid) {
  const Plan pl = make_plan_v(p, nt, grid, false);
  const int64_t pair = 2LL * p.H * p.elt;
  if (pl.GA == 1 && pl.CWA == p.H && pair > kTargetStage / 2 && 2 * pair <= kWideStageBytes) {
    const Plan w = make_plan_v(p, nt, grid, true);
    if (w.nst >= 4) return w;
  }
  return pl;
}

}  // namespace

bool fused_supported(const Problem& p) {
  const int vec = 16 / p.elt;
  if (p.H % vec != 0 || p.I % vec != 0) return false;
  if (p.E > kMaxExperts || p.K > p.E) return false;
  if (p.T < 1 || p.T > kMaxNT) return false;
  const int nt = nt_bucket(p.T);
  if ((int64_t)nt * p.H * 4 > kVecMaxBytes) return false;  // x must fit in shared memory
  if ((int64_t)p.K * nt * p.I >= (1LL << 30)) return false; // 32-bit row indices
  // x (or an activation window) and the per-warp row accumulators must leave
  // room for a ring of at least two stages
  return make_plan(p, nt, device_sm_count()).nst >= 2;
}

size_t fused_workspace_bytes(const Problem& p) {
  const int nt = nt_bucket(p.T < 1 ? 1 : p.T);
  const int64_t slots = p.ep_num < p.K * nt ? p.ep_num : (int64_t)p.K * nt;
  const size_t act = (size_t)slots * p.I * nt * sizeof(float);
  return kActOffset + ((act + 255) & ~size_t(255));
}

wr_status_t launch_fused(const Problem& p, const void* x, const void* gate_w, const void* wbuf,
                         float* out, int32_t* ids, float* w, void* ws, cudaStream_t stream,
                         const CommView* comm) {
  FusedArgs args;
  if (comm) {
    args.comm = *comm;
  } else {
    args.comm = CommView{};  // world 0: no all-reduce
  }
  args.x = x;
  args.res = p.res;
  args.wbuf = static_cast<const uint8_t*>(wbuf);
  args.out = out;
  args.ids_out = ids;
  args.w_out = w;
  args.sync = static_cast<uint32_t*>(ws);
  args.gate_w = gate_w;
  args.bias = p.router_bias;
  args.rparts = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kSyncBytes);
  args.act = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kActOffset);
  args.E = p.E;
  args.H = p.H;
  args.I = p.I;
  args.K = p.K;
  args.T = p.T;
  args.ep_first = p.ep_first;
  args.ep_num = p.ep_num;
  args.lay = make_layout(p.H, p.I, p.elt);
  const int nt = nt_bucket(p.T);
  const int grid = device_sm_count();
  args.pl = make_plan(p, nt, grid);
  if (p.dtype == WR_DTYPE_BF16) {
    if (nt == 1) return launch_stream<uint16_t, 1>(args, grid, stream);
    if (nt == 2) return launch_stream<uint16_t, 2>(args, grid, stream);
    return launch_stream<uint16_t, 4>(args, grid, stream);
  }
  if (nt == 1) return launch_stream<float, 1>(args, grid, stream);
  if (nt == 2) return launch_stream<float, 2>(args, grid, stream);
  return launch_stream<float, 4>(args, grid, stream);
}

}  // namespace wr
