// wr_grouped.cu — the batched layer (two or more bf16 tokens, three or more
// fp32 tokens) as two grouped GEMMs on the 5th-generation tensor cores.
//
// warp-route's batched kernel (src/fused_moe_batched.cu:20-183) gives every
// token its own CTA and streams every selected expert's weights once per
// token, on CUDA cores.  Here the tokens are bucketed per expert first, so
// each expert's weights stream from HBM once per batch and meet all of that
// expert's tokens in tcgen05 MMAs:
//
//   k_route_bucket  one CTA per token: ids / weights (the router of
//                   wr_router.cuh, bit-exact with wr_router_topk); the last
//                   CTA buckets the (token, k) pairs of this rank's experts
//                   into per-expert token lists, each padded to a multiple
//                   of 16 rows with zero-weight rows
//   k_gather        X_g[row] = x[token of row] (bf16), zero for padding
//   k_grouped_gemm<gate/up>
//                   tile = (expert, 128 intermediate rows, <= 256 tokens):
//                   D[token, 256] = X_g rows x [128 gate rows; 128 up rows]
//                   (tokens 128.. of a tile in the second accumulator),
//                   epilogue act = silu(g) * u * w(token, k) stored as bf16
//                   hi + lo (~16 mantissa bits for the second GEMM), in
//                   blocks of 16 act_hi rows each followed by their act_lo
//   k_grouped_gemm<down>
//                   tile = (expert, 256 rows of H, <= 64 / 128 tokens):
//                   D[token half, 256] = act rows x Wd rows, 64 tokens (their
//                   hi and lo rows: 128 A rows) per accumulator, hi + lo
//                   added by a warp shuffle; fp32 partials per K split
//   k_combine       out[t] = sum over k (ascending) of the partials of its
//   (k_combine_ar)  rows (in CTA order): deterministic; with a communicator
//                   the ranks' outputs are also summed over NVLink peer
//                   memory, in rank order.
//
// GEMM structure: the tokens are the MMA's A operand (M = 128 token rows, of
// which a tile's n are loaded), the weights its B operand (N = 256 weight
// rows: one MMA consumes 256 rows x 16 K of weights whatever the token
// count), both K-major bf16 (rows of the packed layout are contiguous along
// K), accumulator fp32 in TMEM.  One persistent CTA per SM, 7 warps: warp 0
// issues the weight TMA loads into a deep ring (they come from HBM), warp 6
// the token-tile loads into a shallow ring (they come from L2), both
// 128-byte swizzled; warp 1 owns TMEM and issues the MMAs (one elected lane,
// tcgen05.commit to release smem stages and to hand accumulators to the
// epilogue); warps 2-5 read the accumulators back with tcgen05.ld (warp w
// reads TMEM lanes 32*(w%4)..+31) and store the results.  Two accumulator
// buffers let the epilogue of one tile overlap the MMAs of the next (down
// tiles above 64 tokens and gate/up tiles above 128 use both).  The K
// chunks of all tiles are dealt to the CTAs in ranges of equal cost
// (stream-K; a chunk of a tile that uses both accumulators costs more).
//
// fp32 (warp-route's dtype): k_gather_f32 and k_grouped_gemm_f32, the same
// structure with every fp32 operand split into bf16 hi + lo (weights by
// converter warps in shared memory); see k_grouped_gemm_f32.
// No TMA multicast anywhere; every wait is bounded and a wait that runs out
// sets the workspace status word and winds the CTA down (copies in flight
// drained, MMAs completed, TMEM freed).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "wr_common.cuh"
#include "wr_internal.h"
#include "wr_router.cuh"

namespace wr {
namespace {

constexpr int kBK = 64;                  // K elements per smem stage: one 128-byte swizzle row
constexpr int kTokM = 128;               // MMA M: token rows (the tile's n, rest unused)
constexpr int kWRows = 256;              // MMA N: weight rows per MMA
constexpr int kRowsA = 128;              // gate/up tile: rows of gate and of up
constexpr int kRowsB = 256;              // down tile: rows of Wd (= rows of H)
constexpr int kNMaxA = kTokM;            // tokens per gate/up tile (one accumulator)
constexpr int kNMaxAWide = 2 * kTokM;    // ... above 128 tokens: both accumulators (T > 128)
constexpr int kNMaxB = 64;               // tokens per down accumulator (act_hi, act_lo: 128 A rows)
constexpr int kNMaxBWide = 128;          // tokens per down tile above 64 tokens: both accumulators
constexpr int kRowB = kBK * 2;           // bytes of one row per stage
constexpr int kWBox = 128;               // weight rows per TMA box
constexpr int kBoxRows = 16;             // token rows: tiles are multiples of this
constexpr int kTokMaps = kTokM / kBoxRows;  // token maps with boxes of 16, 32, .., 128 rows
constexpr int kWStageBytes = kWRows * kRowB;  // 32 KB
constexpr int kTokBytes = kTokM * kRowB;      // 16 KB: the rows one MMA reads as A
constexpr int kGemmThreads = 224;        // 7 warps
constexpr int kTmemCols = 512;           // two accumulator buffers of 256 columns
constexpr int kAccStride = 256;          // columns between accumulator buffers
constexpr int kSmemMax = 232448;         // 227 KB opt-in shared memory per CTA
constexpr int kSmemBase = 1024 + 512;    // alignment slack, barriers
constexpr int kMaxWStages = 8;           // weight ring depth limit
constexpr int kMaxTStages = 6;           // token ring depth limit (6: gate/up above 128 tokens)
// barriers (full/empty of both rings, 2 x accumulator full/empty, drain) and
// three words (TMEM address, abort, fixup flag) in the first 512 bytes
static_assert((2 * kMaxWStages + 2 * kMaxTStages + 5) * 8 + 12 <= 512, "barrier area");
constexpr int kBucketSmemIds = 5632;    // bucketing stages up to this many ids + weights (44 KB)
constexpr int kJMaxA = 3;                // gate/up: CTAs sharing one tile, at most
constexpr int kJMaxB = 4;                // down: partial sums per output tile, at least this cap
constexpr int kJMaxBLimit = 16;          // ... and at most this one (few tiles: expert parallel)

// Bucket metadata (int32 words in the workspace), written by the bucketing:
//   [0] rows in use, [1] gate/up tiles, [2] down tiles, [3] down cost, [4]
//   the largest down chunk cost present, [5] gate/up cost, [6] the largest
//   gate/up chunk cost present, and from word 16 cnt[E], base[E], ntlA[E],
//   ntlB[E] (token tiles per expert), preA[E+1], preB[E+1] (tiles before
//   each expert), costB[E+1], costA[E+1] (down / gate/up cost before each
//   expert, see chunk_cost).
constexpr int kMetaHdr = 16;
__host__ __device__ inline int meta_words(int E) { return kMetaHdr + 8 * E + 4; }
struct MetaView {
  const int* cnt;
  const int* base;
  const int* ntlA;
  const int* ntlB;
  const int* preA;
  const int* preB;
  const int* costB;
  const int* costA;
};
__host__ __device__ inline MetaView meta_view(const int* m, int E) {
  MetaView v;
  v.cnt = m + kMetaHdr;
  v.base = v.cnt + E;
  v.ntlA = v.base + E;
  v.ntlB = v.ntlA + E;
  v.preA = v.ntlB + E;
  v.preB = v.preA + E + 1;
  v.costB = v.preB + E + 1;
  v.costA = v.costB + E + 1;
  return v;
}

// Work is split by cost, not by chunk count.  When a launch has wide tiles
// (gate/up: above 128 tokens, two MMAs and two token slots per K step;
// down: above 64 tokens, two MMAs per K step) a chunk of a wide tile costs
// kCostWideA / kCostWideB units and any other chunk kCostOne (measured: the
// CTAs holding wide down chunks ran about 1.2x as long per chunk, wide
// gate/up chunks about 1.4x); otherwise every chunk costs 1, which is the
// plain chunk split.
constexpr int kCostOne = 5;
constexpr int kCostWideA = 7;
constexpr int kCostWideB = 6;
template <bool kGU>
__host__ __device__ inline int chunk_cost(int n, int nmax) {
  constexpr int narrow = kGU ? kTokM : kNMaxB;
  return nmax > narrow ? (n > narrow ? (kGU ? kCostWideA : kCostWideB) : kCostOne) : 1;
}

// Per-expert cost: chunk costs of its full and last token tiles and the
// cost of one weight-row tile's token tiles (r).
struct TileCost {
  int wfull, wlast;
  int64_t r;
};
template <bool kGU>
__host__ __device__ inline TileCost tile_cost_of(int cnt, int nt, int nmax, int kc) {
  TileCost d;
  const int np = (cnt + 15) & ~15;
  d.wfull = chunk_cost<kGU>(nmax, nmax);
  d.wlast = nt > 0 ? chunk_cost<kGU>(np - (nt - 1) * nmax, nmax) : 0;
  d.r = nt > 0 ? (int64_t)kc * ((int64_t)(nt - 1) * d.wfull + d.wlast) : 0;
  return d;
}

// ---------------------------------------------------------------------------
// tcgen05 / TMA wrappers
// ---------------------------------------------------------------------------

// Shared-memory matrix descriptor for a K-major bf16 tile written by TMA with
// 128-byte swizzling: rows of 128 bytes, 8-row groups 1024 bytes apart (SBO),
// descriptor version 1, layout type 2 (128-byte swizzle).  The tile base must
// be 1024-byte aligned; stepping along K inside the 128-byte row adds the
// byte offset to the start address.
WR_DEVINL uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16: bf16 A and B, fp32 accumulator, both
// K-major, M = m (64 or 128), N = n (multiple of 16, 16..256).
WR_DEVINL uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

WR_DEVINL void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 operation this thread issued so
// far has completed.
WR_DEVINL void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

WR_DEVINL void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
WR_DEVINL void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

WR_DEVINL void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(cols)
               : "memory");
}
WR_DEVINL void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
WR_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}

// 16 consecutive fp32 columns of this warp's 32 TMEM lanes (one per thread).
WR_DEVINL void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
// Waits for this thread's tcgen05.ld results; the registers are threaded
// through the asm so no use of them can be scheduled before the wait.
WR_DEVINL void tmem_wait_ld(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
                 "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]),
                 "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}
WR_DEVINL void reg_dep16(uint32_t (&v)[16]) {
  asm volatile(""
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
                 "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]),
                 "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}

// Tiled TMA loads (no multicast) into this CTA's shared memory, completion
// counted in bytes on `bar`.  The innermost coordinate is always a multiple
// of 64 bf16 elements (128 bytes).
WR_DEVINL void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                           uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
WR_DEVINL void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                           uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// Named barrier `id` over `n` threads that also ORs `v` across them: every
// participant gets the same answer, so a decision taken on it is uniform.
WR_DEVINL bool named_bar_or(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.or.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

WR_DEVINL void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---------------------------------------------------------------------------
// Routing and bucketing
// ---------------------------------------------------------------------------

// One CTA.  Pairs (t, k) whose expert is in [ep_first, ep_first + E) get a
// row: expert e's rows are base[e] .. base[e] + cnt[e] - 1 in ascending
// token order, followed by zero-weight padding up to a multiple of 16.
// Pairs of other ranks' experts get slot -1.  Each row also gets its first
// down tile and the tile stride between H tiles (row_tile), which the
// combine uses.  Writes the tile counts the GEMM kernels walk (per expert
// ntlA / ntlB token tiles of <= nmaxA / nmaxB rows; mtA * ntlA gate/up and
// mtB * ntlB down tiles) and zeroes the gate/up tile counters (robust against
// a call that gave up half-way).
struct BucketArgs {
  const int32_t* ids;  // [TK], written by the routing CTAs of the same launch
  const float* w;
  int TK, K, ep_first, E, nmaxA, nmaxB, mtA, mtB, kcA, kcB;
  int* meta;
  int32_t* slot;
  int32_t* row_tok;
  int4* row_tile;  // per row: {cost position of its down tile at H tile 0, cost per H tile, chunk cost}
  float* row_w;
  uint32_t* tile_cnt;
  int cnt_words;
};

// Row i of expert e: its down tile's cost position at H tile 0, the cost
// between H tiles, its chunk cost (the combine finds the tile's CTAs so).
WR_DEVINL int4 down_row_tile(int i, int e, int nmaxB, int kcB, const int* costB, const int* rowB,
                             const int (*wB)[2], const int* ntlB) {
  const int tn = i / nmaxB;
  const int wt = tn == ntlB[e] - 1 ? wB[e][1] : wB[e][0];
  return make_int4(costB[e] + tn * kcB * wB[e][0], rowB[e], wt, 0);
}

// Warp-wide inclusive prefix sum.
WR_DEVINL int warp_incl_sum(int v, int lane) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += u;
  }
  return v;
}

constexpr int kBucketWarps = kRouterSegments;  // the routing CTA's warps

// Run by one whole CTA of kBucketWarps warps.  s_ids: dynamic shared memory
// of 8 * TK bytes when TK <= kBucketSmemIds (the ids, then the weights, are
// staged there).  The ids and weights were written by other CTAs of this
// launch: read through L2.
//
// Work is linear in the pairs: warp w takes a contiguous span of the (token,
// k) pairs; pass 1 counts its pairs per expert (lanes of one expert found
// with match.any), a scan over the warps gives each warp its first rank in
// every expert, the metadata (per-expert bases, tile counts and cost
// prefixes) is one warp's shuffle scans over the experts, and pass 2 gives
// each pair its row: expert base + the warp's running rank + its rank among
// the warp's lanes of that expert.  Rows of an expert are therefore in pair
// order, i.e. ascending token order (a token picks an expert at most once).
__device__ void bucket_body(const BucketArgs& b, int* s_ids) {
  const int32_t* __restrict__ ids = b.ids;
  const float* __restrict__ w = b.w;
  const int TK = b.TK, K = b.K, ep_first = b.ep_first, E = b.E;
  const int nmaxA = b.nmaxA, nmaxB = b.nmaxB, mtA = b.mtA, mtB = b.mtB, kcA = b.kcA, kcB = b.kcB;
  int* __restrict__ meta = b.meta;
  int32_t* __restrict__ slot = b.slot;
  int32_t* __restrict__ row_tok = b.row_tok;
  int4* __restrict__ row_tile = b.row_tile;
  float* __restrict__ row_w = b.row_w;
  uint32_t* __restrict__ tile_cnt = b.tile_cnt;
  const int cnt_words = b.cnt_words;
  __shared__ int s_cnt[kMaxExperts];
  __shared__ int s_base[kMaxExperts];
  __shared__ int s_costB[kMaxExperts];  // down cost before the expert
  __shared__ int s_rowB[kMaxExperts];   // down cost of one H tile row of its token tiles
  __shared__ int s_wB[kMaxExperts][2];  // chunk cost: full token tiles, last token tile
  __shared__ int s_ntlB[kMaxExperts];
  __shared__ int s_wcnt[kBucketWarps][kMaxExperts];  // per warp: pairs, then running rank
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool staged = TK <= kBucketSmemIds;
  for (int i = threadIdx.x; i < cnt_words; i += blockDim.x) tile_cnt[i] = 0u;
  for (int i = threadIdx.x; i < kBucketWarps * kMaxExperts; i += blockDim.x)
    (&s_wcnt[0][0])[i] = 0;
  float* s_w = reinterpret_cast<float*>(s_ids + TK);
  for (int i = threadIdx.x; i < TK; i += blockDim.x) {
    const int id = __ldcg(ids + i);
    if (staged) {
      s_ids[i] = id;
      s_w[i] = __ldcg(w + i);
    }
    const int e = id - ep_first;
    if (e < 0 || e >= E) slot[i] = -1;
  }
  __syncthreads();
  // (unstaged: the routing is read through L2 again; it was written by other CTAs)
  struct Src {
    const int* p;
    bool smem;
    WR_DEVINL int operator[](int i) const { return smem ? p[i] : __ldcg(p + i); }
  };
  struct SrcF {
    const float* p;
    bool smem;
    WR_DEVINL float operator[](int i) const { return smem ? p[i] : __ldcg(p + i); }
  };
  const Src sid{staged ? s_ids : ids, staged};
  const SrcF sw{staged ? s_w : w, staged};
  // this warp's span of pairs, a multiple of 32
  const int span = ((TK + kBucketWarps - 1) / kBucketWarps + 31) & ~31;
  const int j0 = warp * span;
  const int j1 = min(TK, j0 + span);
  // pass 1: the span's pairs per local expert
  for (int j = j0; j < j1; j += 32) {
    const int i = j + lane;
    const int e = i < j1 ? sid[i] - ep_first : -1;
    const bool mine = e >= 0 && e < E;
    const unsigned peers = __match_any_sync(0xffffffffu, mine ? e : -1);
    if (mine && lane == __ffs(peers) - 1) s_wcnt[warp][e] += __popc(peers);
  }
  __syncthreads();
  // per expert: each warp's first rank (exclusive scan over the warps), the total
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int v = 0; v < kBucketWarps; ++v) {
      const int t = s_wcnt[v][e];
      s_wcnt[v][e] = run;
      run += t;
    }
    s_cnt[e] = run;
  }
  __syncthreads();
  if (warp == 0) {
    // per-expert metadata: lane l takes experts l, l + 32 (E <= 64); bases,
    // tile prefixes and cost prefixes are exclusive scans over the experts
    int* cnt = meta + kMetaHdr;
    int* base = cnt + E;
    int* ntlA = base + E;
    int* ntlB = ntlA + E;
    int* preA = ntlB + E;
    int* preB = preA + E + 1;
    int* costB = preB + E + 1;
    int* costA = costB + E + 1;
    int cb_ = 0, cpa = 0, cpb = 0, ccb = 0, cca = 0, wmax = 1, wmaxA = 1;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const bool on = e < E;
      const int n = on ? s_cnt[e] : 0;
      const int np = (n + 15) & ~15;
      const int na = (np + nmaxA - 1) / nmaxA;
      const int nb = (np + nmaxB - 1) / nmaxB;
      const TileCost dc = tile_cost_of<false>(n, nb, nmaxB, kcB);
      const TileCost da = tile_cost_of<true>(n, na, nmaxA, kcA);
      const int vb = np, vpa = mtA * na, vpb = mtB * nb, vcb = mtB * (int)dc.r,
                vca = mtA * (int)da.r;
      const int ib = warp_incl_sum(vb, lane), ipa = warp_incl_sum(vpa, lane),
                ipb = warp_incl_sum(vpb, lane), icb = warp_incl_sum(vcb, lane),
                ica = warp_incl_sum(vca, lane);
      if (on) {
        const int xb = cb_ + ib - vb, xcb = ccb + icb - vcb;
        cnt[e] = n;
        base[e] = xb;
        s_base[e] = xb;
        ntlA[e] = na;
        ntlB[e] = nb;
        s_ntlB[e] = nb;
        preA[e] = cpa + ipa - vpa;
        preB[e] = cpb + ipb - vpb;
        costA[e] = cca + ica - vca;
        costB[e] = xcb;
        s_costB[e] = xcb;
        s_rowB[e] = (int)dc.r;
        s_wB[e][0] = dc.wfull;
        s_wB[e][1] = dc.wlast;
        if (nb > 0) wmax = max(wmax, nb > 1 ? dc.wfull : dc.wlast);
        if (na > 0) wmaxA = max(wmaxA, na > 1 ? da.wfull : da.wlast);
      }
      cb_ += __shfl_sync(0xffffffffu, ib, 31);
      cpa += __shfl_sync(0xffffffffu, ipa, 31);
      cpb += __shfl_sync(0xffffffffu, ipb, 31);
      ccb += __shfl_sync(0xffffffffu, icb, 31);
      cca += __shfl_sync(0xffffffffu, ica, 31);
    }
    wmax = __reduce_max_sync(0xffffffffu, wmax);
    wmaxA = __reduce_max_sync(0xffffffffu, wmaxA);
    if (lane == 0) {
      preA[E] = cpa;
      preB[E] = cpb;
      costB[E] = ccb;
      costA[E] = cca;
      meta[0] = cb_;
      meta[1] = cpa;
      meta[2] = cpb;
      meta[3] = ccb;
      meta[4] = wmax;
      meta[5] = cca;
      meta[6] = wmaxA;
    }
  }
  __syncthreads();
  // pass 2: each pair's row, in pair order within the warp's span
  for (int j = j0; j < j1; j += 32) {
    const int i = j + lane;
    const int e = i < j1 ? sid[i] - ep_first : -1;
    const bool mine = e >= 0 && e < E;
    const unsigned peers = __match_any_sync(0xffffffffu, mine ? e : -1);
    const int rank = mine ? s_wcnt[warp][e] + __popc(peers & ((1u << lane) - 1u)) : 0;
    __syncwarp();  // every lane has read the running rank before its update
    if (mine) {
      const int b0 = s_base[e];
      const int r = b0 + rank;
      slot[i] = r;
      row_tok[r] = i / K;
      row_tile[r] = down_row_tile(rank, e, nmaxB, kcB, s_costB, s_rowB, s_wB, s_ntlB);
      row_w[r] = sw[i];
      if (lane == __ffs(peers) - 1) s_wcnt[warp][e] += __popc(peers);
    }
    __syncwarp();
  }
  // padding rows of each expert (up to a multiple of 16)
  for (int e = warp; e < E; e += kBucketWarps) {
    const int b0 = s_base[e], n = s_cnt[e];
    const int end = b0 + ((n + 15) & ~15);
    for (int r = b0 + n + lane; r < end; r += 32) {
      row_tok[r] = -1;
      row_tile[r] = down_row_tile(r - b0, e, nmaxB, kcB, s_costB, s_rowB, s_wB, s_ntlB);
      row_w[r] = 0.0f;
    }
  }
}

// Router and bucketing in one launch: CTA t computes token t's logits,
// softmax and top-K (the router of wr_router.cuh, bit-exact with
// wr_router_topk: warp j computes segment j of every router row, reading x
// in 16-byte vectors), writes ids / weights, and counts itself in; the last
// CTA to finish (no waiting) buckets every token.
constexpr int kRouteThreads = 32 * kRouterSegments;
constexpr int kCtlRoute = 4;  // control word: routing CTAs done (zero between launches)

template <typename Tx>
__global__ void __launch_bounds__(kRouteThreads) k_route_bucket(
    const Tx* __restrict__ x, const Tx* __restrict__ gate_w,
    const float* __restrict__ bias, int E_all, int H, bool vec_ok, uint32_t* __restrict__ ctl,
    int32_t* __restrict__ ids_out, float* __restrict__ w_out, const BucketArgs b) {
  extern __shared__ int s_dyn[];
  __shared__ float parts[kRouterSegments * kMaxExperts];
  __shared__ float lg[kMaxExperts];
  __shared__ int tids[kMaxExperts];
  __shared__ float tws[kMaxExperts];
  __shared__ int s_last;
  // While the previous kernel finishes: this CTA's share of the router rows
  // and its token row into L2 (aligned inputs only).  gate_w does not depend
  // on that kernel and x may, but a prefetch into L2, the point of
  // coherence, cannot make a later read return stale data.
  if (threadIdx.x == 0 && vec_ok) {
    prefetch_share_l2(gate_w, (int64_t)E_all * H * sizeof(Tx), blockIdx.x, gridDim.x);
    prefetch_share_l2(x + (int64_t)blockIdx.x * H, (int64_t)H * sizeof(Tx), 0, 1);
  }
  griddep_wait();
  griddep_launch_dependents();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = b.K;
  router_segment_warp<Tx>(gate_w, XGlobal<Tx>{x + (int64_t)t * H}, E_all, H, warp, lane, vec_ok,
                          parts + warp * kMaxExperts);
  __syncthreads();
  for (int e = threadIdx.x; e < E_all; e += blockDim.x)
    lg[e] = router_combine(parts, kMaxExperts, e, bias);
  __syncthreads();
  if (warp == 0) {
    select_topk_warp(lg, E_all, K, lane, tids, tws);
    __syncwarp();
    for (int k = lane; k < K; k += 32) {
      ids_out[(int64_t)t * K + k] = tids[k];
      w_out[(int64_t)t * K + k] = tws[k];
    }
    __threadfence();  // this token's routing is visible before it is counted in
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(ctl + kCtlRoute, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  bucket_body(b, s_dyn);
  if (threadIdx.x == 0) ctl[kCtlRoute] = 0u;  // ready for the next call
}

// X_g[row, :] = x[row_tok[row], :] (bf16, 16-byte chunks), zero for padding.
__global__ void __launch_bounds__(256) k_gather(const uint4* __restrict__ x, int H8,
                                                const int* __restrict__ meta,
                                                const int32_t* __restrict__ row_tok,
                                                uint4* __restrict__ xg) {
  griddep_wait();
  griddep_launch_dependents();
  const int rows = meta[0];
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int t = row_tok[r];
    uint4* dst = xg + (int64_t)r * H8;
    if (t >= 0) {
      const uint4* src = x + (int64_t)t * H8;
      for (int c = threadIdx.x; c < H8; c += blockDim.x) dst[c] = src[c];
    } else {
      for (int c = threadIdx.x; c < H8; c += blockDim.x) dst[c] = make_uint4(0, 0, 0, 0);
    }
  }
}

// Activation rows: token row r's act_hi is row act_row_hi(r) and its act_lo
// 16 rows further: blocks of 16 act_hi rows, each followed by the same 16
// tokens' act_lo rows.  A down tile's 2n rows are then one TMA box per 64
// tokens, and as an MMA's A rows they put token t's two halves (t < 64) in
// accumulator lanes 32q + l and 32q + 16 + l (q = t / 16, l = t % 16): the
// same warp, 16 lanes apart.
WR_DEVINL int64_t act_row_hi(int r) { return 2 * (int64_t)(r & ~15) + (r & 15); }

// fp32 tokens: X_g holds each row split into bf16 hi = rn(x) and lo =
// rn(x - hi), laid out like the activations (act_row_hi): blocks of 16 hi
// rows, each followed by the same 16 rows' lo parts; zero for padding.
__global__ void __launch_bounds__(256) k_gather_f32(const float4* __restrict__ x, int H8,
                                                    const int* __restrict__ meta,
                                                    const int32_t* __restrict__ row_tok,
                                                    uint4* __restrict__ xg) {
  griddep_wait();
  griddep_launch_dependents();
  const int rows = meta[0];
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int t = row_tok[r];
    uint4* hi = xg + act_row_hi(r) * H8;
    uint4* lo = hi + 16 * (int64_t)H8;
    for (int c = threadIdx.x; c < H8; c += blockDim.x) {
      if (t < 0) {
        hi[c] = lo[c] = make_uint4(0, 0, 0, 0);
        continue;
      }
      const float4 a = x[((int64_t)t * H8 + c) * 2], b = x[((int64_t)t * H8 + c) * 2 + 1];
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      uint32_t ph[4], pl[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const __nv_bfloat16 h0 = __float2bfloat16_rn(v[2 * k]), h1 = __float2bfloat16_rn(v[2 * k + 1]);
        ph[k] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
        const __nv_bfloat16 l0 = __float2bfloat16_rn(v[2 * k] - __bfloat162float(h0));
        const __nv_bfloat16 l1 = __float2bfloat16_rn(v[2 * k + 1] - __bfloat162float(h1));
        pl[k] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
      }
      hi[c] = make_uint4(ph[0], ph[1], ph[2], ph[3]);
      lo[c] = make_uint4(pl[0], pl[1], pl[2], pl[3]);
    }
  }
}

// ---------------------------------------------------------------------------
// Work split (stream-K), both GEMMs: the tiles' K chunks, laid end to end
// (tile-major), chunk (tile, k) at cost position pos(tile) + k * w(tile)
// (w: chunk_cost), are cut into G ranges of equal cost, one per CTA: CTA c
// takes the chunks whose position lies in [c C / G, (c + 1) C / G).  A tile
// whose chunks straddle several ranges is finished from partial sums: for
// the down projection each CTA writes an fp32 partial that the combine adds
// (in CTA order); for gate/up the partial accumulators go to a scratch
// buffer and the last CTA to finish the tile adds them (in CTA order) and
// applies SwiGLU.  G is capped so that every range holds at least
// L = ceil(kc / (jmax - 1)) chunks of the dearest kind present, which bounds
// the CTAs per tile by jmax.
// ---------------------------------------------------------------------------
struct CostSplit {
  int64_t C;  // total cost
  int G;      // CTAs with work
  // CTA whose range holds position p: the largest c with floor(c C / G) <= p.
  WR_DEVINL int cta_of(int64_t p) const { return (int)(((p + 1) * G - 1) / C); }
  WR_DEVINL int64_t lo(int c) const { return (int64_t)c * C / G; }
};

WR_DEVINL CostSplit make_costsplit(int64_t C, int kc, int grid, int jmax, int wmax) {
  CostSplit s;
  s.C = C;
  const int64_t L = (kc + jmax - 2) / (jmax - 1);
  int64_t g = C / (L * wmax);
  if (g < 1) g = 1;
  if (g > grid) g = grid;
  s.G = (int)g;
  return s;
}

// out[t, :] = sum over k ascending of (slot >= 0 ? sum over the tile's
// partials in slot order : 0).  One fixed order: deterministic.
__global__ void __launch_bounds__(256) k_combine(const float4* __restrict__ ypart,
                                                 const int32_t* __restrict__ slot,
                                                 const int4* __restrict__ row_tile,
                                                 const int* __restrict__ meta, int K, int H4,
                                                 int rmax, int kcB, int rowsB, int grid,
                                                 int jmax, const Residual res,
                                                 float4* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  const int t = blockIdx.x;
  const int h = blockIdx.y * blockDim.x + threadIdx.x;
  if (h >= H4) return;
  const CostSplit cs = make_costsplit(meta[3], kcB, grid, jmax, meta[4]);
  const int mt = (h * 4) / rowsB;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < K; ++k) {
    const int r = slot[(int64_t)t * K + k];
    if (r < 0) continue;
    const int4 rt = row_tile[r];
    const int64_t pos = rt.x + (int64_t)mt * rt.y;
    const int c0 = cs.cta_of(pos);
    const int c1 = cs.cta_of(pos + (int64_t)(kcB - 1) * rt.z);
    for (int j = 0; j <= c1 - c0; ++j) {
      const float4 v = ypart[((int64_t)j * rmax + r) * H4 + h];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
  }
  const int64_t i = ((int64_t)t * H4 + h) * 4;
  acc.x = residual_out(res, i + 0, acc.x);
  acc.y = residual_out(res, i + 1, acc.y);
  acc.z = residual_out(res, i + 2, acc.z);
  acc.w = residual_out(res, i + 3, acc.w);
  out[(int64_t)t * H4 + h] = acc;
}

// The combine with the ranks' outputs summed over NVLink peer memory, for
// tokens [t0, t0 + Tc) (Tc <= kCommMaxTokens).  Each thread's (token, 4
// columns) items: the partial output is written as words (fp32 | epoch << 32)
// into this rank's slot of every rank's mailbox (relaxed system-scope
// stores), then the words of every source rank are polled in this rank's
// mailbox until they carry this launch's epoch and summed in rank order
// (bit-identical on every rank).  An aligned 64-bit store is single-copy
// atomic, so a word with the right epoch has the right value.  The grid is
// small enough to be resident at once on every rank (no CTA waits for a
// peer CTA that cannot run); the last CTA to finish publishes the epoch.
constexpr int kCtlExit = 1;  // control word: CTAs done (the streaming kernel's, zero between launches)

__global__ void __launch_bounds__(256) k_combine_ar(const float4* __restrict__ ypart,
                                                    const int32_t* __restrict__ slot,
                                                    const int4* __restrict__ row_tile,
                                                    const int* __restrict__ meta, int K, int H,
                                                    int rmax, int kcB, int rowsB, int grid,
                                                    int jmax, int t0,
                                                    int Tc, const CommView comm,
                                                    const Residual res,
                                                    uint32_t* __restrict__ ctl,
                                                    float* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ uint32_t s_ep;
  if (threadIdx.x == 0) s_ep = *comm.epoch + 1;
  __syncthreads();
  const uint32_t ep = s_ep;
  const CostSplit cs = make_costsplit(meta[3], kcB, grid, jmax, meta[4]);
  const int H4 = H / 4;
  const int items = Tc * H4;
  const int stride = gridDim.x * blockDim.x;
  const uint64_t tag = (uint64_t)ep << 32;
  for (int it = blockIdx.x * blockDim.x + threadIdx.x; it < items; it += stride) {
    const int tl = it / H4, h4 = it - tl * H4;
    const int t = t0 + tl;
    const int mt = (h4 * 4) / rowsB;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < K; ++k) {
      const int r = slot[(int64_t)t * K + k];
      if (r < 0) continue;
      const int4 rt = row_tile[r];
      const int64_t pos = rt.x + (int64_t)mt * rt.y;
      const int c0 = cs.cta_of(pos), c1 = cs.cta_of(pos + (int64_t)(kcB - 1) * rt.z);
      for (int j = 0; j <= c1 - c0; ++j) {
        const float4 v = ypart[((int64_t)j * rmax + r) * H4 + h4];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
    }
    const size_t off =
        (((size_t)comm.rank * 2 + (ep & 1u)) * kCommMaxTokens + tl) * (size_t)H + 4 * h4;
    for (int q = 0; q < comm.world; ++q) {
      uint64_t* d = comm.box[q] + off;
      st_relaxed_sys_u64(d + 0, tag | __float_as_uint(acc.x));
      st_relaxed_sys_u64(d + 1, tag | __float_as_uint(acc.y));
      st_relaxed_sys_u64(d + 2, tag | __float_as_uint(acc.z));
      st_relaxed_sys_u64(d + 3, tag | __float_as_uint(acc.w));
    }
  }
  const uint64_t tstart = globaltimer_ns();
  bool late = false;
  for (int it = blockIdx.x * blockDim.x + threadIdx.x; it < items; it += stride) {
    const int tl = it / H4, h4 = it - tl * H4;
    // every source's four words loaded at once, then any missing one polled
    // alone; summed in source-rank order
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    const uint64_t* pb =
        comm.box[comm.rank] + ((size_t)(ep & 1u) * kCommMaxTokens + tl) * (size_t)H + 4 * h4;
    const size_t qs = (size_t)2 * kCommMaxTokens * H;  // words between sources
    uint64_t wv[kMaxRanks][4];
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q)
      if (q < comm.world) {
#pragma unroll
        for (int c = 0; c < 4; ++c) wv[q][c] = ld_relaxed_sys_u64(pb + q * qs + c);
      }
#pragma unroll
    for (int q = 0; q < kMaxRanks; ++q) {
      if (q < comm.world) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          for (uint32_t spin = 1; (uint32_t)(wv[q][c] >> 32) != ep && !late; ++spin) {
            if ((spin & 63u) == 0 && globaltimer_ns() - tstart > comm.peer_wait_ns) {
              atomicOr(ctl + 2, DEV_TIMEOUT_PEER);
              late = true;
            }
            wv[q][c] = ld_relaxed_sys_u64(pb + q * qs + c);
          }
          o[c] += __uint_as_float((uint32_t)wv[q][c]);
        }
      }
    }
    const int64_t i = (int64_t)(t0 + tl) * H + 4 * h4;
#pragma unroll
    for (int c = 0; c < 4; ++c) o[c] = residual_out(res, i + c, o[c]);
    *reinterpret_cast<float4*>(out + i) = make_float4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(ctl + kCtlExit, 1u);
    if (prev == gridDim.x - 1) {  // every CTA has left its waits
      *comm.epoch = ep;          // the next launch uses epoch + 1
      atomicExch(ctl + kCtlExit, 0u);
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------------------
// Grouped GEMM
// ---------------------------------------------------------------------------

struct GemmArgs {
  const int* meta;
  int E;               // experts of this rank
  int H, I;
  int nmax;            // token rows per tile
  int kc_total;        // K chunks of kBK per tile (gate/up: over H, down: over I)
  int mrows;           // weight rows per tile (gate/up: of gate and of up; down: of Wd)
  int rmax;            // token rows (padded per expert)
  int wstages, tstages;  // weight ring / token ring depth
  int tstage_bytes;      // token slot: gate/up min(nmax, 128) rows, down 2 * nmax rows
  const float* row_w;  // gate/up epilogue: per-row routing weight
  uint16_t* act;       // gate/up output: [2 rmax][I] bf16, rows as act_row_hi / + 16
  float* ypart;        // down output: [jmax][rmax][H] fp32
  int jmax;            // CTAs per tile, at most (gate/up: kJMaxA)
  float* pbuf;         // gate/up partial accumulators: [CTA][2][nmax][256] fp32 (nmax <= 256)
  uint32_t* cnt;       // gate/up: CTAs done with each cut tile (zeroed by the bucketing)
  uint32_t* status;
};

// One unit of a CTA's work: weight rows starting at m0 (gate/up: rows
// m0..m0+127 of gate and of up; down: rows m0..m0+255 of Wd) of expert e
// against token rows [row0, row0 + n), K chunks [kc0, kc1) taken in the
// rotated order kc0 + (rot + i) % (kc1 - kc0); j = partial slot (down);
// pos, wt = the tile's cost position and chunk cost (the gate/up fixup
// finds the tile's CTAs from them).  The rotation depends only on the tile,
// so the summation order is fixed; it spreads the CTAs that share a token
// tile over different K chunks, so they do not all fetch the same L2 lines
// at the same moment.
struct Work {
  int tile, e, m0, row0, n, kc0, kc1, rot, j, wt;
  int64_t pos;
  WR_DEVINL int kc_at(int i) const {
    const int len = kc1 - kc0;
    int k = rot + i;
    if (k >= len) k -= len;
    return kc0 + k;
  }
};

// The sequence of work one CTA runs: the pieces of the tiles whose chunks'
// cost positions lie in its range, cut at tile boundaries; every role of the
// CTA walks the same sequence.  Tiles are numbered expert-major; inside an
// expert the token tile varies fastest, then the weight-row tile.  The grid
// cap uses the largest chunk cost present, as the down combine does.
//
// gate/up: when the range ends inside a tile, that piece runs first.  The
// CTA holding a tile's last piece sums the tile's partials (the fixup); run
// at the end of the range, that sum is the tail of the kernel, run first it
// overlaps the MMAs of the whole tiles that follow.  The order of pieces
// changes no sum: partials are added in CTA order.
template <bool kGU>
struct WorkIter {
  CostSplit cs;
  int64_t p, p1;  // next chunk position to take, end of the stretch being walked
  int64_t q, q1;  // then the stretch [q, q1) (empty when q >= q1)
  int e, m, tn;   // the tile p lies in (or the next one)

  WR_DEVINL const int* cost_prefix(const MetaView& mv) const { return kGU ? mv.costA : mv.costB; }
  WR_DEVINL int tiles_of(const MetaView& mv, int x) const {
    return __ldg((kGU ? mv.ntlA : mv.ntlB) + x);
  }

  // (e, m, tn) = the tile whose cost span holds position x.
  WR_DEVINL void seek(const GemmArgs& a, const MetaView& mv, int64_t x) {
    const int* cost = cost_prefix(mv);
    e = 0;
    while (e + 1 < a.E && __ldg(cost + e + 1) <= x) ++e;  // experts without tiles cost 0
    const int nt = tiles_of(mv, e);
    const TileCost tc = tile_cost_of<kGU>(__ldg(mv.cnt + e), nt, a.nmax, a.kc_total);
    const int64_t rel = x - __ldg(cost + e);
    m = (int)(rel / tc.r);
    tn = (int)((rel - (int64_t)m * tc.r) / ((int64_t)a.kc_total * tc.wfull));
    if (tn > nt - 1) tn = nt - 1;
  }

  // Cost position and chunk cost of tile (e, m, tn).
  WR_DEVINL void tile_pos(const GemmArgs& a, const MetaView& mv, int64_t& pos, int& wt) const {
    const int nt = tiles_of(mv, e);
    const TileCost tc = tile_cost_of<kGU>(__ldg(mv.cnt + e), nt, a.nmax, a.kc_total);
    wt = tn == nt - 1 ? tc.wlast : tc.wfull;
    pos = __ldg(cost_prefix(mv) + e) + (int64_t)m * tc.r + (int64_t)tn * a.kc_total * tc.wfull;
  }

  WR_DEVINL bool init(const GemmArgs& a) {
    const int64_t C = __ldg(a.meta + (kGU ? 5 : 3));
    cs = make_costsplit(C, a.kc_total, gridDim.x, a.jmax, __ldg(a.meta + (kGU ? 6 : 4)));
    if (C == 0 || (int)blockIdx.x >= cs.G) return false;
    p = cs.lo(blockIdx.x);
    p1 = cs.lo(blockIdx.x + 1);
    q = q1 = 0;
    if (p >= p1) return false;
    const MetaView mv = meta_view(a.meta, a.E);
    if (kGU) {
      // the tile holding the range's last position: if the range ends inside
      // it and it is not the range's first tile, walk [its start, p1) first
      seek(a, mv, p1 - 1);
      int64_t pos;
      int wt;
      tile_pos(a, mv, pos, wt);
      const int64_t k1 = (p1 - pos + wt - 1) / wt;
      if (k1 < a.kc_total && pos > p) {
        q = p;
        q1 = pos;
        p = pos;
        return true;
      }
    }
    seek(a, mv, p);
    return true;
  }

  // The next piece of the stretch [p, p1), or false at its end.
  WR_DEVINL bool take(const GemmArgs& a, const MetaView& mv, Work& w) {
    const int kc = a.kc_total;
    const int mt = ((kGU ? a.I : a.H) + a.mrows - 1) / a.mrows;
    while (p < p1 && e < a.E) {
      const int nt = tiles_of(mv, e);
      int64_t pos;
      int wt;
      tile_pos(a, mv, pos, wt);
      const int64_t k0 = p > pos ? (p - pos + wt - 1) / wt : 0;
      int64_t k1 = (p1 - pos + wt - 1) / wt;
      if (k1 > kc) k1 = kc;
      const int ce = e, cm = m, ctn = tn;
      if (++tn == nt) {  // the tile after this one
        tn = 0;
        if (++m == mt) {
          m = 0;
          do {
            ++e;
          } while (e < a.E && tiles_of(mv, e) == 0);
        }
      }
      if (k0 >= kc) continue;  // p is past this tile's last chunk
      if (k1 <= k0) break;
      p = pos + k1 * wt;
      w.tile = __ldg((kGU ? mv.preA : mv.preB) + ce) + cm * nt + ctn;
      w.kc0 = (int)k0;
      w.kc1 = (int)k1;
      w.j = (int)blockIdx.x - cs.cta_of(pos);
      w.e = ce;
      w.m0 = cm * a.mrows;
      const int np = (__ldg(mv.cnt + ce) + 15) & ~15;
      w.row0 = __ldg(mv.base + ce) + ctn * a.nmax;
      w.n = min(a.nmax, np - ctn * a.nmax);
      w.rot = (int)(((unsigned)w.tile * 37u) % (unsigned)(k1 - k0));
      w.pos = pos;
      w.wt = wt;
      return true;
    }
    p = p1;
    return false;
  }

  WR_DEVINL bool next(const GemmArgs& a, const MetaView& mv, Work& w) {
    for (;;) {
      if (take(a, mv, w)) return true;
      if (q >= q1) return false;
      p = q;
      p1 = q1;
      q = q1 = 0;
      seek(a, mv, p);
    }
  }

  // The CTAs holding pieces of tile w: first and last.
  WR_DEVINL int first_cta(const Work& w) const { return cs.cta_of(w.pos); }
  WR_DEVINL int last_cta(const GemmArgs& a, const Work& w) const {
    return cs.cta_of(w.pos + (int64_t)(a.kc_total - 1) * w.wt);
  }
};

// gate/up partial slots: a CTA has at most two cut tiles, the one its range
// starts in (its piece starts after chunk 0) and the one its range ends in
// (its piece starts at chunk 0: the tile's first CTA); slot 1 is the latter.
WR_DEVINL int part_slot_of_piece(const Work& w) { return w.kc0 == 0 ? 1 : 0; }
WR_DEVINL int part_slot_of_cta(int c, int first) { return c == first ? 1 : 0; }

// TMEM accumulators: two buffers of 256 columns.  A tile of at most 128
// tokens (gate/up) or 64 tokens (down) takes one buffer, the two in turn, so
// the epilogue of one tile overlaps the MMAs of the next; a wider tile takes
// both (its tokens 128.. / 64.. in the second).  The MMA lane and the
// epilogue warps walk the same tiles and derive the same buffers and phases.
struct AccTurns {
  uint32_t use0, use1;  // uses of buffer 0 / 1 so far
  int next;
  WR_DEVINL void init() {
    use0 = use1 = 0u;
    next = 0;
  }
  // This tile's buffers [b0, b0 + nb) and each one's phase for this use.
  WR_DEVINL void take(bool wide, int& b0, int& nb, uint32_t (&ph)[2]) {
    if (wide) {
      b0 = 0;
      nb = 2;
      ph[0] = use0++ & 1u;
      ph[1] = use1++ & 1u;
      next = 0;
    } else if (next == 0) {
      b0 = 0;
      nb = 1;
      ph[0] = use0++ & 1u;
      next = 1;
    } else {
      b0 = 1;
      nb = 1;
      ph[0] = use1++ & 1u;
      next = 0;
    }
  }
};

// An epilogue warp is done reading buffers [b0, b0 + nb): one arrival each.
WR_DEVINL void release_acc(uint64_t* tempty, int b0, int nb, int lane) {
  tc_fence_before();
  __syncwarp();
  if (lane == 0) {
    mbar_arrive(&tempty[b0]);
    if (nb > 1) mbar_arrive(&tempty[b0 + 1]);
  }
}

template <bool kGU>
WR_DEVINL bool tile_is_wide(const Work& w) {
  return w.n > (kGU ? kTokM : kNMaxB);
}

WR_DEVINL void flag_timeout(const GemmArgs& a, volatile int* abort, uint32_t bit) {
  *abort = 1;
  atomicOr(a.status, bit);
}

// Waits until the last arming of each of the `stages` barriers (armed
// `issued` times in ring order) has completed: the copies they count must
// land before this CTA's shared memory is released.
WR_DEVINL void drain_ring(uint64_t* full, int stages, uint32_t issued, uint32_t* status) {
  for (int s = 0; s < stages; ++s) {
    const uint32_t n_s = issued / stages + ((uint32_t)s < issued % stages ? 1u : 0u);
    if (n_s == 0) continue;
    if (!mbar_wait(&full[s], (n_s - 1u) & 1u, nullptr)) {
      atomicOr(status, DEV_TIMEOUT_DRAIN);
      return;
    }
  }
}

// SiLU with the fast exponential and division intrinsics (a few ulp).
WR_DEVINL float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

WR_DEVINL uint32_t pack_bf16x2(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}


// act = silu(g) * u * wt for 16 consecutive intermediate rows i.. of one
// token, stored as bf16 hi (act rounded) and lo (act - hi rounded).
WR_DEVINL void swiglu_store16(const float (&g)[16], const float (&u)[16], float wt, uint16_t* hi,
                              uint16_t* lo, int i, int I) {
  uint32_t ph[8], pl[8];
#pragma unroll
  for (int c = 0; c < 16; c += 2) {
    float av[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) av[k] = silu_fast(g[c + k]) * u[c + k] * wt;
    const __nv_bfloat16 h0 = __float2bfloat16_rn(av[0]);
    const __nv_bfloat16 h1 = __float2bfloat16_rn(av[1]);
    ph[c / 2] = pack_bf16x2(h0, h1);
    pl[c / 2] = pack_bf16x2(__float2bfloat16_rn(av[0] - __bfloat162float(h0)),
                            __float2bfloat16_rn(av[1] - __bfloat162float(h1)));
  }
#pragma unroll
  for (int h = 0; h < 2; ++h)
    if (i + 8 * h < I) {
      *reinterpret_cast<uint4*>(hi + i + 8 * h) =
          make_uint4(ph[4 * h], ph[4 * h + 1], ph[4 * h + 2], ph[4 * h + 3]);
      *reinterpret_cast<uint4*>(lo + i + 8 * h) =
          make_uint4(pl[4 * h], pl[4 * h + 1], pl[4 * h + 2], pl[4 * h + 3]);
    }
}

// D[token, weight row] = tokens (MMA A: M = 128 token rows, of which the
// tile's n are loaded; the rest of the smem tile is stale and only feeds
// accumulator lanes nobody reads) x weights (MMA B: N = 256 weight rows).
// Each MMA takes 256 weight rows x 16 K, whatever the token count.
//
// gate/up: B rows 0..127 = gate rows m0.., 128..255 = up rows m0.., so
//   accumulator lane t (token) holds gate and up of the same rows in columns
//   c and 128 + c: SwiGLU runs in the thread that owns the token.
// down:    up to 64 tokens per tile; A = the tile's 2n activation rows
//   (act_hi and act_lo in blocks of 16, see act_row_hi), so lanes 32q + l
//   and 32q + 16 + l hold the two halves of token 16q + l's output and a
//   warp shuffle adds them.  One MMA per K step at every token count.
//
// Warp roles: 0 weight loads, 6 token loads (one elected lane each), 1 TMEM
// owner + MMA issue (one elected lane), 2..5 epilogue (TMEM lane quarter
// warp % 4).  Weights and tokens have separate smem rings: weights come from
// HBM and need a deep ring, token tiles come from L2 and a shallow one does.
// One token tensor map per tile height: a tile of n rows (a multiple of 16)
// is one TMA box of exactly n rows (every copy instruction costs the single
// issuing thread time in each K step, so 16-row boxes slowed large tiles).
struct TokenMaps {
  CUtensorMap m[kTokMaps];  // m[h - 1]: boxes of 16 h rows
};

template <bool kGU>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_grouped_gemm(const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ TokenMaps tm_b, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  griddep_launch_dependents();

  // [token ring][weight ring][barriers, exchange]: a token slot may be
  // shorter than the 128 rows an MMA reads as A; the overhang reads the
  // following slots or the weight ring (stale rows, unread accumulator lanes).
  uint8_t* tring = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem = tring + (size_t)a.tstages * a.tstage_bytes;
  uint64_t* fullW = reinterpret_cast<uint64_t*>(smem + (size_t)a.wstages * kWStageBytes);
  uint64_t* emptyW = fullW + kMaxWStages;
  uint64_t* fullT = emptyW + kMaxWStages;
  uint64_t* emptyT = fullT + kMaxTStages;
  uint64_t* tfull = emptyT + kMaxTStages;  // [2]
  uint64_t* tempty = tfull + 2;            // [2]
  uint64_t* drain = tempty + 2;            // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.wstages; ++s) {
      mbar_init(&fullW[s], 1);
      mbar_init(&emptyW[s], 1);
    }
    for (int s = 0; s < a.tstages; ++s) {
      mbar_init(&fullT[s], 1);
      mbar_init(&emptyT[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_w);
    for (int h = 0; h < kTokMaps; ++h) prefetch_tmap(&tm_b.m[h]);
  }
  // Everything above touches only this CTA; the previous kernel's outputs
  // (bucket metadata, gathered tokens, activations) are read from here on.
  griddep_wait();
  {
    WorkIter<kGU> probe;
    if (!probe.init(a)) return;  // whole CTA: no work (uniform)
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const MetaView mv = meta_view(a.meta, a.E);

  if (warp == 0 || warp == 6) {
    // ---- TMA producers: warp 0 weights, warp 6 token tiles ----
    if (lane == 0) {
      const bool wprod = warp == 0;
      const uint64_t pol = wprod ? l2_policy_evict_first() : l2_policy_evict_last();
      uint64_t* full = wprod ? fullW : fullT;
      uint64_t* empty = wprod ? emptyW : emptyT;
      const int stages = wprod ? a.wstages : a.tstages;
      uint8_t* ring = wprod ? smem : tring;
      const int sbytes = wprod ? kWStageBytes : a.tstage_bytes;
      int st = 0;
      uint32_t ph = 0;
      uint32_t issued = 0;
      bool ok = true;
      WorkIter<kGU> it;
      it.init(a);
      Work w;
      while (ok && it.next(a, mv, w)) {
        const int nbox = w.n / kBoxRows;
        // a gate/up tile of more than 128 tokens takes two token slots per K
        // step: rows 0..127, then rows 128.. (each slot one MMA's A operand)
        const bool split = kGU && !wprod && w.n > kTokM;
        for (int i = 0; i < w.kc1 - w.kc0 && ok; ++i) {
          const int kc = w.kc_at(i);
          const int kx = kc * kBK;
          for (int h = 0; h < (split ? 2 : 1); ++h) {
            if (!mbar_wait(&empty[st], ph ^ 1u, abort)) {
              if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_EMPTY);
              ok = false;
              break;
            }
            uint8_t* s = ring + (size_t)st * sbytes;
            if (wprod) {
              // gate/up: gate rows m0.. then up rows m0..; down: Wd rows m0..m0+255
              mbar_arrive_expect_tx(&full[st], (uint32_t)kWStageBytes);
              tma_load_3d(s, &tm_w, kx, w.m0, w.e, &full[st], pol);
              tma_load_3d(s + kWBox * kRowB, &tm_w, kx, kGU ? a.I + w.m0 : w.m0 + kWBox, w.e,
                          &full[st], pol);
            } else if (kGU) {
              // the tile's token rows (one half of a split tile)
              const int nb = split ? (h == 0 ? kTokMaps : nbox - kTokMaps) : nbox;
              mbar_arrive_expect_tx(&full[st], (uint32_t)(nb * kBoxRows * kRowB));
              tma_load_2d(s, &tm_b.m[nb - 1], kx, w.row0 + h * kTokM, &full[st], pol);
            } else {
              // its 2n activation rows (act_hi / act_lo blocks of 16, row0 a
              // multiple of 16), at most 128 rows per box: a wide tile's
              // tokens 64.. in a second box
              mbar_arrive_expect_tx(&full[st], (uint32_t)(2 * w.n * kRowB));
              const int b0 = nbox < kTokMaps / 2 ? nbox : kTokMaps / 2;
              tma_load_2d(s, &tm_b.m[2 * b0 - 1], kx, 2 * w.row0, &full[st], pol);
              if (nbox > b0)
                tma_load_2d(s + kTokBytes, &tm_b.m[2 * (nbox - b0) - 1], kx,
                            2 * w.row0 + kTokM, &full[st], pol);
            }
            ++issued;
            if (++st == stages) {
              st = 0;
              ph ^= 1u;
            }
          }
        }
      }
      drain_ring(full, stages, issued, a.status);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      int sw = 0, stt = 0;
      uint32_t phw = 0, pht = 0;
      bool ok = true;
      const uint32_t idesc = idesc_bf16(kTokM, kWRows);
      WorkIter<kGU> it;
      it.init(a);
      Work w;
      AccTurns acc;
      acc.init();
      while (ok && it.next(a, mv, w)) {
        const bool wide = tile_is_wide<kGU>(w);
        int b0, nb;
        uint32_t aph[2];
        acc.take(wide, b0, nb, aph);
#pragma unroll
        for (int b = 0; b < 2; ++b)
          if (b < nb && ok && !mbar_wait(&tempty[b0 + b], aph[b] ^ 1u, abort)) {
            if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_FULL);
            ok = false;
          }
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(b0 * kAccStride);
        for (int i = 0; i < w.kc1 - w.kc0; ++i) {
          if (!mbar_wait(&fullW[sw], phw, abort) || !mbar_wait(&fullT[stt], pht, abort)) {
            if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_FULL);
            ok = false;
            break;
          }
          // a wide gate/up tile's tokens 128.. are in the next token slot; a
          // wide down tile's tokens 64.. (A rows 128..) in the same slot
          int st2 = stt;
          uint32_t ph2 = pht;
          if (kGU && wide) {
            if (++st2 == a.tstages) {
              st2 = 0;
              ph2 ^= 1u;
            }
            if (!mbar_wait(&fullT[st2], ph2, abort)) {
              if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_FULL);
              ok = false;
              break;
            }
          }
          tc_fence_after();
          const uint32_t sw_addr = smem_u32(smem + (size_t)sw * kWStageBytes);
          const uint32_t st_addr = smem_u32(tring + (size_t)stt * a.tstage_bytes);
          const uint32_t st2_addr =
              kGU ? smem_u32(tring + (size_t)st2 * a.tstage_bytes) : st_addr + kTokBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint32_t accum = (i > 0 || kk > 0) ? 1u : 0u;
            const uint64_t wdesc = sw128_desc(sw_addr + kk * 32);
            umma_bf16(d, sw128_desc(st_addr + kk * 32), wdesc, idesc, accum);
            if (wide)
              umma_bf16(d + kAccStride, sw128_desc(st2_addr + kk * 32), wdesc, idesc, accum);
          }
          umma_commit(&emptyW[sw]);
          umma_commit(&emptyT[stt]);
          if (kGU && wide) umma_commit(&emptyT[st2]);
          if (++sw == a.wstages) {
            sw = 0;
            phw ^= 1u;
          }
          stt = st2;
          pht = ph2;
          if (++stt == a.tstages) {
            stt = 0;
            pht ^= 1u;
          }
        }
        if (!ok) break;
#pragma unroll
        for (int b = 0; b < 2; ++b)
          if (b < nb) umma_commit(&tfull[b0 + b]);
      }
      // Every MMA issued above must complete before TMEM is released.
      umma_commit(drain);
      if (!mbar_wait(drain, 0, nullptr)) atomicOr(a.status, DEV_TIMEOUT_DRAIN);
    }
  } else {
    // ---- epilogue: warps 2..5, TMEM lane quarter warp % 4 ----
    const int q = warp & 3;
    WorkIter<kGU> it;
    it.init(a);
    Work w;
    AccTurns acc;
    acc.init();
    while (it.next(a, mv, w)) {
      int b0, nb;
      uint32_t aph[2];
      acc.take(tile_is_wide<kGU>(w), b0, nb, aph);
      bool bad = *abort != 0;
#pragma unroll
      for (int b = 0; b < 2; ++b)
        if (b < nb && !bad && !mbar_wait(&tfull[b0 + b], aph[b], abort)) {
          if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_ACT);
          bad = true;
        }
      // The four epilogue warps leave together or not at all: the down
      // epilogue synchronises them on a named barrier.
      if (named_bar_or(2, 128, bad)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(b0 * kAccStride);
      if (kGU) {
        // lane = token t of the tile (buffer h holds tokens 128h..); columns
        // c / 128 + c = gate / up row m0 + c
        const bool whole = w.kc0 == 0 && w.kc1 == a.kc_total;  // whole tile in this CTA
        for (int h = 0; h < nb; ++h) {
          const int t = kTokM * h + 32 * q + lane;
          if (t - lane >= w.n) continue;  // warp-uniform: this quarter holds no tokens
          const bool live = t < w.n;
          const uint32_t tb = taddr + (uint32_t)(h * kAccStride);
          if (whole) {
            const int r = w.row0 + t;
            uint16_t* hi = a.act + act_row_hi(r) * a.I;
            uint16_t* lo = hi + 16 * (int64_t)a.I;
            const float wt = live ? __ldg(a.row_w + r) : 0.0f;
            for (int c0 = 0; c0 < kRowsA; c0 += 16) {
              uint32_t gv[16], uv[16];
              tmem_ld16(tb + c0, gv);
              tmem_ld16(tb + kRowsA + c0, uv);
              tmem_wait_ld(gv);
              reg_dep16(uv);
              float g[16], u[16];
#pragma unroll
              for (int c = 0; c < 16; ++c) {
                g[c] = __uint_as_float(gv[c]);
                u[c] = __uint_as_float(uv[c]);
              }
              if (live) swiglu_store16(g, u, wt, hi, lo, w.m0 + c0, a.I);
            }
          } else {
            // Cut tile: park this CTA's partial sums (below: count it in; the
            // last CTA of the tile adds the partials in CTA order and applies
            // SwiGLU).
            float* pb =
                a.pbuf +
                (((size_t)blockIdx.x * 2 + part_slot_of_piece(w)) * a.nmax + t) *
                    kWRows;
            for (int c0 = 0; c0 < kWRows; c0 += 16) {
              uint32_t v[16];
              tmem_ld16(tb + c0, v);
              tmem_wait_ld(v);
              if (live) {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  *reinterpret_cast<float4*>(pb + c0 + 4 * k) =
                      make_float4(__uint_as_float(v[4 * k]), __uint_as_float(v[4 * k + 1]),
                                  __uint_as_float(v[4 * k + 2]), __uint_as_float(v[4 * k + 3]));
              }
            }
          }
        }
        // The accumulators are read: hand them back to the MMA lane before
        // the fixup below, so the next tile's MMAs overlap it.
        release_acc(tempty, b0, nb, lane);
        if (!whole) {
          __threadfence();
          named_bar_sync(1, 128);
          const int cf = it.first_cta(w), cl = it.last_cta(a, w);
          if (threadIdx.x == 64) {
            const uint32_t done = atomicAdd(&a.cnt[w.tile], 1u);
            *last_flag = done == (uint32_t)(cl - cf) ? 1 : 0;
          }
          named_bar_sync(1, 128);
          if (*last_flag) {
            __threadfence();
            // The partials live in global memory, so all 128 epilogue threads
            // share the work: item = (token, 16 intermediate rows).
            const int et = threadIdx.x - 64;
            for (int item = et; item < w.n * (kRowsA / 16); item += 128) {
              const int tt = item / (kRowsA / 16);
              const int c0 = (item % (kRowsA / 16)) * 16;
              const int rr = w.row0 + tt;
              // All partials' loads in flight at once (at most kJMaxA CTAs
              // share a tile), then the adds in CTA order.
              float4 gv[kJMaxA][4], uv[kJMaxA][4];
#pragma unroll
              for (int cc = 0; cc < kJMaxA; ++cc) {
                if (cf + cc <= cl) {
                  const float* src = a.pbuf + (((size_t)(cf + cc) * 2 +
                                                part_slot_of_cta(cf + cc, cf)) * a.nmax + tt) *
                                                  kWRows;
#pragma unroll
                  for (int k = 0; k < 4; ++k) {
                    gv[cc][k] = __ldcg(reinterpret_cast<const float4*>(src + c0) + k);
                    uv[cc][k] = __ldcg(reinterpret_cast<const float4*>(src + kRowsA + c0) + k);
                  }
                }
              }
              float g[16], u[16];
#pragma unroll
              for (int c = 0; c < 16; ++c) g[c] = u[c] = 0.0f;
#pragma unroll
              for (int cc = 0; cc < kJMaxA; ++cc) {
                if (cf + cc <= cl) {
#pragma unroll
                  for (int k = 0; k < 4; ++k) {
                    g[4 * k] += gv[cc][k].x; g[4 * k + 1] += gv[cc][k].y;
                    g[4 * k + 2] += gv[cc][k].z; g[4 * k + 3] += gv[cc][k].w;
                    u[4 * k] += uv[cc][k].x; u[4 * k + 1] += uv[cc][k].y;
                    u[4 * k + 2] += uv[cc][k].z; u[4 * k + 3] += uv[cc][k].w;
                  }
                }
              }
              uint16_t* hrow = a.act + act_row_hi(rr) * a.I;
              swiglu_store16(g, u, __ldg(a.row_w + rr), hrow, hrow + 16 * (int64_t)a.I,
                             w.m0 + c0, a.I);
            }
            if (threadIdx.x == 64) a.cnt[w.tile] = 0;  // ready for the next call
          }
        }
      } else {
        // Lane l < 16 of quarter q holds the act_hi part of token 16q + l,
        // lane l + 16 its act_lo part: one shuffle adds them (the same sum in
        // both lanes), and each lane stores 8 of every 16 outputs.
        // A wide tile's tokens 64.. are in the second accumulator, same lanes.
        for (int acc_i = 0; acc_i * kNMaxB < w.n; ++acc_i) {
          const int tok = acc_i * kNMaxB + 16 * q + (lane & 15);
          if (tok - (lane & 15) >= w.n) continue;  // warp-uniform: this quarter holds no tokens
          const bool live = tok < w.n;
          const bool upper = lane >= 16;  // stores columns 8..15 of each 16
          float* yrow = a.ypart + ((int64_t)w.j * a.rmax + w.row0 + tok) * a.H;
          for (int c0 = 0; c0 < kWRows; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(taddr + acc_i * kAccStride + c0, v);
            tmem_wait_ld(v);
            float o[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const float x0 = __uint_as_float(v[c]), x1 = __uint_as_float(v[c + 8]);
              const float s0 = x0 + __shfl_xor_sync(0xffffffffu, x0, 16);
              const float s1 = x1 + __shfl_xor_sync(0xffffffffu, x1, 16);
              o[c] = upper ? s1 : s0;
            }
            const int h = w.m0 + c0 + (upper ? 8 : 0);
            if (live) {
#pragma unroll
              for (int k = 0; k < 2; ++k)
                if (h + 4 * k < a.H)
                  *reinterpret_cast<float4*>(yrow + h + 4 * k) =
                      make_float4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
            }
          }
        }
      }
      if (!kGU) release_acc(tempty, b0, nb, lane);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// fp32 weights (warp-route's own dtype) on the same tensor cores.  The MMAs
// take bf16 operands, so every fp32 value is split into two bf16 parts:
//   * tokens and activations: hi = rn(v), lo = rn(v - hi) (about 2^-17
//     relative), hi and lo rows interleaved in blocks of 16 (act_row_hi), so
//     one MMA's 128 A rows hold 64 tokens' hi and lo parts in accumulator
//     lanes 32q + l and 32q + 16 + l, added by one shuffle;
//   * weights: the fp32 rows land in shared memory by TMA (two 128-byte
//     swizzled boxes of 32 K elements per stage) and four converter warps
//     write hi = the upper 16 bits of v and lo = the upper 16 bits of the
//     exact remainder v - hi (bit operations only; |v - hi - lo| < 2^-14 |v|)
//     as 128 hi rows followed by 128 lo rows in the MMA layout.
// Per K step of 16 one MMA with N = 256: B = [W_hi; W_lo], so accumulator
// columns c and 128 + c hold A.w_hi and A.w_lo of weight row c, added in
// the epilogue; the sum is (x_hi + x_lo) . (w_hi + w_lo) in fp32.  Tiles:
// gate/up 64 gate + 64 up rows (columns 0..63 / 64..127 of each half), down
// 128 rows of Wd; at most 64 tokens per tile.  The weights stream from HBM
// once per batch; each byte of them is read by the TMA and once more by a
// converter.  Shared-memory traffic (TMA writes, the converters' reads and
// writes, the MMA's operand reads) is about 160 KB per 32 KB weight stage.
// ---------------------------------------------------------------------------
constexpr int kF32Rows = 128;                     // weight rows per stage and MMA N
constexpr int kRowsAF = 64;                       // gate/up tile: rows of gate and of up
constexpr int kRowsBF = 128;                      // down tile: rows of Wd
constexpr int kNMaxF = 64;                        // tokens per tile
constexpr int kLStageBytes = kF32Rows * kBK * 4;  // 32 KB fp32 landing stage: two K halves
constexpr int kLHalfBytes = kLStageBytes / 2;     // 128 rows x 32 fp32 (128-byte rows)
constexpr int kCHalfBytes = kF32Rows * kRowB;     // 16 KB: 128 bf16 rows of 64 K
constexpr int kCStageBytes = 2 * kCHalfBytes;     // hi rows, then lo rows
constexpr int kLStagesF = 4, kCStagesF = 2, kTStagesF = 2;
constexpr int kConvWarps = 4;                     // warps 7..10
constexpr int kConvRows = 4;                      // rows a converter lane has in flight
constexpr int kGemmThreadsF = 32 * (7 + kConvWarps);
constexpr int kTmemColsF = 512;                   // two accumulators of 256 columns
constexpr int kAccStrideF = 256;
constexpr int kSmemF = kTStagesF * kTokBytes + kLStagesF * kLStageBytes +
                       kCStagesF * kCStageBytes + kSmemBase;
static_assert(kSmemF <= kSmemMax, "fp32 grouped GEMM shared memory");
static_assert((2 * kLStagesF + 2 * kCStagesF + 2 * kTStagesF + 5) * 8 + 12 <= 512, "barriers");

// act = silu(g) * u * wt for 8 consecutive intermediate rows i.. of one
// token (i a multiple of 8, I a multiple of 8), stored as bf16 hi and lo.
WR_DEVINL void swiglu_store8(const float (&g)[8], const float (&u)[8], float wt, uint16_t* hi,
                             uint16_t* lo, int i, int I) {
  if (i >= I) return;
  uint32_t ph[4], pl[4];
#pragma unroll
  for (int c = 0; c < 8; c += 2) {
    float av[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) av[k] = silu_fast(g[c + k]) * u[c + k] * wt;
    const __nv_bfloat16 h0 = __float2bfloat16_rn(av[0]);
    const __nv_bfloat16 h1 = __float2bfloat16_rn(av[1]);
    ph[c / 2] = pack_bf16x2(h0, h1);
    pl[c / 2] = pack_bf16x2(__float2bfloat16_rn(av[0] - __bfloat162float(h0)),
                            __float2bfloat16_rn(av[1] - __bfloat162float(h1)));
  }
  *reinterpret_cast<uint4*>(hi + i) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
  *reinterpret_cast<uint4*>(lo + i) = make_uint4(pl[0], pl[1], pl[2], pl[3]);
}

// Weight rows c0..c0+15 of this lane's accumulator row: the W_hi column
// c plus the W_lo column 128 + c, hi and lo token lanes added: lanes l < 16
// get rows c0..c0+7, lanes l + 16 rows c0+8..c0+15 (of the same token
// 16q + l).
WR_DEVINL void acc_sum8(uint32_t taddr, int c0, bool upper, float (&o)[8]) {
  uint32_t v[16], u[16];
  tmem_ld16(taddr + c0, v);
  tmem_ld16(taddr + kF32Rows + c0, u);
  tmem_wait_ld(v);
  reg_dep16(u);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const float x0 = __uint_as_float(v[c]) + __uint_as_float(u[c]);
    const float x1 = __uint_as_float(v[c + 8]) + __uint_as_float(u[c + 8]);
    const float s0 = x0 + __shfl_xor_sync(0xffffffffu, x0, 16);
    const float s1 = x1 + __shfl_xor_sync(0xffffffffu, x1, 16);
    o[c] = upper ? s1 : s0;
  }
}

template <bool kGU>
__global__ void __launch_bounds__(kGemmThreadsF, 1)
    k_grouped_gemm_f32(const __grid_constant__ CUtensorMap tm_w,
                       const __grid_constant__ TokenMaps tm_b, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  griddep_launch_dependents();

  // [token ring][fp32 landing ring][bf16 hi/lo ring][barriers]: a token slot
  // holds 2n <= 128 rows; the MMA reads 128 (the overhang: stale rows of the
  // next slot or the landing ring, feeding accumulator lanes nobody reads).
  uint8_t* tring = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* land = tring + kTStagesF * kTokBytes;
  uint8_t* conv = land + kLStagesF * kLStageBytes;
  uint64_t* fullL = reinterpret_cast<uint64_t*>(conv + kCStagesF * kCStageBytes);
  uint64_t* emptyL = fullL + kLStagesF;
  uint64_t* fullC = emptyL + kLStagesF;
  uint64_t* emptyC = fullC + kCStagesF;
  uint64_t* fullT = emptyC + kCStagesF;
  uint64_t* emptyT = fullT + kTStagesF;
  uint64_t* tfull = emptyT + kTStagesF;  // [2]
  uint64_t* tempty = tfull + 2;          // [2]
  uint64_t* drain = tempty + 2;          // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kLStagesF; ++s) {
      mbar_init(&fullL[s], 1);
      mbar_init(&emptyL[s], kConvWarps);
    }
    for (int s = 0; s < kCStagesF; ++s) {
      mbar_init(&fullC[s], kConvWarps);
      mbar_init(&emptyC[s], 1);
    }
    for (int s = 0; s < kTStagesF; ++s) {
      mbar_init(&fullT[s], 1);
      mbar_init(&emptyT[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_w);
    for (int h = 0; h < kTokMaps; ++h) prefetch_tmap(&tm_b.m[h]);
  }
  griddep_wait();
  {
    WorkIter<kGU> probe;
    if (!probe.init(a)) return;  // whole CTA: no work (uniform)
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemColsF);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const MetaView mv = meta_view(a.meta, a.E);

  if (warp == 0 || warp == 6) {
    // ---- TMA producers: warp 0 fp32 weights, warp 6 token tiles ----
    if (lane == 0) {
      const bool wprod = warp == 0;
      const uint64_t pol = wprod ? l2_policy_evict_first() : l2_policy_evict_last();
      uint64_t* full = wprod ? fullL : fullT;
      uint64_t* empty = wprod ? emptyL : emptyT;
      const int stages = wprod ? kLStagesF : kTStagesF;
      uint8_t* ring = wprod ? land : tring;
      const int sbytes = wprod ? kLStageBytes : kTokBytes;
      int st = 0;
      uint32_t ph = 0;
      uint32_t issued = 0;
      bool ok = true;
      WorkIter<kGU> it;
      it.init(a);
      Work w;
      while (ok && it.next(a, mv, w)) {
        const int nbox = w.n / kBoxRows;  // <= 4: the 2n A rows are one box
        for (int i = 0; i < w.kc1 - w.kc0; ++i) {
          const int kx = w.kc_at(i) * kBK;
          if (!mbar_wait(&empty[st], ph ^ 1u, abort)) {
            if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_EMPTY);
            ok = false;
            break;
          }
          uint8_t* s = ring + (size_t)st * sbytes;
          if (wprod) {
            // per K half: gate rows m0.. then up rows m0.. (64 each), or 128 rows of Wd
            mbar_arrive_expect_tx(&full[st], (uint32_t)kLStageBytes);
            for (int kh = 0; kh < 2; ++kh) {
              uint8_t* d = s + kh * kLHalfBytes;
              tma_load_3d(d, &tm_w, kx + 32 * kh, w.m0, w.e, &full[st], pol);
              if (kGU)
                tma_load_3d(d + kRowsAF * 128, &tm_w, kx + 32 * kh, a.I + w.m0, w.e, &full[st],
                            pol);
            }
          } else {
            mbar_arrive_expect_tx(&full[st], (uint32_t)(2 * w.n * kRowB));
            tma_load_2d(s, &tm_b.m[2 * nbox - 1], kx, 2 * w.row0, &full[st], pol);
          }
          ++issued;
          if (++st == stages) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      drain_ring(full, stages, issued, a.status);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      int sc = 0, stt = 0;
      uint32_t phc = 0, pht = 0;
      bool ok = true;
      const uint32_t idesc = idesc_bf16(kTokM, 2 * kF32Rows);  // B = [W_hi; W_lo]
      WorkIter<kGU> it;
      it.init(a);
      Work w;
      AccTurns acc;
      acc.init();
      while (ok && it.next(a, mv, w)) {
        int b0, nb;
        uint32_t aph[2];
        acc.take(false, b0, nb, aph);
        if (!mbar_wait(&tempty[b0], aph[0] ^ 1u, abort)) {
          if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_FULL);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(b0 * kAccStrideF);
        for (int i = 0; i < w.kc1 - w.kc0; ++i) {
          if (!mbar_wait(&fullC[sc], phc, abort) || !mbar_wait(&fullT[stt], pht, abort)) {
            if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_FULL);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t wh = smem_u32(conv + (size_t)sc * kCStageBytes);
          const uint32_t ta = smem_u32(tring + (size_t)stt * kTokBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            umma_bf16(d, sw128_desc(ta + kk * 32), sw128_desc(wh + kk * 32), idesc,
                      (i > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&emptyC[sc]);
          umma_commit(&emptyT[stt]);
          if (++sc == kCStagesF) {
            sc = 0;
            phc ^= 1u;
          }
          if (++stt == kTStagesF) {
            stt = 0;
            pht ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[b0]);
      }
      // Every MMA issued above must complete before TMEM is released.
      umma_commit(drain);
      if (!mbar_wait(drain, 0, nullptr)) atomicOr(a.status, DEV_TIMEOUT_DRAIN);
    }
  } else if (warp >= 7) {
    // ---- converters: fp32 landing stage -> bf16 hi and lo stages ----
    // Lane l takes K elements 4c..4c+3 (c = l % 16: one 16-byte chunk of
    // the landing row, half c / 8) of row 2p + l / 16 of each row pair p the
    // warp converts (pairs cw, cw + 4, ..): one 16-byte load, the hi parts
    // (upper halves) and the exact remainders by bit masks and subtractions,
    // byte permutes to pack, one 8-byte store into each of hi and lo; each
    // 8-lane group reads and writes whole 128-byte rows (no bank conflicts).
    // A lane's rows r = 2 (cw + 4 j) + l / 16 all have the same r % 8, so its
    // swizzled chunk positions are fixed and the rows 1 KB apart.
    const int cw = warp - 7;
    const int c = lane & 15, rp = lane >> 4;
    const int sw = (2 * cw + rp) & 7;
    const int row0 = (2 * cw + rp) * 128;
    const int ld_off = (c >> 3) * kLHalfBytes + row0 + (((c & 7) ^ sw) << 4);
    const int st_off = row0 + ((((c >> 1) ^ sw) << 4) | ((c & 1) << 3));
    constexpr int kRowStep = 2 * kConvWarps * 128;  // bytes between a lane's rows
    constexpr int kLaneRows = kF32Rows / (2 * kConvWarps);
    int sl = 0, sc = 0;
    uint32_t phl = 0, phc = 0;
    bool ok = true;
    WorkIter<kGU> it;
    it.init(a);
    Work w;
    while (ok && it.next(a, mv, w)) {
      for (int i = 0; i < w.kc1 - w.kc0; ++i) {
        const bool got =
            mbar_wait(&fullL[sl], phl, abort) && mbar_wait(&emptyC[sc], phc ^ 1u, abort);
        if (!__all_sync(0xffffffffu, got)) {
          if (lane == 0 && !*abort) flag_timeout(a, abort, DEV_TIMEOUT_FULL);
          ok = false;
          break;
        }
        const uint8_t* L = land + (size_t)sl * kLStageBytes + ld_off;
        uint8_t* C = conv + (size_t)sc * kCStageBytes + st_off;
        // kConvRows rows in flight per lane: all loads first, so they overlap
#pragma unroll
        for (int j0 = 0; j0 < kLaneRows; j0 += kConvRows) {
          float4 v[kConvRows];
#pragma unroll
          for (int j = 0; j < kConvRows; ++j)
            v[j] = *reinterpret_cast<const float4*>(L + (j0 + j) * kRowStep);
#pragma unroll
          for (int j = 0; j < kConvRows; ++j) {
            const uint32_t u0 = __float_as_uint(v[j].x), u1 = __float_as_uint(v[j].y);
            const uint32_t u2 = __float_as_uint(v[j].z), u3 = __float_as_uint(v[j].w);
            const float r0 = v[j].x - __uint_as_float(u0 & 0xffff0000u);
            const float r1 = v[j].y - __uint_as_float(u1 & 0xffff0000u);
            const float r2 = v[j].z - __uint_as_float(u2 & 0xffff0000u);
            const float r3 = v[j].w - __uint_as_float(u3 & 0xffff0000u);
            uint8_t* d = C + (j0 + j) * kRowStep;
            *reinterpret_cast<uint2*>(d) = make_uint2(__byte_perm(u0, u1, 0x7632),
                                                      __byte_perm(u2, u3, 0x7632));
            *reinterpret_cast<uint2*>(d + kCHalfBytes) =
                make_uint2(__byte_perm(__float_as_uint(r0), __float_as_uint(r1), 0x7632),
                           __byte_perm(__float_as_uint(r2), __float_as_uint(r3), 0x7632));
          }
        }
        fence_proxy_async_smem();  // the tensor core reads these stores
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&emptyL[sl]);
          mbar_arrive(&fullC[sc]);
        }
        if (++sl == kLStagesF) {
          sl = 0;
          phl ^= 1u;
        }
        if (++sc == kCStagesF) {
          sc = 0;
          phc ^= 1u;
        }
      }
    }
  } else {
    // ---- epilogue: warps 2..5, TMEM lane quarter warp % 4 ----
    // Lane l < 16 of quarter q holds the hi part of token 16q + l, lane
    // l + 16 its lo part: acc_sum8 adds them.
    const int q = warp & 3;
    const bool upper = lane >= 16;
    const int half = upper ? 8 : 0;
    WorkIter<kGU> it;
    it.init(a);
    Work w;
    AccTurns acc;
    acc.init();
    while (it.next(a, mv, w)) {
      int b0, nb;
      uint32_t aph[2];
      acc.take(false, b0, nb, aph);
      bool bad = *abort != 0;
      if (!bad && !mbar_wait(&tfull[b0], aph[0], abort)) {
        if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_ACT);
        bad = true;
      }
      if (named_bar_or(2, 128, bad)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(b0 * kAccStrideF);
      const int tok = 16 * q + (lane & 15);
      const bool has = 16 * q < w.n;  // warp-uniform: this quarter holds tokens
      const bool live = tok < w.n;
      if (kGU) {
        const bool whole = w.kc0 == 0 && w.kc1 == a.kc_total;
        const int r = w.row0 + tok;
        float* pb = a.pbuf +
                    (((size_t)blockIdx.x * 2 + part_slot_of_piece(w)) * a.nmax + tok) * kF32Rows;
        if (has) {
          const float wt = live ? __ldg(a.row_w + r) : 0.0f;
          uint16_t* hi = a.act + act_row_hi(r) * a.I;
          uint16_t* lo = hi + 16 * (int64_t)a.I;
          for (int c0 = 0; c0 < kRowsAF; c0 += 16) {
            float g[8], u[8];
            acc_sum8(taddr, c0, upper, g);
            acc_sum8(taddr, kRowsAF + c0, upper, u);
            if (!live) continue;
            if (whole) {
              swiglu_store8(g, u, wt, hi, lo, w.m0 + c0 + half, a.I);
            } else {
#pragma unroll
              for (int k2 = 0; k2 < 2; ++k2) {
                *reinterpret_cast<float4*>(pb + c0 + half + 4 * k2) =
                    make_float4(g[4 * k2], g[4 * k2 + 1], g[4 * k2 + 2], g[4 * k2 + 3]);
                *reinterpret_cast<float4*>(pb + kRowsAF + c0 + half + 4 * k2) =
                    make_float4(u[4 * k2], u[4 * k2 + 1], u[4 * k2 + 2], u[4 * k2 + 3]);
              }
            }
          }
        }
        release_acc(tempty, b0, 1, lane);
        if (!whole) {
          __threadfence();
          named_bar_sync(1, 128);
          const int cf = it.first_cta(w), cl = it.last_cta(a, w);
          if (threadIdx.x == 64) {
            const uint32_t done = atomicAdd(&a.cnt[w.tile], 1u);
            *last_flag = done == (uint32_t)(cl - cf) ? 1 : 0;
          }
          named_bar_sync(1, 128);
          if (*last_flag) {
            __threadfence();
            // item = (token, 16 rows of gate and of up); partials added in CTA order
            const int et = threadIdx.x - 64;
            for (int item = et; item < w.n * (kRowsAF / 16); item += 128) {
              const int tt = item / (kRowsAF / 16);
              const int c0 = (item % (kRowsAF / 16)) * 16;
              const int rr = w.row0 + tt;
              float4 gv[kJMaxA][4], uv[kJMaxA][4];
#pragma unroll
              for (int cc = 0; cc < kJMaxA; ++cc) {
                if (cf + cc <= cl) {
                  const float* src =
                      a.pbuf +
                      (((size_t)(cf + cc) * 2 + part_slot_of_cta(cf + cc, cf)) * a.nmax + tt) *
                          kF32Rows;
#pragma unroll
                  for (int k4 = 0; k4 < 4; ++k4) {
                    gv[cc][k4] = __ldcg(reinterpret_cast<const float4*>(src + c0) + k4);
                    uv[cc][k4] = __ldcg(reinterpret_cast<const float4*>(src + kRowsAF + c0) + k4);
                  }
                }
              }
              float g[16], u[16];
#pragma unroll
              for (int c = 0; c < 16; ++c) g[c] = u[c] = 0.0f;
#pragma unroll
              for (int cc = 0; cc < kJMaxA; ++cc) {
                if (cf + cc <= cl) {
#pragma unroll
                  for (int k4 = 0; k4 < 4; ++k4) {
                    g[4 * k4] += gv[cc][k4].x; g[4 * k4 + 1] += gv[cc][k4].y;
                    g[4 * k4 + 2] += gv[cc][k4].z; g[4 * k4 + 3] += gv[cc][k4].w;
                    u[4 * k4] += uv[cc][k4].x; u[4 * k4 + 1] += uv[cc][k4].y;
                    u[4 * k4 + 2] += uv[cc][k4].z; u[4 * k4 + 3] += uv[cc][k4].w;
                  }
                }
              }
              uint16_t* hrow = a.act + act_row_hi(rr) * a.I;
              swiglu_store16(g, u, __ldg(a.row_w + rr), hrow, hrow + 16 * (int64_t)a.I,
                             w.m0 + c0, a.I);
            }
            if (threadIdx.x == 64) a.cnt[w.tile] = 0;  // ready for the next call
          }
        }
      } else {
        if (has) {
          float* yrow = a.ypart + ((int64_t)w.j * a.rmax + w.row0 + tok) * a.H;
          for (int c0 = 0; c0 < kF32Rows; c0 += 16) {
            float o[8];
            acc_sum8(taddr, c0, upper, o);
            const int h = w.m0 + c0 + half;
            if (live) {
#pragma unroll
              for (int k2 = 0; k2 < 2; ++k2)
                if (h + 4 * k2 < a.H)
                  *reinterpret_cast<float4*>(yrow + h + 4 * k2) =
                      make_float4(o[4 * k2], o[4 * k2 + 1], o[4 * k2 + 2], o[4 * k2 + 3]);
            }
          }
        }
        release_acc(tempty, b0, 1, lane);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemColsF);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

wr_status_t get_encoder(EncodeTiledFn* out) {
  static std::once_flag once;
  static void* fn = nullptr;
  static cudaError_t err = cudaSuccess;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (err == cudaSuccess && q != cudaDriverEntryPointSuccess) fn = nullptr;
  });
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
  if (!fn) return fail(WR_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  *out = reinterpret_cast<EncodeTiledFn>(fn);
  return WR_OK;
}

// bf16 tensor map with 128-byte swizzling, zero fill outside the tensor.
wr_status_t encode_map(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
                       const cuuint64_t* strides_bytes, const cuuint32_t* box,
                       CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  EncodeTiledFn enc;
  wr_status_t st = get_encoder(&enc);
  if (st != WR_OK) return st;
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, dtype, (cuuint32_t)rank, const_cast<void*>(base),
                   dims, strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(WR_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return WR_OK;
}

// Token maps with boxes of 16, 32, .. rows.  Heights above the largest tile
// (nmax, and never above the rows a tile can start in) are never used and
// repeat the 16-row map.
wr_status_t encode_token_maps(TokenMaps* t, const void* base, const cuuint64_t* dims,
                              const cuuint64_t* str, int nmax, int rmax) {
  for (int h = 1; h <= kTokMaps; ++h) {
    const int rows = h * kBoxRows;
    if (h > 1 && (rows > nmax || rows > rmax)) {
      t->m[h - 1] = t->m[0];
      continue;
    }
    const cuuint32_t box[2] = {kBK, (cuuint32_t)rows};
    const wr_status_t st = encode_map(&t->m[h - 1], base, 2, dims, str, box);
    if (st != WR_OK) return st;
  }
  return WR_OK;
}

size_t a256(size_t n) { return (n + 255) & ~size_t(255); }

// Everything the grouped path derives from the problem on the host.
struct GroupedPlan {
  bool f32;          // fp32 weights and tokens (k_grouped_gemm_f32)
  int rowsA, rowsB;  // weight rows per tile (gate/up: of gate and of up; down: of Wd)
  int nmaxA, nmaxB;  // token rows per tile
  int rmax;          // row capacity (>= padded rows in use)
  int mtA, mtB;      // weight-row tiles per expert (gate/up over I, down over H)
  int kcA, kcB;      // K chunks (over H, over I)
  int wstA, tstA, tbA;  // gate/up rings: weight depth, token depth, token slot bytes
  int wstB, tstB, tbB;  // down rings
  int cnt_words;     // gate/up tile counters (>= gate/up tiles)
  int jmaxB;         // down: partial sums per tile, at most
  size_t off_ids, off_w, off_slot, off_meta, off_rtok, off_re, off_rw, off_xg, off_act, off_y,
      off_pbuf, off_cnt, total;
};

// Ring depths.  Weights come from HBM and want >= 5 stages of 32 KB in
// flight; token tiles come from L2, but a slot is held until its MMAs finish,
// so 2 slots leave the MMA waiting on L2 latency.  Take the most token slots
// (<= 4) that still leave 5 weight stages; large token slots (>= 32 KB) may
// drop to 4 weight stages for a third slot.
void ring_split(int tbytes, int reserve, int* wst, int* tst) {
  const int avail = kSmemMax - reserve;
  int t = 4, w = 0;
  for (; t >= 2; --t) {
    w = (avail - t * tbytes) / kWStageBytes;
    if (w >= 5 || (tbytes >= 32768 && t >= 3 && w >= 4)) break;
  }
  if (t < 2) {
    t = 2;
    w = (avail - t * tbytes) / kWStageBytes;
  }
  // the last token slot's 128-row MMA window must end inside the allocation
  static_assert(kTokBytes <= 4 * kWStageBytes, "token window overhang");
  *tst = t;
  *wst = w > kMaxWStages ? kMaxWStages : w;
}

GroupedPlan make_plan(const Problem& p) {
  GroupedPlan g;
  const int TK = p.T * p.K;
  const int n16 = (p.T + 15) & ~15;
  g.f32 = p.dtype != WR_DTYPE_BF16;
  if (g.f32) {
    g.nmaxA = g.nmaxB = n16 < kNMaxF ? n16 : kNMaxF;
    g.rowsA = kRowsAF;
    g.rowsB = kRowsBF;
  } else {
    g.nmaxA = n16 <= kNMaxA ? n16 : kNMaxAWide;
    g.nmaxB = n16 <= kNMaxB ? n16 : kNMaxBWide;
    g.rowsA = kRowsA;
    g.rowsB = kRowsB;
  }
  g.rmax = (TK + 15 * p.ep_num + 15) & ~15;
  g.mtA = (p.I + g.rowsA - 1) / g.rowsA;
  g.mtB = (p.H + g.rowsB - 1) / g.rowsB;
  g.kcA = (p.H + kBK - 1) / kBK;
  g.kcB = (p.I + kBK - 1) / kBK;
  g.tbA = (g.nmaxA < kTokM ? g.nmaxA : kTokM) * kRowB;  // a wide tile takes two slots
  g.tbB = 2 * g.nmaxB * kRowB;
  ring_split(g.tbA, kSmemBase, &g.wstA, &g.tstA);
  if (!g.f32 && g.nmaxA > kTokM) {
    // Wide gate/up tiles take two token slots per K step: six slots (three
    // steps of token lookahead) and four weight stages measured 2 % faster
    // on the Mixtral T = 256 layer than four slots and five stages.
    g.tstA = 6;
    g.wstA = (kSmemMax - kSmemBase - 6 * g.tbA) / kWStageBytes;
  }
  ring_split(g.tbB, kSmemBase, &g.wstB, &g.tstB);
  size_t o = kWsControlBytes;
  g.off_ids = o; o += a256(4 * (size_t)TK);
  g.off_w = o; o += a256(4 * (size_t)TK);
  g.off_slot = o; o += a256(4 * (size_t)TK);
  g.off_meta = o; o += a256(4 * (size_t)meta_words(p.ep_num));
  g.off_rtok = o; o += a256(4 * (size_t)g.rmax);
  g.off_re = o; o += a256(16 * (size_t)g.rmax);
  g.off_rw = o; o += a256(4 * (size_t)g.rmax);
  g.off_xg = o; o += a256((g.f32 ? 4 : 2) * (size_t)g.rmax * p.H);  // fp32: hi and lo rows
  g.off_act = o; o += a256(2 * 2 * (size_t)g.rmax * p.I);
  // Down partials per tile: enough that the fewest possible tiles (one active
  // expert) still spread over every SM.
  g.jmaxB = (device_sm_count() + g.mtB - 1) / g.mtB + 1;
  if (g.jmaxB < kJMaxB) g.jmaxB = kJMaxB;
  if (g.jmaxB > kJMaxBLimit) g.jmaxB = kJMaxBLimit;
  g.off_y = o; o += a256(4 * (size_t)g.jmaxB * g.rmax * p.H);
  g.off_pbuf = o;
  o += a256(4 * (size_t)device_sm_count() * 2 * g.nmaxA * (g.f32 ? kF32Rows : kWRows));
  g.cnt_words = g.mtA * (p.ep_num + (g.rmax + g.nmaxA - 1) / g.nmaxA);
  g.off_cnt = o; o += a256(4 * (size_t)g.cnt_words);
  g.total = o;
  return g;
}

// Launches `kern` with programmatic stream serialization: it may start while
// the previous kernel on the stream finishes, and waits for it with
// griddep_wait() before touching its outputs.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

template <bool kGU, bool kF32>
wr_status_t set_smem_attr() {
  static std::once_flag once[64];
  static cudaError_t err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    err[dev & 63] = kF32 ? cudaFuncSetAttribute(k_grouped_gemm_f32<kGU>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemF)
                         : cudaFuncSetAttribute(k_grouped_gemm<kGU>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  });
  if (err[dev & 63] != cudaSuccess)
    return cuda_fail(err[dev & 63], "cudaFuncSetAttribute(grouped gemm)");
  return WR_OK;
}

}  // namespace

bool grouped_supported(const Problem& p) {
  const int min_t = p.dtype == WR_DTYPE_BF16 ? kGroupedMinTokens : kGroupedMinTokensF32;
  return p.T >= min_t && p.H % 8 == 0 && p.I % 8 == 0 && p.ep_num >= 1;
}

size_t grouped_workspace_bytes(const Problem& p) { return make_plan(p).total; }

wr_status_t launch_grouped(const Problem& p, const void* x, const void* gate_w, const void* wbuf,
                           float* out, int32_t* ids, float* w, void* ws, cudaStream_t stream,
                           const CommView* comm) {
  const int sms = device_sm_count();
  const GroupedPlan g = make_plan(p);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  int32_t* ids_d = ids ? ids : reinterpret_cast<int32_t*>(wsb + g.off_ids);
  float* w_d = w ? w : reinterpret_cast<float*>(wsb + g.off_w);
  int32_t* slot = reinterpret_cast<int32_t*>(wsb + g.off_slot);
  int* meta = reinterpret_cast<int*>(wsb + g.off_meta);
  int32_t* rtok = reinterpret_cast<int32_t*>(wsb + g.off_rtok);
  int4* rtile = reinterpret_cast<int4*>(wsb + g.off_re);
  float* rw = reinterpret_cast<float*>(wsb + g.off_rw);
  uint16_t* xg = reinterpret_cast<uint16_t*>(wsb + g.off_xg);
  uint16_t* act = reinterpret_cast<uint16_t*>(wsb + g.off_act);
  float* ypart = reinterpret_cast<float*>(wsb + g.off_y);
  float* pbuf = reinterpret_cast<float*>(wsb + g.off_pbuf);
  uint32_t* tcnt = reinterpret_cast<uint32_t*>(wsb + g.off_cnt);
  uint32_t* status = reinterpret_cast<uint32_t*>(ws) + 2;

  wr_status_t st = WR_OK;
  const int TK = p.T * p.K;
  const size_t bucket_smem = TK <= kBucketSmemIds ? 8 * (size_t)TK : 0;
  BucketArgs ba;
  ba.ids = ids_d;
  ba.w = w_d;
  ba.TK = TK;
  ba.K = p.K;
  ba.ep_first = p.ep_first;
  ba.E = p.ep_num;
  ba.nmaxA = g.nmaxA;
  ba.nmaxB = g.nmaxB;
  ba.mtA = g.mtA;
  ba.mtB = g.mtB;
  ba.kcA = g.kcA;
  ba.kcB = g.kcB;
  ba.meta = meta;
  ba.slot = slot;
  ba.row_tok = rtok;
  ba.row_tile = rtile;
  ba.row_w = rw;
  ba.tile_cnt = tcnt;
  ba.cnt_words = g.cnt_words;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(gate_w) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(x) & 15) == 0;  // H % 8 == 0 here
  cudaError_t ce =
      g.f32 ? launch_pdl(k_route_bucket<float>, dim3(p.T), dim3(kRouteThreads), bucket_smem,
                         stream, static_cast<const float*>(x), static_cast<const float*>(gate_w),
                         p.router_bias, p.E, p.H, vec_ok, reinterpret_cast<uint32_t*>(ws), ids_d,
                         w_d, ba)
            : launch_pdl(k_route_bucket<uint16_t>, dim3(p.T), dim3(kRouteThreads), bucket_smem,
                         stream, static_cast<const uint16_t*>(x),
                         static_cast<const uint16_t*>(gate_w), p.router_bias, p.E, p.H, vec_ok,
                         reinterpret_cast<uint32_t*>(ws), ids_d, w_d, ba);
  const int gather_blocks = g.rmax < 4 * sms ? g.rmax : 4 * sms;
  if (ce == cudaSuccess)
    ce = g.f32 ? launch_pdl(k_gather_f32, dim3(gather_blocks), dim3(256), 0, stream,
                            static_cast<const float4*>(x), p.H / 8, (const int*)meta,
                            (const int32_t*)rtok, reinterpret_cast<uint4*>(xg))
               : launch_pdl(k_gather, dim3(gather_blocks), dim3(256), 0, stream,
                            static_cast<const uint4*>(x), p.H / 8, (const int*)meta,
                            (const int32_t*)rtok, reinterpret_cast<uint4*>(xg));
  if (ce != cudaSuccess) return cuda_fail(ce, "bucket / gather launch");

  const Layout lay = make_layout(p.H, p.I, g.f32 ? 4 : 2);
  const uint8_t* wb = static_cast<const uint8_t*>(wbuf);
  CUtensorMap tm_gu, tm_dn;
  TokenMaps tm_x, tm_act;
  if (g.f32) {
    // fp32 weights: per stage two K halves of 32 elements (128-byte rows);
    // gate/up boxes of 64 rows (gate, then up), down boxes of 128 rows
    constexpr CUtensorMapDataType f32t = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const cuuint64_t dgu[3] = {(cuuint64_t)p.H, (cuuint64_t)2 * p.I, (cuuint64_t)p.ep_num};
    const cuuint64_t sgu[2] = {(cuuint64_t)p.H * 4, (cuuint64_t)lay.stride};
    const cuuint32_t bgu[3] = {32, kRowsAF, 1};
    if ((st = encode_map(&tm_gu, wb + lay.off_gate, 3, dgu, sgu, bgu, f32t)) != WR_OK) return st;
    const cuuint64_t ddn[3] = {(cuuint64_t)p.I, (cuuint64_t)p.H, (cuuint64_t)p.ep_num};
    const cuuint64_t sdn[2] = {(cuuint64_t)p.I * 4, (cuuint64_t)lay.stride};
    const cuuint32_t bdn[3] = {32, kRowsBF, 1};
    if ((st = encode_map(&tm_dn, wb + lay.off_down, 3, ddn, sdn, bdn, f32t)) != WR_OK) return st;
    // tokens: 2 rmax rows (hi / lo blocks of 16), boxes of up to 2 nmax rows
    const cuuint64_t dx[2] = {(cuuint64_t)p.H, (cuuint64_t)2 * g.rmax};
    const cuuint64_t sx[1] = {(cuuint64_t)p.H * 2};
    if ((st = encode_token_maps(&tm_x, xg, dx, sx, 2 * g.nmaxA, 2 * g.rmax)) != WR_OK) return st;
  } else {
    {
      const cuuint64_t dims[3] = {(cuuint64_t)p.H, (cuuint64_t)2 * p.I, (cuuint64_t)p.ep_num};
      const cuuint64_t str[2] = {(cuuint64_t)p.H * 2, (cuuint64_t)lay.stride};
      const cuuint32_t box[3] = {kBK, kWBox, 1};
      if ((st = encode_map(&tm_gu, wb + lay.off_gate, 3, dims, str, box)) != WR_OK) return st;
    }
    {
      const cuuint64_t dims[2] = {(cuuint64_t)p.H, (cuuint64_t)g.rmax};
      const cuuint64_t str[1] = {(cuuint64_t)p.H * 2};
      if ((st = encode_token_maps(&tm_x, xg, dims, str, g.nmaxA, g.rmax)) != WR_OK) return st;
    }
    {
      const cuuint64_t dims[3] = {(cuuint64_t)p.I, (cuuint64_t)p.H, (cuuint64_t)p.ep_num};
      const cuuint64_t str[2] = {(cuuint64_t)p.I * 2, (cuuint64_t)lay.stride};
      const cuuint32_t box[3] = {kBK, kWBox, 1};
      if ((st = encode_map(&tm_dn, wb + lay.off_down, 3, dims, str, box)) != WR_OK) return st;
    }
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)p.I, (cuuint64_t)2 * g.rmax};
    const cuuint64_t str[1] = {(cuuint64_t)p.I * 2};
    if ((st = encode_token_maps(&tm_act, act, dims, str, 2 * g.nmaxB, 2 * g.rmax)) != WR_OK)
      return st;
  }
  if (g.f32) {
    if ((st = set_smem_attr<true, true>()) != WR_OK) return st;
    if ((st = set_smem_attr<false, true>()) != WR_OK) return st;
  } else {
    if ((st = set_smem_attr<true, false>()) != WR_OK) return st;
    if ((st = set_smem_attr<false, false>()) != WR_OK) return st;
  }

  GemmArgs ga;
  ga.meta = meta;
  ga.E = p.ep_num;
  ga.H = p.H;
  ga.I = p.I;
  ga.rmax = g.rmax;
  ga.row_w = rw;
  ga.act = act;
  ga.ypart = ypart;
  ga.pbuf = pbuf;
  ga.cnt = tcnt;
  ga.status = status;

  GemmArgs a1 = ga;
  a1.nmax = g.nmaxA;
  a1.kc_total = g.kcA;
  a1.jmax = kJMaxA;
  a1.wstages = g.wstA;
  a1.tstages = g.tstA;
  a1.tstage_bytes = g.tbA;
  a1.mrows = g.rowsA;
  const size_t smemA = (size_t)g.wstA * kWStageBytes + (size_t)g.tstA * g.tbA + kSmemBase;
  ce = g.f32 ? launch_pdl(k_grouped_gemm_f32<true>, dim3(sms), dim3(kGemmThreadsF),
                          (size_t)kSmemF, stream, tm_gu, tm_x, a1)
             : launch_pdl(k_grouped_gemm<true>, dim3(sms), dim3(kGemmThreads), smemA, stream,
                          tm_gu, tm_x, a1);
  if (ce != cudaSuccess) return cuda_fail(ce, "grouped GEMM (gate/up) launch");

  GemmArgs a2 = ga;
  a2.nmax = g.nmaxB;
  a2.kc_total = g.kcB;
  a2.jmax = g.jmaxB;
  a2.wstages = g.wstB;
  a2.tstages = g.tstB;
  a2.tstage_bytes = g.tbB;
  a2.mrows = g.rowsB;
  const size_t smemB = (size_t)g.wstB * kWStageBytes + (size_t)g.tstB * g.tbB +
                       kSmemBase;
  ce = g.f32 ? launch_pdl(k_grouped_gemm_f32<false>, dim3(sms), dim3(kGemmThreadsF),
                          (size_t)kSmemF, stream, tm_dn, tm_act, a2)
             : launch_pdl(k_grouped_gemm<false>, dim3(sms), dim3(kGemmThreads), smemB, stream,
                          tm_dn, tm_act, a2);
  if (ce != cudaSuccess) return cuda_fail(ce, "grouped GEMM (down) launch");

  const int H4 = p.H / 4;
  if (comm) {
    // all-reduce in the combine, one launch (one epoch) per kCommMaxTokens tokens
    for (int t0 = 0; t0 < p.T; t0 += kCommMaxTokens) {
      const int Tc = p.T - t0 < kCommMaxTokens ? p.T - t0 : kCommMaxTokens;
      int blocks = (Tc * H4 + 255) / 256;
      if (blocks > 4 * sms) blocks = 4 * sms;
      ce = launch_pdl(k_combine_ar, dim3(blocks), dim3(256), 0, stream,
                      reinterpret_cast<const float4*>(ypart), (const int32_t*)slot,
                      (const int4*)rtile, (const int*)meta, p.K, p.H, g.rmax, g.kcB, g.rowsB,
                      sms, g.jmaxB, t0, Tc, *comm, p.res,
                      reinterpret_cast<uint32_t*>(ws), out);
      if (ce != cudaSuccess) return cuda_fail(ce, "combine (all-reduce) launch");
    }
    return WR_OK;
  }
  ce = launch_pdl(k_combine, dim3(p.T, (H4 + 255) / 256), dim3(256), 0, stream,
                  reinterpret_cast<const float4*>(ypart), (const int32_t*)slot,
                  (const int4*)rtile, (const int*)meta, p.K, H4, g.rmax, g.kcB, g.rowsB, sms,
                  g.jmaxB, p.res, reinterpret_cast<float4*>(out));
  return ce == cudaSuccess ? WR_OK : cuda_fail(ce, "combine launch");
}

}  // namespace wr
