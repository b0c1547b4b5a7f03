// wr_grouped.cu — the batched layer for larger token batches as two grouped
// GEMMs on the 5th-generation tensor cores.
//
// warp-route's batched kernel (src/fused_moe_batched.cu:20-183) gives every
// token its own CTA and streams every selected expert's weights once per
// token, on CUDA cores.  Here the tokens are bucketed per expert first, so
// each expert's weights stream from HBM once per batch and meet all of that
// expert's tokens in a tcgen05 MMA:
//
//   k_router        ids / weights of every token (bit-exact with the fused
//                   path: same kernel as wr_router_topk)
//   k_bucket        (token, k) pairs of this rank's experts -> rows of a
//                   per-expert token list, each expert's list padded to a
//                   multiple of 16 rows with zero-weight rows
//   k_gather        X_g[row] = x[token of row] (bf16), zero for padding
//   k_grouped_gemm<gate/up>
//                   per (expert, 128 rows of I, <=128 tokens): gate and up
//                   accumulators in TMEM over K = H, epilogue
//                   act = silu(g) * u * w(token, k) stored as bf16 hi + lo
//   k_grouped_gemm<down>
//                   per (expert, 128 rows of H, K split, <=128 tokens):
//                   Wd . act_hi + Wd . act_lo (the hi/lo pair keeps the
//                   activation to ~16 mantissa bits), fp32 partials per split
//   k_combine       out[t] = sum over k (ascending) and splits (ascending):
//                   one fixed order, so the result is deterministic.
//
// GEMM structure: weights are the MMA's A operand (M = 128 weight rows,
// K-major: rows of the packed layout are contiguous along K), tokens the B
// operand (N = 16..128, K-major), both bf16, accumulator fp32 in TMEM.  One
// persistent CTA per SM, 6 warps: warp 0 issues the TMA loads (one elected
// lane, 128-byte swizzled tiles), warp 1 owns TMEM and issues the MMAs (one
// elected lane, tcgen05.commit to release smem stages and to hand
// accumulators to the epilogue), warps 2-5 read the accumulators back with
// tcgen05.ld (warp w reads TMEM lanes 32*(w%4)..+31) and store the results.
// Two accumulator buffers let the epilogue of one tile overlap the MMAs of
// the next.  No TMA multicast anywhere; every wait is bounded and a wait
// that runs out sets the workspace status word and winds the CTA down
// (copies in flight drained, MMAs completed, TMEM freed).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "wr_common.cuh"
#include "wr_internal.h"
#include "wr_router.cuh"

namespace wr {
namespace {

constexpr int kBM = 128;                  // weight rows per tile (MMA M)
constexpr int kBK = 64;                   // K elements per smem stage: one 128-byte swizzle row
constexpr int kNMax = 128;                // tokens per tile (MMA N)
constexpr int kTileA = kBM * kBK * 2;     // 16 KB of weights per operand per stage
constexpr int kRowB = kBK * 2;            // bytes of one token row per stage
constexpr int kBoxRows = 16;              // token rows per TMA box
constexpr int kGemmThreads = 192;
constexpr int kTmemCols = 512;            // two accumulator buffers of 256 columns
constexpr int kAccStride = 256;           // columns between accumulator buffers
constexpr int kUpCol = 128;               // up accumulator column offset (gate at 0)
constexpr int kSmemMax = 232448;          // 227 KB opt-in shared memory per CTA
constexpr int kSmemReserve = 1024 + 256;  // alignment slack + barriers
constexpr int kMaxStages = 8;

// Bucket metadata (int32 words in the workspace), written by k_bucket:
//   [0] rows in use, [1] gate/up items, [2] down items,
//   cnt[E], base[E], ntl[E] (token tiles), preA[E+1], preB[E+1] from word 16.
constexpr int kMetaHdr = 16;
__host__ __device__ inline int meta_words(int E) { return kMetaHdr + 5 * E + 2; }
struct MetaView {
  const int* cnt;
  const int* base;
  const int* ntl;
  const int* preA;
  const int* preB;
};
__host__ __device__ inline MetaView meta_view(const int* m, int E) {
  MetaView v;
  v.cnt = m + kMetaHdr;
  v.base = v.cnt + E;
  v.ntl = v.base + E;
  v.preA = v.ntl + E;
  v.preB = v.preA + E + 1;
  return v;
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
// K-major, M = 128, N = n (multiple of 16, 16..256).
WR_DEVINL uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
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
WR_DEVINL void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---------------------------------------------------------------------------
// Routing and bucketing
// ---------------------------------------------------------------------------

// One CTA.  Pairs (t, k) whose expert is in [ep_first, ep_first + E) get a
// row: expert e's rows are base[e] .. base[e] + cnt[e] - 1 in ascending
// token order, followed by zero-weight padding up to a multiple of 16.
// Pairs of other ranks' experts get slot -1.  Also writes the tile counts
// the GEMM kernels walk: per expert ntl token tiles of <= nmax rows,
// mtA * ntl gate/up items and mtB * S * ntl down items.
__global__ void __launch_bounds__(512) k_bucket(const int32_t* __restrict__ ids,
                                                 const float* __restrict__ w, int TK, int K,
                                                 int ep_first, int E, int nmax, int mtA, int mtB,
                                                 int S, int* __restrict__ meta,
                                                 int32_t* __restrict__ slot,
                                                 int32_t* __restrict__ row_tok,
                                                 float* __restrict__ row_w) {
  __shared__ int s_cnt[kMaxExperts];
  __shared__ int s_base[kMaxExperts];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int i = threadIdx.x; i < TK; i += blockDim.x) {
    const int e = ids[i] - ep_first;
    if (e < 0 || e >= E) slot[i] = -1;
  }
  for (int e = warp; e < E; e += nw) {
    int c = 0;
    for (int j = 0; j < TK; j += 32) {
      const bool m = j + lane < TK && ids[j + lane] == e + ep_first;
      c += __popc(__ballot_sync(0xffffffffu, m));
    }
    if (lane == 0) s_cnt[e] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    MetaView v = meta_view(meta, E);
    int* cnt = const_cast<int*>(v.cnt);
    int* base = const_cast<int*>(v.base);
    int* ntl = const_cast<int*>(v.ntl);
    int* preA = const_cast<int*>(v.preA);
    int* preB = const_cast<int*>(v.preB);
    int b = 0, pa = 0, pb = 0;
    for (int e = 0; e < E; ++e) {
      const int n = s_cnt[e];
      const int np = (n + 15) & ~15;
      const int nt = (np + nmax - 1) / nmax;
      cnt[e] = n;
      base[e] = b;
      s_base[e] = b;
      ntl[e] = nt;
      preA[e] = pa;
      preB[e] = pb;
      b += np;
      pa += mtA * nt;
      pb += mtB * S * nt;
    }
    preA[E] = pa;
    preB[E] = pb;
    meta[0] = b;
    meta[1] = pa;
    meta[2] = pb;
  }
  __syncthreads();
  for (int e = warp; e < E; e += nw) {
    int run = s_base[e];
    for (int j = 0; j < TK; j += 32) {
      const bool m = j + lane < TK && ids[j + lane] == e + ep_first;
      const unsigned bal = __ballot_sync(0xffffffffu, m);
      if (m) {
        const int r = run + __popc(bal & ((1u << lane) - 1u));
        slot[j + lane] = r;
        row_tok[r] = (j + lane) / K;
        row_w[r] = w[j + lane];
      }
      run += __popc(bal);
    }
    const int end = s_base[e] + ((s_cnt[e] + 15) & ~15);
    for (int r = run + lane; r < end; r += 32) {
      row_tok[r] = -1;
      row_w[r] = 0.0f;
    }
  }
}

// X_g[row, :] = x[row_tok[row], :] (bf16, 16-byte chunks), zero for padding.
__global__ void __launch_bounds__(256) k_gather(const uint4* __restrict__ x, int H8,
                                                const int* __restrict__ meta,
                                                const int32_t* __restrict__ row_tok,
                                                uint4* __restrict__ xg) {
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

// out[t, :] = sum over k of (slot >= 0 ? sum over splits of Y[split][slot] : 0),
// k and splits ascending.
__global__ void __launch_bounds__(256) k_combine(const float4* __restrict__ ypart,
                                                 const int32_t* __restrict__ slot, int K, int H4,
                                                 int S, int rmax, float4* __restrict__ out) {
  const int t = blockIdx.x;
  for (int h = threadIdx.x; h < H4; h += blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < K; ++k) {
      const int r = slot[(int64_t)t * K + k];
      if (r < 0) continue;
      for (int s = 0; s < S; ++s) {
        const float4 v = ypart[((int64_t)s * rmax + r) * H4 + h];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
    }
    out[(int64_t)t * H4 + h] = acc;
  }
}

// ---------------------------------------------------------------------------
// Grouped GEMM
// ---------------------------------------------------------------------------

struct GemmArgs {
  const int* meta;
  int E;            // experts of this rank
  int H, I;
  int nmax;         // token rows per tile
  int S;            // down: K splits
  int kc_total;     // K chunks of kBK (gate/up: over H, down: over I)
  int kc_split;     // down: chunks per split
  int mt;           // weight-row tiles per expert
  int rmax;         // rows of one activation half (lo rows start at rmax)
  int stages;
  int stage_bytes;
  const float* row_w;  // gate/up epilogue: per-row routing weight
  uint16_t* act;       // gate/up output: [2][rmax][I] bf16 (hi, lo)
  float* ypart;        // down output: [S][rmax][H] fp32
  uint32_t* status;
};

struct Item {
  int e, m0, row0, n, kc0, kc1, s;
};

// Item i of this phase: experts in order; inside an expert the token tile
// varies fastest (tiles that share a weight tile run on neighbouring CTAs at
// the same time, so the second read of the weights mostly hits L2), then the
// K split (down), then the weight-row tile.  `e` is advanced monotonically:
// each role walks its items in increasing order.
template <bool kGU>
WR_DEVINL Item decode_item(const GemmArgs& a, const MetaView& mv, int i, int& e) {
  const int* pre = kGU ? mv.preA : mv.preB;
  while (e + 1 < a.E && __ldg(pre + e + 1) <= i) ++e;
  const int local = i - __ldg(pre + e);
  const int nt = __ldg(mv.ntl + e);
  const int tn = local % nt;
  const int rest = local / nt;
  Item it;
  it.e = e;
  int mtile;
  if (kGU) {
    it.s = 0;
    mtile = rest;
    it.kc0 = 0;
    it.kc1 = a.kc_total;
  } else {
    it.s = rest % a.S;
    mtile = rest / a.S;
    it.kc0 = it.s * a.kc_split;
    it.kc1 = min(a.kc_total, it.kc0 + a.kc_split);
  }
  it.m0 = mtile * kBM;
  const int np = (__ldg(mv.cnt + e) + 15) & ~15;
  it.row0 = __ldg(mv.base + e) + tn * a.nmax;
  it.n = min(a.nmax, np - tn * a.nmax);
  return it;
}

WR_DEVINL void flag_timeout(const GemmArgs& a, volatile int* abort, uint32_t bit) {
  *abort = 1;
  atomicOr(a.status, bit);
}

template <bool kGU>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_grouped_gemm(const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_b, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const int total = __ldg(a.meta + (kGU ? 1 : 2));
  if ((int)blockIdx.x >= total) return;  // whole CTA: no work

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)a.stages * a.stage_bytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;  // [2]
  uint64_t* tempty = tfull + 2;          // [2]
  uint64_t* drain = tempty + 2;          // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    *abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_b);
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

  if (warp == 0) {
    // ---- TMA producer ----
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_b = l2_policy_evict_last();
      int st = 0;
      uint32_t ph = 0;
      uint32_t issued = 0;
      int e = 0;
      bool ok = true;
      for (int i = blockIdx.x; ok && i < total; i += gridDim.x) {
        const Item it = decode_item<kGU>(a, mv, i, e);
        const int nbox = it.n / kBoxRows;
        const uint32_t bytes = (kGU ? 2 : 1) * kTileA + (kGU ? 1 : 2) * it.n * kRowB;
        for (int kc = it.kc0; kc < it.kc1; ++kc) {
          if (!mbar_wait(&empty[st], ph ^ 1u, abort)) {
            if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_EMPTY);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[st], bytes);
          uint8_t* sa = smem + (size_t)st * a.stage_bytes;
          const int kx = kc * kBK;
          if (kGU) {
            tma_load_3d(sa, &tm_w, kx, it.m0, it.e, &full[st], pol_w);
            tma_load_3d(sa + kTileA, &tm_w, kx, a.I + it.m0, it.e, &full[st], pol_w);
            uint8_t* sb = sa + 2 * kTileA;
            for (int r = 0; r < nbox; ++r)
              tma_load_2d(sb + r * kBoxRows * kRowB, &tm_b, kx, it.row0 + r * kBoxRows, &full[st],
                          pol_b);
          } else {
            tma_load_3d(sa, &tm_w, kx, it.m0, it.e, &full[st], pol_w);
            uint8_t* sh = sa + kTileA;
            uint8_t* sl = sh + a.nmax * kRowB;
            for (int r = 0; r < nbox; ++r) {
              tma_load_2d(sh + r * kBoxRows * kRowB, &tm_b, kx, it.row0 + r * kBoxRows, &full[st],
                          pol_b);
              tma_load_2d(sl + r * kBoxRows * kRowB, &tm_b, kx, a.rmax + it.row0 + r * kBoxRows,
                          &full[st], pol_b);
            }
          }
          ++issued;
          if (++st == a.stages) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      // Drain: the last arming of each stage must have landed before this
      // CTA's shared memory can be released.
      for (int s = 0; s < a.stages; ++s) {
        const uint32_t n_s = issued / a.stages + ((uint32_t)s < issued % a.stages ? 1u : 0u);
        if (n_s == 0) continue;
        if (!mbar_wait(&full[s], (n_s - 1u) & 1u, nullptr)) {
          atomicOr(a.status, DEV_TIMEOUT_DRAIN);
          break;
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      int st = 0;
      uint32_t ph = 0;
      int j = 0;
      int e = 0;
      bool ok = true;
      for (int i = blockIdx.x; ok && i < total; i += gridDim.x, ++j) {
        const Item it = decode_item<kGU>(a, mv, i, e);
        const int ab = j & 1;
        const uint32_t aph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(&tempty[ab], aph ^ 1u, abort)) {
          if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_FULL);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(ab * kAccStride);
        const uint32_t idesc = idesc_bf16(it.n);
        for (int kc = it.kc0; kc < it.kc1; ++kc) {
          if (!mbar_wait(&full[st], ph, abort)) {
            if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_FULL);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + (size_t)st * a.stage_bytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint32_t acc = (kc > it.kc0 || kk > 0) ? 1u : 0u;
            if (kGU) {
              const uint64_t bdesc = sw128_desc(sa + 2 * kTileA + kk * 32);
              umma_bf16(d, sw128_desc(sa + kk * 32), bdesc, idesc, acc);
              umma_bf16(d + kUpCol, sw128_desc(sa + kTileA + kk * 32), bdesc, idesc, acc);
            } else {
              const uint64_t adesc = sw128_desc(sa + kk * 32);
              const uint32_t sh = sa + kTileA;
              const uint32_t sl = sh + a.nmax * kRowB;
              umma_bf16(d, adesc, sw128_desc(sh + kk * 32), idesc, acc);
              umma_bf16(d, adesc, sw128_desc(sl + kk * 32), idesc, 1u);
            }
          }
          umma_commit(&empty[st]);
          if (++st == a.stages) {
            st = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[ab]);
      }
      // Every MMA issued above must complete before TMEM is released.
      umma_commit(drain);
      if (!mbar_wait(drain, 0, nullptr)) atomicOr(a.status, DEV_TIMEOUT_DRAIN);
    }
  } else {
    // ---- epilogue: warps 2..5, TMEM lane quarter warp % 4 ----
    const int q = warp & 3;
    const int rloc = 32 * q + lane;
    int j = 0;
    int e = 0;
    for (int i = blockIdx.x; i < total; i += gridDim.x, ++j) {
      if (*abort) break;
      const Item it = decode_item<kGU>(a, mv, i, e);
      const int ab = j & 1;
      const uint32_t aph = (uint32_t)(j >> 1) & 1u;
      if (!mbar_wait(&tfull[ab], aph, abort)) {
        if (!*abort) flag_timeout(a, abort, DEV_TIMEOUT_ACT);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(ab * kAccStride);
      if (kGU) {
        const int irow = it.m0 + rloc;
        const bool inb = irow < a.I;
        __nv_bfloat16* hi = reinterpret_cast<__nv_bfloat16*>(a.act);
        __nv_bfloat16* lo = hi + (int64_t)a.rmax * a.I;
        for (int c0 = 0; c0 < it.n; c0 += 16) {
          uint32_t g[16], u[16];
          tmem_ld16(taddr + c0, g);
          tmem_ld16(taddr + kUpCol + c0, u);
          tmem_wait_ld(g);
          reg_dep16(u);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int r = it.row0 + c0 + c;
            const float wv = __ldg(a.row_w + r);
            const float av = silu(__uint_as_float(g[c])) * __uint_as_float(u[c]) * wv;
            const __nv_bfloat16 h = __float2bfloat16_rn(av);
            const __nv_bfloat16 l = __float2bfloat16_rn(av - __bfloat162float(h));
            if (inb) {
              hi[(int64_t)r * a.I + irow] = h;
              lo[(int64_t)r * a.I + irow] = l;
            }
          }
        }
      } else {
        const int hrow = it.m0 + rloc;
        const bool inb = hrow < a.H;
        float* yp = a.ypart + (int64_t)it.s * a.rmax * a.H;
        for (int c0 = 0; c0 < it.n; c0 += 16) {
          uint32_t v[16];
          tmem_ld16(taddr + c0, v);
          tmem_wait_ld(v);
#pragma unroll
          for (int c = 0; c < 16; ++c)
            if (inb) yp[(int64_t)(it.row0 + c0 + c) * a.H + hrow] = __uint_as_float(v[c]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[ab]);
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
                       const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  EncodeTiledFn enc;
  wr_status_t st = get_encoder(&enc);
  if (st != WR_OK) return st;
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base),
                   dims, strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(WR_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return WR_OK;
}

size_t a256(size_t n) { return (n + 255) & ~size_t(255); }

// Everything the grouped path derives from the problem on the host.
struct GroupedPlan {
  int nmax;       // token rows per tile
  int rmax;       // row capacity (>= padded rows in use)
  int mtA, mtB;   // weight-row tiles per expert (gate/up over I, down over H)
  int kcA, kcB;   // K chunks (over H, over I)
  int S, kc_split;
  int stagesA, stagesB, stage_bytesA, stage_bytesB;
  size_t off_ids, off_w, off_slot, off_meta, off_rtok, off_rw, off_xg, off_act, off_y, total;
};

int split_count(int kcB, int units, int sms) {
  int best = 1;
  double best_eff = 0.0;
  for (int s = 1; s <= 8; ++s) {
    if (s > 1 && kcB / s < 8) break;
    const int items = units * s;
    const int rounds = (items + sms - 1) / sms;
    const double eff = (double)items / ((double)rounds * sms);
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      best = s;
    }
  }
  return best;
}

GroupedPlan make_plan(const Problem& p, int sms) {
  GroupedPlan g;
  const int TK = p.T * p.K;
  const int n16 = (p.T + 15) & ~15;
  g.nmax = n16 < kNMax ? n16 : kNMax;
  g.rmax = (TK + 15 * p.ep_num + 15) & ~15;
  g.mtA = (p.I + kBM - 1) / kBM;
  g.mtB = (p.H + kBM - 1) / kBM;
  g.kcA = (p.H + kBK - 1) / kBK;
  g.kcB = (p.I + kBK - 1) / kBK;
  const int active = TK < p.ep_num ? TK : p.ep_num;
  const int s0 = split_count(g.kcB, active * g.mtB, sms);
  g.kc_split = (g.kcB + s0 - 1) / s0;
  g.S = (g.kcB + g.kc_split - 1) / g.kc_split;
  const int avail = kSmemMax - kSmemReserve;
  g.stage_bytesA = 2 * kTileA + g.nmax * kRowB;
  g.stage_bytesA = (g.stage_bytesA + 1023) & ~1023;
  g.stage_bytesB = kTileA + 2 * g.nmax * kRowB;
  g.stage_bytesB = (g.stage_bytesB + 1023) & ~1023;
  g.stagesA = avail / g.stage_bytesA;
  g.stagesB = avail / g.stage_bytesB;
  if (g.stagesA > kMaxStages) g.stagesA = kMaxStages;
  if (g.stagesB > kMaxStages) g.stagesB = kMaxStages;
  size_t o = kWsControlBytes;
  g.off_ids = o; o += a256(4 * (size_t)TK);
  g.off_w = o; o += a256(4 * (size_t)TK);
  g.off_slot = o; o += a256(4 * (size_t)TK);
  g.off_meta = o; o += a256(4 * (size_t)meta_words(p.ep_num));
  g.off_rtok = o; o += a256(4 * (size_t)g.rmax);
  g.off_rw = o; o += a256(4 * (size_t)g.rmax);
  g.off_xg = o; o += a256(2 * (size_t)g.rmax * p.H);
  g.off_act = o; o += a256(2 * 2 * (size_t)g.rmax * p.I);
  g.off_y = o; o += a256(4 * (size_t)g.S * g.rmax * p.H);
  g.total = o;
  return g;
}

template <bool kGU>
wr_status_t set_smem_attr() {
  static std::once_flag once[64];
  static cudaError_t err[64];
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&] {
    err[dev & 63] = cudaFuncSetAttribute(k_grouped_gemm<kGU>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  });
  if (err[dev & 63] != cudaSuccess)
    return cuda_fail(err[dev & 63], "cudaFuncSetAttribute(grouped gemm)");
  return WR_OK;
}

}  // namespace

bool grouped_supported(const Problem& p) {
  return p.dtype == WR_DTYPE_BF16 && p.T >= kGroupedMinTokens && p.H % 8 == 0 && p.I % 8 == 0 &&
         p.ep_num >= 1;
}

size_t grouped_workspace_bytes(const Problem& p) {
  return make_plan(p, device_sm_count()).total;
}

wr_status_t launch_grouped(const Problem& p, const void* x, const void* gate_w, const void* wbuf,
                           float* out, int32_t* ids, float* w, void* ws, cudaStream_t stream) {
  const int sms = device_sm_count();
  const GroupedPlan g = make_plan(p, sms);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  int32_t* ids_d = ids ? ids : reinterpret_cast<int32_t*>(wsb + g.off_ids);
  float* w_d = w ? w : reinterpret_cast<float*>(wsb + g.off_w);
  int32_t* slot = reinterpret_cast<int32_t*>(wsb + g.off_slot);
  int* meta = reinterpret_cast<int*>(wsb + g.off_meta);
  int32_t* rtok = reinterpret_cast<int32_t*>(wsb + g.off_rtok);
  float* rw = reinterpret_cast<float*>(wsb + g.off_rw);
  uint16_t* xg = reinterpret_cast<uint16_t*>(wsb + g.off_xg);
  uint16_t* act = reinterpret_cast<uint16_t*>(wsb + g.off_act);
  float* ypart = reinterpret_cast<float*>(wsb + g.off_y);
  uint32_t* status = reinterpret_cast<uint32_t*>(ws) + 2;

  wr_status_t st = launch_router(p, x, gate_w, nullptr, ids_d, w_d, stream);
  if (st != WR_OK) return st;
  k_bucket<<<1, 512, 0, stream>>>(ids_d, w_d, p.T * p.K, p.K, p.ep_first, p.ep_num, g.nmax,
                                   g.mtA, g.mtB, g.S, meta, slot, rtok, rw);
  const int gather_blocks = g.rmax < 4 * sms ? g.rmax : 4 * sms;
  k_gather<<<gather_blocks, 256, 0, stream>>>(static_cast<const uint4*>(x), p.H / 8, meta, rtok,
                                              reinterpret_cast<uint4*>(xg));
  cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) return cuda_fail(ce, "bucket / gather launch");

  const Layout lay = make_layout(p.H, p.I, 2);
  const uint8_t* wb = static_cast<const uint8_t*>(wbuf);
  CUtensorMap tm_gu, tm_x, tm_dn, tm_act;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)p.H, (cuuint64_t)2 * p.I, (cuuint64_t)p.ep_num};
    const cuuint64_t str[2] = {(cuuint64_t)p.H * 2, (cuuint64_t)lay.stride};
    const cuuint32_t box[3] = {kBK, kBM, 1};
    if ((st = encode_map(&tm_gu, wb + lay.off_gate, 3, dims, str, box)) != WR_OK) return st;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)p.H, (cuuint64_t)g.rmax};
    const cuuint64_t str[1] = {(cuuint64_t)p.H * 2};
    const cuuint32_t box[2] = {kBK, kBoxRows};
    if ((st = encode_map(&tm_x, xg, 2, dims, str, box)) != WR_OK) return st;
  }
  {
    const cuuint64_t dims[3] = {(cuuint64_t)p.I, (cuuint64_t)p.H, (cuuint64_t)p.ep_num};
    const cuuint64_t str[2] = {(cuuint64_t)p.I * 2, (cuuint64_t)lay.stride};
    const cuuint32_t box[3] = {kBK, kBM, 1};
    if ((st = encode_map(&tm_dn, wb + lay.off_down, 3, dims, str, box)) != WR_OK) return st;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)p.I, (cuuint64_t)2 * g.rmax};
    const cuuint64_t str[1] = {(cuuint64_t)p.I * 2};
    const cuuint32_t box[2] = {kBK, kBoxRows};
    if ((st = encode_map(&tm_act, act, 2, dims, str, box)) != WR_OK) return st;
  }
  if ((st = set_smem_attr<true>()) != WR_OK) return st;
  if ((st = set_smem_attr<false>()) != WR_OK) return st;

  GemmArgs ga;
  ga.meta = meta;
  ga.E = p.ep_num;
  ga.H = p.H;
  ga.I = p.I;
  ga.nmax = g.nmax;
  ga.rmax = g.rmax;
  ga.row_w = rw;
  ga.act = act;
  ga.ypart = ypart;
  ga.status = status;

  GemmArgs a1 = ga;
  a1.S = 1;
  a1.kc_total = g.kcA;
  a1.kc_split = g.kcA;
  a1.mt = g.mtA;
  a1.stages = g.stagesA;
  a1.stage_bytes = g.stage_bytesA;
  const size_t smemA = (size_t)g.stagesA * g.stage_bytesA + kSmemReserve;
  k_grouped_gemm<true><<<sms, kGemmThreads, smemA, stream>>>(tm_gu, tm_x, a1);

  GemmArgs a2 = ga;
  a2.S = g.S;
  a2.kc_total = g.kcB;
  a2.kc_split = g.kc_split;
  a2.mt = g.mtB;
  a2.stages = g.stagesB;
  a2.stage_bytes = g.stage_bytesB;
  const size_t smemB = (size_t)g.stagesB * g.stage_bytesB + kSmemReserve;
  k_grouped_gemm<false><<<sms, kGemmThreads, smemB, stream>>>(tm_dn, tm_act, a2);

  k_combine<<<p.T, 256, 0, stream>>>(reinterpret_cast<const float4*>(ypart), slot, p.K, p.H / 4,
                                     g.S, g.rmax, reinterpret_cast<float4*>(out));
  ce = cudaGetLastError();
  return ce == cudaSuccess ? WR_OK : cuda_fail(ce, "grouped GEMM launch");
}

}  // namespace wr
