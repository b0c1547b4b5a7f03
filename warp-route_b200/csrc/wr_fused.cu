// wr_fused.cu — the fused decode-time MoE layer for 1..4 tokens, streamed
// through shared memory with bulk (TMA) copies at HBM bandwidth.
//
// Replaces warp-route's k_fused_moe / k_fused_moe_batched
// (src/fused_moe.cu:76-227, src/fused_moe_batched.cu:66-180): the same
// router -> top-K -> SwiGLU over the selected experts -> weighted combine,
// but spread over every SM instead of one warp.
//
// One persistent CTA per SM (cooperative launch, 227 KB of shared memory):
//   warps 0-7  consumers: router, then dot products out of shared memory;
//   warp 8     producer: one elected lane issues cp.async.bulk copies of
//              weight rows into a 4-stage ring (mbarrier full/empty pairs),
//              L2 evict-first, never waiting on the math.
// Every CTA computes the router redundantly (the router rows are L2
// resident), so all CTAs agree on the selection without a grid sync.
// The selected experts become "slots"; the layer is then two matvecs over
// virtual matrices built from the slots' packed blocks:
//   phase A  rows p = slot*I + i of [Wg; Wu] . x  ->  act[p] =
//            w_slot * silu(g) * u        (fp32, workspace, per token)
//   phase B  out[h] = sum_c Wd_virtual[h, c] * act[c],  c over slot*I + i
// Phase A rows and phase B rows are split evenly over the CTAs.  Between
// the phases one grid-wide barrier (bounded spin) makes act visible; the
// producer keeps streaming phase-B weights across it, so HBM never idles.
// Phase B reads act through shared memory in windows of up to ~93 KB.
// Results are deterministic: fixed lane order, fixed xor trees, fixed
// window order, no floating-point atomics.
#include <cuda_runtime.h>

#include <mutex>

#include "wr_common.cuh"
#include "wr_internal.h"
#include "wr_router.cuh"

namespace wr {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;  // + producer warp
constexpr int kStageBytes = 32 * 1024;
constexpr int kStages = 4;
constexpr int kRingBytes = kStages * kStageBytes;
constexpr int kSmemBytes = 232448;  // 227 KB: the sm_100 per-CTA opt-in maximum
constexpr int kMiscBytes = 6144;
constexpr int kVecBytes = kSmemBytes - kRingBytes - kMiscBytes;  // x / act window
constexpr int kMaxNT = 4;
static_assert(kVecBytes % 16 == 0, "vector region must keep 16-byte alignment");

// Offsets inside the misc region.
constexpr int kOffBars = 0;        // full[kStages], empty[kStages], act
constexpr int kOffAbort = 128;     // int
constexpr int kOffNSlots = 132;    // int
constexpr int kOffSlotE = 256;     // int [64]: local expert of each slot
constexpr int kOffSlotW = 512;     // float [64 * NT]: routing weight (0: not routed)
constexpr int kOffLogits = 1536;   // float [NT * 64]
constexpr int kOffTokIds = 2560;   // int [NT * 64]
constexpr int kOffTokW = 3584;     // float [NT * 64]
static_assert(kOffTokW + 4 * kMaxNT * kMaxExperts <= kMiscBytes, "misc region overflow");

// Workspace words (uint32) in front of the activation buffer.
constexpr int kSyncArrive = 0;
constexpr int kSyncExit = 1;
constexpr int kSyncStatus = 2;
constexpr size_t kSyncBytes = 256;

struct FusedArgs {
  const void* x;
  const void* gate_w;
  const float* router_bias;
  const uint8_t* wbuf;
  float* out;
  int32_t* ids_out;
  float* w_out;
  float* act;
  uint32_t* sync;
  int E, H, I, K, T;
  int ep_first, ep_num;
  Layout lay;
};

// Balanced split of n items into parts: [n*i/parts, n*(i+1)/parts).
WR_DEVINL int split_lo(int64_t n, int i, int parts) { return (int)((n * i) / parts); }

template <typename Tw, int NT>
__global__ void __launch_bounds__(kThreads, 1) k_fused_stream(const FusedArgs a) {
  constexpr int VEC = Chunk<Tw>::kVec;
  constexpr int ELT = (int)sizeof(Tw);
  constexpr int CWA = kStageBytes / (2 * kConsumerWarps * ELT);  // phase A columns per stage
  constexpr int CWB = kStageBytes / (kConsumerWarps * ELT);      // phase B columns per stage

  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ring = smem;
  float* vreg = reinterpret_cast<float*>(smem + kRingBytes);
  uint8_t* misc = smem + kRingBytes + kVecBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(misc + kOffBars);
  uint64_t* empty = full + kStages;
  uint64_t* actbar = empty + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + kOffAbort);
  int* s_nslots = reinterpret_cast<int*>(misc + kOffNSlots);
  int* slot_e = reinterpret_cast<int*>(misc + kOffSlotE);
  float* slot_w = reinterpret_cast<float*>(misc + kOffSlotW);
  float* s_logits = reinterpret_cast<float*>(misc + kOffLogits);
  int* tok_ids = reinterpret_cast<int*>(misc + kOffTokIds);
  float* tok_w = reinterpret_cast<float*>(misc + kOffTokW);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int H = a.H, I = a.I, E = a.E, K = a.K, T = a.T;
  const int G = gridDim.x, b = blockIdx.x;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    mbar_init(actbar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }

  // ---- x -> shared memory as fp32 [NT][H] (tokens >= T are zero) ----------
  {
    const Tw* xg = static_cast<const Tw*>(a.x);
    const int nvec = H / VEC;  // host guarantees H % VEC == 0 on this path
    for (int idx = tid; idx < NT * nvec; idx += kThreads) {
      const int t = idx / nvec;
      const int v = idx - t * nvec;
      float f[VEC];
      if (t < T) {
        Chunk<Tw>::widen(ldg_nc_v4(xg + (int64_t)t * H + (int64_t)v * VEC), f);
      } else {
#pragma unroll
        for (int q = 0; q < VEC; ++q) f[q] = 0.0f;
      }
      float4* dst = reinterpret_cast<float4*>(vreg + (int64_t)t * H + (int64_t)v * VEC);
#pragma unroll
      for (int q = 0; q < VEC / 4; ++q) dst[q] = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
    }
  }
  __syncthreads();

  // ---- router: every warp takes (token, expert) pairs ----------------------
  for (int j = warp; j < T * E; j += kThreads / 32) {
    const int t = j / E;
    const int e = j - t * E;
    float l = router_logit_warp<Tw>(static_cast<const Tw*>(a.gate_w) + (int64_t)e * H,
                                    vreg + (int64_t)t * H, H, lane, true);
    if (lane == 0) {
      if (a.router_bias) l = __fadd_rn(l, a.router_bias[e]);
      s_logits[t * kMaxExperts + e] = l;
    }
  }
  __syncthreads();

  // ---- selection + slots (one thread; E <= 64, K <= E) ---------------------
  if (tid == 0) {
    int ns = 0;
    for (int t = 0; t < T; ++t) {
      softmax_topk(s_logits + t * kMaxExperts, E, K, tok_ids + t * kMaxExperts,
                   tok_w + t * kMaxExperts);
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
      if (b == 0) {
        for (int k = 0; k < K; ++k) {
          if (a.ids_out) a.ids_out[t * K + k] = tok_ids[t * kMaxExperts + k];
          if (a.w_out) a.w_out[t * K + k] = tok_w[t * kMaxExperts + k];
        }
      }
    }
    *s_nslots = ns;
  }
  __syncthreads();

  const int S = *s_nslots;
  const int64_t P = (int64_t)S * I;  // phase A rows == phase B columns
  const int pa0 = split_lo(P, b, G), pa1 = split_lo(P, b + 1, G);
  const int hb0 = split_lo(H, b, G), hb1 = split_lo(H, b + 1, G);
  const int na = pa1 - pa0, nb = hb1 - hb0;
  const int nga = (na + kConsumerWarps - 1) / kConsumerWarps;
  const int ngb = (nb + kConsumerWarps - 1) / kConsumerWarps;
  // Activation windows over the P columns of phase B.
  const int64_t wmax = (int64_t)(kVecBytes / (NT * 4)) / VEC * VEC;
  const int nwin = (int)((P + wmax - 1) / wmax);
  int64_t wsz = nwin ? (P + nwin - 1) / nwin : 0;
  wsz = (wsz + VEC - 1) / VEC * VEC;

  if (S == 0) {
    // No local expert selected (expert-parallel rank): this rank adds zero.
    for (int idx = tid; idx < T * nb; idx += kThreads) {
      const int t = idx / nb;
      a.out[(int64_t)t * H + hb0 + (idx - t * nb)] = 0.0f;
    }
  } else if (warp == kConsumerWarps) {
    // =========================== producer ===================================
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      uint32_t it = 0;
      bool ok = true;
      for (int gi = 0; gi < nga && ok; ++gi) {
        const int r0 = pa0 + split_lo(na, gi, nga), r1 = pa0 + split_lo(na, gi + 1, nga);
        for (int c0 = 0; c0 < H; c0 += CWA) {
          const int cw = min(CWA, H - c0);
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
          uint8_t* st = ring + s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * (r1 - r0) * cw * ELT));
          for (int r = r0; r < r1; ++r) {
            const int sl = r / I;
            const int i = r - sl * I;
            const uint8_t* src = a.wbuf + (int64_t)slot_e[sl] * a.lay.stride +
                                 ((int64_t)i * H + c0) * ELT;
            bulk_g2s(st + (r - r0) * CWA * ELT, src + a.lay.off_gate, cw * ELT, &full[s], pol);
            bulk_g2s(st + (kConsumerWarps + r - r0) * CWA * ELT, src + a.lay.off_up, cw * ELT,
                     &full[s], pol);
          }
          ++it;
        }
      }
      for (int w = 0; w < nwin && ok; ++w) {
        const int64_t ws0 = (int64_t)w * wsz;
        const int64_t ws1 = min(P, ws0 + wsz);
        for (int gi = 0; gi < ngb && ok; ++gi) {
          const int r0 = hb0 + split_lo(nb, gi, ngb), r1 = hb0 + split_lo(nb, gi + 1, ngb);
          for (int64_t c0 = ws0; c0 < ws1; c0 += CWB) {
            const int cw = (int)min((int64_t)CWB, ws1 - c0);
            const int s = it % kStages;
            const uint32_t ph = (it / kStages) & 1u;
            if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag)) { ok = false; break; }
            uint8_t* st = ring + s * kStageBytes;
            mbar_arrive_expect_tx(&full[s], (uint32_t)((r1 - r0) * cw * ELT));
            for (int r = r0; r < r1; ++r) {
              uint8_t* dst = st + (r - r0) * CWB * ELT;
              int64_t c = c0;
              while (c < c0 + cw) {
                const int sl = (int)(c / I);
                const int64_t i0 = c - (int64_t)sl * I;
                const int len = (int)(min(c0 + cw, (int64_t)(sl + 1) * I) - c);
                const uint8_t* src = a.wbuf + (int64_t)slot_e[sl] * a.lay.stride +
                                     a.lay.off_down + ((int64_t)r * I + i0) * ELT;
                bulk_g2s(dst + (c - c0) * ELT, src, len * ELT, &full[s], pol);
                c += len;
              }
            }
            ++it;
          }
        }
      }
      if (!ok) {
        // Let every copy already issued land before the CTA can exit.
        *abort_flag = 1;
        const uint32_t first = it > (uint32_t)kStages ? it - kStages : 0u;
        for (uint32_t j = first; j < it; ++j)
          if (!mbar_wait(&full[j % kStages], (j / kStages) & 1u, nullptr))
            atomicOr(&a.sync[kSyncStatus], DEV_TIMEOUT_DRAIN);
        atomicOr(&a.sync[kSyncStatus], DEV_TIMEOUT_EMPTY);
      }
    }
  } else {
    // =========================== consumers ==================================
    // Abort-safe structure: loop trip counts depend only on the problem, so
    // every consumer warp passes every named barrier exactly once even after
    // a failed wait; `ok` is kept warp-uniform with __all_sync.
    const int cw_id = warp;  // 0..7
    uint32_t it = 0;
    bool ok = true;
    // ---- phase A: gate/up rows -> activations ----
    for (int gi = 0; gi < nga; ++gi) {
      const int r0 = pa0 + split_lo(na, gi, nga), r1 = pa0 + split_lo(na, gi + 1, nga);
      const bool active = cw_id < r1 - r0;
      float g[NT], u[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) g[t] = u[t] = 0.0f;
      for (int c0 = 0; c0 < H; c0 += CWA) {
        const int cw = min(CWA, H - c0);
        const int s = it % kStages;
        const uint32_t ph = (it / kStages) & 1u;
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&full[s], ph, abort_flag));
        if (ok && active) {
          const uint8_t* st = ring + s * kStageBytes;
          const uint4* gp = reinterpret_cast<const uint4*>(st + cw_id * CWA * ELT);
          const uint4* up = reinterpret_cast<const uint4*>(st + (kConsumerWarps + cw_id) * CWA * ELT);
          const int nch = cw / VEC;
          for (int j = lane; j < nch; j += 32) {
            float gf[VEC], uf[VEC];
            Chunk<Tw>::widen(gp[j], gf);
            Chunk<Tw>::widen(up[j], uf);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              const float4* xv = reinterpret_cast<const float4*>(vreg + (int64_t)t * H + c0 + j * VEC);
#pragma unroll
              for (int q4 = 0; q4 < VEC / 4; ++q4) {
                const float4 x4 = xv[q4];
                g[t] = fmaf(gf[4 * q4 + 0], x4.x, g[t]);
                g[t] = fmaf(gf[4 * q4 + 1], x4.y, g[t]);
                g[t] = fmaf(gf[4 * q4 + 2], x4.z, g[t]);
                g[t] = fmaf(gf[4 * q4 + 3], x4.w, g[t]);
                u[t] = fmaf(uf[4 * q4 + 0], x4.x, u[t]);
                u[t] = fmaf(uf[4 * q4 + 1], x4.y, u[t]);
                u[t] = fmaf(uf[4 * q4 + 2], x4.z, u[t]);
                u[t] = fmaf(uf[4 * q4 + 3], x4.w, u[t]);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        ++it;
      }
      if (ok && active) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) {
            g[t] += __shfl_xor_sync(0xffffffffu, g[t], off);
            u[t] += __shfl_xor_sync(0xffffffffu, u[t], off);
          }
        }
        if (lane == 0) {
          const int r = r0 + cw_id;
          const int sl = r / I;
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const float wt = slot_w[sl * NT + t];
            a.act[(int64_t)r * NT + t] = (wt != 0.0f) ? wt * (silu(g[t]) * u[t]) : 0.0f;
          }
        }
      }
    }
    if (!ok && lane == 0) *abort_flag = 1;

    // ---- grid-wide barrier: every CTA's activations are written ----
    named_bar_sync(1, kConsumerThreads);
    if (tid == 0) {
      __threadfence();
      fence_proxy_async_global();
      red_release_gpu_add(&a.sync[kSyncArrive], 1u);
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_gpu(&a.sync[kSyncArrive]) < (uint32_t)G) {
        if ((++spins & 63u) == 0) {
          if (*abort_flag || globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(&a.sync[kSyncStatus], DEV_TIMEOUT_GRID);
            *abort_flag = 1;
            break;
          }
        }
      }
      fence_proxy_async_global();
    }

    // ---- phase B: down rows over activation windows ----
    int act_issued = 0;
    for (int w = 0; w < nwin; ++w) {
      const int64_t ws0 = (int64_t)w * wsz;
      const int64_t ws1 = min(P, ws0 + wsz);
      named_bar_sync(1, kConsumerThreads);  // window w-1 fully read (or the grid barrier done)
      if (*abort_flag) ok = false;
      if (tid == 0 && ok) {
        fence_proxy_async_smem();
        const uint32_t bytes = (uint32_t)((ws1 - ws0) * NT * 4);
        const uint64_t pol = l2_policy_evict_last();
        mbar_arrive_expect_tx(actbar, bytes);
        const uint8_t* src = reinterpret_cast<const uint8_t*>(a.act + ws0 * NT);
        for (uint32_t off = 0; off < bytes; off += 32768u)
          bulk_g2s(reinterpret_cast<uint8_t*>(vreg) + off, src + off, min(32768u, bytes - off),
                   actbar, pol);
        act_issued = w + 1;
      }
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(actbar, (uint32_t)(w & 1), abort_flag));
      for (int gi = 0; gi < ngb; ++gi) {
        const int r0 = hb0 + split_lo(nb, gi, ngb), r1 = hb0 + split_lo(nb, gi + 1, ngb);
        const bool active = cw_id < r1 - r0;
        float acc[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
        for (int64_t c0 = ws0; c0 < ws1; c0 += CWB) {
          const int cw = (int)min((int64_t)CWB, ws1 - c0);
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1u;
          if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&full[s], ph, abort_flag));
          if (ok && active) {
            const uint4* wp = reinterpret_cast<const uint4*>(ring + s * kStageBytes + cw_id * CWB * ELT);
            const float* abase = vreg + (c0 - ws0) * NT;
            const int nch = cw / VEC;
            for (int j = lane; j < nch; j += 32) {
              float wf[VEC];
              Chunk<Tw>::widen(wp[j], wf);
              const float4* av = reinterpret_cast<const float4*>(abase + j * VEC * NT);
#pragma unroll
              for (int q4 = 0; q4 < VEC * NT / 4; ++q4) {
                const float4 a4 = av[q4];
                const float av4[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
                for (int z = 0; z < 4; ++z) {
                  const int flat = 4 * q4 + z;  // = q * NT + t
                  acc[flat % NT] = fmaf(wf[flat / NT], av4[z], acc[flat % NT]);
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
          ++it;
        }
        if (ok && active) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], off);
          }
          if (lane == 0) {
            const int h = r0 + cw_id;
            for (int t = 0; t < T; ++t) {
              float* o = a.out + (int64_t)t * H + h;
              *o = (w == 0) ? acc[t] : *o + acc[t];
            }
          }
        }
      }
      if (!ok && lane == 0) *abort_flag = 1;
    }
    if (tid == 0 && act_issued > 0 && !ok) {
      // The last activation copy must land before the CTA exits.
      if (!mbar_wait(actbar, (uint32_t)((act_issued - 1) & 1), nullptr))
        atomicOr(&a.sync[kSyncStatus], DEV_TIMEOUT_DRAIN);
    }
    if (lane == 0 && !ok) atomicOr(&a.sync[kSyncStatus], DEV_TIMEOUT_FULL);
  }

  __syncthreads();
  if (tid == 0) {
    // Self-reset of the grid barrier: every CTA has left its wait once it
    // counts itself out, so the last one can clear both counters.
    __threadfence();
    const uint32_t prev = atomicAdd(&a.sync[kSyncExit], 1u);
    if (prev == (uint32_t)G - 1) {
      atomicExch(&a.sync[kSyncArrive], 0u);
      atomicExch(&a.sync[kSyncExit], 0u);
      __threadfence();
    }
  }
}

template <typename Tw, int NT>
wr_status_t launch_one(const FusedArgs& args, int grid, cudaStream_t stream) {
  auto kern = k_fused_stream<Tw, NT>;
  static std::once_flag once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  static cudaError_t attr_err[64];
  std::call_once(once[dev & 63], [&] {
    attr_err[dev & 63] =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  });
  if (attr_err[dev & 63] != cudaSuccess) return cuda_fail(attr_err[dev & 63], "cudaFuncSetAttribute(fused)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(fused)");
  return WR_OK;
}

int nt_bucket(int T) { return T <= 1 ? 1 : (T <= 2 ? 2 : 4); }

}  // namespace

bool fused_supported(const Problem& p) {
  const int vec = 16 / p.elt;
  if (p.H % vec != 0 || p.I % vec != 0) return false;
  if (p.E > kMaxExperts || p.K > p.E) return false;
  if (p.T < 1 || p.T > kMaxNT) return false;
  const int nt = nt_bucket(p.T);
  if ((int64_t)nt * p.H * 4 > kVecBytes) return false;  // x must fit in shared memory
  return true;
}

size_t fused_workspace_bytes(const Problem& p) {
  const int nt = nt_bucket(p.T < 1 ? 1 : p.T);
  const int64_t slots = p.ep_num < p.K * nt ? p.ep_num : (int64_t)p.K * nt;
  const size_t act = (size_t)slots * p.I * nt * sizeof(float);
  return kSyncBytes + ((act + 255) & ~size_t(255));
}

wr_status_t launch_fused(const Problem& p, const void* x, const void* gate_w, const void* wbuf,
                         float* out, int32_t* ids, float* w, void* ws, cudaStream_t stream) {
  FusedArgs args;
  args.x = x;
  args.gate_w = gate_w;
  args.router_bias = p.router_bias;
  args.wbuf = static_cast<const uint8_t*>(wbuf);
  args.out = out;
  args.ids_out = ids;
  args.w_out = w;
  args.sync = static_cast<uint32_t*>(ws);
  args.act = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kSyncBytes);
  args.E = p.E;
  args.H = p.H;
  args.I = p.I;
  args.K = p.K;
  args.T = p.T;
  args.ep_first = p.ep_first;
  args.ep_num = p.ep_num;
  args.lay = make_layout(p.H, p.I, p.elt);
  const int grid = device_sm_count();
  const int nt = nt_bucket(p.T);
  if (p.dtype == WR_DTYPE_BF16) {
    if (nt == 1) return launch_one<uint16_t, 1>(args, grid, stream);
    if (nt == 2) return launch_one<uint16_t, 2>(args, grid, stream);
    return launch_one<uint16_t, 4>(args, grid, stream);
  }
  if (nt == 1) return launch_one<float, 1>(args, grid, stream);
  if (nt == 2) return launch_one<float, 2>(args, grid, stream);
  return launch_one<float, 4>(args, grid, stream);
}

}  // namespace wr
