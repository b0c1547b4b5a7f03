// wr_router.cuh — router logits, softmax and top-K (device side).
//
// Follows warp-route's inlined router (src/fused_moe.cu:100-150,
// src/gate.cu:6-101): fp32 logits = gate_w[e,:] . x, softmax over all E,
// iterative argmax with strict '>' (ties -> lowest index), weights are the
// probabilities, not renormalised.  Differences, on purpose:
//   * one fixed reduction order for each logit — lane l of a warp runs an
//     explicit-fma sweep over the 16-byte vectors v = l, l+32, l+64, ...
//     (elements of a vector in order), then a 16/8/4/2/1 xor tree — so the
//     logits are bit-identical across devices and to the CPU oracle;
//   * the argmax runs on the logits (softmax is monotonic), so selection
//     never depends on the last bit of exp();
//   * an optional fp32 router bias is added after the tree.
#pragma once

#include "wr_common.cuh"

namespace wr {

constexpr int kMaxExperts = 64;

// One logit, computed by a full warp.  `xs` is the token's fp32 activation
// vector (shared or global memory), `wrow` the router row (global).
// `vec_ok`: the row and H allow 16-byte vector loads.  Result valid on all
// lanes.
template <typename Tw>
WR_DEVINL float router_logit_warp(const Tw* __restrict__ wrow, const float* __restrict__ xs,
                                  int H, int lane, bool vec_ok) {
  constexpr int VEC = Chunk<Tw>::kVec;
  float acc = 0.0f;
  if (vec_ok) {
    const int nvec = H / VEC;
#pragma unroll 4
    for (int v = lane; v < nvec; v += 32) {
      const uint4 raw = ldg_nc_v4(wrow + (int64_t)v * VEC);
      float f[VEC];
      Chunk<Tw>::widen(raw, f);
      const float* xv = xs + (int64_t)v * VEC;
#pragma unroll
      for (int q = 0; q < VEC; ++q) acc = __fmaf_rn(f[q], xv[q], acc);
    }
  } else {
    const int nvec = (H + VEC - 1) / VEC;
    for (int v = lane; v < nvec; v += 32) {
#pragma unroll
      for (int q = 0; q < VEC; ++q) {
        const int j = v * VEC + q;
        if (j < H) acc = __fmaf_rn(load_scalar<Tw>(wrow, j), xs[j], acc);
      }
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1)
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  return acc;
}

// Softmax + top-K for one token, run by a single thread.
// logits [E] (E <= 64) -> ids [K], weights [K] (probabilities of the picks).
WR_DEVINL void softmax_topk(const float* logits, int E, int K, int* ids, float* weights) {
  float m = logits[0];
  for (int e = 1; e < E; ++e) m = fmaxf(m, logits[e]);
  float s = 0.0f;
  for (int e = 0; e < E; ++e) s = __fadd_rn(s, expf(logits[e] - m));
  uint64_t used = 0;
  for (int k = 0; k < K; ++k) {
    int best = -1;
    for (int e = 0; e < E; ++e) {
      if ((used >> e) & 1ull) continue;
      if (best < 0 || logits[e] > logits[best]) best = e;
    }
    used |= 1ull << best;
    ids[k] = best;
    weights[k] = __fdiv_rn(expf(logits[best] - m), s);
  }
}

}  // namespace wr
