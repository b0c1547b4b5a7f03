// wr_router.cuh — router logits, softmax and top-K (device side).
//
// Follows warp-route's inlined router (src/fused_moe.cu:100-150,
// src/gate.cu:6-101): fp32 logits = gate_w[e,:] . x, softmax over all E,
// iterative argmax with strict '>' (ties -> lowest index), weights are the
// probabilities, not renormalised.  Differences, on purpose:
//   * one fixed reduction order for each logit, so logits are bit-identical
//     across devices and to the CPU oracle.  The row's 16-byte vectors
//     (nvec = ceil(H / VEC)) are cut into 8 segments [nvec*j/8,
//     nvec*(j+1)/8); in segment j, lane l runs an explicit-fma sweep over the
//     vectors lo+l, lo+l+32, ... (elements of a vector in order), a 16/8/4/2/1
//     xor tree gives the segment sum s_j, and logit = (((s_0 + s_1) + s_2) +
//     ... + s_7).  One warp per segment lets every warp keep many router rows
//     in flight at once;
//   * the argmax runs on the logits (softmax is monotonic), so selection
//     never depends on the last bit of exp();
//   * an optional fp32 router bias is added after the sum.
#pragma once

#include "wr_common.cuh"

namespace wr {

constexpr int kMaxExperts = 64;
constexpr int kRouterSegments = 8;
constexpr int kRouterRowBatch = 8;  // router rows a warp keeps in flight

// Where router_segment_warp reads x: an fp32 copy in shared memory, or the
// caller's x in global memory (widened on the fly; widening is exact, so both
// give the same fp32 values and the same sums).
struct XSmem {
  const float* p;
  template <int VEC>
  WR_DEVINL void vec(int v, float (&f)[VEC]) const {
#pragma unroll
    for (int q = 0; q < VEC; ++q) f[q] = p[(int64_t)v * VEC + q];
  }
  WR_DEVINL float at(int j) const { return p[j]; }
};
template <typename Tw>
struct XGlobal {
  const Tw* p;
  template <int VEC>
  WR_DEVINL void vec(int v, float (&f)[VEC]) const {
    Chunk<Tw>::widen(ldg_nc_v4(p + (int64_t)v * VEC), f);
  }
  WR_DEVINL float at(int j) const { return load_scalar<Tw>(p, j); }
};

// Segment `seg` partial sums of rows [0, E) of gate_w against x, computed by
// one warp.  Writes part[e] (lane 0) for every row.  vec_ok: rows and H allow
// 16-byte vector loads.
template <typename Tw, typename XS = XSmem>
WR_DEVINL void router_segment_warp(const Tw* __restrict__ gate_w, const XS xs, int E, int H,
                                   int seg, int lane, bool vec_ok, float* __restrict__ part) {
  constexpr int VEC = Chunk<Tw>::kVec;
  constexpr int RB = kRouterRowBatch;
  const int nvec = (H + VEC - 1) / VEC;
  const int lo = (int)((int64_t)nvec * seg / kRouterSegments);
  const int hi = (int)((int64_t)nvec * (seg + 1) / kRouterSegments);
  for (int e0 = 0; e0 < E; e0 += RB) {
    float acc[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) acc[r] = 0.0f;
    if (vec_ok) {
      for (int v = lo + lane; v < hi; v += 32) {
        uint4 raw[RB];
#pragma unroll
        for (int r = 0; r < RB; ++r)
          if (e0 + r < E) raw[r] = ldg_nc_v4(gate_w + (int64_t)(e0 + r) * H + (int64_t)v * VEC);
        float xf[VEC];
        xs.template vec<VEC>(v, xf);
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          if (e0 + r < E) {
            float f[VEC];
            Chunk<Tw>::widen(raw[r], f);
#pragma unroll
            for (int q = 0; q < VEC; ++q) acc[r] = __fmaf_rn(f[q], xf[q], acc[r]);
          }
        }
      }
    } else {
      for (int v = lo + lane; v < hi; v += 32) {
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          if (e0 + r >= E) continue;
          const Tw* row = gate_w + (int64_t)(e0 + r) * H;
#pragma unroll
          for (int q = 0; q < VEC; ++q) {
            const int j = v * VEC + q;
            if (j < H) acc[r] = __fmaf_rn(load_scalar<Tw>(row, j), xs.at(j), acc[r]);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < RB; ++r) {
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1)
        acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], off));
      if (lane == 0 && e0 + r < E) part[e0 + r] = acc[r];
    }
  }
}

// logit = (((s_0 + s_1) + s_2) + ... + s_7) [+ bias]; parts laid out
// [segment][stride] with the expert index as the fastest dimension.
WR_DEVINL float router_combine(const float* parts, int stride, int e, const float* bias) {
  float l = parts[e];
#pragma unroll
  for (int j = 1; j < kRouterSegments; ++j) l = __fadd_rn(l, parts[j * stride + e]);
  if (bias) l = __fadd_rn(l, bias[e]);
  return l;
}

// Order-preserving key of a logit for the top-K rounds: a larger float gives
// a larger unsigned key; NaN ranks as -inf and -0 as +0 (so the keys compare
// exactly as the floats do under '>').  Key 0 is below every logit.
WR_DEVINL uint32_t logit_key(float v) {
  if (v != v) v = __int_as_float(0xff800000);
  if (v == 0.0f) v = 0.0f;
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Softmax + top-K for one token, run by one full warp.
// logits [E] (E <= 64, any memory) -> ids [K], weights [K] (written by lanes
// 0..K-1).
// Selection: K rounds of "largest key, lowest index on ties" over the unused
// experts, key = logit (NaN counts as -inf) — warp-route's strict-'>'
// argmax (src/fused_moe.cu:134-142) with ties to the lowest index.  A round
// is one warp max-reduction of the keys (lane l holds experts l and l + 32)
// and two ballots for the lowest index holding the maximum.
// Softmax: m = max logit; p_e = exp(l_e - m); the sum is a fixed tree —
// lane l adds p_l + p_{l+32}, then a 16/8/4/2/1 xor tree; weight_k =
// p_{id_k} / sum.
WR_DEVINL void select_topk_warp(const float* logits, int E, int K, int lane, int* ids,
                                float* weights) {
  const float ninf = __int_as_float(0xff800000);
  const int e0 = lane, e1 = lane + 32;
  const float l0 = e0 < E ? logits[e0] : ninf;
  const float l1 = e1 < E ? logits[e1] : ninf;
  float m = fmaxf(l0, l1);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  const float p0 = e0 < E ? expf(l0 - m) : 0.0f;
  const float p1 = e1 < E ? expf(l1 - m) : 0.0f;
  float s = __fadd_rn(p0, p1);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
  uint32_t k0 = e0 < E ? logit_key(l0) : 0u;  // 0: absent or already selected
  uint32_t k1 = e1 < E ? logit_key(l1) : 0u;
  int mine = -1;  // lane k keeps the k-th selected expert
  for (int k = 0; k < K; ++k) {
    const uint32_t best = __reduce_max_sync(0xffffffffu, k0 > k1 ? k0 : k1);
    const unsigned b0 = __ballot_sync(0xffffffffu, k0 == best);
    const unsigned b1 = __ballot_sync(0xffffffffu, k1 == best);
    const int ki = b0 ? __ffs(b0) - 1 : 32 + __ffs(b1) - 1;  // experts l < experts l + 32
    if (ki == e0) k0 = 0u;
    if (ki == e1) k1 = 0u;
    if (lane == k) mine = ki;
  }
  if (lane < K) {
    const float pe = expf(logits[mine] - m);  // the same value as p0 / p1 of its lane
    ids[lane] = mine;
    weights[lane] = __fdiv_rn(pe, s);
  }
}

}  // namespace wr
