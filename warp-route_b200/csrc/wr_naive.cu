// wr_naive.cu — standalone router kernel and the unfused ("naive") layer.
//
// k_router replaces warp-route's warp_gate_topk (src/gate.cu:103-116) and
// k_router_matmul + cpu_softmax_topk (src/naive_moe.cu:49-72,152-175): the
// softmax and top-K run on the device, so the naive path has no device->host
// round trip in the middle of the layer (src/naive_moe.cu:196-199 has one).
// The naive layer keeps warp-route's kernel-per-step structure
// (src/naive_moe.cu:181-241: gate, up, SwiGLU, down, weighted accumulate per
// selected expert) and takes any H and I (no alignment requirements); it is
// also the path the fused entry points use for shapes the streaming kernel
// does not take.
#include <cuda_runtime.h>

#include <mutex>

#include "wr_common.cuh"
#include "wr_internal.h"
#include "wr_router.cuh"

namespace wr {
namespace {

constexpr int kRouterThreads = 32 * kRouterSegments;

// One CTA per token: warp j computes segment j of every router row, reading
// x straight from global memory in 16-byte vectors (no staging: the loads of
// all rows and x are in flight together); softmax + top-K by warp 0.
template <typename Tw>
__global__ void __launch_bounds__(kRouterThreads) k_router(const Tw* __restrict__ x,
                                                           const Tw* __restrict__ gate_w,
                                                           const float* __restrict__ bias, int E,
                                                           int H, int K, bool vec_ok,
                                                           float* __restrict__ logits_out,
                                                           int32_t* __restrict__ ids_out,
                                                           float* __restrict__ w_out) {
  __shared__ float parts[kRouterSegments * kMaxExperts];
  __shared__ float lg[kMaxExperts];
  __shared__ int ids[kMaxExperts];
  __shared__ float ws[kMaxExperts];
  const int t = blockIdx.x;
  const Tw* xt = x + (int64_t)t * H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // blockDim.x == 32 * kRouterSegments: warp j computes segment j of every row.
  router_segment_warp<Tw>(gate_w, XGlobal<Tw>{xt}, E, H, warp, lane, vec_ok,
                          parts + warp * kMaxExperts);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    lg[e] = router_combine(parts, kMaxExperts, e, bias);
  __syncthreads();
  if (warp == 0) {
    select_topk_warp(lg, E, K, lane, ids, ws);
    __syncwarp();
    for (int k = lane; k < K; k += 32) {
      ids_out[(int64_t)t * K + k] = ids[k];
      w_out[(int64_t)t * K + k] = ws[k];
    }
  }
  if (logits_out)
    for (int e = threadIdx.x; e < E; e += blockDim.x) logits_out[(int64_t)t * E + e] = lg[e];
}

// y[row] = W[row, :] . v for the expert in selection slot `sel` (ids[sel]);
// zero when that expert is not in this rank's shard.  One warp per row,
// lanes stride the columns (coalesced), any row length.
template <typename Tw, typename Tv>
__global__ void __launch_bounds__(256) k_matvec_sel(const uint8_t* __restrict__ wbuf,
                                                    int64_t stride, int64_t off,
                                                    const int32_t* __restrict__ ids, int sel,
                                                    int ep_first, int ep_num, int rows, int cols,
                                                    const Tv* __restrict__ v,
                                                    float* __restrict__ y) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int e = ids[sel];
  if (e < ep_first || e >= ep_first + ep_num) {
    if (lane == 0) y[row] = 0.0f;
    return;
  }
  const Tw* W = reinterpret_cast<const Tw*>(wbuf + (int64_t)(e - ep_first) * stride + off) +
                (int64_t)row * cols;
  float acc = 0.0f;
  for (int c = lane; c < cols; c += 32) {
    float vv;
    if constexpr (sizeof(Tv) == 2)
      vv = __uint_as_float(static_cast<uint32_t>(v[c]) << 16);
    else
      vv = v[c];
    acc = fmaf(load_scalar<Tw>(W, c), vv, acc);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) y[row] = acc;
}

__global__ void k_swiglu(const float* __restrict__ g, const float* __restrict__ u,
                         float* __restrict__ act, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) act[i] = silu(g[i]) * u[i];
}

// out = (first ? 0 : out) + weights[sel] * y
__global__ void k_weighted_accum(float* __restrict__ out, const float* __restrict__ y,
                                 const float* __restrict__ weights, int sel, int n, int first) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = (first ? 0.0f : out[i]) + weights[sel] * y[i];
}

template <typename Tw>
wr_status_t router_impl(const Problem& p, const void* x, const void* gate_w, float* logits,
                        int32_t* ids, float* w, cudaStream_t stream) {
  const int vec = 16 / p.elt;
  const bool vec_ok = (p.H % vec == 0) && ((reinterpret_cast<uintptr_t>(gate_w) & 15) == 0) &&
                      ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  k_router<Tw><<<p.T, kRouterThreads, 0, stream>>>(
      static_cast<const Tw*>(x), static_cast<const Tw*>(gate_w), p.router_bias, p.E, p.H, p.K,
      vec_ok, logits, ids, w);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? WR_OK : cuda_fail(e, "k_router launch");
}

struct NaiveScratch {
  float* logits;  // [E]
  int32_t* ids;   // [K]
  float* w;       // [K]
  float* g;       // [I]
  float* u;       // [I]
  float* act;     // [I]
  float* y;       // [H]
};

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// The start of every workspace holds the streaming kernel's control words;
// the naive path leaves them alone so one workspace can serve both paths.
constexpr size_t kWsReserved = kWsControlBytes;

NaiveScratch carve(const Problem& p, void* ws) {
  uint8_t* b = static_cast<uint8_t*>(ws) + kWsReserved;
  NaiveScratch s;
  s.logits = reinterpret_cast<float*>(b); b += align256(4 * (size_t)p.E);
  s.ids = reinterpret_cast<int32_t*>(b); b += align256(4 * (size_t)p.K);
  s.w = reinterpret_cast<float*>(b); b += align256(4 * (size_t)p.K);
  s.g = reinterpret_cast<float*>(b); b += align256(4 * (size_t)p.I);
  s.u = reinterpret_cast<float*>(b); b += align256(4 * (size_t)p.I);
  s.act = reinterpret_cast<float*>(b); b += align256(4 * (size_t)p.I);
  s.y = reinterpret_cast<float*>(b);
  return s;
}

template <typename Tw>
wr_status_t naive_impl(const Problem& p, const void* x, const void* gate_w, const void* wbuf,
                       float* out, int32_t* ids_out, float* w_out, void* ws,
                       cudaStream_t stream) {
  const Layout lay = make_layout(p.H, p.I, p.elt);
  const uint8_t* wb = static_cast<const uint8_t*>(wbuf);
  for (int t = 0; t < p.T; ++t) {
    NaiveScratch s = carve(p, ws);
    Problem one = p;
    one.T = 1;
    const Tw* xt = static_cast<const Tw*>(x) + (int64_t)t * p.H;
    wr_status_t st = router_impl<Tw>(one, xt, gate_w, s.logits, s.ids, s.w, stream);
    if (st != WR_OK) return st;
    float* ot = out + (int64_t)t * p.H;
    const int rpb = 256 / 32;
    for (int k = 0; k < p.K; ++k) {
      k_matvec_sel<Tw, Tw><<<(p.I + rpb - 1) / rpb, 256, 0, stream>>>(
          wb, lay.stride, lay.off_gate, s.ids, k, p.ep_first, p.ep_num, p.I, p.H, xt, s.g);
      k_matvec_sel<Tw, Tw><<<(p.I + rpb - 1) / rpb, 256, 0, stream>>>(
          wb, lay.stride, lay.off_up, s.ids, k, p.ep_first, p.ep_num, p.I, p.H, xt, s.u);
      k_swiglu<<<(p.I + 255) / 256, 256, 0, stream>>>(s.g, s.u, s.act, p.I);
      k_matvec_sel<Tw, float><<<(p.H + rpb - 1) / rpb, 256, 0, stream>>>(
          wb, lay.stride, lay.off_down, s.ids, k, p.ep_first, p.ep_num, p.H, p.I, s.act, s.y);
      k_weighted_accum<<<(p.H + 255) / 256, 256, 0, stream>>>(ot, s.y, s.w, k, p.H, k == 0);
    }
    if (ids_out)
      cudaMemcpyAsync(ids_out + (int64_t)t * p.K, s.ids, 4 * (size_t)p.K,
                      cudaMemcpyDeviceToDevice, stream);
    if (w_out)
      cudaMemcpyAsync(w_out + (int64_t)t * p.K, s.w, 4 * (size_t)p.K, cudaMemcpyDeviceToDevice,
                      stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "naive layer launch");
  }
  return WR_OK;
}

}  // namespace

wr_status_t launch_router(const Problem& p, const void* x, const void* gate_w, float* logits,
                          int32_t* ids, float* w, cudaStream_t stream) {
  if (p.dtype == WR_DTYPE_BF16) return router_impl<uint16_t>(p, x, gate_w, logits, ids, w, stream);
  return router_impl<float>(p, x, gate_w, logits, ids, w, stream);
}

size_t naive_workspace_bytes(const Problem& p) {
  return kWsReserved + align256(4 * (size_t)p.E) + 2 * align256(4 * (size_t)p.K) +
         3 * align256(4 * (size_t)p.I) + align256(4 * (size_t)p.H);
}

wr_status_t launch_naive(const Problem& p, const void* x, const void* gate_w, const void* wbuf,
                         float* out, int32_t* ids, float* w, void* ws, cudaStream_t stream) {
  if (p.dtype == WR_DTYPE_BF16)
    return naive_impl<uint16_t>(p, x, gate_w, wbuf, out, ids, w, ws, stream);
  return naive_impl<float>(p, x, gate_w, wbuf, out, ids, w, ws, stream);
}

}  // namespace wr
