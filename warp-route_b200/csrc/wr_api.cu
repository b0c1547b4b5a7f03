// wr_api.cu — the extern "C" entry points of include/warp_route_b200.h:
// argument checks (status codes instead of warp-route's exit(1),
// src/fused_moe.cu:239-247), dispatch to the streaming kernel or the naive
// path, and the layout helpers.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "wr_common.cuh"
#include "wr_internal.h"
#include "wr_router.cuh"

namespace wr {

namespace {
thread_local char g_last_error[512] = "";
}

wr_status_t fail(wr_status_t s, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return s;
}

wr_status_t cuda_fail(cudaError_t e, const char* what) {
  return fail(WR_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int device_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int& c = cache[dev & 63];
  if (c == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    c = n > 0 ? n : 1;
  }
  return c;
}

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Checks the descriptor and fills `p`.  Messages follow warp-route's
// TORCH_CHECK texts (src/bindings.cpp:13-23,40-43,75-77) where one exists.
wr_status_t make_problem(const wr_moe_desc_t* d, int tokens, Problem* p) {
  if (!d) return fail(WR_ERR_INVALID, "desc must not be NULL");
  if (d->dtype != WR_DTYPE_F32 && d->dtype != WR_DTYPE_BF16)
    return fail(WR_ERR_INVALID, "dtype must be float32 or bfloat16, got code %d", d->dtype);
  if (d->num_experts < 1 || d->hidden_dim < 1 || d->intermediate_dim < 1)
    return fail(WR_ERR_INVALID, "num_experts, hidden_dim and intermediate_dim must be positive, got %d, %d, %d",
                d->num_experts, d->hidden_dim, d->intermediate_dim);
  if (d->num_experts > kMaxExperts)
    return fail(WR_ERR_UNSUPPORTED, "num_experts %d exceeds GATE_MAX_EXPERTS %d", d->num_experts,
                kMaxExperts);
  if (d->top_k < 1 || d->top_k > d->num_experts)
    return fail(WR_ERR_INVALID, "top_k must be in [1, num_experts=%d], got %d", d->num_experts,
                d->top_k);
  if (tokens < 0) return fail(WR_ERR_INVALID, "num_tokens must be >= 0, got %d", tokens);
  p->E = d->num_experts;
  p->H = d->hidden_dim;
  p->I = d->intermediate_dim;
  p->K = d->top_k;
  p->T = tokens;
  p->dtype = d->dtype;
  p->elt = d->dtype == WR_DTYPE_BF16 ? 2 : 4;
  p->router_bias = d->router_bias;
  p->res = Residual{nullptr, nullptr, d->dtype == WR_DTYPE_BF16 ? 1 : 0};
  if (d->ep_num_local == 0) {
    p->ep_first = 0;
    p->ep_num = p->E;
  } else {
    if (d->ep_first_expert < 0 || d->ep_num_local < 0 ||
        d->ep_first_expert + d->ep_num_local > p->E)
      return fail(WR_ERR_INVALID, "expert shard [%d, %d) is outside [0, %d)", d->ep_first_expert,
                  d->ep_first_expert + d->ep_num_local, p->E);
    p->ep_first = d->ep_first_expert;
    p->ep_num = d->ep_num_local;
  }
  return WR_OK;
}

wr_status_t check_weights(const Problem& p, const void* wbuf, int64_t bytes) {
  const Layout l = make_layout(p.H, p.I, p.elt);
  const int64_t need = (int64_t)p.ep_num * l.stride;
  if (!wbuf) return fail(WR_ERR_INVALID, "weight_buf must not be NULL");
  if (bytes < need)
    return fail(WR_ERR_TOO_SMALL, "weight_buf too small: need %lld bytes, got %lld",
                (long long)need, (long long)bytes);
  return WR_OK;
}

wr_status_t check_ws(void* ws, size_t have, size_t need) {
  if (need == 0) return WR_OK;
  if (!ws) return fail(WR_ERR_WORKSPACE, "workspace must not be NULL (%zu bytes needed)", need);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0)
    return fail(WR_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  if (have < need)
    return fail(WR_ERR_WORKSPACE, "workspace too small: need %zu bytes, got %zu", need, have);
  return WR_OK;
}

size_t fused_ws_for(const Problem& p) {
  // Batches of kGroupedMinTokens or more bf16 tokens (kGroupedMinTokensF32
  // fp32 tokens) run as grouped GEMMs; otherwise the batched entry point runs
  // blocks of up to 4 tokens through the streaming kernel, and unsupported
  // shapes go through the naive path.
  Problem q = p;
  q.T = p.T < 1 ? 1 : (p.T > 4 ? 4 : p.T);
  size_t need = naive_workspace_bytes(p);
  if (fused_supported(q)) {
    const size_t fused = fused_workspace_bytes(q);
    need = fused > need ? fused : need;
  }
  if (grouped_supported(p)) {
    const size_t g = grouped_workspace_bytes(p);
    need = g > need ? g : need;
  }
  return need;
}

// Blocks of up to 4 tokens through the streaming kernel (or the naive path
// for shapes it does not take).  comm: all-reduce the ranks' partial outputs
// inside each launch; the naive path has no all-reduce, so with a
// communicator the shape must suit the streaming kernel.
wr_status_t run_layer(const Problem& p, const void* x, const void* gate_w, const void* wbuf,
                      float* out, int32_t* ids, float* w, void* ws, cudaStream_t stream,
                      const CommView* comm = nullptr) {
  if (p.T == 0) return WR_OK;
  const bool ptr_ok = aligned16(x) && aligned16(gate_w) && aligned16(wbuf);
  if (ptr_ok && grouped_supported(p))
    return launch_grouped(p, x, gate_w, wbuf, out, ids, w, ws, stream, comm);
  for (int t0 = 0; t0 < p.T; t0 += 4) {
    Problem q = p;
    q.T = p.T - t0 < 4 ? p.T - t0 : 4;
    const size_t xoff = (size_t)t0 * p.H * p.elt;
    const void* xq = static_cast<const uint8_t*>(x) + xoff;
    float* oq = out + (size_t)t0 * p.H;
    int32_t* iq = ids ? ids + (size_t)t0 * p.K : nullptr;
    float* wq = w ? w + (size_t)t0 * p.K : nullptr;
    if (p.res.x) {  // this block's rows of x and next_x
      q.res.x = xq;
      q.res.next_x = p.res.next_x ? static_cast<uint8_t*>(p.res.next_x) + xoff : nullptr;
    }
    wr_status_t st;
    if (ptr_ok && aligned16(xq) && fused_supported(q))
      st = launch_fused(q, xq, gate_w, wbuf, oq, iq, wq, ws, stream, comm);
    else if (comm)
      st = fail(WR_ERR_UNSUPPORTED,
                "the all-reduce layer needs the streaming kernel: 16-byte aligned x, gate_w and "
                "weight_buf, and H, I multiples of 16 bytes of elements");
    else if (p.res.x)
      st = fail(WR_ERR_UNSUPPORTED,
                "the fused residual needs the streaming or grouped kernels: 16-byte aligned x, "
                "gate_w and weight_buf, and H, I multiples of 16 bytes of elements");
    else
      st = launch_naive(q, xq, gate_w, wbuf, oq, iq, wq, ws, stream);
    if (st != WR_OK) return st;
  }
  return WR_OK;
}

}  // namespace
}  // namespace wr

using namespace wr;

extern "C" {

const char* wr_version(void) { return "warp-route-b200 0.1.0 (sm_100a)"; }

const char* wr_status_string(wr_status_t s) {
  switch (s) {
    case WR_OK: return "ok";
    case WR_ERR_INVALID: return "invalid argument";
    case WR_ERR_UNSUPPORTED: return "unsupported configuration";
    case WR_ERR_CUDA: return "CUDA error";
    case WR_ERR_TIMEOUT: return "device wait timed out";
    case WR_ERR_WORKSPACE: return "bad workspace";
    case WR_ERR_TOO_SMALL: return "weight buffer too small";
    case WR_ERR_COMM: return "communicator error";
  }
  return "unknown status";
}

const char* wr_last_error_string(void) { return g_last_error; }

wr_status_t wr_expert_offsets(int32_t hidden_dim, int32_t intermediate_dim, int32_t elt_bytes,
                              wr_expert_offsets_t* out) {
  if (!out) return fail(WR_ERR_INVALID, "out must not be NULL");
  if (hidden_dim < 1 || intermediate_dim < 1 || (elt_bytes != 2 && elt_bytes != 4))
    return fail(WR_ERR_INVALID, "bad layout arguments (%d, %d, %d)", hidden_dim, intermediate_dim,
                elt_bytes);
  const Layout l = make_layout(hidden_dim, intermediate_dim, elt_bytes);
  out->gate_proj_offset = l.off_gate;
  out->up_proj_offset = l.off_up;
  out->down_proj_offset = l.off_down;
  out->expert_stride = l.stride;
  return WR_OK;
}

int64_t wr_total_weight_bytes(int32_t num_experts, int32_t hidden_dim, int32_t intermediate_dim,
                              int32_t elt_bytes) {
  if (num_experts < 0 || hidden_dim < 1 || intermediate_dim < 1) return -1;
  return (int64_t)num_experts * make_layout(hidden_dim, intermediate_dim, elt_bytes).stride;
}

wr_status_t wr_router_topk(const wr_moe_desc_t* desc, int32_t num_tokens, const void* x,
                           const void* gate_w, float* logits_out, int32_t* topk_ids,
                           float* topk_weights, wr_stream_t stream) {
  Problem p;
  wr_status_t st = make_problem(desc, num_tokens, &p);
  if (st != WR_OK) return st;
  if (!x || !gate_w || !topk_ids || !topk_weights)
    return fail(WR_ERR_INVALID, "x, gate_w, topk_ids and topk_weights must not be NULL");
  if (num_tokens == 0) return WR_OK;
  return launch_router(p, x, gate_w, logits_out, topk_ids, topk_weights,
                       static_cast<cudaStream_t>(stream));
}

size_t wr_fused_moe_workspace_size(const wr_moe_desc_t* desc, int32_t num_tokens) {
  Problem p;
  if (make_problem(desc, num_tokens < 1 ? 1 : num_tokens, &p) != WR_OK) return 0;
  return fused_ws_for(p);
}

wr_status_t wr_fused_moe(const wr_moe_desc_t* desc, const void* x, const void* gate_w,
                         const void* weight_buf, int64_t weight_buf_bytes, float* out,
                         int32_t* topk_ids, float* topk_weights, void* workspace,
                         size_t workspace_bytes, wr_stream_t stream) {
  Problem p;
  wr_status_t st = make_problem(desc, 1, &p);
  if (st != WR_OK) return st;
  if (!x || !gate_w || !out) return fail(WR_ERR_INVALID, "x, gate_w and out must not be NULL");
  if ((st = check_weights(p, weight_buf, weight_buf_bytes)) != WR_OK) return st;
  if ((st = check_ws(workspace, workspace_bytes, fused_ws_for(p))) != WR_OK) return st;
  return run_layer(p, x, gate_w, weight_buf, out, topk_ids, topk_weights, workspace,
                   static_cast<cudaStream_t>(stream));
}

wr_status_t wr_batched_fused_moe(const wr_moe_desc_t* desc, int32_t num_tokens, const void* x,
                                 const void* gate_w, const void* weight_buf,
                                 int64_t weight_buf_bytes, float* out, int32_t* topk_ids,
                                 float* topk_weights, void* workspace, size_t workspace_bytes,
                                 wr_stream_t stream) {
  Problem p;
  wr_status_t st = make_problem(desc, num_tokens, &p);
  if (st != WR_OK) return st;
  if (num_tokens == 0) return WR_OK;
  if (!x || !gate_w || !out) return fail(WR_ERR_INVALID, "x, gate_w and out must not be NULL");
  if ((st = check_weights(p, weight_buf, weight_buf_bytes)) != WR_OK) return st;
  if ((st = check_ws(workspace, workspace_bytes, fused_ws_for(p))) != WR_OK) return st;
  return run_layer(p, x, gate_w, weight_buf, out, topk_ids, topk_weights, workspace,
                   static_cast<cudaStream_t>(stream));
}

wr_status_t wr_fused_moe_allreduce(const wr_moe_desc_t* desc, int32_t num_tokens, const void* x,
                                   const void* gate_w, const void* weight_buf,
                                   int64_t weight_buf_bytes, float* out, int32_t* topk_ids,
                                   float* topk_weights, void* workspace, size_t workspace_bytes,
                                   wr_comm_t comm, wr_stream_t stream) {
  Problem p;
  wr_status_t st = make_problem(desc, num_tokens, &p);
  if (st != WR_OK) return st;
  if (!comm) return fail(WR_ERR_INVALID, "comm must not be NULL");
  CommView v;
  if ((st = comm_view(comm, &v)) != WR_OK) return st;
  if (v.H != p.H)
    return fail(WR_ERR_INVALID, "hidden_dim %d differs from the communicator's %d", p.H, v.H);
  if (num_tokens == 0) return WR_OK;
  if (!x || !gate_w || !out) return fail(WR_ERR_INVALID, "x, gate_w and out must not be NULL");
  if ((st = check_weights(p, weight_buf, weight_buf_bytes)) != WR_OK) return st;
  if ((st = check_ws(workspace, workspace_bytes, fused_ws_for(p))) != WR_OK) return st;
  return run_layer(p, x, gate_w, weight_buf, out, topk_ids, topk_weights, workspace,
                   static_cast<cudaStream_t>(stream), &v);
}

wr_status_t wr_moe_decode_layer(const wr_moe_desc_t* desc, int32_t num_tokens, const void* x,
                                const void* gate_w, const void* weight_buf,
                                int64_t weight_buf_bytes, float* out, void* next_x,
                                int32_t* topk_ids, float* topk_weights, void* workspace,
                                size_t workspace_bytes, wr_comm_t comm, wr_stream_t stream) {
  Problem p;
  wr_status_t st = make_problem(desc, num_tokens, &p);
  if (st != WR_OK) return st;
  if (num_tokens == 0) return WR_OK;
  if (!x || !gate_w || !out) return fail(WR_ERR_INVALID, "x, gate_w and out must not be NULL");
  if (next_x == x) return fail(WR_ERR_INVALID, "next_x must not alias x");
  if ((st = check_weights(p, weight_buf, weight_buf_bytes)) != WR_OK) return st;
  if ((st = check_ws(workspace, workspace_bytes, fused_ws_for(p))) != WR_OK) return st;
  CommView v;
  if (comm) {
    if ((st = comm_view(comm, &v)) != WR_OK) return st;
    if (v.H != p.H)
      return fail(WR_ERR_INVALID, "hidden_dim %d differs from the communicator's %d", p.H, v.H);
  }
  p.res.x = x;
  p.res.next_x = next_x;
  return run_layer(p, x, gate_w, weight_buf, out, topk_ids, topk_weights, workspace,
                   static_cast<cudaStream_t>(stream), comm ? &v : nullptr);
}

size_t wr_naive_moe_workspace_size(const wr_moe_desc_t* desc) {
  Problem p;
  if (make_problem(desc, 1, &p) != WR_OK) return 0;
  return naive_workspace_bytes(p);
}

wr_status_t wr_naive_moe(const wr_moe_desc_t* desc, const void* x, const void* gate_w,
                         const void* weight_buf, int64_t weight_buf_bytes, float* out,
                         void* workspace, size_t workspace_bytes, wr_stream_t stream) {
  Problem p;
  wr_status_t st = make_problem(desc, 1, &p);
  if (st != WR_OK) return st;
  if (!x || !gate_w || !out) return fail(WR_ERR_INVALID, "x, gate_w and out must not be NULL");
  if ((st = check_weights(p, weight_buf, weight_buf_bytes)) != WR_OK) return st;
  if ((st = check_ws(workspace, workspace_bytes, naive_workspace_bytes(p))) != WR_OK) return st;
  return launch_naive(p, x, gate_w, weight_buf, out, nullptr, nullptr, workspace,
                      static_cast<cudaStream_t>(stream));
}

wr_status_t wr_workspace_status(void* workspace, wr_stream_t stream) {
  if (!workspace) return fail(WR_ERR_INVALID, "workspace must not be NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, static_cast<uint32_t*>(workspace) + 2, 4,
                                  cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "wr_workspace_status");
  if (host != 0) {
    e = cudaMemsetAsync(static_cast<uint32_t*>(workspace) + 2, 0, 4, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "wr_workspace_status (clear)");
    return fail(WR_ERR_TIMEOUT, "a bounded device wait gave up (status bits 0x%x)", host);
  }
  return WR_OK;
}

}  // extern "C"
