// wr_bindings.cpp — the `warp_route._C` torch extension.
//
// Keeps warp-route's binding surface (src/bindings.cpp:145-152):
//   naive_moe_forward, fused_moe_forward, batched_fused_moe_forward, each
//   (Tensor hidden, Tensor gate_w, Tensor weight_buf, int E, int H, int I,
//    int top_k) -> Tensor,
// with the same argument checks and messages (src/bindings.cpp:9-23,40-43,
// 75-83), raised as RuntimeError.  Differences: float32 or bfloat16 inputs
// (one dtype for all three tensors; the output is always float32), top_k up
// to num_experts, work on the current torch stream, and no device-wide
// synchronisation after the launch.  Everything below the tensor checks is a
// call into the C ABI (include/warp_route_b200.h); torch is only the binding.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "warp_route_b200.h"

namespace {

#define CHECK_CONTIGUOUS(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")
#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_DTYPE(t)                                                                     \
  TORCH_CHECK((t).scalar_type() == torch::kFloat32 || (t).scalar_type() == torch::kBFloat16, \
              #t " must be float32 or bfloat16")

// warp-route's validate_1d/2d (src/bindings.cpp:13-23) stringify their own
// parameter ("t must be ..."); these name the argument instead.
void check_tensor(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(t.scalar_type() == torch::kFloat32 || t.scalar_type() == torch::kBFloat16, name,
              " must be float32 or bfloat16");
}

void validate_1d(const torch::Tensor& t, const char* name, int64_t expected) {
  check_tensor(t, name);
  TORCH_CHECK(t.dim() == 1 && t.size(0) == expected, name, " must have shape [", expected,
              "], got shape ", t.sizes());
}

void validate_2d(const torch::Tensor& t, const char* name, int64_t rows, int64_t cols) {
  check_tensor(t, name);
  TORCH_CHECK(t.dim() == 2 && t.size(0) == rows && t.size(1) == cols, name,
              " must have shape [", rows, ", ", cols, "], got shape ", t.sizes());
}

int32_t dtype_code(const torch::Tensor& t) {
  return t.scalar_type() == torch::kBFloat16 ? WR_DTYPE_BF16 : WR_DTYPE_F32;
}

void check_same(const torch::Tensor& a, const torch::Tensor& b, const char* an, const char* bn) {
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), an, " and ", bn,
              " must have the same dtype, got ", a.scalar_type(), " and ", b.scalar_type());
  TORCH_CHECK(a.device() == b.device(), an, " and ", bn, " must be on the same device");
}

void check_status(wr_status_t st) {
  TORCH_CHECK(st == WR_OK, wr_last_error_string());
}

// One zero-initialised workspace per (device, stream), grown on demand.  Calls
// on one stream are ordered, so sharing is safe; distinct streams get distinct
// workspaces.  The map is never destroyed (process exit frees device memory).
struct WsCache {
  std::mutex mu;
  std::map<std::pair<int, cudaStream_t>, torch::Tensor> bufs;
};
WsCache& ws_cache() {
  static WsCache* c = new WsCache();
  return *c;
}

torch::Tensor workspace_for(const torch::Device& dev, cudaStream_t stream, size_t bytes) {
  auto& c = ws_cache();
  std::lock_guard<std::mutex> lk(c.mu);
  auto key = std::make_pair((int)dev.index(), stream);
  auto it = c.bufs.find(key);
  if (it != c.bufs.end() && (size_t)it->second.numel() >= bytes) return it->second;
  size_t grow = bytes < (1u << 20) ? (1u << 20) : bytes;
  torch::Tensor t = torch::zeros({(int64_t)grow}, torch::TensorOptions().dtype(torch::kUInt8).device(dev));
  c.bufs[key] = t;
  return t;
}

wr_moe_desc_t make_desc(const torch::Tensor& hidden, int E, int H, int I, int top_k,
                        const c10::optional<torch::Tensor>& bias, int ep_first, int ep_num) {
  wr_moe_desc_t d{};
  d.num_experts = E;
  d.hidden_dim = H;
  d.intermediate_dim = I;
  d.top_k = top_k;
  d.dtype = dtype_code(hidden);
  d.ep_first_expert = ep_first;
  d.ep_num_local = ep_num;
  d.router_bias = nullptr;
  if (bias.has_value() && bias->defined()) {
    const auto& b = *bias;
    CHECK_CUDA(b);
    CHECK_CONTIGUOUS(b);
    TORCH_CHECK(b.scalar_type() == torch::kFloat32, "router_bias must be float32");
    TORCH_CHECK(b.dim() == 1 && b.size(0) == E, "router_bias must have shape [", E, "], got shape ",
                b.sizes());
    d.router_bias = b.data_ptr<float>();
  }
  return d;
}

void check_weight_buf(const torch::Tensor& hidden, const torch::Tensor& weight_buf) {
  CHECK_CUDA(weight_buf);
  CHECK_CONTIGUOUS(weight_buf);
  CHECK_DTYPE(weight_buf);
  check_same(hidden, weight_buf, "hidden", "weight_buf");
}

// Shared body of the fused entry points.  hidden: [H] or [T,H].
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> fused_impl(
    const torch::Tensor& hidden, const torch::Tensor& gate_w, const torch::Tensor& weight_buf,
    int E, int H, int I, int top_k, const c10::optional<torch::Tensor>& bias, int ep_first,
    int ep_num, bool want_routing, wr_comm_t comm = nullptr) {
  const bool one = hidden.dim() == 1;
  const int64_t T = one ? 1 : hidden.size(0);
  validate_2d(gate_w, "gate_w", E, H);
  check_same(hidden, gate_w, "hidden", "gate_w");
  check_weight_buf(hidden, weight_buf);
  const c10::cuda::CUDAGuard guard(hidden.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(hidden.device().index()).stream();
  wr_moe_desc_t d = make_desc(hidden, E, H, I, top_k, bias, ep_first, ep_num);
  auto fopt = torch::TensorOptions().dtype(torch::kFloat32).device(hidden.device());
  torch::Tensor out = one ? torch::empty({H}, fopt) : torch::empty({T, H}, fopt);
  torch::Tensor ids, w;
  if (want_routing) {
    ids = torch::empty({T, top_k}, fopt.dtype(torch::kInt32));
    w = torch::empty({T, top_k}, fopt);
  }
  if (T == 0) return {out, ids, w};
  const size_t need = wr_fused_moe_workspace_size(&d, (int32_t)T);
  TORCH_CHECK(need > 0, wr_last_error_string());
  torch::Tensor ws = workspace_for(hidden.device(), stream, need);
  const int64_t wbytes = weight_buf.numel() * (int64_t)weight_buf.element_size();
  wr_status_t st;
  if (comm)
    st = wr_fused_moe_allreduce(&d, (int32_t)T, hidden.data_ptr(), gate_w.data_ptr(),
                                weight_buf.data_ptr(), wbytes, out.data_ptr<float>(),
                                want_routing ? ids.data_ptr<int32_t>() : nullptr,
                                want_routing ? w.data_ptr<float>() : nullptr, ws.data_ptr(),
                                (size_t)ws.numel(), comm, stream);
  else if (one)
    st = wr_fused_moe(&d, hidden.data_ptr(), gate_w.data_ptr(), weight_buf.data_ptr(), wbytes,
                      out.data_ptr<float>(), want_routing ? ids.data_ptr<int32_t>() : nullptr,
                      want_routing ? w.data_ptr<float>() : nullptr, ws.data_ptr(),
                      (size_t)ws.numel(), stream);
  else
    st = wr_batched_fused_moe(&d, (int32_t)T, hidden.data_ptr(), gate_w.data_ptr(),
                              weight_buf.data_ptr(), wbytes, out.data_ptr<float>(),
                              want_routing ? ids.data_ptr<int32_t>() : nullptr,
                              want_routing ? w.data_ptr<float>() : nullptr, ws.data_ptr(),
                              (size_t)ws.numel(), stream);
  check_status(st);
  return {out, ids, w};
}

// ---- warp-route's three entry points ---------------------------------------

torch::Tensor naive_moe_forward_torch(torch::Tensor hidden, torch::Tensor gate_w,
                                      torch::Tensor weight_buf, int num_experts, int hidden_dim,
                                      int intermediate_dim, int top_k) {
  validate_1d(hidden, "hidden", hidden_dim);
  validate_2d(gate_w, "gate_w", num_experts, hidden_dim);
  check_same(hidden, gate_w, "hidden", "gate_w");
  check_weight_buf(hidden, weight_buf);
  const c10::cuda::CUDAGuard guard(hidden.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(hidden.device().index()).stream();
  wr_moe_desc_t d = make_desc(hidden, num_experts, hidden_dim, intermediate_dim, top_k,
                              c10::nullopt, 0, 0);
  const size_t need = wr_naive_moe_workspace_size(&d);
  TORCH_CHECK(need > 0, wr_last_error_string());
  torch::Tensor ws = workspace_for(hidden.device(), stream, need);
  torch::Tensor out =
      torch::empty({hidden_dim}, torch::TensorOptions().dtype(torch::kFloat32).device(hidden.device()));
  check_status(wr_naive_moe(&d, hidden.data_ptr(), gate_w.data_ptr(), weight_buf.data_ptr(),
                            weight_buf.numel() * (int64_t)weight_buf.element_size(),
                            out.data_ptr<float>(), ws.data_ptr(), (size_t)ws.numel(), stream));
  return out;
}

torch::Tensor fused_moe_forward_torch(torch::Tensor hidden, torch::Tensor gate_w,
                                      torch::Tensor weight_buf, int num_experts, int hidden_dim,
                                      int intermediate_dim, int top_k) {
  validate_1d(hidden, "hidden", hidden_dim);
  return std::get<0>(fused_impl(hidden, gate_w, weight_buf, num_experts, hidden_dim,
                                intermediate_dim, top_k, c10::nullopt, 0, 0, false));
}

torch::Tensor batched_fused_moe_forward_torch(torch::Tensor hidden_batch, torch::Tensor gate_w,
                                              torch::Tensor weight_buf, int num_experts,
                                              int hidden_dim, int intermediate_dim, int top_k) {
  CHECK_CUDA(hidden_batch);
  CHECK_CONTIGUOUS(hidden_batch);
  CHECK_DTYPE(hidden_batch);
  TORCH_CHECK(hidden_batch.dim() == 2 && hidden_batch.size(1) == hidden_dim,
              "hidden_batch must have shape [batch_size, ", hidden_dim, "], got shape ",
              hidden_batch.sizes());
  return std::get<0>(fused_impl(hidden_batch, gate_w, weight_buf, num_experts, hidden_dim,
                                intermediate_dim, top_k, c10::nullopt, 0, 0, false));
}

// ---- additions (keyword-only extras in warp_route.functional) -------------

// Layer with optional router bias / expert-parallel shard, returning the
// routing as well: (out fp32 [..,H], ids int32 [T,K], weights fp32 [T,K]).
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> fused_moe_routed(
    torch::Tensor hidden, torch::Tensor gate_w, torch::Tensor weight_buf, int num_experts,
    int hidden_dim, int intermediate_dim, int top_k, c10::optional<torch::Tensor> router_bias,
    int ep_first_expert, int ep_num_local) {
  CHECK_CUDA(hidden);
  CHECK_CONTIGUOUS(hidden);
  CHECK_DTYPE(hidden);
  TORCH_CHECK((hidden.dim() == 1 && hidden.size(0) == hidden_dim) ||
                  (hidden.dim() == 2 && hidden.size(1) == hidden_dim),
              "hidden must have shape [", hidden_dim, "] or [batch_size, ", hidden_dim,
              "], got shape ", hidden.sizes());
  return fused_impl(hidden, gate_w, weight_buf, num_experts, hidden_dim, intermediate_dim, top_k,
                    router_bias, ep_first_expert, ep_num_local, true);
}

// Router only: (logits fp32 [T,E], ids int32 [T,K], weights fp32 [T,K]).
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> router_topk(
    torch::Tensor hidden, torch::Tensor gate_w, int num_experts, int hidden_dim, int top_k,
    c10::optional<torch::Tensor> router_bias) {
  CHECK_CUDA(hidden);
  CHECK_CONTIGUOUS(hidden);
  CHECK_DTYPE(hidden);
  const int64_t T = hidden.dim() == 1 ? 1 : hidden.size(0);
  TORCH_CHECK(hidden.size(-1) == hidden_dim, "hidden last dimension must be ", hidden_dim);
  validate_2d(gate_w, "gate_w", num_experts, hidden_dim);
  check_same(hidden, gate_w, "hidden", "gate_w");
  const c10::cuda::CUDAGuard guard(hidden.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(hidden.device().index()).stream();
  wr_moe_desc_t d = make_desc(hidden, num_experts, hidden_dim, 1, top_k, router_bias, 0, 0);
  auto fopt = torch::TensorOptions().dtype(torch::kFloat32).device(hidden.device());
  torch::Tensor logits = torch::empty({T, num_experts}, fopt);
  torch::Tensor ids = torch::empty({T, top_k}, fopt.dtype(torch::kInt32));
  torch::Tensor w = torch::empty({T, top_k}, fopt);
  check_status(wr_router_topk(&d, (int32_t)T, hidden.data_ptr(), gate_w.data_ptr(),
                              logits.data_ptr<float>(), ids.data_ptr<int32_t>(),
                              w.data_ptr<float>(), stream));
  return {logits, ids, w};
}

// ---- communicator for the all-reduce fused into the layer ---------------
// The handle is the C pointer as an integer; the Python wrapper owns it.

int64_t comm_create(int rank, int world_size, int hidden_dim) {
  wr_comm_t c = nullptr;
  check_status(wr_comm_create(rank, world_size, hidden_dim, &c));
  return reinterpret_cast<int64_t>(c);
}

torch::Tensor comm_handle(int64_t comm) {
  torch::Tensor h = torch::empty({(int64_t)wr_comm_handle_bytes()}, torch::kUInt8);
  check_status(wr_comm_get_handle(reinterpret_cast<wr_comm_t>(comm), h.data_ptr()));
  return h;
}

void comm_open(int64_t comm, torch::Tensor handles) {
  TORCH_CHECK(handles.device().is_cpu() && handles.scalar_type() == torch::kUInt8 &&
                  handles.is_contiguous(),
              "handles must be a contiguous uint8 CPU tensor");
  check_status(wr_comm_open(reinterpret_cast<wr_comm_t>(comm), handles.data_ptr()));
}

void comm_destroy(int64_t comm) { check_status(wr_comm_destroy(reinterpret_cast<wr_comm_t>(comm))); }

void comm_set_peer_timeout_ns(int64_t comm, int64_t ns) {
  TORCH_CHECK(ns >= 0, "peer timeout must be >= 0 ns");
  check_status(wr_comm_set_peer_timeout_ns(reinterpret_cast<wr_comm_t>(comm), (uint64_t)ns));
}

void comm_reset(int64_t comm) {
  cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
  check_status(wr_comm_reset(reinterpret_cast<wr_comm_t>(comm), stream));
}

// This rank's shard of the layer with the ranks' outputs summed in-kernel:
// (out fp32 [..,H], ids int32 [T,K], weights fp32 [T,K]).
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> fused_moe_allreduce(
    torch::Tensor hidden, torch::Tensor gate_w, torch::Tensor weight_buf, int num_experts,
    int hidden_dim, int intermediate_dim, int top_k, int64_t comm,
    c10::optional<torch::Tensor> router_bias, int ep_first_expert, int ep_num_local) {
  CHECK_CUDA(hidden);
  CHECK_CONTIGUOUS(hidden);
  CHECK_DTYPE(hidden);
  TORCH_CHECK(comm != 0, "comm must not be NULL");
  TORCH_CHECK((hidden.dim() == 1 && hidden.size(0) == hidden_dim) ||
                  (hidden.dim() == 2 && hidden.size(1) == hidden_dim),
              "hidden must have shape [", hidden_dim, "] or [batch_size, ", hidden_dim,
              "], got shape ", hidden.sizes());
  return fused_impl(hidden, gate_w, weight_buf, num_experts, hidden_dim, intermediate_dim, top_k,
                    router_bias, ep_first_expert, ep_num_local, true,
                    reinterpret_cast<wr_comm_t>(comm));
}

// One layer of a decode stack with the residual fused (wr_moe_decode_layer):
// returns out = hidden + layer(hidden) (fp32, summed over the ranks when comm
// is given) and writes next_x = out in hidden's dtype when next_x is given.
torch::Tensor moe_decode_layer(torch::Tensor hidden, torch::Tensor gate_w,
                               torch::Tensor weight_buf, int num_experts, int hidden_dim,
                               int intermediate_dim, int top_k, int64_t comm,
                               c10::optional<torch::Tensor> router_bias, int ep_first_expert,
                               int ep_num_local, c10::optional<torch::Tensor> next_x) {
  CHECK_CUDA(hidden);
  CHECK_CONTIGUOUS(hidden);
  CHECK_DTYPE(hidden);
  TORCH_CHECK((hidden.dim() == 1 && hidden.size(0) == hidden_dim) ||
                  (hidden.dim() == 2 && hidden.size(1) == hidden_dim),
              "hidden must have shape [", hidden_dim, "] or [batch_size, ", hidden_dim,
              "], got shape ", hidden.sizes());
  validate_2d(gate_w, "gate_w", num_experts, hidden_dim);
  check_same(hidden, gate_w, "hidden", "gate_w");
  check_weight_buf(hidden, weight_buf);
  void* nx = nullptr;
  if (next_x.has_value() && next_x->defined()) {
    const auto& n = *next_x;
    CHECK_CUDA(n);
    CHECK_CONTIGUOUS(n);
    check_same(hidden, n, "hidden", "next_x");
    TORCH_CHECK(n.sizes() == hidden.sizes(), "next_x must have hidden's shape ", hidden.sizes(),
                ", got ", n.sizes());
    nx = n.data_ptr();
  }
  const c10::cuda::CUDAGuard guard(hidden.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(hidden.device().index()).stream();
  wr_moe_desc_t d = make_desc(hidden, num_experts, hidden_dim, intermediate_dim, top_k,
                              router_bias, ep_first_expert, ep_num_local);
  const int64_t T = hidden.dim() == 1 ? 1 : hidden.size(0);
  auto fopt = torch::TensorOptions().dtype(torch::kFloat32).device(hidden.device());
  torch::Tensor out = torch::empty(hidden.sizes(), fopt);
  if (T == 0) return out;
  const size_t need = wr_fused_moe_workspace_size(&d, (int32_t)T);
  TORCH_CHECK(need > 0, wr_last_error_string());
  torch::Tensor ws = workspace_for(hidden.device(), stream, need);
  check_status(wr_moe_decode_layer(&d, (int32_t)T, hidden.data_ptr(), gate_w.data_ptr(),
                                   weight_buf.data_ptr(),
                                   weight_buf.numel() * (int64_t)weight_buf.element_size(),
                                   out.data_ptr<float>(), nx, nullptr, nullptr, ws.data_ptr(),
                                   (size_t)ws.numel(), reinterpret_cast<wr_comm_t>(comm), stream));
  return out;
}

// One rank's shard of per-expert weight lists packed on the device
// (wr_pack_experts): experts [ep_first, ep_first + ep_num), intermediate
// slice tp_rank of tp_size.  Entries outside the shard are not read.
torch::Tensor pack_experts(const std::vector<torch::Tensor>& gate,
                           const std::vector<torch::Tensor>& up,
                           const std::vector<torch::Tensor>& down, int num_experts,
                           int hidden_dim, int intermediate_dim, int ep_first, int ep_num,
                           int tp_rank, int tp_size) {
  TORCH_CHECK((int)gate.size() == num_experts && (int)up.size() == num_experts &&
                  (int)down.size() == num_experts,
              "gate_proj, up_proj and down_proj must each hold num_experts=", num_experts,
              " tensors");
  TORCH_CHECK(ep_num >= 1 && ep_first >= 0 && ep_first + ep_num <= num_experts,
              "expert shard [", ep_first, ", ", ep_first + ep_num, ") is outside [0, ",
              num_experts, ")");
  const torch::Tensor& ref = gate[ep_first];
  CHECK_CUDA(ref);
  CHECK_DTYPE(ref);
  std::vector<const void*> g(num_experts, nullptr), u(num_experts, nullptr),
      d(num_experts, nullptr);
  for (int e = ep_first; e < ep_first + ep_num; ++e) {
    const torch::Tensor* mats[3] = {&gate[e], &up[e], &down[e]};
    const char* names[3] = {"gate_proj", "up_proj", "down_proj"};
    for (int m = 0; m < 3; ++m) {
      const torch::Tensor& t = *mats[m];
      CHECK_CUDA(t);
      CHECK_CONTIGUOUS(t);
      check_same(ref, t, "gate_proj", names[m]);
      const int64_t rows = m == 2 ? hidden_dim : intermediate_dim;
      const int64_t cols = m == 2 ? intermediate_dim : hidden_dim;
      TORCH_CHECK(t.dim() == 2 && t.size(0) == rows && t.size(1) == cols, names[m], "[", e,
                  "] must have shape [", rows, ", ", cols, "], got shape ", t.sizes());
    }
    g[e] = gate[e].data_ptr();
    u[e] = up[e].data_ptr();
    d[e] = down[e].data_ptr();
  }
  TORCH_CHECK(tp_size >= 1 && intermediate_dim % tp_size == 0,
              "tp_size must divide intermediate_dim");
  const int elt = (int)ref.element_size();
  const int64_t stride = wr_total_weight_bytes(1, hidden_dim, intermediate_dim / tp_size, elt);
  const c10::cuda::CUDAGuard guard(ref.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(ref.device().index()).stream();
  torch::Tensor buf = torch::empty({ep_num * stride / elt}, ref.options());
  check_status(wr_pack_experts(num_experts, hidden_dim, intermediate_dim,
                               ref.scalar_type() == torch::kBFloat16 ? WR_DTYPE_BF16
                                                                     : WR_DTYPE_F32,
                               ep_first, ep_num, tp_rank, tp_size, g.data(), u.data(), d.data(),
                               buf.data_ptr(), ep_num * stride, stream));
  return buf;
}

int64_t workspace_status(torch::Tensor hidden) {
  // Reads and clears the status word of this device/stream's cached workspace.
  const c10::cuda::CUDAGuard guard(hidden.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(hidden.device().index()).stream();
  torch::Tensor ws = workspace_for(hidden.device(), stream, 256);
  return (int64_t)wr_workspace_status(ws.data_ptr(), stream);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("naive_moe_forward", &naive_moe_forward_torch,
        "Naive multi-kernel MoE forward (float32 or bfloat16 inputs, float32 output)");
  m.def("fused_moe_forward", &fused_moe_forward_torch,
        "Fused MoE forward for one decode token (float32 or bfloat16 inputs, float32 output)");
  m.def("batched_fused_moe_forward", &batched_fused_moe_forward_torch,
        "Fused MoE forward for B decode tokens (float32 or bfloat16 inputs, float32 output)");
  m.def("fused_moe_routed", &fused_moe_routed, "Fused MoE forward returning (out, ids, weights)",
        py::arg("hidden"), py::arg("gate_w"), py::arg("weight_buf"), py::arg("num_experts"),
        py::arg("hidden_dim"), py::arg("intermediate_dim"), py::arg("top_k"),
        py::arg("router_bias") = py::none(), py::arg("ep_first_expert") = 0,
        py::arg("ep_num_local") = 0);
  m.def("router_topk", &router_topk, "Router + softmax + top-K: (logits, ids, weights)",
        py::arg("hidden"), py::arg("gate_w"), py::arg("num_experts"), py::arg("hidden_dim"),
        py::arg("top_k"), py::arg("router_bias") = py::none());
  m.def("comm_create", &comm_create, "Communicator of one rank (returns an opaque handle)",
        py::arg("rank"), py::arg("world_size"), py::arg("hidden_dim"));
  m.def("comm_handle", &comm_handle, "This rank's IPC handle bytes (uint8 CPU tensor)");
  m.def("comm_open", &comm_open, "Map every rank's buffer (handles in rank order)");
  m.def("comm_destroy", &comm_destroy, "Unmap and free a communicator");
  m.def("comm_set_peer_timeout_ns", &comm_set_peer_timeout_ns,
        "Bound of each wait for a peer's partial outputs (ns; 0 = default)");
  m.def("comm_reset", &comm_reset,
        "Back to the initial state after a timed-out call (every rank, between host barriers)");
  m.def("fused_moe_allreduce", &fused_moe_allreduce,
        "This rank's shard of the layer with the ranks' outputs summed in the same kernel",
        py::arg("hidden"), py::arg("gate_w"), py::arg("weight_buf"), py::arg("num_experts"),
        py::arg("hidden_dim"), py::arg("intermediate_dim"), py::arg("top_k"), py::arg("comm"),
        py::arg("router_bias") = py::none(), py::arg("ep_first_expert") = 0,
        py::arg("ep_num_local") = 0);
  m.def("moe_decode_layer", &moe_decode_layer,
        "Layer with the residual fused: out = hidden + layer(hidden); next_x = out in the "
        "layer dtype",
        py::arg("hidden"), py::arg("gate_w"), py::arg("weight_buf"), py::arg("num_experts"),
        py::arg("hidden_dim"), py::arg("intermediate_dim"), py::arg("top_k"), py::arg("comm"),
        py::arg("router_bias") = py::none(), py::arg("ep_first_expert") = 0,
        py::arg("ep_num_local") = 0, py::arg("next_x") = py::none());
  m.def("pack_experts", &pack_experts,
        "Pack one rank's shard (experts, intermediate slice) of per-expert weights on the "
        "device");
  m.def("workspace_status", &workspace_status,
        "Read and clear the device status word of the current stream's workspace");
  m.def("version", []() { return std::string(wr_version()); });
}
