// wr_noalloc.cu — wr_fused_moe for callers that cannot allocate device
// memory.
//
// Some hosts own the whole device heap — an inference server's memory pool,
// a plugin interface that hands its plugins no workspace — and do not let
// the code they load call cudaMalloc (which can also stall the device while
// it runs).  wr_fused_moe needs a small device workspace (counters and a status
// word, router partial sums, fp32 activations); this entry point takes it
// from a fixed array compiled into the library instead, so the caller passes
// only inputs and outputs.
//
// Costs and limits:
//   * every GPU that loads the library holds kNoAllocScratchBytes (1 MiB)
//     of device memory until the process exits;
//   * one decode token per call, and the layer's workspace must fit:
//     roughly top_k * intermediate_dim * 4 + 8704 bytes <= 1 MiB (Mixtral,
//     DBRX and DeepSeek shapes fit); larger shapes are rejected with
//     WR_ERR_UNSUPPORTED before anything is launched;
//   * all calls on a device share the one array, which keeps the last call's
//     contents: the counters that must start at zero are cleared on the
//     caller's stream before every launch, and calls that overlap on the GPU
//     (several streams, several host threads) race on the array — serialise
//     them;
//   * the status word (set when a bounded wait inside a kernel gave up) is
//     not cleared by a call: wr_fused_moe_noalloc_status reads and clears
//     it, as wr_workspace_status does for a caller's workspace;
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it; make
//     that first call before any stream capture begins.
// No cudaMalloc, cudaFree or allocating library routine is called here.
#include <cuda_runtime.h>

#include <mutex>

#include "wr_internal.h"

namespace wr {
namespace {

constexpr size_t kNoAllocScratchBytes = 1u << 20;
constexpr size_t kControlBytes = kWsControlBytes;  // counters and the status word
constexpr size_t kStatusOffset = 8;                // the status word (32-bit word 2)

// The shared scratch.  Host code must not use this name as a device address:
// on the host it denotes a host-side stand-in.  Its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_dev[kMaxDevices] = {nullptr};

// Device address of the scratch on the current device (looked up once).
wr_status_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "wr_fused_moe_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return fail(WR_ERR_UNSUPPORTED, "wr_fused_moe_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_scratch_dev[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "wr_fused_moe_noalloc: cudaGetSymbolAddress");
    g_scratch_dev[dev] = p;
  }
  *out = g_scratch_dev[dev];
  return WR_OK;
}

}  // namespace
}  // namespace wr

using namespace wr;

extern "C" wr_status_t wr_fused_moe_noalloc(const wr_moe_desc_t* desc, const void* x,
                                            const void* gate_w, const void* weight_buf,
                                            int64_t weight_buf_bytes, float* out,
                                            int32_t* topk_ids, float* topk_weights,
                                            wr_stream_t stream) {
  const size_t need = wr_fused_moe_workspace_size(desc, 1);
  bool args_ok = need != 0 && x && gate_w && out && weight_buf;
  if (args_ok) {
    const int32_t local = desc->ep_num_local ? desc->ep_num_local : desc->num_experts;
    const int32_t elt = desc->dtype == WR_DTYPE_BF16 ? 2 : 4;
    args_ok = weight_buf_bytes >= wr_total_weight_bytes(local, desc->hidden_dim,
                                                        desc->intermediate_dim, elt);
  }
  if (!args_ok) {
    // Let the regular entry point report the bad argument: its descriptor,
    // pointer and weight checks all come before the workspace check, so it
    // returns that error and launches nothing.
    return wr_fused_moe(desc, x, gate_w, weight_buf, weight_buf_bytes, out, topk_ids,
                        topk_weights, nullptr, 0, stream);
  }
  if (need > kNoAllocScratchBytes)
    return fail(WR_ERR_UNSUPPORTED,
                "wr_fused_moe_noalloc: this layer needs %zu bytes of scratch; the built-in "
                "scratch holds %zu (use wr_fused_moe with a caller-allocated workspace)",
                need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  wr_status_t st = scratch_address(&scratch);
  if (st != WR_OK) return st;
  // Every control word but the status word, which keeps a failed wait's bits
  // until wr_fused_moe_noalloc_status reads them.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ctl = static_cast<uint8_t*>(scratch);
  cudaError_t e = cudaMemsetAsync(ctl, 0, kStatusOffset, s);
  if (e == cudaSuccess)
    e = cudaMemsetAsync(ctl + kStatusOffset + 4, 0, kControlBytes - kStatusOffset - 4, s);
  if (e != cudaSuccess) return cuda_fail(e, "wr_fused_moe_noalloc: clearing the control words");
  return wr_fused_moe(desc, x, gate_w, weight_buf, weight_buf_bytes, out, topk_ids, topk_weights,
                      scratch, kNoAllocScratchBytes, stream);
}

extern "C" wr_status_t wr_fused_moe_noalloc_status(wr_stream_t stream) {
  void* scratch = nullptr;
  wr_status_t st = scratch_address(&scratch);
  if (st != WR_OK) return st;
  return wr_workspace_status(scratch, stream);
}
