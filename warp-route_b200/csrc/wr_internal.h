// wr_internal.h — host-side declarations shared by the C ABI (wr_api.cu) and
// the kernel translation units.  Not part of the public ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/warp_route_b200.h"

namespace wr {

// Bytes at the start of every workspace reserved for the fused kernel's
// control words (per-slot completion counters, exit counter, status word):
// zero before the first call, left zero by every call.  The naive path keeps
// its scratch behind them so both can share one workspace.
constexpr size_t kWsControlBytes = 512;

// ---- peer-memory all-reduce (wr_comm.cu) ----
constexpr int kMaxRanks = 8;
constexpr int kCommMaxTokens = 64;  // tokens one kernel launch all-reduces

// What the fused kernel needs of a communicator: every rank's mailbox,
// mapped into this process, and this rank's launch counter.  A mailbox is
// [source rank][2 parities][kCommMaxTokens][H] 64-bit words, each the fp32
// partial output of one (token, row) in its low half and the epoch of the
// launch that wrote it in its high half.
struct CommView {
  uint64_t* box[kMaxRanks];
  uint32_t* epoch;
  int rank, world, H;
  uint64_t peer_wait_ns;  // bound of each wait for a peer's words (ns)
};

// Default bound of a wait for a peer rank's partial outputs (ns).
constexpr uint64_t kPeerWaitDefaultNs = 2000000000ull;

// The kernel's view of an open communicator on the current device.
wr_status_t comm_view(const wr_comm* c, CommView* v);

// The residual connection of a decode stack, fused into a layer's last
// step: out = x + layer(x) (fp32), and next_x = out rounded to the layer's
// dtype (the next layer's input).  x == null: no residual.
struct Residual {
  const void* x;   // [T, H] in the layer dtype
  void* next_x;    // [T, H] in the layer dtype, or null
  int bf16;        // layer dtype is bf16 (else fp32)
};

// Per-call problem description after validation.
struct Problem {
  int E, H, I, K, T;          // experts, hidden, intermediate, top_k, tokens
  int ep_first, ep_num;       // expert-parallel shard (ep_num = E: no EP)
  int dtype;                  // wr_dtype_t
  int elt;                    // bytes per element
  const float* router_bias;   // optional [E]
  Residual res;               // res.x == null: no fused residual
};

// Sets the thread's last-error text (printf-style) and returns `s`.
wr_status_t fail(wr_status_t s, const char* fmt, ...);

// Maps a CUDA error to WR_ERR_CUDA with a message naming `what`.
wr_status_t cuda_fail(cudaError_t e, const char* what);

// ---- fused streaming kernel (wr_fused.cu) ----
// True when the streaming kernel can take this problem (alignment, sizes).
bool fused_supported(const Problem& p);
size_t fused_workspace_bytes(const Problem& p);
// comm: null, or the communicator whose ranks' partial outputs are summed
// into `out` (identical on every rank).
wr_status_t launch_fused(const Problem& p, const void* x, const void* gate_w,
                         const void* wbuf, float* out, int32_t* ids, float* w,
                         void* ws, cudaStream_t stream, const CommView* comm = nullptr);

// ---- grouped tensor-core path for token batches (wr_grouped.cu) ----
// Batches of at least this many tokens run as grouped GEMMs over tokens
// bucketed per expert (fewer take the streaming kernel).
constexpr int kGroupedMinTokens = 2;     // bf16 batches from 2 tokens run as grouped GEMMs
constexpr int kGroupedMinTokensF32 = 3;  // fp32: 2 tokens stream faster (measured)
bool grouped_supported(const Problem& p);
size_t grouped_workspace_bytes(const Problem& p);
// comm: null, or the communicator whose ranks' partial outputs the combine
// step sums over peer memory (identical on every rank).
wr_status_t launch_grouped(const Problem& p, const void* x, const void* gate_w,
                           const void* wbuf, float* out, int32_t* ids, float* w, void* ws,
                           cudaStream_t stream, const CommView* comm = nullptr);

// ---- router kernel (wr_naive.cu) ----
wr_status_t launch_router(const Problem& p, const void* x, const void* gate_w,
                          float* logits, int32_t* ids, float* w, cudaStream_t stream);

// ---- naive multi-kernel path (wr_naive.cu) ----
size_t naive_workspace_bytes(const Problem& p);
wr_status_t launch_naive(const Problem& p, const void* x, const void* gate_w,
                         const void* wbuf, float* out, int32_t* ids, float* w,
                         void* ws, cudaStream_t stream);

// Number of SMs of the current device (cached per device).
int device_sm_count();

}  // namespace wr
