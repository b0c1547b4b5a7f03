// wr_comm.cu — communicator for the one-shot all-reduce fused into the tail
// of the streaming kernel (tensor- and expert-parallel layers).
//
// Each rank allocates one device block at set-up — 256 bytes holding its
// launch counter (epoch), then its mailbox of
// [source rank][2 parities][64 tokens][H] 64-bit words — and shares it with
// the other ranks of the node through a CUDA IPC handle.  A fused launch
// with epoch e on rank r stores each of its CTAs' partial output rows as
// words (fp32 value | e << 32) into slot r of every rank's mailbox (peer
// stores over NVLink), then reads its own mailbox: each word is polled
// (bounded) until its epoch is e, and the values are summed in source-rank
// order, so every rank ends with the same fp32 sums.  An aligned 64-bit
// store is single-copy atomic, so a word that shows epoch e also shows its
// value: no flags or memory fences are needed.  Parity e & 1: a rank writes
// a slot for launch e + 2 only after reading every rank's words of launch
// e + 1, which each rank writes only after finishing launch e.
//
// A wait for a peer's words gives up after the communicator's peer timeout
// (2 s unless set) and flags DEV_TIMEOUT_PEER in the workspace status word.
// The launch that gave up still counts its epoch, while a rank that never
// made the call does not, so after such a failure the ranks' epochs differ
// for good: wr_comm_reset on every rank (between two host barriers) puts
// them back in step.
//
// warp-route is single-GPU; this replaces the separate NCCL all-reduce a
// tensor- or expert-parallel caller would run after each layer.
#include <cuda_runtime.h>

#include <cstring>
#include <new>

#include "wr_internal.h"

struct wr_comm {
  int rank = 0, world = 1, H = 0, device = 0;
  uint64_t peer_wait_ns = wr::kPeerWaitDefaultNs;
  void* local = nullptr;
  size_t bytes = 0;
  cudaIpcMemHandle_t handle{};
  void* peers[wr::kMaxRanks] = {nullptr};
  bool open = false;
};

namespace wr {
namespace {

constexpr size_t kCtrlBytes = 256;

size_t comm_bytes(int H) {
  return kCtrlBytes + (size_t)kMaxRanks * 2 * kCommMaxTokens * H * sizeof(uint64_t);
}

}  // namespace

// The view a kernel launch needs (valid once the communicator is open).
wr_status_t comm_view(const wr_comm* c, CommView* v) {
  if (!c || !c->open) return fail(WR_ERR_COMM, "communicator is not open (call wr_comm_open)");
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != c->device)
    return fail(WR_ERR_COMM, "communicator belongs to device %d, current device is %d", c->device,
                dev);
  std::memset(v, 0, sizeof(*v));
  for (int q = 0; q < c->world; ++q)
    v->box[q] = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(c->peers[q]) + kCtrlBytes);
  v->epoch = static_cast<uint32_t*>(c->local);
  v->rank = c->rank;
  v->world = c->world;
  v->H = c->H;
  v->peer_wait_ns = c->peer_wait_ns;
  return WR_OK;
}

}  // namespace wr

using namespace wr;

extern "C" {

size_t wr_comm_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

wr_status_t wr_comm_create(int32_t rank, int32_t world_size, int32_t hidden_dim, wr_comm_t* out) {
  if (!out) return fail(WR_ERR_INVALID, "out must not be NULL");
  *out = nullptr;
  if (world_size < 1 || world_size > kMaxRanks)
    return fail(WR_ERR_UNSUPPORTED, "world_size must be in [1, %d], got %d", kMaxRanks, world_size);
  if (rank < 0 || rank >= world_size)
    return fail(WR_ERR_INVALID, "rank must be in [0, %d), got %d", world_size, rank);
  if (hidden_dim < 1) return fail(WR_ERR_INVALID, "hidden_dim must be positive, got %d", hidden_dim);
  wr_comm* c = new (std::nothrow) wr_comm();
  if (!c) return fail(WR_ERR_COMM, "out of host memory");
  c->rank = rank;
  c->world = world_size;
  c->H = hidden_dim;
  cudaGetDevice(&c->device);
  c->bytes = comm_bytes(hidden_dim);
  cudaError_t e = cudaMalloc(&c->local, c->bytes);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, c->bytes);
  if (e == cudaSuccess && world_size > 1) e = cudaIpcGetMemHandle(&c->handle, c->local);
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    return cuda_fail(e, "wr_comm_create");
  }
  c->peers[rank] = c->local;
  if (world_size == 1) c->open = true;
  *out = c;
  return WR_OK;
}

wr_status_t wr_comm_get_handle(wr_comm_t comm, void* handle) {
  if (!comm || !handle) return fail(WR_ERR_INVALID, "comm and handle must not be NULL");
  std::memcpy(handle, &comm->handle, sizeof(cudaIpcMemHandle_t));
  return WR_OK;
}

wr_status_t wr_comm_open(wr_comm_t comm, const void* handles) {
  if (!comm || !handles) return fail(WR_ERR_INVALID, "comm and handles must not be NULL");
  if (comm->open) return WR_OK;
  const cudaIpcMemHandle_t* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (int q = 0; q < comm->world; ++q) {
    if (q == comm->rank) continue;
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h[q], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int z = 0; z < q; ++z)
        if (z != comm->rank && comm->peers[z]) {
          cudaIpcCloseMemHandle(comm->peers[z]);
          comm->peers[z] = nullptr;
        }
      return cuda_fail(e, "wr_comm_open: cudaIpcOpenMemHandle");
    }
    comm->peers[q] = p;
  }
  comm->open = true;
  return WR_OK;
}

wr_status_t wr_comm_set_peer_timeout_ns(wr_comm_t comm, uint64_t ns) {
  if (!comm) return fail(WR_ERR_INVALID, "comm must not be NULL");
  comm->peer_wait_ns = ns ? ns : kPeerWaitDefaultNs;
  return WR_OK;
}

wr_status_t wr_comm_reset(wr_comm_t comm, wr_stream_t stream) {
  if (!comm) return fail(WR_ERR_INVALID, "comm must not be NULL");
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != comm->device)
    return fail(WR_ERR_COMM, "communicator belongs to device %d, current device is %d",
                comm->device, dev);
  // Epoch 0 and an all-zero mailbox: no launch uses epoch 0, so no word left
  // over from before the reset can pass for a new launch's.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(comm->local, 0, comm->bytes, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "wr_comm_reset");
  return WR_OK;
}

wr_status_t wr_comm_destroy(wr_comm_t comm) {
  if (!comm) return WR_OK;
  for (int q = 0; q < comm->world; ++q)
    if (q != comm->rank && comm->peers[q]) cudaIpcCloseMemHandle(comm->peers[q]);
  if (comm->local) cudaFree(comm->local);
  delete comm;
  return WR_OK;
}

}  // extern "C"
