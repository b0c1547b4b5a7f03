// wr_pack.cu — packs one rank's shard of the experts into the flat layout
// on the device, in one launch.
//
// warp-route packs with one torch copy per matrix and expert
// (warp_route/functional.py:21-57); a multi-GPU caller would also have to
// slice every matrix for its rank first.  Here every row segment of the
// shard is one CTA's contiguous copy:
//   gate / up row i of the slice  <- source row (tp_rank * I_l + i), H elements
//   down row h of the slice       <- source row h, columns [tp_rank * I_l, +I_l)
// written at the layout's offsets (expert stride rounded up to 128 bytes,
// the rounding bytes zeroed).
#include <cuda_runtime.h>

#include "wr_common.cuh"
#include "wr_internal.h"

namespace wr {
namespace {

constexpr int kPackMaxExperts = 64;

struct PackArgs {
  const uint8_t* gate[kPackMaxExperts];  // indexed by local slot
  const uint8_t* up[kPackMaxExperts];
  const uint8_t* down[kPackMaxExperts];
  uint8_t* dst;
  int64_t stride;   // bytes per packed expert
  int H, I, Il;     // hidden, full intermediate, intermediate of the slice
  int i0;           // first intermediate row of the slice
  int elt;
};

// Copies `bytes` from src to dst with 16-byte vectors when both are aligned
// and the length allows, else byte by byte.  Called by a whole CTA.
__device__ void copy_row(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src,
                         int64_t bytes) {
  const bool vec = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) |
                     static_cast<uintptr_t>(bytes)) & 15) == 0;
  if (vec) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int64_t j = threadIdx.x; j < bytes / 16; j += blockDim.x) d[j] = s[j];
  } else {
    for (int64_t j = threadIdx.x; j < bytes; j += blockDim.x) dst[j] = src[j];
  }
}

// blockIdx.y = local expert slot, blockIdx.x = row of the packed expert:
// [0, Il) gate, [Il, 2 Il) up, [2 Il, 2 Il + H) down.
__global__ void __launch_bounds__(128) k_pack(const PackArgs a) {
  const int e = blockIdx.y;
  const int row = blockIdx.x;
  uint8_t* base = a.dst + (int64_t)e * a.stride;
  const int64_t gu_row = (int64_t)a.H * a.elt;
  if (row < 2 * a.Il) {
    const bool is_up = row >= a.Il;
    const int i = is_up ? row - a.Il : row;
    const uint8_t* src = (is_up ? a.up[e] : a.gate[e]) + (int64_t)(a.i0 + i) * gu_row;
    copy_row(base + (int64_t)row * gu_row, src, gu_row);
  } else {
    const int h = row - 2 * a.Il;
    const uint8_t* src = a.down[e] + ((int64_t)h * a.I + a.i0) * a.elt;
    const int64_t seg = (int64_t)a.Il * a.elt;
    copy_row(base + 2 * (int64_t)a.Il * gu_row + (int64_t)h * seg, src, seg);
  }
  if (row == 0) {  // the bytes that round the expert stride up to 128
    const int64_t used = 3 * (int64_t)a.Il * a.H * a.elt;
    for (int64_t j = used + threadIdx.x; j < a.stride; j += blockDim.x) base[j] = 0;
  }
}

}  // namespace
}  // namespace wr

using namespace wr;

extern "C" wr_status_t wr_pack_experts(int32_t num_experts, int32_t hidden_dim,
                                       int32_t intermediate_dim, int32_t dtype,
                                       int32_t ep_first, int32_t ep_num, int32_t tp_rank,
                                       int32_t tp_size, const void* const* gate,
                                       const void* const* up, const void* const* down, void* dst,
                                       int64_t dst_bytes, wr_stream_t stream) {
  if (dtype != WR_DTYPE_F32 && dtype != WR_DTYPE_BF16)
    return fail(WR_ERR_INVALID, "dtype must be float32 or bfloat16, got code %d", dtype);
  if (num_experts < 1 || hidden_dim < 1 || intermediate_dim < 1)
    return fail(WR_ERR_INVALID, "num_experts, hidden_dim and intermediate_dim must be positive");
  if (ep_first < 0 || ep_num < 1 || ep_first + ep_num > num_experts)
    return fail(WR_ERR_INVALID, "expert shard [%d, %d) is outside [0, %d)", ep_first,
                ep_first + ep_num, num_experts);
  if (ep_num > kPackMaxExperts)
    return fail(WR_ERR_UNSUPPORTED, "a shard packs at most %d experts, got %d", kPackMaxExperts,
                ep_num);
  if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size || intermediate_dim % tp_size != 0)
    return fail(WR_ERR_INVALID,
                "tensor-parallel rank %d of %d must split intermediate_dim %d evenly", tp_rank,
                tp_size, intermediate_dim);
  if (!gate || !up || !down || !dst)
    return fail(WR_ERR_INVALID, "gate, up, down and dst must not be NULL");
  const int elt = dtype == WR_DTYPE_BF16 ? 2 : 4;
  const int Il = intermediate_dim / tp_size;
  const Layout lay = make_layout(hidden_dim, Il, elt);
  const int64_t need = (int64_t)ep_num * lay.stride;
  if (dst_bytes < need)
    return fail(WR_ERR_TOO_SMALL, "weight_buf too small: need %lld bytes, got %lld",
                (long long)need, (long long)dst_bytes);
  PackArgs a;
  for (int j = 0; j < ep_num; ++j) {
    const int e = ep_first + j;
    if (!gate[e] || !up[e] || !down[e])
      return fail(WR_ERR_INVALID, "expert %d of the shard has a NULL matrix", e);
    a.gate[j] = static_cast<const uint8_t*>(gate[e]);
    a.up[j] = static_cast<const uint8_t*>(up[e]);
    a.down[j] = static_cast<const uint8_t*>(down[e]);
  }
  a.dst = static_cast<uint8_t*>(dst);
  a.stride = lay.stride;
  a.H = hidden_dim;
  a.I = intermediate_dim;
  a.Il = Il;
  a.i0 = tp_rank * Il;
  a.elt = elt;
  const int rows = 2 * Il + hidden_dim;
  k_pack<<<dim3(rows, ep_num), 128, 0, static_cast<cudaStream_t>(stream)>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? WR_OK : cuda_fail(e, "k_pack launch");
}
